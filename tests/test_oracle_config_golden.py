"""The oracle against the reference at the benchmark configurations' scale and on the
reference's own at-scale statistics networks, before it is trusted at full size.

``config_c1`` is configuration 1 at its specified size (1,000 neurons, 8 trials, 1,000
steps); ``config_c2/c4/c5`` are configurations 2, 4 and 5 built the same way at 2,000
neurons (``tests/golden/make_golden.py``). The reference ran each through its own CPU
dynamics (``conductance/dynamics.py:146-237``). The acceptance bar: identical spike
rasters, and voltages within 1e-5 relative at every recorded step before the first
spike that differs (the reference's fp32 against the oracle's fp32 with synaptic sums
in double: an ulp apart at most until then).

The statistics networks (``tests/fixtures/generate.py`` ``STATS_NETWORKS`` of the
reference) are judged as the reference's ``tests/test_statistics.py:50-85`` judges its
own simulators: per-type mean rates within twice the difference between the two
recorded inputs, or 2%, of the recording; the feedforward network's spikes within 0.1%.
"""

import numpy as np
import pytest

import golden_io
from oracle import oracle

V_RTOL = 1e-5


def _kw(d, prefix):
    return {k: d[f"{prefix}{k}"] for k in ("refractory", "gating", "adaptation") if f"{prefix}{k}" in d}


def check_free_run(spikes, v_snap, d, meta, min_identical=None):
    """Spikes against the case's raster; voltages at the recorded steps before the first
    difference within ``V_RTOL``. Returns the first differing step (T if none)."""
    ref = d["out.spikes"]
    T = ref.shape[1]
    first = golden_io.first_divergence(spikes, ref)
    snap = meta["snap"]
    for w in range(T // snap):
        if (w + 1) * snap > first:
            break
        np.testing.assert_allclose(v_snap[w], d["out.v_snap"][w], rtol=V_RTOL, atol=0,
                                   err_msg=f"voltages after step {(w + 1) * snap}")  # fmt: skip
    assert first >= (T if min_identical is None else min_identical), f"rasters differ from step {first} of {T}"
    return first


def oracle_snapshots(net, x, v, g, kw, snap):
    spikes, v_snap = [], []
    for start in range(0, x.shape[1], snap):
        out = net.simulate(x[:, start : start + snap], v, g, **kw, track=False)
        spikes.append(out["spikes"])
        v, g = out["v"], out["g"]
        kw = {k: (out[k] if out[k] is not None else kw[k]) for k in kw}
        v_snap.append(v.copy())
    return np.concatenate(spikes, 1), np.stack(v_snap), v, g, kw


@pytest.mark.parametrize("name", golden_io.config_cases())
def test_oracle_reproduces_the_reference_at_config_scale(name):
    drive, p, d, meta = golden_io.load(name)
    x = d["in.x"]
    oracle.set_threads(4)
    net = oracle.Network(drive, p, x.shape[0], x.shape[2])
    spikes, v_snap, v, g, kw = oracle_snapshots(net, x, d["in.v"], d["in.g"], _kw(d, "in."), meta["snap"])
    assert d["out.spikes"].sum() > 200  # the network is active
    check_free_run(spikes, v_snap, d, meta)
    np.testing.assert_allclose(v, d["out.v"], rtol=V_RTOL, atol=0)
    np.testing.assert_allclose(g, d["out.g"], rtol=1e-5, atol=1e-6)
    for key, value in kw.items():
        np.testing.assert_allclose(value, d[f"out.{key}"], rtol=1e-5, atol=1e-6)


def statistics_rates(run, name):
    """``(rates (N,), population means per type)`` of one input's free run after the
    burn-in, and the case's allowed deviation per type and the recorded means."""
    drive, p, d, meta = golden_io.load(name)
    types = d["in.types"]
    A, B = meta["seeds"]
    spikes = run(drive, p, d, meta, d[f"in.x_{A}"])[:, meta["burn_in"] :]
    rates = spikes.mean(axis=(0, 1)) * 1000.0 / float(p.dt)
    means = np.array([rates[types == t].mean() for t in np.unique(types)])
    rec_a, rec_b = d[f"rec.rates_{A}"], d[f"rec.rates_{B}"]
    ref = np.array([rec_a[types == t].mean() for t in np.unique(types)])
    ref_b = np.array([rec_b[types == t].mean() for t in np.unique(types)])
    allowed = np.maximum(2 * np.abs(ref_b - ref), 0.02 * ref)
    return spikes, rates, means, ref, allowed, d


def oracle_run(drive, p, d, meta, x):
    oracle.set_threads(4)
    net = oracle.Network(drive, p, x.shape[0], x.shape[2])
    spikes, _, _, _, _ = oracle_snapshots(net, x, d["in.v"], d["in.g"], _kw(d, "in."), meta["chunk"])
    return spikes


def test_oracle_statistics_recurrent():
    spikes, rates, means, ref, allowed, d = statistics_rates(oracle_run, "statistics_recurrent")
    assert np.all(np.abs(means - ref) <= allowed), (means, ref, allowed)
    A, B = 0, 1
    floor = np.corrcoef(d[f"rec.rates_{A}"], d[f"rec.rates_{B}"])[0, 1]
    assert np.corrcoef(rates, d[f"rec.rates_{A}"])[0, 1] >= floor - 0.01
    # and the reference's CPU run of the same input, as far as its raster goes
    cpu = d["out.spikes"]
    cpu_means = golden_io.population_rates(cpu, d["in.types"], 1.0)
    assert np.all(np.abs(means - cpu_means) <= allowed)


def test_oracle_statistics_feedforward():
    spikes, rates, means, ref, allowed, d = statistics_rates(oracle_run, "statistics_feedforward")
    recorded = d["rec.spikes"]
    mismatched = (spikes != recorded).sum() / recorded.sum()
    assert mismatched < 1e-3, f"{mismatched:.2%} of spikes differ from the recording"
    assert (spikes != d["out.spikes"]).sum() / d["out.spikes"].sum() < 1e-3
