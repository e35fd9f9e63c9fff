"""The oracle's current-based step (``cond_lif.c`` with ``current`` set, restating
``network_simulators/current/dynamics.py:116-205``) against the reference's own runs of
its current-based test networks (golden cases ``current_*``; three also match the
reference suite's recordings): the spike raster exactly, voltages within 1e-5 (natural
units, threshold 1) and the final currents within 1e-5 relative. Both of the oracle's
schedules (whole trials per thread, and each step's neurons over all threads) are run."""

import numpy as np
import pytest

import golden_io
from oracle import oracle

CASES = golden_io.current_cases()


@pytest.mark.parametrize("threads", [1, 4])
@pytest.mark.parametrize("name", CASES)
def test_oracle_free_run_matches_reference(name, threads):
    drive, p, d, meta = golden_io.load(name)
    oracle.set_threads(threads)
    try:
        net = oracle.Network(drive, p, d["in.x"].shape[0], d["in.x"].shape[2])
        kw = {k: d[f"in.{k}"] for k in ("refractory", "gating", "adaptation") if f"in.{k}" in d}
        out = net.simulate(d["in.x"], d["in.v"], d["in.g"], probabilities=meta["probabilities"], **kw)
    finally:
        oracle.set_threads(1)
    differs = (out["spikes"] != d["out.spikes"]).any(axis=(0, 2))
    assert not differs.any(), f"first divergence at step {int(np.argmax(differs))}"
    np.testing.assert_allclose(out["v_track"], d["out.v_track"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(out["g"], d["out.g"], rtol=1e-5, atol=1e-6)
    if meta["probabilities"]:
        np.testing.assert_allclose(out["prob"], d["out.prob"], rtol=0, atol=1e-5)
    if "rec.spikes" in d:
        assert (out["spikes"] == d["rec.spikes"]).all()


def test_c2c_configuration_at_a_tenth():
    """The current-based C2 configuration (``configs.c2_current``) at a tenth of its
    neurons with the same in-degrees: each cell type's synapse type carries the type's
    sign and time constant, the state is the currents (B, N, S), and the oracle's
    current-based step fires it in the benchmark's range (a few Hz, not silent, not
    saturated)."""
    from wiretorch_b200 import configs

    cfg = configs.c2_current(B=2, T=500, device="cpu", N=2000, p_max=0.5)
    v, I, kw = cfg.state()
    S = cfg.drive.made.shape[1]
    assert I.shape == (2, 2000, S) and v.shape == (2, 2000)
    assert set(cfg.p.sign.tolist()) == {1.0, -1.0} and float(cfg.p.sign[-1]) == 1.0
    exc = cfg.p.sign > 0
    np.testing.assert_allclose(cfg.p.decay[exc].numpy(), np.exp(-0.1 / 5.0), rtol=1e-6)
    np.testing.assert_allclose(cfg.p.decay[~exc].numpy(), np.exp(-0.1 / 10.0), rtol=1e-6)
    net = oracle.Network(cfg.drive, cfg.p, cfg.B, cfg.n_in)
    out = net.simulate(cfg.inputs(seed=1), v, I, **kw, track=False)
    rate = out["spikes"].mean() / 1e-4
    assert 1.0 < rate < 30.0, rate


def test_field_mapping_follows_the_physiology():
    """The current-based physiology as the kernel's fields: U_rest as E_L, R as C_m, the
    signs as E_syn, each type a decay component with a unit jump; cached per physiology
    and its tensors, so that a field replaced on the same object is seen."""
    import torch

    from wiretorch_b200 import current
    from wiretorch_b200.types import CurrentPhysiology

    N = 4
    p = CurrentPhysiology(theta=torch.ones(N), U_reset=torch.zeros(N), beta=torch.full((N,), 0.9),
                          U_rest=torch.full((N,), 0.1), R=torch.full((N,), 2.0), sign=torch.tensor([1.0, -1.0]),
                          decay=torch.tensor([0.9, 0.8]), surr_scale=torch.tensor(5.0))  # fmt: skip
    f = current._fields(p)
    assert f.E_L is p.U_rest and f.C_m is p.R and f.beta is p.beta and f.current
    assert torch.equal(f.E_syn, p.sign) and torch.equal(f.decay[1], p.decay) and not f.decay[0].any()
    assert torch.equal(f.jump, torch.tensor([[0.0, 0.0], [1.0, 1.0]]))
    assert current._fields(p) is f
    p.theta = torch.full((N,), 2.0)
    assert current._fields(p).theta is p.theta


# ---- at the reference's statistics scale (2,000 and 1,000 neurons, 3,000 / 2,000 steps) ----


def _curstats_run(name):
    """The oracle's free run of a ``curstats_*`` case's first input in 250-step calls (the
    state carried), after the burn-in; and the case."""
    drive, p, d, meta = golden_io.load(name)
    A = meta["seeds"][0]
    x = d[f"in.x_{A}"]
    oracle.set_threads(4)
    try:
        net = oracle.Network(drive, p, x.shape[0], x.shape[2])
        v, g = d["in.v"], d["in.g"]
        kw = {k: d[f"in.{k}"] for k in ("refractory", "gating", "adaptation") if f"in.{k}" in d}
        spikes = []
        for start in range(0, x.shape[1], meta["chunk"]):
            out = net.simulate(x[:, start : start + meta["chunk"]], v, g, **kw, track=False)
            spikes.append(out["spikes"])
            v, g = out["v"], out["g"]
            kw = {k: (out[k] if out[k] is not None else kw[k]) for k in kw}
    finally:
        oracle.set_threads(1)
    return np.concatenate(spikes, 1)[:, meta["burn_in"] :], d, meta


def test_oracle_current_statistics_recurrent():
    """The current-based recurrent network of the reference's statistics test: per-type
    population rates within the reference's own tolerance (twice the spread between its
    two recorded inputs, at least 2%) of its recording, and the raster of the reference's
    CPU run of the same input reproduced spike for spike (4 trials x 2,000 neurons x 2,500
    steps after the burn-in)."""
    spikes, d, meta = _curstats_run("curstats_recurrent")
    types = d["in.types"]
    A, B = meta["seeds"]
    means = golden_io.population_rates(spikes, types, meta["dt"])
    rec_a, rec_b = d[f"rec.rates_{A}"], d[f"rec.rates_{B}"]
    ref = np.array([rec_a[types == t].mean() for t in np.unique(types)])
    ref_b = np.array([rec_b[types == t].mean() for t in np.unique(types)])
    allowed = np.maximum(2 * np.abs(ref_b - ref), 0.02 * ref)
    assert np.all(np.abs(means - ref) <= allowed), (means, ref, allowed)
    cpu_means = golden_io.population_rates(d["out.spikes"], types, meta["dt"])
    assert np.all(np.abs(means - cpu_means) <= allowed)
    assert (spikes == d["out.spikes"]).all()


def test_oracle_current_statistics_feedforward():
    """The current-based feedforward network: the reference's CPU run here reproduced
    spike for spike (4 trials x 1,000 neurons x 1,500 steps), and its recorded raster to
    within 0.1% of the spikes (the recording itself differs from the CPU run here by 36 of
    171,310 spikes, 2e-4: another machine's float32 rounding)."""
    spikes, d, meta = _curstats_run("curstats_feedforward")
    assert (spikes == d["out.spikes"]).all()
    assert (spikes != d["rec.spikes"]).sum() / d["rec.spikes"].sum() < 1e-3
