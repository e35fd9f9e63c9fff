"""The forward kernel against wiretorch's own results (golden cases), on the B200.

* **Lockstep** (the reference's definition of "the same simulator",
  ``tests/test_lockstep.py``): restart from every recorded window state and take the
  window's steps; spikes must match exactly (a neuron within 1e-3 mV of threshold
  excused, at most 1% of trial-windows), voltages and conductances within the tolerances
  below.
* **Free run**: the whole 200-step input from the initial state gives exactly the
  recorded spike raster.
* **Determinism**: the synaptic input is accumulated in fixed point, so two runs are
  bit-for-bit identical.

Tolerances: voltages 2e-4 mV absolute (the reference's own CUDA lockstep test allows
1e-3, ``tests/test_lockstep.py:24-27``), conductances 1e-5 relative (the target of
this build).
"""

import numpy as np
import pytest
import torch

import golden_io
from wiretorch_b200 import engine

pytestmark = pytest.mark.gpu

CASES = golden_io.cases()
THRESHOLD_MARGIN = 1e-3
V_ATOL = 2e-4
G_RTOL, G_ATOL = 1e-5, 1e-6


def _state_kw(d, prefix, w=None, device="cuda"):
    out = {}
    for key in ("refractory", "gating", "adaptation"):
        name = f"{prefix}{key}"
        if name in d:
            a = d[name] if w is None else d[name][w]
            out[key] = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return out


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _engine_run(drive, p, d, meta, x, v, g, kw, pool):
    engine.POOL_SYNAPSES = pool
    try:
        with torch.no_grad():
            return engine.simulate(_t(v), _t(g), _t(x), drive, p, **kw,
                                   probabilities=meta["probabilities"], track=True,
                                   track_batch_idx=None)  # fmt: skip
    finally:
        engine.POOL_SYNAPSES = False


@pytest.mark.parametrize("pool", [False, True], ids=["exact", "pooled"])
@pytest.mark.parametrize("name", CASES)
def test_lockstep(name, pool):
    drive, p, d, meta = golden_io.load(name, "cuda")
    x = d["in.x"]
    W, B = meta["window"], x.shape[0]
    theta = p.theta.cpu().numpy()
    excused, worst_v, worst_g = 0, 0.0, 0.0
    for w, start in enumerate(range(0, x.shape[1], W)):
        stop = start + W
        run = _engine_run(drive, p, d, meta, x[:, start:stop], d["out.win_v"][w],
                          d["out.win_g"][w], _state_kw(d, "out.win_", w), pool)  # fmt: skip
        spikes = run.output.cpu().numpy() > 0.5
        ok = np.ones(B, bool)
        diff = spikes != d["out.spikes"][:, start:stop]
        if diff.any():
            v_enter = np.concatenate([d["out.win_v"][w][:, None],
                                      d["out.v_track"][:, start : stop - 1]], 1)  # fmt: skip
            for b, t, n in zip(*np.nonzero(diff)):
                if ok[b]:
                    margin = abs(v_enter[b, t, n] - theta[n])
                    assert margin < THRESHOLD_MARGIN, (w, b, t, n, margin)
                    ok[b] = False
                    excused += 1
        v_track = run.tracked["v"].cpu().numpy()
        np.testing.assert_allclose(v_track[ok], d["out.v_track"][ok, start:stop], rtol=0,
                                   atol=V_ATOL, err_msg=f"window {w}")  # fmt: skip
        g_next = d["out.win_g"][w + 1]
        got = run.syn.cpu().numpy()
        if pool:  # compare the pooled sums
            got = _pool_sums(got, engine.get_plan(drive, p, B, x.shape[2], "cuda", True))
            g_next = _pool_sums(g_next, engine.get_plan(drive, p, B, x.shape[2], "cuda", True))
        np.testing.assert_allclose(got[ok], g_next[ok], rtol=G_RTOL, atol=G_ATOL,
                                   err_msg=f"window {w}")  # fmt: skip
        for key in ("refractory", "gating", "adaptation"):
            if f"out.win_{key}" in d and getattr(run, key) is not None:
                np.testing.assert_allclose(getattr(run, key).cpu().numpy()[ok],
                                           d[f"out.win_{key}"][w + 1][ok], rtol=1e-5, atol=1e-6)  # fmt: skip
        if meta["probabilities"]:
            np.testing.assert_allclose(run.probabilities.cpu().numpy()[ok],
                                       d["out.prob"][ok, start:stop], rtol=0, atol=1e-5)  # fmt: skip
        worst_v = max(worst_v, float(np.abs(v_track[ok] - d["out.v_track"][ok, start:stop]).max(initial=0)))
    assert excused <= 0.01 * (x.shape[1] // W) * B


def _pool_sums(g, plan):
    """(B, N, 2, S) -> (B, N, 2, S') summed over each pool."""
    return np.stack([g[..., m].sum(-1) for m in plan.ch.member], -1)


@pytest.mark.parametrize("pool", [False, True], ids=["exact", "pooled"])
@pytest.mark.parametrize("name", CASES)
def test_free_run_is_spike_exact(name, pool):
    drive, p, d, meta = golden_io.load(name, "cuda")
    run = _engine_run(drive, p, d, meta, d["in.x"], d["in.v"], d["in.g"],
                      _state_kw(d, "in."), pool)  # fmt: skip
    spikes = run.output.cpu().numpy() > 0.5
    differs = (spikes != d["out.spikes"]).any(axis=(0, 2))
    assert not differs.any(), f"first divergence at step {int(np.argmax(differs))}"
    np.testing.assert_allclose(run.tracked["v"].cpu().numpy(), d["out.v_track"], rtol=0,
                               atol=V_ATOL)  # fmt: skip


@pytest.mark.parametrize("name", ["recurrent_frozen", "recurrent_stp", "feedforward_features"])
def test_runs_are_bitwise_reproducible(name):
    drive, p, d, meta = golden_io.load(name, "cuda")
    runs = [
        _engine_run(drive, p, d, meta, d["in.x"], d["in.v"], d["in.g"], _state_kw(d, "in."), False)
        for _ in range(2)
    ]
    assert torch.equal(runs[0].output, runs[1].output)
    assert torch.equal(runs[0].v, runs[1].v)
    assert torch.equal(runs[0].syn, runs[1].syn)


@pytest.mark.parametrize("name", ["recurrent_scaling_factors", "recurrent_refractory"])
def test_chunking_does_not_matter(name):
    """Splitting the input into chunks gives the same run (``test_invariants.py:36``)."""
    drive, p, d, meta = golden_io.load(name, "cuda")
    x = d["in.x"]
    whole = _engine_run(drive, p, d, meta, x, d["in.v"], d["in.g"], _state_kw(d, "in."), False)
    v, g, kw = _t(d["in.v"]), _t(d["in.g"]), _state_kw(d, "in.")
    outs = []
    for start in range(0, x.shape[1], 7):
        with torch.no_grad():
            run = engine.simulate(v, g, _t(x[:, start : start + 7]), drive, p, **kw)
        outs.append(run.output)
        v, g = run.v, run.syn
        kw = {k: getattr(run, k) for k in kw}
    assert torch.equal(torch.cat(outs, 1), whole.output)
    assert torch.equal(v, whole.v)
