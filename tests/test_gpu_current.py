"""The current-based family (``wiretorch_b200.current``, the forward kernel's
``WT_F_CURRENT`` mode) against the reference's own current-based dynamics
(``network_simulators/current/dynamics.py``) on its test networks (golden cases
``current_*``; three of them also match the reference suite's recordings), on the B200.

* **Lockstep**: restart from every recorded window state and take the window's steps;
  spikes must match exactly (a neuron within 1e-4 of threshold excused, at most 1% of
  trial-windows), voltages within 1e-5 and currents within 1e-5 relative.
* **Free run**: the whole 200-step input from the initial state gives exactly the
  recorded spike raster.

Voltages are in the family's natural units (reset 0, threshold 1): 1e-5 is a hundred-
thousandth of the reset-to-threshold gap. The kernel sums a step's synaptic input over all
pathways in fixed point; the reference adds pathway after pathway in float32.
"""

import numpy as np
import pytest
import torch

import golden_io
from wiretorch_b200 import current

pytestmark = pytest.mark.gpu

CASES = golden_io.current_cases()
THRESHOLD_MARGIN = 1e-4
V_ATOL = 1e-5
I_RTOL, I_ATOL = 1e-5, 1e-6


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _kw(d, prefix, w=None):
    out = {}
    for key in ("refractory", "gating", "adaptation"):
        name = f"{prefix}{key}"
        if name in d:
            out[key] = _t(d[name] if w is None else d[name][w])
    return out


def _run(drive, p, meta, x, v, I, kw):
    with torch.no_grad():
        return current.simulate(_t(v), _t(I), _t(x), drive, p, **kw, probabilities=meta["probabilities"],
                                track=True, track_batch_idx=None)  # fmt: skip


def test_cases_exist():
    assert len(CASES) >= 4, CASES


@pytest.mark.parametrize("name", CASES)
def test_lockstep(name):
    drive, p, d, meta = golden_io.load(name, "cuda")
    x = d["in.x"]
    W, B = meta["window"], x.shape[0]
    theta = p.theta.cpu().numpy()
    excused = 0
    for w, start in enumerate(range(0, x.shape[1], W)):
        stop = start + W
        run = _run(drive, p, meta, x[:, start:stop], d["out.win_v"][w], d["out.win_g"][w], _kw(d, "out.win_", w))
        spikes = run.output.cpu().numpy() > 0.5
        ok = np.ones(B, bool)
        diff = spikes != d["out.spikes"][:, start:stop]
        if diff.any():
            v_enter = np.concatenate([d["out.win_v"][w][:, None], d["out.v_track"][:, start : stop - 1]], 1)
            for b, t, n in zip(*np.nonzero(diff)):
                if ok[b]:
                    margin = abs(v_enter[b, t, n] - theta[n])
                    assert margin < THRESHOLD_MARGIN, (w, b, t, n, margin)
                    ok[b] = False
                    excused += 1
        np.testing.assert_allclose(run.tracked["v"].cpu().numpy()[ok], d["out.v_track"][ok, start:stop], rtol=0,
                                   atol=V_ATOL, err_msg=f"window {w}")  # fmt: skip
        np.testing.assert_allclose(run.syn.cpu().numpy()[ok], d["out.win_g"][w + 1][ok], rtol=I_RTOL, atol=I_ATOL,
                                   err_msg=f"window {w}")  # fmt: skip
        for key in ("refractory", "gating", "adaptation"):
            if f"out.win_{key}" in d and getattr(run, key) is not None:
                np.testing.assert_allclose(getattr(run, key).cpu().numpy()[ok], d[f"out.win_{key}"][w + 1][ok],
                                           rtol=1e-5, atol=1e-6, err_msg=f"{key}, window {w}")  # fmt: skip
        if meta["probabilities"]:
            np.testing.assert_allclose(run.probabilities.cpu().numpy()[ok], d["out.prob"][ok, start:stop], rtol=0,
                                       atol=1e-5)  # fmt: skip
    assert excused <= 0.01 * (x.shape[1] // W) * B


@pytest.mark.parametrize("name", CASES)
def test_free_run_is_spike_exact(name):
    drive, p, d, meta = golden_io.load(name, "cuda")
    run = _run(drive, p, meta, d["in.x"], d["in.v"], d["in.g"], _kw(d, "in."))
    spikes = run.output.cpu().numpy() > 0.5
    differs = (spikes != d["out.spikes"]).any(axis=(0, 2))
    assert not differs.any(), f"first divergence at step {int(np.argmax(differs))}"
    np.testing.assert_allclose(run.tracked["v"].cpu().numpy(), d["out.v_track"], rtol=0, atol=V_ATOL)
    if "rec.spikes" in d:  # the reference suite's own recording
        assert (spikes == d["rec.spikes"]).all()


def test_tracked_currents_and_chunking():
    """The tracked currents are the state after each step's input (the last equals the
    final state), and a run split into two calls equals one call."""
    drive, p, d, meta = golden_io.load("current_recurrent", "cuda")
    x = d["in.x"]
    whole = _run(drive, p, meta, x, d["in.v"], d["in.g"], {})
    np.testing.assert_array_equal(whole.tracked["I"][:, -1].cpu().numpy(), whole.syn.cpu().numpy())
    first = _run(drive, p, meta, x[:, :70], d["in.v"], d["in.g"], {})
    second = _run(drive, p, meta, x[:, 70:], first.v.cpu().numpy(), first.syn.cpu().numpy(), {})
    assert torch.equal(torch.cat([first.output, second.output], 1), whole.output)
    assert torch.equal(second.v, whole.v)


def test_gradients_are_refused():
    drive, p, d, meta = golden_io.load("current_feedforward", "cuda")
    x = _t(d["in.x"]).requires_grad_(True)
    with pytest.raises(NotImplementedError, match="forward only"):
        current.simulate(_t(d["in.v"]), _t(d["in.g"]), x, drive, p)
