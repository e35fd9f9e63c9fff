"""The oracle reproduces wiretorch's own results: it is pinned before anything is
checked against it.

Every golden case was produced by the reference's ``dynamics.simulate`` on the CPU
(``tests/golden/make_golden.py``). The oracle must

* restart from every recorded window state and take the window's steps with exactly
  the recorded spikes and voltages within 1e-4 mV (the reference's own CPU lockstep
  tolerance, ``tests/test_lockstep.py:24-27``) and the state within 1e-4 relative;
* run the whole input from the initial state with exactly the recorded spikes;
* and, for the scenarios the reference's own suite recorded (``rec.*``, from
  ``tests/fixtures/*.npz``), do the same against that recording.
"""

import numpy as np
import pytest

import golden_io
from oracle import oracle

CASES = golden_io.cases()
THRESHOLD_MARGIN = 1e-3  # mV: a flip this close to threshold is a legitimate rounding


def _kw(d, prefix, w=None):
    out = {}
    for key in ("refractory", "gating", "adaptation"):
        name = f"{prefix}{key}"
        if name in d:
            out[key] = d[name] if w is None else d[name][w]
    return out


def lockstep(net, x, v_states, g_states, spikes, voltages, theta, window, kw_states,
             probabilities=None):  # fmt: skip
    """Restart at every window; returns the number of excused near-threshold flips."""
    excused = 0
    for w, start in enumerate(range(0, x.shape[1], window)):
        stop = start + window
        kw = {k: v[w] for k, v in kw_states.items()}
        out = net.simulate(x[:, start:stop], v_states[w], g_states[w], **kw,
                           probabilities=probabilities is not None)  # fmt: skip
        diff = out["spikes"] != spikes[:, start:stop]
        ok = np.ones(x.shape[0], bool)
        if diff.any():
            v_enter = np.concatenate([v_states[w][:, None], voltages[:, start : stop - 1]], 1)
            for b, t, n in zip(*np.nonzero(diff)):
                if ok[b]:
                    assert abs(v_enter[b, t, n] - theta[n]) < THRESHOLD_MARGIN
                    ok[b] = False
                    excused += 1
        np.testing.assert_allclose(out["v_track"][ok], voltages[ok, start:stop],
                                   rtol=0, atol=1e-4, err_msg=f"window {w}")  # fmt: skip
        np.testing.assert_allclose(out["g"][ok], g_states[w + 1][ok], rtol=1e-4,
                                   atol=1e-5, err_msg=f"window {w}")  # fmt: skip
        if probabilities is not None:
            np.testing.assert_allclose(out["prob"][ok], probabilities[ok, start:stop],
                                       rtol=0, atol=1e-4)  # fmt: skip
    return excused


@pytest.mark.parametrize("name", CASES)
def test_oracle_lockstep_matches_reference(name):
    drive, p, d, meta = golden_io.load(name)
    x = d["in.x"]
    net = oracle.Network(drive, p, x.shape[0], x.shape[2])
    kw = _kw(d, "out.win_")
    excused = lockstep(net, x, d["out.win_v"], d["out.win_g"], d["out.spikes"],
                       d["out.v_track"], p.theta.numpy(), meta["window"], kw,
                       d.get("out.prob"))  # fmt: skip
    assert excused == 0


@pytest.mark.parametrize("name", CASES)
def test_oracle_free_run_is_spike_exact(name):
    drive, p, d, meta = golden_io.load(name)
    x = d["in.x"]
    net = oracle.Network(drive, p, x.shape[0], x.shape[2])
    out = net.simulate(x, d["in.v"], d["in.g"], **_kw(d, "in."))
    assert (out["spikes"] == d["out.spikes"]).all()
    np.testing.assert_allclose(out["v_track"], d["out.v_track"], rtol=0, atol=1e-4)
    np.testing.assert_allclose(out["g"], d["out.g"], rtol=1e-4, atol=1e-5)
    for key in ("refractory", "gating", "adaptation"):
        if f"out.{key}" in d and out[key] is not None:
            np.testing.assert_allclose(out[key], d[f"out.{key}"], rtol=1e-5, atol=1e-6)


RECORDED = [n for n in CASES if "rec.state_v" in golden_io.load(n)[2]]


@pytest.mark.parametrize("name", RECORDED)
def test_oracle_matches_the_reference_suites_recording(name):
    """Lockstep against ``tests/fixtures/<name>.npz`` of the reference's own suite,
    recorded from its pre-optimisation simulator."""
    drive, p, d, meta = golden_io.load(name)
    x = d["in.x"]
    net = oracle.Network(drive, p, x.shape[0], x.shape[2])
    excused = lockstep(net, x, d["rec.state_v"], d["rec.state_g"], d["rec.spikes"],
                       d["rec.voltages"], p.theta.numpy(), meta["window"], {},
                       d.get("rec.probabilities"))  # fmt: skip
    assert excused <= 0.01 * (x.shape[1] // meta["window"]) * x.shape[0]
