"""The lockstep comparison of the engine with the oracle, shared by the GPU tests and
``__graft_entry__.smoke``.

The oracle runs the whole input, recording its state every ``window`` steps; the engine
restarts from each recorded state and runs the window. Spikes must match exactly, except
a neuron whose voltage entering the step was within ``margin`` mV of threshold (either
outcome is a legitimate rounding of the same equations; that trial's window is then
excused); voltages, conductances and the gating state (release probabilities and
resources, within g_atol + g_rtol: they lie in [0, 1]) must match to the tolerances given. This is the
reference suite's own definition of "the same simulator" (its tests/test_lockstep.py).
"""

from __future__ import annotations

import numpy as np
import torch


def oracle_windows(net, x, v, g, kw, window):
    """The oracle's free run in windows: per-window entering states and outputs."""
    states = {"v": [], "g": [], **{k: [] for k in kw}}
    spikes, v_track = [], []
    v = v.detach().cpu().numpy()
    g = g.detach().cpu().numpy()
    kw = {k: val.detach().cpu().numpy() for k, val in kw.items()}
    x = x.detach().cpu().numpy()
    for start in range(0, x.shape[1], window):
        for key, value in (("v", v), ("g", g), *kw.items()):
            states[key].append(np.array(value))
        out = net.simulate(x[:, start : start + window], v, g, **kw)
        spikes.append(out["spikes"])
        v_track.append(out["v_track"])
        v, g = out["v"], out["g"]
        kw = {k: (out[k] if out[k] is not None else kw[k]) for k in kw}
    for key, value in (("v", v), ("g", g), *kw.items()):
        states[key].append(np.array(value))
    return states, np.concatenate(spikes, 1), np.concatenate(v_track, 1)


def _pooled(g, pools):
    """``(B, N, 2, S)`` conductances summed over each pool's member types."""
    if not pools:
        return g
    return np.stack([g[..., list(m)].sum(-1) for m in pools], -1)


def compare(engine_sim, net, drive, p, x, v, g, kw, window=10, margin=1e-3, v_atol=2e-4,
            g_rtol=1e-5, g_atol=1e-6, pools=None, oracle=None):  # fmt: skip
    """Lockstep of ``engine_sim(v, g, x_window, kw) -> Run`` against the oracle.

    ``pools``: the engine's pooled channels (lists of synapse types), whose state holds
    each pool's sum at its first member; the conductances are then compared pool by pool.
    ``oracle``: the result of ``oracle_windows`` for these inputs, if already run.

    Returns ``(excused, trial_windows, worst_dv, worst_dg)``; raises AssertionError on a
    flip away from threshold or a trace outside tolerance."""
    states, spikes, v_track = oracle if oracle is not None else oracle_windows(net, x, v, g, kw, window)
    theta = p.theta.detach().cpu().numpy()
    dev = x.device
    B = x.shape[0]
    excused, worst_dv, worst_dg = 0, 0.0, 0.0
    for w, start in enumerate(range(0, x.shape[1], window)):
        stop = start + window
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        kw_w = {k: t(states[k][w]) for k in kw}
        run = engine_sim(t(states["v"][w]), t(states["g"][w]), x[:, start:stop], kw_w)
        got = run.output.detach().cpu().numpy() > 0.5
        ok = np.ones(B, bool)
        diff = got != spikes[:, start:stop]
        if diff.any():
            v_enter = np.concatenate([states["v"][w][:, None], v_track[:, start : stop - 1]], 1)
            for b, tt, n in zip(*np.nonzero(diff)):
                if ok[b]:
                    m = abs(v_enter[b, tt, n] - theta[n])
                    assert m < margin, f"window {w} step {start + tt} trial {b} neuron {n}: flip {m:.2e} mV from threshold"
                    ok[b] = False
                    excused += 1
        if run.tracked is not None:
            vt = run.tracked["v"].detach().cpu().numpy()
            dv = np.abs(vt[ok] - v_track[ok, start:stop]).max(initial=0.0)
        else:  # an engine without tracking: the voltages the window leaves
            dv = np.abs(run.v.detach().cpu().numpy()[ok] - states["v"][w + 1][ok]).max(initial=0.0)
        assert dv <= v_atol, f"window {w}: voltage differs by {dv:.2e} mV"
        gk = _pooled(run.syn.detach().cpu().numpy(), pools)
        ref = _pooled(states["g"][w + 1], pools)
        err = np.abs(gk[ok] - ref[ok]) - (g_atol + g_rtol * np.abs(ref[ok]))
        assert err.max(initial=-1.0) <= 0, f"window {w}: conductances differ by {np.abs(gk[ok]-ref[ok]).max():.2e}"
        if "gating" in kw and run.gating is not None:
            gt = run.gating.detach().cpu().numpy()
            ref_gt = states["gating"][w + 1]
            dgt = np.abs(gt[ok] - ref_gt[ok]).max(initial=0.0)
            assert dgt <= g_atol + g_rtol, f"window {w}: gating state differs by {dgt:.2e}"
        worst_dv = max(worst_dv, float(dv))
        worst_dg = max(worst_dg, float(np.abs(gk[ok] - ref[ok]).max(initial=0.0)))
    return excused, B * (x.shape[1] // window), worst_dv, worst_dg
