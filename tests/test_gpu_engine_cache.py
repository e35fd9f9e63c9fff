"""The engine's caches: the folded edges (weights times the per-target scale, in fixed
point) are kept while the same scale tensor is passed unchanged, and refolded when it
changes in place or is replaced."""

import pytest
import torch

from wiretorch_b200 import _lib, engine
from wiretorch_b200.testing import random_network

pytestmark = pytest.mark.gpu


def _folds():
    return len(_lib.TIMER.get("wt_fold_weights", []))


def test_fold_is_kept_while_the_scale_is_unchanged():
    drive, p, x, v, g, kw = random_network(N=500, n_in=100, B=2, T=60, seed=11, device="cuda")
    _lib.TIMER = {}
    try:
        with torch.no_grad():
            r1 = engine.simulate(v, g, x, drive, p, **kw)
            r2 = engine.simulate(v, g, x, drive, p, **kw)
            assert _folds() == 1
            assert torch.equal(r1.output, r2.output) and torch.equal(r1.v, r2.v)
            drive.scale.mul_(1.5)  # in place: refolded
            r3 = engine.simulate(v, g, x, drive, p, **kw)
            assert _folds() == 2
            drive.scale = torch.full_like(drive.scale, 1.5)  # replaced by equal values: refolded
            r4 = engine.simulate(v, g, x, drive, p, **kw)
            assert _folds() == 3
    finally:
        _lib.TIMER = None
    assert not torch.equal(r1.v, r3.v)  # the new scale took effect
    assert torch.equal(r3.output, r4.output) and torch.equal(r3.v, r4.v)


def test_the_callers_state_is_not_written():
    """The kernels write the state in place, into copies: the caller's tensors (here
    ``(B, N, 2, S)`` views of ``(B, 2, S, N)`` storage, the kernel's own layout) keep
    their values, and a second call from them repeats the first."""
    from wiretorch_b200 import configs

    cfg = configs.c5(B=2, T=80, device="cuda", N=2000, mean_degree=200.0, lam=0.05 * 500 ** (1 / 3),
                     w_e=6.0, w_in=30.0)  # fmt: skip
    x = cfg.inputs(seed=2)
    v, g, kw = cfg.state()
    g.add_(0.01)  # a non-trivial state in the kernel's layout
    before = (v.clone(), g.clone(), {k: t.clone() for k, t in kw.items()})
    with torch.no_grad():
        r1 = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
        r2 = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
    assert torch.equal(v, before[0]) and torch.equal(g, before[1])
    assert all(torch.equal(kw[k], before[2][k]) for k in kw)
    assert float(r1.output.sum()) > 0
    assert torch.equal(r1.output, r2.output) and torch.equal(r1.v, r2.v) and torch.equal(r1.gating, r2.gating)
