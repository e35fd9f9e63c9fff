"""The forward kernels specialised on a run's features against the generic kernel.

Forward runs with a refractory period and the Mg block and/or gating, or adaptation,
take a kernel with those features compiled in (fewer registers, more warps per SM);
tracking the same run sends it through the generic kernel, which tests every feature at
run time. Both must give identical spikes and state, bit for bit (the synaptic sums are
fixed point, the membrane arithmetic the same float32 operations in the same order).
"""

import pytest
import torch

from test_gpu_gating import _c5_small, _doubled
from wiretorch_b200 import engine
from wiretorch_b200.testing import random_network

pytestmark = pytest.mark.gpu

STATE = ("output", "v", "syn", "gating", "refractory", "adaptation")


def _both(drive, p, x, v, g, kw, pool):
    engine.POOL_SYNAPSES = pool
    try:
        with torch.no_grad():
            fast = engine.simulate(v, g, x, drive, p, **kw)
            generic = engine.simulate(v, g, x, drive, p, **kw, track=True)
    finally:
        engine.POOL_SYNAPSES = False
    return fast, generic


def _same(fast, generic):
    assert float(fast.output.sum()) > 20  # the network is active
    for name in STATE:
        a, b = getattr(fast, name), getattr(generic, name)
        assert (a is None) == (b is None), name
        if a is not None:
            assert torch.equal(a, b), name


@pytest.mark.parametrize("pool", [False, True], ids=["exact", "pooled"])
def test_mg_block_and_gating(pool):
    cfg = _doubled(_c5_small())
    v, g, kw = cfg.state()
    _same(*_both(cfg.drive, cfg.p, cfg.inputs(seed=7), v, g, kw, pool))


@pytest.mark.parametrize("pool", [False, True], ids=["exact", "pooled"])
def test_adaptation(pool):
    drive, p, x, v, g, kw = random_network(N=3000, n_in=200, B=4, T=150, seed=11, device="cuda",
                                           tau_ref=2.0, adapt=0.4)  # fmt: skip
    assert "adaptation" in kw and "refractory" in kw
    _same(*_both(drive, p, x, v, g, kw, pool))
