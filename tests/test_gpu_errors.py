"""A kernel's device error word reaches the caller as an exception: read at once after the
forward launch by default, or — with ``engine.DEFER_CHECKS`` — copied behind the launch
and raised by ``engine.check_errors()`` (or the next engine call).

The error is made on the host: the weights are scaled up 2^30-fold after the plan chose
its fixed point, so the scatter meets products beyond the accumulators' range, skips
them and records ``WT_ERR_FIXED_POINT``; the kernel then leaves at its next grid
barrier. No fault, no hang.
"""

import pytest
import torch

from wiretorch_b200 import engine
from wiretorch_b200.testing import random_network

pytestmark = pytest.mark.gpu


def test_device_error_raises_at_once_or_deferred():
    drive, p, x, v, g, kw = random_network(N=500, n_in=50, B=2, T=30, seed=3, device="cuda", tau_ref=2.0)
    kw = {"refractory": kw["refractory"]}
    assert float(x.sum()) > 0  # input events reach the scatter
    with torch.no_grad():
        engine.simulate(v, g, x, drive, p, **kw)  # the plan's fixed point is chosen here
        drive.scale = drive.scale * 2.0**30
        with pytest.raises(RuntimeError, match="fixed-point"):
            engine.simulate(v, g, x, drive, p, **kw)
        engine.DEFER_CHECKS = True
        try:
            engine.simulate(v, g, x, drive, p, **kw)  # returns: its error word is read later
            with pytest.raises(RuntimeError, match="fixed-point"):
                engine.check_errors()
            engine.check_errors()  # nothing left to raise
        finally:
            engine.DEFER_CHECKS = False
            engine._PENDING.clear()
