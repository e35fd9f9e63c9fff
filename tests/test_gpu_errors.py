"""A kernel's device error word reaches the caller as an exception: read at once after the
forward launch by default, or — with ``engine.DEFER_CHECKS`` — copied behind the launch
and raised by ``engine.check_errors()`` (or the next engine call).

The errors are made on the host. The weights are scaled up 2^30-fold after the plan
chose its fixed point, so the scatter meets products beyond the accumulators' range,
skips them and records ``WT_ERR_FIXED_POINT``; the kernel then leaves at its next grid
barrier. And a neuron-partitioned run is given a partner rank that never runs (its
buffers are this GPU's own), so the bounded wait for its progress runs out and records
``WT_ERR_BARRIER``. No fault, no hang.
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


class _LonelyPartition:
    """One rank (0) of a two-rank neuron partition on a single GPU whose partner never
    runs: every buffer the kernel touches is this GPU's own memory (the partner's
    replicas are plain local buffers), and the partner's progress slot is never written."""

    def __init__(self, N, B, device):
        words = -(-N // 32)
        self.words = [torch.zeros(2 * B * words, dtype=torch.int32, device=device) for _ in range(2)]
        self.progress = [torch.zeros(8, dtype=torch.int64, device=device) for _ in range(2)]

    def fill(self, run, plan=None):
        run.words, run.progress = self.words[0].data_ptr(), self.progress[0].data_ptr()
        for r in range(2):
            run.peer_words[r] = self.words[r].data_ptr()
            run.peer_progress[r] = self.progress[r].data_ptr()
        run.n_ranks, run.rank, run.word0, run.epoch = 2, 0, 0, 1


def test_partition_progress_wait_gives_up():
    """A bounded device wait that runs out: the barrier of a neuron-partitioned step
    waits for every rank's progress slot; with the partner's slot never written, the
    spin gives up after its poll limit (well under a second), the kernel records
    ``WT_ERR_BARRIER`` and every block leaves at that barrier; the host raises.
    The context stays usable: a normal run follows and succeeds."""
    from wiretorch_b200 import plan as P

    drive, p, x, v, g, kw = random_network(N=600, n_in=40, B=2, T=20, seed=4, device="cuda")
    plan = engine.get_plan(drive, p, x.shape[0], x.shape[2], x.device)
    P.fold(plan, drive.scale)
    v_k, g_k, counter, g_a, gating = engine._prepare_state(plan, v, g, None, None, None, p)
    part = _LonelyPartition(plan.N, x.shape[0], x.device)
    with torch.no_grad(), pytest.raises(RuntimeError, match="barrier"):
        engine.run_forward(plan, p, x, v_k, g_k, counter, g_a, gating, part=part)
    assert int(part.progress[1][0]) >> 32 == 1  # its progress (epoch 1) reached the partner's replica
    with torch.no_grad():
        run = engine.simulate(v, g, x, drive, p)
    assert run.output.shape == x.shape[:2] + (plan.N,)
