"""``wt_forward_noalloc``: the forward run with its scratch in a static device array.

Called through the C ABI, two calls in a row (the second continuing from the state the
first left) must give what ``wt_forward`` with a caller-allocated workspace gives on the
same inputs; a run whose workspace exceeds the static array is rejected before any
device work. Named to be collected last: the entry point's set-up happens in whichever
test calls it first, so the file must pass both alone and after every other test.
"""

import ctypes

import pytest
import torch

from wiretorch_b200 import _lib, engine
from wiretorch_b200.testing import random_network

NOALLOC_LIMIT = 32 << 20  # bytes of the static scratch per device


def _net_and_state(T):
    drive, p, x, v, g, kw = random_network(N=700, n_in=120, B=3, T=T, seed=5, tau_ref=2.0,
                                           device="cuda")  # fmt: skip
    plan = engine.get_plan(drive, p, x.shape[0], x.shape[2], x.device)
    from wiretorch_b200 import plan as P

    P.fold(plan, drive.scale)
    v_k, g_k, counter, _, _ = engine._prepare_state(plan, v, g, kw["refractory"], None, None, p)
    return plan, p, x, v_k, g_k, counter


def _noalloc(plan, p, x, v, g, counter):
    """One ``wt_forward_noalloc`` call over all of ``x``; updates the state in place."""
    lib = _lib.lib()
    net = plan.net(p)
    run = _lib.WtForward()
    B, T, _ = x.shape
    run.T, run.T_total, run.t0, run.flags = T, T, 0, _lib.F_REFRACTORY
    spikes = torch.empty((B, T, plan.N), device=x.device)
    run.v, run.g, run.counter = v.data_ptr(), g.data_ptr(), counter.data_ptr()
    run.x, run.spikes, run.track_b = x.data_ptr(), spikes.data_ptr(), -1
    stream = ctypes.c_void_p(_lib.stream_of(x.device))
    rc = lib.wt_forward_noalloc(ctypes.byref(net), ctypes.byref(run), stream)
    assert rc == 0, lib.wt_last_error().decode()
    code = ctypes.c_int32(-1)
    assert lib.wt_noalloc_error(stream, ctypes.byref(code)) == 0
    assert code.value == 0
    return spikes


@pytest.mark.gpu
def test_noalloc_matches_wt_forward_two_calls():
    T = 80
    plan, p, x, v, g, counter = _net_and_state(T)
    xs = x.contiguous()
    state_a = [v.clone(), g.clone(), counter.clone()]
    state_b = [v.clone(), g.clone(), counter.clone()]
    total = 0.0
    for half in (xs[:, : T // 2].contiguous(), xs[:, T // 2 :].contiguous()):
        with torch.no_grad():
            out = engine.run_forward(plan, p, half, *state_a, None, None)
        spikes = _noalloc(plan, p, half, *state_b)
        torch.cuda.synchronize()
        assert torch.equal(spikes, out["spikes"])
        torch.testing.assert_close(state_b[0], state_a[0], rtol=0, atol=1e-5)  # v, mV
        torch.testing.assert_close(state_b[1], state_a[1], rtol=1e-6, atol=1e-7)  # g, nS
        assert torch.equal(state_b[2], state_a[2])  # refractory counters
        total += float(spikes.sum())
    assert total > 0  # the comparison saw spikes


def test_noalloc_rejects_a_run_above_its_scratch():
    """Checked on the host before any device work (runs without a GPU): a net whose
    accumulators alone exceed the static array."""
    lib = _lib.lib()
    one = (ctypes.c_float * 4)(1.0, 1.0, 1.0, 1.0)
    ints = (ctypes.c_int32 * 4)(0, 0, 0, 0)
    net = _lib.WtNet()
    net.B, net.N, net.n_in, net.S, net.C = 64, 100_000, 0, 2, 2  # X alone: 205 MB
    addr = ctypes.cast(one, ctypes.c_void_p).value
    net.theta = net.U_reset = net.E_L = net.C_m = net.beta = addr
    iaddr = ctypes.cast(ints, ctypes.c_void_p).value
    net.src_slot = net.slot_chunk = net.src_chunk = iaddr
    run = _lib.WtForward()
    run.T, run.T_total = 10, 10
    rc = lib.wt_forward_noalloc(ctypes.byref(net), ctypes.byref(run), None)
    assert rc == 1  # WT_ERR_ARGS
    msg = lib.wt_last_error().decode()
    assert "static limit" in msg and str(NOALLOC_LIMIT) in msg
