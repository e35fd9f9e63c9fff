"""The loss filter's kernels against its definition (wiretorch's
``tests/test_losses.py:28-55``): ``y[t] = sum_{k <= t} exp(-k dt / tau) x[t - k] +
carried exp(-t dt / tau)``, rise then decay, the state carried from chunk to chunk and no
gradient across chunks. Both kernel variants run: the per-column scan (many trains) and
the warp-shuffle parallel scan over time (few trains)."""

import numpy as np
import pytest
import torch

from wiretorch_b200 import filtering

pytestmark = pytest.mark.gpu

TAU_RISE, TAU_DECAY, DT = 10.0, 100.0, 1.0


def exponential_filter(x, tau, carried):
    T = x.shape[1]
    k = torch.exp(-torch.arange(T, dtype=torch.float64, device=x.device) * DT / tau)
    lag = torch.arange(T, device=x.device)
    lag = lag[:, None] - lag[None, :]
    M = torch.where(lag >= 0, k[lag.clamp(min=0)], torch.zeros((), dtype=torch.float64, device=x.device))
    y = torch.einsum("ts,bsn->btn", M, x.double())
    return y if carried is None else y + carried.double() * k[None, :, None]


@pytest.mark.parametrize("B,N,T", [(2, 7, 300), (64, 2000, 123)], ids=["parallel-T", "per-column"])
def test_filter_matches_definition_across_chunks(B, N, T):
    rng = np.random.default_rng(0)
    x = torch.from_numpy((rng.random((B, 3 * T, N)) < 0.05).astype(np.float32)).cuda()
    x.requires_grad_(True)
    t = torch.arange(T, dtype=torch.float32, device="cuda") * DT
    kr, kd = torch.exp(-t / TAU_RISE), torch.exp(-t / TAU_DECAY)
    rise = smooth = None
    ref_r = ref_s = None
    R = torch.from_numpy(rng.normal(size=(B, T, N)).astype(np.float32)).cuda()
    for c in range(3):
        xc = x[:, c * T : (c + 1) * T]
        r, s = filtering.double_exponential(xc, kr, kd, rise, smooth)
        er = exponential_filter(xc.detach(), TAU_RISE, ref_r)
        es = exponential_filter(er, TAU_DECAY, ref_s)
        torch.testing.assert_close(s.double(), es, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(r.double(), er, rtol=1e-4, atol=1e-4)
        # gradient of sum(s R) w.r.t. this chunk's input: the transposed filters
        (g,) = torch.autograd.grad((s * R).sum(), xc)
        x64 = xc.detach().double().requires_grad_(True)
        e64 = exponential_filter(exponential_filter(x64, TAU_RISE, None), TAU_DECAY, None)
        (g64,) = torch.autograd.grad((e64 * R.double()).sum(), x64)
        torch.testing.assert_close(g.double(), g64, rtol=1e-4, atol=1e-3)
        rise, smooth = r[:, -1:].detach(), s[:, -1:].detach()
        ref_r, ref_s = er[:, -1:], es[:, -1:]


@pytest.mark.parametrize("use_prob", [False, True])
def test_van_rossum_rate_loss_matches_definition_across_chunks(use_prob):
    """The fused loss against its definition, three chunks with the filter state carried
    and no gradient across chunks; spikes or probabilities as the output."""
    rng = np.random.default_rng(1)
    B, T, N = 4, 203, 300  # T not a multiple of the scans' 8-step load groups
    out = torch.from_numpy((rng.random((B, 3 * T, N)) < 0.02).astype(np.float32)).cuda()
    if use_prob:
        out = torch.from_numpy(rng.random((B, 3 * T, N)).astype(np.float32) * 0.05).cuda()
    out.requires_grad_(True)
    rate = torch.from_numpy(rng.uniform(0.0, 0.05, (B, 1, N)).astype(np.float32)).cuda()
    loss_fn = filtering.VanRossumRateLoss(TAU_RISE, TAU_DECAY, DT, T)
    carry = None
    for c in range(3):
        oc = out[:, c * T : (c + 1) * T]
        kw = {"output_probabilities": oc} if use_prob else {"output_spikes": oc}
        loss = loss_fn(rate.expand(B, T, N), **kw)
        o64 = oc.detach().double().requires_grad_(True)
        r_o = exponential_filter(o64, TAU_RISE, None if carry is None else carry[0])
        s_o = exponential_filter(r_o, TAU_DECAY, None if carry is None else carry[1])
        tgt = rate.expand(B, T, N).double()
        r_t = exponential_filter(tgt, TAU_RISE, None if carry is None else carry[2])
        s_t = exponential_filter(r_t, TAU_DECAY, None if carry is None else carry[3])
        expected = ((s_o - s_t) ** 2).mean()
        torch.testing.assert_close(loss.double(), expected, rtol=1e-4, atol=1e-9)
        (g,) = torch.autograd.grad(loss, oc)
        (g64,) = torch.autograd.grad(expected, o64)
        # float32 err = smooth(x) - smooth(y) cancels: compare at 1e-3 of the largest entry
        torch.testing.assert_close(g.double(), g64, rtol=1e-3, atol=1e-3 * float(g64.abs().max()))
        torch.testing.assert_close(loss_fn.prev_output_smooth.double(), s_o[:, -1:].detach(), rtol=1e-4, atol=1e-6)
        carry = [q[:, -1:].detach() for q in (r_o, s_o, r_t, s_t)]
