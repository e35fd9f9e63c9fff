"""The factorised drive's tensor-core product (``wt_lowrank_product``, tcgen05.mma)
against the same product in float64: V rounded to bf16 on both sides, P kept to fp32
accuracy by its three-part bf16 split. Sizes that are and are not multiples of the
128 x 128 tile, one to four pathways."""

import pytest
import torch

from wiretorch_b200 import lowrank

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,N,KP,r", [(128, 128, 1, 64), (200, 300, 2, 64), (300, 129, 3, 40), (64, 1000, 4, 16)])
def test_product_matches_float64(B, N, KP, r):
    g = torch.Generator().manual_seed(B * 7 + N)
    V = (torch.randn(N, r, generator=g) / 8).to(torch.bfloat16).cuda()
    P = torch.randn(B, KP, r, generator=g).cuda()
    D = lowrank.product(V, P)
    ref = torch.einsum("nr,bkr->kbn", V.double(), P.double())
    torch.testing.assert_close(D.double(), ref, rtol=1e-5, atol=1e-5 * float(ref.abs().max()))


def test_product_of_spike_sums_is_exact_enough():
    """P as the simulation forms it: sums of a few bf16 U rows (exactly representable in
    fp32), so D matches the dense W = U V^T gather."""
    g = torch.Generator().manual_seed(3)
    N, B, n_src, r = 256, 130, 400, 64
    U = (torch.randn(n_src, r, generator=g) / 8).to(torch.bfloat16)
    V = (torch.randn(N, r, generator=g) / 8).to(torch.bfloat16)
    S = (torch.rand(B, n_src, generator=g) < 0.02).float()
    P = (S.double() @ U.double()).float()[:, None, :]
    D = lowrank.product(V.cuda(), P.cuda())[0].double().cpu()
    W = U.double() @ V.double().T
    torch.testing.assert_close(D, S.double() @ W, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("double_exp", [False, True])
def test_factorised_simulation_matches_oracle_lockstep(double_exp):
    """The fused factorised kernel (wt_lowrank_forward) against the oracle run on the
    assembled dense network: two 128-trial blocks (130 trials) and a ragged neuron tile,
    spikes identical in lockstep windows, voltages and conductances within tolerance."""
    import lockstep
    from oracle import oracle as O
    from wiretorch_b200 import engine
    from wiretorch_b200.testing import lowrank_network

    drive_lr, drive_dense, p, x, v, g, kw = lowrank_network(double_exp=double_exp, device="cuda")
    net = O.Network(drive_dense, p, x.shape[0], x.shape[2])

    def sim(v_, g_, x_, kw_):
        return engine.simulate(v_, g_, x_, drive_lr, p, **kw_)

    excused, windows, dv, dg = lockstep.compare(sim, net, drive_dense, p, x, v, g, kw, window=10,
                                                v_atol=2e-4, g_rtol=1e-5, g_atol=1e-5)  # fmt: skip
    assert excused <= windows // 20
    out = engine.simulate(v, g, x, drive_lr, p, **kw).output
    assert float(out.sum()) > 50  # the run fires: the comparison saw spikes
