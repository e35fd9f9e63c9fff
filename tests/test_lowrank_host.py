"""The factorised path's host side, without a GPU: the equivalence of a ``LowRank``
pathway with its assembled weights, and the checks that send a network the fused kernel
does not cover to a clear error (and never to a CPU fallback)."""

import pytest
import torch

from wiretorch_b200 import lowrank
from wiretorch_b200.testing import lowrank_network


def test_lowrank_dense_is_the_product():
    U = torch.randn(7, 5).to(torch.bfloat16)
    V = torch.randn(11, 5).to(torch.bfloat16)
    W = lowrank.LowRank(U, V)
    assert W.shape == (7, 11)
    torch.testing.assert_close(W.dense().double(), U.double() @ V.double().T, rtol=1e-6, atol=1e-6)


def test_a_supported_network_passes_the_checks_and_needs_cuda():
    drive_lr, _, p, x, v, g, kw = lowrank_network(N=64, B=3, T=5)
    with pytest.raises(RuntimeError, match="CUDA"):
        lowrank.simulate(v, g, x, drive_lr, p, **kw)


def test_unsupported_features_are_rejected():
    drive_lr, _, p, x, v, g, kw = lowrank_network(N=64, B=3, T=5)
    with pytest.raises(NotImplementedError, match="tracking"):
        lowrank.simulate(v, g, x, drive_lr, p, track=True, **kw)
    p.mg_c = torch.zeros(2)
    with pytest.raises(NotImplementedError, match="Mg block"):
        lowrank.simulate(v, g, x, drive_lr, p, **kw)


def test_non_diagonal_input_is_rejected():
    drive_lr, _, p, x, v, g, kw = lowrank_network(N=64, B=3, T=5)
    rows, _ = drive_lr.feedforward[0]
    drive_lr.feedforward = [(rows, torch.ones(64, 64))]
    with pytest.raises(NotImplementedError, match="one input column per neuron"):
        lowrank.simulate(v, g, x, drive_lr, p, **kw)
