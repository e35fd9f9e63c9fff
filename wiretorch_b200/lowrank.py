"""The factorised recurrent drive on the tensor cores (``wt_lowrank_product``).

For pathways whose weights are a low-rank product W_k = U_k V^T (the factorised
configuration of the benchmark: a linear rank-r product, where wiretorch's
``LowRankProjection``, ``network_simulators/projections.py:167-216``, assembles a dense
W every forward, ``network.py:731-752``), a step's recurrent input is
``a_k[b, n] = sum_r V[n, r] P_k[b, r]`` with ``P_k = S_k U_k`` the fired sources' sum of
U rows: one GEMM with K = the rank, which ``product`` runs as tcgen05.mma tiles.
"""

from __future__ import annotations

import torch

from wiretorch_b200 import _lib

RANK_SLOTS = 64  #: K of the product; a lower rank is zero-padded


class _ProductArgs(_lib.C.Structure):
    _fields_ = [
        ("B", _lib.C.c_int32), ("N", _lib.C.c_int32), ("KP", _lib.C.c_int32),
        ("V", _lib.P), ("P", _lib.P), ("D", _lib.P), ("err", _lib.P),
    ]  # fmt: skip


def pad_rank(V: torch.Tensor) -> torch.Tensor:
    """``(N, r)`` -> ``(N, 64)`` bf16, contiguous, zero-padded rank slots."""
    N, r = V.shape
    if r > RANK_SLOTS:
        raise ValueError(f"rank {r} above the {RANK_SLOTS} slots of the tensor-core product")
    out = torch.zeros((N, RANK_SLOTS), dtype=torch.bfloat16, device=V.device)
    out[:, :r] = V.to(torch.bfloat16)
    return out


def product(V: torch.Tensor, P: torch.Tensor) -> torch.Tensor:
    """``D[k, b, n] = sum_r V[n, r] P[b, k, r]``: V ``(N, r)`` (rounded to bf16), P
    ``(B, KP, r)`` float32 (kept to fp32 accuracy), KP <= 4."""
    if not V.is_cuda:
        raise RuntimeError("wiretorch_b200 runs on CUDA tensors only (no CPU path)")
    B, KP, r = P.shape
    Vp = pad_rank(V)
    Pp = torch.zeros((B, KP, RANK_SLOTS), device=P.device)
    Pp[..., :r] = P.float()
    N = Vp.shape[0]
    D = torch.empty((KP, B, N), device=P.device)
    err = torch.zeros(1, dtype=torch.int32, device=P.device)
    a = _ProductArgs()
    a.B, a.N, a.KP = B, N, KP
    a.V, a.P, a.D, a.err = Vp.data_ptr(), Pp.data_ptr(), D.data_ptr(), err.data_ptr()
    with _lib.timed("wt_lowrank_product"):
        rc = _lib.lib().wt_lowrank_product(_lib.C.byref(a), _lib.C.c_void_p(_lib.stream_of(P.device)))
    _lib.check(rc, "wt_lowrank_product")
    _lib.count_launches(1)
    from wiretorch_b200.engine import check_device

    check_device(err, "wt_lowrank_product")
    return D
