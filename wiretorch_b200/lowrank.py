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


class LowRank:
    """A pathway's weights in factorised form, ``W = U @ V.T``: ``U`` ``(n_rows, r)`` for
    the pathway's source rows, ``V`` ``(N, r)`` shared by the network's factorised
    pathways; rank ``r <= 64``, both held as bf16. Used in a ``Drive`` in place of a
    dense ``W``; ``dense()`` assembles the equivalent dense weights."""

    def __init__(self, U: torch.Tensor, V: torch.Tensor):
        if U.shape[1] != V.shape[1] or U.shape[1] > RANK_SLOTS:
            raise ValueError("U and V need the same rank, at most 64")
        self.U, self.V = U.to(torch.bfloat16), V.to(torch.bfloat16)
        self.requires_grad = False

    @property
    def shape(self) -> tuple[int, int]:
        return (self.U.shape[0], self.V.shape[0])

    def dense(self) -> torch.Tensor:
        return (self.U.double() @ self.V.double().T).float()


class _LrNet(_lib.C.Structure):
    _fields_ = [
        ("B", _lib.C.c_int32), ("N", _lib.C.c_int32), ("S", _lib.C.c_int32), ("KP", _lib.C.c_int32),
        ("theta", _lib.P), ("U_reset", _lib.P), ("E_L", _lib.P), ("C_m", _lib.P), ("beta", _lib.P),
        ("n_ref", _lib.P),
        ("decay_r", _lib.C.c_float * _lib.MAX_CHANNELS), ("decay_d", _lib.C.c_float * _lib.MAX_CHANNELS),
        ("jump_r", _lib.C.c_float * _lib.MAX_CHANNELS), ("jump_d", _lib.C.c_float * _lib.MAX_CHANNELS),
        ("E_syn", _lib.C.c_float * _lib.MAX_CHANNELS), ("g_clip", _lib.C.c_float * _lib.MAX_CHANNELS),
        ("dt", _lib.C.c_float),
        ("U", _lib.P), ("path_of", _lib.P), ("V", _lib.P), ("scale", _lib.P), ("w_in", _lib.P),
        ("made", _lib.C.c_uint32),
    ]  # fmt: skip


class _LrRun(_lib.C.Structure):
    _fields_ = [
        ("T", _lib.C.c_int32), ("T_total", _lib.C.c_int32), ("t0", _lib.C.c_int32),
        ("v", _lib.P), ("g", _lib.P), ("counter", _lib.P), ("x", _lib.P), ("spikes", _lib.P),
        ("P", _lib.P), ("barrier", _lib.P), ("err", _lib.P),
    ]  # fmt: skip


def is_factorised(drive) -> bool:
    return any(isinstance(W, LowRank) for _, W in drive.recurrent)


def _diagonal_input(W, N: int, device) -> torch.Tensor:
    """The per-neuron weight of a feedforward pathway that gives neuron n exactly input
    column n (a ``SparseRows`` or dense ``(N, N)`` diagonal), else raise."""
    from wiretorch_b200.types import SparseRows

    if isinstance(W, SparseRows):
        ar = torch.arange(N + 1, device=W.row_ptr.device)
        if W.shape == (N, N) and torch.equal(W.row_ptr.to(ar.dtype), ar) and torch.equal(
            W.cols.long(), ar[:-1]
        ):
            return W.values.detach().to(device, torch.float32).contiguous()
    elif W.shape == (N, N):
        d = torch.diagonal(W.detach()).to(device, torch.float32)
        if torch.count_nonzero(W.detach()) <= N:
            return d.contiguous()
    raise NotImplementedError(
        "the factorised kernel takes one input column per neuron (a diagonal feedforward pathway)"
    )


def simulate(v, g, x, drive, p, *, refractory=None, gating=None, adaptation=None,
             probabilities=False, track=False, track_batch_idx=None, retain=None):  # fmt: skip
    """``engine.simulate`` for a network whose recurrent pathways are all ``LowRank`` with
    one shared ``V`` (at most two pathways), driven by one input column per neuron;
    conductance LIF with refractoriness, no Mg block, adaptation, gating, escape noise,
    tracking or gradients (``NotImplementedError`` otherwise)."""
    from wiretorch_b200.types import Run

    unsupported = [name for name, bad in (
        ("gating", gating is not None or bool(getattr(drive, "gates", None))),
        ("adaptation", p.adapt is not None or adaptation is not None), ("the Mg block", p.mg_c is not None),
        ("escape noise", getattr(p, "spike_mode", "deterministic") == "sample"),
        ("probabilities", probabilities), ("tracking", track), ("retained graphs", retain is not None),
        ("gradients", torch.is_grad_enabled() and (x.requires_grad or drive.scale.requires_grad)),
    ) if bad]  # fmt: skip
    if unsupported:
        raise NotImplementedError("the factorised kernel does not support " + ", ".join(unsupported))
    dev = x.device
    B, T, n_in = x.shape
    N = v.shape[1]
    rec = list(drive.recurrent)
    KP = len(rec)
    if not all(isinstance(W, LowRank) for _, W in rec) or KP > 2:
        raise NotImplementedError("the factorised kernel takes one or two LowRank recurrent pathways")
    if any(W.V is not rec[0][1].V and not torch.equal(W.V, rec[0][1].V) for _, W in rec):
        raise NotImplementedError("the factorised pathways must share V")
    if len(drive.feedforward) != 1 or n_in != N:
        raise NotImplementedError("the factorised kernel takes one input column per neuron")
    S = p.E_syn.shape[0]
    if S > 4:
        raise NotImplementedError("the factorised kernel carries at most 4 synapse types")
    _diagonal_input(drive.feedforward[0][1], N, dev)
    if not x.is_cuda:
        raise RuntimeError("wiretorch_b200 runs on CUDA tensors only (no CPU path)")
    keep = {}
    U = torch.zeros((N, RANK_SLOTS), dtype=torch.bfloat16, device=dev)
    path_of = torch.full((N,), -1, dtype=torch.int8, device=dev)
    for k, (rows, W) in enumerate(rec):
        rows = rows.to(dev).long()
        if bool((path_of[rows] >= 0).any()):
            raise NotImplementedError("a neuron is a source of two factorised pathways")
        U[rows, : W.U.shape[1]] = W.U.to(dev)
        path_of[rows] = k
    keep["U"], keep["path_of"] = U, path_of
    keep["V"] = pad_rank(rec[0][1].V.to(dev))
    keep["w_in"] = _diagonal_input(drive.feedforward[0][1], N, dev)
    keep["scale"] = drive.scale.detach().to(dev, torch.float32).contiguous()
    net = _LrNet()
    net.B, net.N, net.S, net.KP = B, N, S, KP
    for name in ("theta", "U_reset", "E_L", "C_m", "beta"):
        keep[name] = getattr(p, name).detach().to(dev, torch.float32).contiguous()
        setattr(net, name, keep[name].data_ptr())
    if p.n_ref is not None:
        keep["n_ref"] = p.n_ref.to(dev, torch.int32).contiguous()
        net.n_ref = keep["n_ref"].data_ptr()
    dec, jmp = p.decay.detach().float().cpu(), p.jump.detach().float().cpu()
    E, clip = p.E_syn.detach().float().cpu(), p.g_clip.detach().float().cpu()
    for s in range(S):
        net.decay_r[s], net.decay_d[s] = float(dec[0, s]), float(dec[1, s])
        net.jump_r[s], net.jump_d[s] = float(jmp[0, s]), float(jmp[1, s])
        net.E_syn[s], net.g_clip[s] = float(E[s]), float(clip[s])
    net.dt = float(p.dt)
    net.U, net.path_of, net.V = U.data_ptr(), path_of.data_ptr(), keep["V"].data_ptr()
    net.scale, net.w_in = keep["scale"].data_ptr(), keep["w_in"].data_ptr()
    made = drive.made.detach().cpu().bool()
    bits = 0
    for k in range(KP + 1):
        for s in range(S):
            if made[k, s]:
                bits |= 1 << (8 * k + s)
    net.made = bits

    v_k = v.detach().to(dev, torch.float32).contiguous().clone()
    g_k = g.detach().to(dev, torch.float32).permute(0, 2, 3, 1).clone(memory_format=torch.contiguous_format)
    counter = (torch.zeros((B, N), dtype=torch.int32, device=dev) if refractory is None
               else refractory.detach().to(dev, torch.int32).contiguous().clone())  # fmt: skip
    xs = x.detach().float().contiguous()
    spikes = torch.empty((B, T, N), device=dev)
    scratch = torch.empty(3 * B * KP * RANK_SLOTS + 128, device=dev)
    barrier = torch.zeros(64, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    run = _LrRun()
    run.T, run.T_total, run.t0 = T, T, 0
    run.v, run.g, run.counter = v_k.data_ptr(), g_k.data_ptr(), counter.data_ptr()
    run.x, run.spikes, run.P = xs.data_ptr(), spikes.data_ptr(), scratch.data_ptr()
    run.barrier, run.err = barrier.data_ptr(), err.data_ptr()
    with _lib.timed("wt_lowrank_forward"):
        rc = _lib.lib().wt_lowrank_forward(_lib.C.byref(net), _lib.C.byref(run), _lib.C.c_void_p(_lib.stream_of(dev)))
    _lib.check(rc, "wt_lowrank_forward")
    _lib.count_launches(1)
    from wiretorch_b200.engine import check_device

    check_device(err, "wt_lowrank_forward")
    return Run(output=spikes, v=v_k, syn=g_k.permute(0, 3, 1, 2), probabilities=None, tracked=None,
               refractory=counter if (refractory is not None or p.n_ref is not None) else None,
               gating=None, adaptation=None)  # fmt: skip
