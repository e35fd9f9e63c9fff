"""The drop-in engine: ``simulate`` with the signature of wiretorch's
``conductance/engine.py:71-89``, run by this package's sm_100a kernels.

A wiretorch network calls its engine through its ``_engine`` class attribute
(``conductance/network.py:68``, called at ``network.py:896-909``); setting

    ConductanceNetwork._engine = wiretorch_b200.engine

routes every conductance-based network through this module, with nothing else in the
network changed. The arguments and the returned ``Run`` are the reference's: state
``v`` ``(B, N)``, conductances ``g`` ``(B, N, 2, S)`` (any view), input ``x``
``(B, T, n_in)``, the ``Drive`` and ``Physiology``; the engine copies its inputs, updates
the copies and returns them, and never synchronises with the host inside a call after
the first call of a network (which builds and caches its tables).

There is no CPU path and no PyTorch fallback: inputs must be CUDA tensors on a B200 and
the compiled library must be present, or the call raises.
"""

from __future__ import annotations

import os
import weakref

import torch

from wiretorch_b200 import _lib, plan as _plan
from wiretorch_b200.types import PHYSIOLOGY, Run

#: Pool synapse types with identical dynamics into one channel (see ``plan``). Off by
#: default: the state then holds every synapse type's conductance, as the reference's.
POOL_SYNAPSES = os.environ.get("WIRETORCH_POOL_SYNAPSES", "0") == "1"

_PLANS: dict = {}

#: If set to a (2,) int64 CUDA tensor, the forward kernel adds to it the edges it
#: traverses (recurrent, input): the synaptic events of the run, counted on the device.
EDGE_COUNTER = None

#: Keep the forward kernel's state in HBM, streamed through shared memory every step,
#: even where it would fit on chip (the path of networks too large for it; for tests).
FORCE_STREAM = False

#: If set to a list, every forward launch appends to it a (T, warps, WT_PHASES) int64
#: tensor: per step and warp of the grid the global timer (ns) at the end of each phase
#: of the step (instrumented runs; see ``WT_PHASES`` in the C header).
PHASE_RECORD = None


def _key(drive, p, B, n_in, device, pool):
    pathways = list(drive.recurrent) + list(drive.feedforward)
    gates = tuple(None if g is None else (g.start, g.n, g.stp, g.saturates, id(g.params))
                  for g in (drive.gates or []))  # fmt: skip
    learnt = tuple(_requires_grad(getattr(p, n)) for n in ("E_syn", "decay", "jump"))
    return (tuple(id(r) for r, _ in pathways), tuple(id(W) for _, W in pathways), gates,
            tuple(drive.made.shape), B, n_in, str(device), pool, tuple(p.decay.shape),
            p.mg_c is not None, learnt)  # fmt: skip


def _same_objects(plan, drive) -> bool:
    """The cached plan was built from these very weight and row tensors, unmodified (an
    ``id`` can be reused once its tensor is freed). The reference builds ``made`` afresh
    every call from a fixed buffer, so only its shape is part of the key."""
    pathways = list(drive.recurrent) + list(drive.feedforward)
    objs = [o for r, W in pathways for o in (r, W.values if hasattr(W, "row_ptr") else W)]
    refs = plan.sources
    return len(refs) == len(objs) and all(
        ref() is o and ver == getattr(o, "_version", 0) for (ref, ver), o in zip(refs, objs)
    )


def get_plan(drive, p, B, n_in, device, pool=None):
    """The compiled tables of this network (cached while its weight tensors live)."""
    pool = POOL_SYNAPSES if pool is None else pool
    key = _key(drive, p, B, n_in, device, pool)
    plan = _PLANS.get(key)
    if plan is None or not _same_objects(plan, drive):
        if len(_PLANS) > 32:
            _PLANS.clear()
        plan = _plan.build(drive, p, B, n_in, device, pool=pool)
        pathways = list(drive.recurrent) + list(drive.feedforward)
        objs = [o for r, W in pathways for o in (r, W.values if hasattr(W, "row_ptr") else W)]
        plan.sources = [(weakref.ref(o), getattr(o, "_version", 0)) for o in objs]
        _PLANS[key] = plan
    return plan


def _internal_g(plan, g):
    """``(B, N, 2, S)`` reference state -> ``(B, 2, S', N)`` kernel state (pools summed)."""
    g = g.detach().to(plan.device, torch.float32)
    out = g.permute(0, 2, 3, 1)  # (B, 2, S, N)
    if plan.ch.pooled:
        parts = [out[:, :, m].sum(2) for m in plan.ch.member]
        return torch.stack(parts, 2).contiguous()
    # always a copy: the kernel writes the state in place, and a caller's (B, N, 2, S)
    # view of (B, 2, S, N) storage would otherwise be that very memory
    return out.clone(memory_format=torch.contiguous_format)


def _external_g(plan, g):
    """Kernel state ``(B, 2, S', N)`` -> reference ``(B, N, 2, S)`` view."""
    if plan.ch.pooled:
        B, _, _, N = g.shape
        full = g.new_zeros((B, 2, plan.ch.S, N))
        for c, m in enumerate(plan.ch.member):
            full[:, :, m[0]] = g[:, :, c]
        g = full
    return g.permute(0, 3, 1, 2)


def _workspace(plan, T, device):
    B, N, C = plan.B, plan.N, plan.ch.C
    cap = B * max(plan.n_chunks, 1)
    Np = -(-N // 32) * 32  # accumulator rows are padded to whole 32-neuron groups
    ws = {
        "X": torch.empty(2 * C * B * Np, dtype=torch.int64, device=device),
        "ev": torch.empty(2 * cap * _lib.EVENT_BYTES, dtype=torch.uint8, device=device),
        "ev_count": torch.empty(T + 1, dtype=torch.int32, device=device),
        "barrier": torch.zeros(64, dtype=torch.int32, device=device),
        "err": torch.zeros(1, dtype=torch.int32, device=device),
    }
    w = _lib.WtWorkspace()
    for name in ("X", "ev", "ev_count", "barrier", "err"):
        setattr(w, name, ws[name].data_ptr())
    w.ev_cap = cap
    if EDGE_COUNTER is not None:
        w.edges = EDGE_COUNTER.data_ptr()
    return ws, w


def check_device(err: torch.Tensor, what: str) -> None:
    """Raise if a kernel recorded an error (synchronises)."""
    code = int(err.item())
    if code:
        raise RuntimeError(f"{what}: {_lib.ERRORS.get(code & 255, code)} (code {code})")


#: When True, a forward launch's device error word is not read at once (a host
#: synchronisation per call) but copied to pinned host memory behind the launch, on its
#: stream, and checked by the next engine call or by ``check_errors()`` — the first
#: error raises there. For loops that keep the GPU fed (training, benchmarks); the
#: default reads the word before the call returns.
DEFER_CHECKS = False
_PENDING: list = []


def _defer_check(err: torch.Tensor, what: str) -> None:
    host = torch.empty(1, dtype=torch.int32, pin_memory=True)
    host.copy_(err, non_blocking=True)
    done = torch.cuda.Event()
    done.record(torch.cuda.current_stream(err.device))
    _PENDING.append((done, host, what))


def check_errors(block: bool = True) -> None:
    """Raise for the first device error recorded by a deferred check (``DEFER_CHECKS``);
    ``block``: wait for the launches still running, else check only finished ones."""
    while _PENDING:
        done, host, what = _PENDING[0]
        if not block and not done.query():
            return
        done.synchronize()
        _PENDING.pop(0)
        code = int(host[0])
        if code:
            _PENDING.clear()
            raise RuntimeError(f"{what}: {_lib.ERRORS.get(code & 255, code)} (code {code})")


def run_forward(plan, p, x, v, g, counter, g_a, gating, *, probabilities=False, track=False,
                track_b=-1, save=None, noise=None, check=True, part=None):  # fmt: skip
    """Launch the forward kernel over all of ``x``; returns the outputs (dict)."""
    if _PENDING:
        check_errors(block=False)  # earlier deferred checks that have finished
    device = plan.device
    B, T, n_in = x.shape
    N, Sp = plan.N, plan.ch.Sp
    net = plan.net(p)
    plan.net_struct = net
    run = _lib.WtForward()
    run.T, run.T_total, run.t0 = T, T, 0
    flags = 0
    if p.n_ref is not None:
        flags |= _lib.F_REFRACTORY
    if p.mg_c is not None:
        flags |= _lib.F_MG_BLOCK
    if p.adapt is not None:
        flags |= _lib.F_ADAPT
    if p.spike_mode == "sample":
        flags |= _lib.F_SAMPLE
    if plan.gated:
        flags |= _lib.F_GATED
    if FORCE_STREAM:
        flags |= _lib.F_STREAM
    if getattr(p, "current", False):  # current-based neurons (wiretorch_b200.current)
        flags |= _lib.F_CURRENT
    out = {"spikes": torch.empty((B, T, N), device=device)}
    run.v, run.g = v.data_ptr(), g.data_ptr()
    run.counter = _lib.ptr(counter) if flags & _lib.F_REFRACTORY else None
    run.g_a = _lib.ptr(g_a) if flags & _lib.F_ADAPT else None
    run.gating = _lib.ptr(gating) if plan.gated else None
    x = x.contiguous()
    run.x = x.data_ptr() if n_in else None
    if flags & _lib.F_SAMPLE:
        if noise is None:
            noise = torch.rand((B, T, N), device=device)
        run.noise = noise.data_ptr()
    out["noise"] = noise
    run.spikes = out["spikes"].data_ptr()
    if probabilities:
        flags |= _lib.F_PROB
        out["prob"] = torch.empty((B, T, N), device=device)
        run.prob = out["prob"].data_ptr()
    if track:
        flags |= _lib.F_TRACK
        Bt = B if track_b < 0 else 1
        out["track_v"] = torch.empty((Bt, T, N), device=device)
        out["track_I"] = torch.empty((Bt, T, N, Sp + 1), device=device)
        out["track_g"] = torch.empty((Bt, T, N, 2, Sp), device=device)
        run.track_v, run.track_I = out["track_v"].data_ptr(), out["track_I"].data_ptr()
        run.track_g = out["track_g"].data_ptr()
        if flags & _lib.F_ADAPT:
            out["track_a"] = torch.empty((Bt, T, N), device=device)
            run.track_a = out["track_a"].data_ptr()
        run.track_b = track_b
    if save is not None:
        flags |= _lib.F_SAVE
        words = (N + 31) // 32
        save["v"] = torch.empty((B, T, N), device=device)
        save["G"] = torch.empty((B, T, Sp, N), device=device)
        save["spike_bits"] = torch.empty((B, T, words), dtype=torch.int32, device=device)
        run.v_saved, run.G_saved = save["v"].data_ptr(), save["G"].data_ptr()
        run.spike_bits = save["spike_bits"].data_ptr()
        if flags & _lib.F_REFRACTORY:
            save["held_bits"] = torch.empty((B, T, words), dtype=torch.int32, device=device)
            run.held_bits = save["held_bits"].data_ptr()
        if flags & _lib.F_ADAPT:
            save["a"] = torch.empty((B, T, N), device=device)
            run.a_saved = save["a"].data_ptr()
        if plan.gated:
            save["f"] = torch.empty((B, T, max(plan.R_f, 1)), device=device)
            run.f_saved = save["f"].data_ptr()
        if save.get("want_input"):
            flags |= _lib.F_SAVE_INPUT
            save["X"] = torch.empty((B, T, plan.ch.C, N), device=device)
            run.X_saved = save["X"].data_ptr()
    if part is not None:  # one rank of a neuron-partitioned run (wiretorch_b200.partition)
        flags |= _lib.F_PARTITION
        part.fill(run, plan)
    if PHASE_RECORD is not None:  # instrumented run: every warp's phase stamps, every step
        warps = torch.cuda.get_device_properties(device).multi_processor_count * 32
        stamps = torch.zeros((T, warps, _lib.PHASES), dtype=torch.int64, device=device)
        run.phases, run.phase_warps = stamps.data_ptr(), warps
        PHASE_RECORD.append(stamps)
    run.flags = flags
    ws, w = _workspace(plan, T, device)
    out["_ws"] = ws
    with _lib.timed("wt_forward"):
        rc = _lib.lib().wt_forward(_ctypes_ref(net), _ctypes_ref(run), _ctypes_ref(w),
                                   _lib.C.c_void_p(_lib.stream_of(device)))  # fmt: skip
    _lib.check(rc, "wt_forward")
    _lib.count_launches(1)
    if check and DEFER_CHECKS:
        _defer_check(ws["err"], "wt_forward")
    elif check:
        check_device(ws["err"], "wt_forward")
    return out


def _ctypes_ref(s):
    return _lib.C.byref(s)


def _prepare_state(plan, v, g, refractory, gating, adaptation, p):
    device = plan.device
    v_k = v.detach().to(device, torch.float32).contiguous().clone()
    g_k = _internal_g(plan, g)
    if refractory is None:
        refractory = torch.zeros(v.shape, dtype=torch.int32, device=device)
    counter = refractory.detach().to(device, torch.int32).contiguous().clone()
    g_a = None
    if p.adapt is not None:
        g_a = (torch.zeros_like(v_k) if adaptation is None
               else adaptation.detach().to(device, torch.float32).contiguous().clone())  # fmt: skip
    gating_k = None
    if gating is not None:
        gating_k = gating.detach().to(device, torch.float32).contiguous().clone()
    return v_k, g_k, counter, g_a, gating_k


def simulate(
    v, g, x, drive, p, *, refractory=None, gating=None, adaptation=None,
    probabilities=False, track=False, track_batch_idx=None, retain=None,
) -> Run:  # fmt: skip
    """Simulate ``x.shape[1]`` steps from state ``(v, g)`` with input ``x``: the
    reference's ``engine.simulate`` (``conductance/engine.py:71-89``), same arguments and
    result. Differentiable in ``drive.scale``, the weights, ``x`` and the physiology
    (``PHYSIOLOGY``) when any of them requires grad."""
    if retain is not None:
        raise NotImplementedError(
            "track_gradients retains the autograd graph of every step, which only the "
            "reference's PyTorch path builds; the fused kernels do not"
        )
    from wiretorch_b200 import lowrank

    if lowrank.is_factorised(drive):
        return lowrank.simulate(v, g, x, drive, p, refractory=refractory, gating=gating,
                                adaptation=adaptation, probabilities=probabilities, track=track,
                                track_batch_idx=track_batch_idx, retain=retain)  # fmt: skip
    if not x.is_cuda:
        raise RuntimeError("wiretorch_b200 runs on CUDA tensors only (no CPU path)")
    B, T, n_in = x.shape
    device = x.device
    plan = get_plan(drive, p, B, n_in, device)
    weights = [W for _, W in drive.recurrent] + [W for _, W in drive.feedforward]
    grad = torch.is_grad_enabled() and (
        drive.scale.requires_grad or x.requires_grad
        or any(getattr(W, "requires_grad", False) for W in weights)
        or any(_requires_grad(getattr(p, n, None)) for n in PHYSIOLOGY)
    )  # fmt: skip
    if grad:
        from wiretorch_b200 import autograd

        return autograd.simulate_with_grad(plan, v, g, x, drive, p, refractory, gating,
                                           adaptation, probabilities, track, track_batch_idx)  # fmt: skip
    _plan.fold(plan, drive.scale)
    v_k, g_k, counter, g_a, gating_k = _prepare_state(plan, v, g, refractory, gating, adaptation, p)
    track_b = -1 if track_batch_idx is None else int(track_batch_idx)
    with torch.no_grad():
        out = run_forward(plan, p, x.detach().float(), v_k, g_k, counter, g_a, gating_k,
                          probabilities=probabilities, track=track, track_b=track_b)  # fmt: skip
    return _run(plan, out, v_k, g_k, counter, g_a, gating_k, p, track, refractory)


def _run(plan, out, v_k, g_k, counter, g_a, gating_k, p, track, refractory, spikes=None,
         prob=None):  # fmt: skip
    tracked = None
    if track:
        tracked = {"v": out["track_v"], "I": _external_I(plan, out["track_I"]),
                   "g": _external_tracked_g(plan, out["track_g"])}  # fmt: skip
        if "track_a" in out:
            tracked["a"] = out["track_a"]
    return Run(
        output=out["spikes"] if spikes is None else spikes,
        v=v_k,
        syn=_external_g(plan, g_k),
        probabilities=out.get("prob") if prob is None else prob,
        tracked=tracked,
        refractory=counter if refractory is not None or p.n_ref is not None else None,
        gating=gating_k,
        adaptation=g_a,
    )


def _external_I(plan, I):
    """Tracked currents ``(Bt, T, N, S' + 1)`` -> ``(Bt, T, N, S + 1)`` (leak last)."""
    if not plan.ch.pooled:
        return I
    S = plan.ch.S
    full = I.new_zeros((*I.shape[:-1], S + 1))
    for c, m in enumerate(plan.ch.member):
        full[..., m[0]] = I[..., c]
    full[..., S] = I[..., -1]
    return full


def _external_tracked_g(plan, g):
    """Tracked conductances ``(Bt, T, N, 2, S')`` -> ``(Bt, T, N, 2, S)``."""
    if not plan.ch.pooled:
        return g
    full = g.new_zeros((*g.shape[:-1], plan.ch.S))
    for c, m in enumerate(plan.ch.member):
        full[..., m[0]] = g[..., c]
    return full


def _requires_grad(t) -> bool:
    return isinstance(t, torch.Tensor) and t.requires_grad
