"""Backpropagation through time for the engine, as one ``torch.autograd.Function``.

The forward pass is the persistent kernel with ``WT_F_SAVE``: it keeps, per step, the
voltage entering it, the summed conductances, spike and refractory bits, the adaptation,
the gating factors (and, when decays or jumps are learnt, the synaptic input). The
backward pass is:

1. ``wt_backward``: the reverse scan per (trial, neuron) — the adjoint of every input
   channel at every step, ``Q``, and per-(trial, neuron) partial sums of the physiology
   gradients (the reference's ``scan_backward``, ``conductance/kernels.py:382-568``);
2. ``wt_edge_grads``: ``Q`` carried along the connectome's edges to the kernel scales
   ``(K, N)``, the weights (on their non-zero entries) and the input.

Gradients flow through the voltages and conductances and, via the fast-sigmoid
surrogate, into the spikes; never through the reset. By default (``Drive.recurrent_gradients``
False, the reference's default for conductance-based networks) not through the recurrent
spikes into their presynaptic neurons: the recurrent input is then input like any other.
With ``recurrent_gradients`` the scan is taken one step at a time: each step's input
adjoints are carried back along the recurrent edges to that step's source spikes
(``wt_recurrent_carry``) before the step's membrane adjoint. The gradient of a dense weight matrix is computed on its non-zero
entries: every parametrisation of the reference multiplies its weights by their mask
or connectome, so the entries that are zero carry no gradient to any parameter.
"""

from __future__ import annotations

import torch

from wiretorch_b200 import _lib, engine, plan as _plan
from wiretorch_b200.types import PHYSIOLOGY

WANT_BITS = {name: 1 << i for i, name in enumerate(PHYSIOLOGY)}


class _BackwardArgs(_lib.C.Structure):
    _fields_ = [
        ("T", _lib.C.c_int32), ("flags", _lib.C.c_int32), ("wants", _lib.C.c_int32),
        ("grad_spikes", _lib.P), ("grad_prob", _lib.P),
        ("v_saved", _lib.P), ("G_saved", _lib.P), ("a_saved", _lib.P), ("X_saved", _lib.P),
        ("g_init", _lib.P), ("spike_bits", _lib.P), ("held_bits", _lib.P), ("Q", _lib.P),
        ("g_theta", _lib.P), ("g_reset", _lib.P), ("g_E_L", _lib.P), ("g_C_m", _lib.P),
        ("g_beta", _lib.P), ("g_E_syn", _lib.P), ("g_decay", _lib.P), ("g_jump", _lib.P),
        ("g_adapt", _lib.P), ("g_adapt_decay", _lib.P), ("g_E_adapt", _lib.P),
        ("t_lo", _lib.C.c_int32), ("t_hi", _lib.C.c_int32), ("adj", _lib.P), ("R", _lib.P),
        ("QT", _lib.P),
    ]  # fmt: skip


class _CarryArgs(_lib.C.Structure):
    _fields_ = [
        ("T", _lib.C.c_int32), ("t", _lib.C.c_int32), ("adj", _lib.P), ("f_saved", _lib.P),
        ("Qt", _lib.P), ("R", _lib.P),
    ]  # fmt: skip


class _EdgeArgs(_lib.C.Structure):
    _fields_ = [
        ("T", _lib.C.c_int32), ("spike_bits", _lib.P), ("x", _lib.P), ("f_saved", _lib.P),
        ("Q", _lib.P), ("w_raw", _lib.P), ("scale", _lib.P), ("jf", _lib.P),
        ("chunk_path", _lib.P), ("g_scale", _lib.P), ("g_w", _lib.P), ("g_x", _lib.P),
        ("fired", _lib.P), ("work", _lib.P),
        ("QT", _lib.P), ("in_ptr", _lib.P), ("in_edge", _lib.P), ("in_src", _lib.P), ("in_path", _lib.P),
        ("in_fcol", _lib.P), ("ev_start", _lib.P), ("ev", _lib.P), ("ev_cap", _lib.C.c_longlong),
        ("in_acc", _lib.P), ("err", _lib.P),
    ]  # fmt: skip


class Context:
    """What the autograd function needs besides its tensor inputs."""

    def __init__(self, plan, p, drive, state, probabilities, track, track_b):
        self.plan, self.p, self.drive = plan, p, drive
        self.state = state  # (v, g, counter, g_a, gating) kernel copies, updated in place
        self.probabilities, self.track, self.track_b = probabilities, track, track_b
        self.out = None


def _unique_weights(drive):
    """The distinct weight tensors of the drive (pathways of one source cell type share
    theirs), as the tensors autograd sees (a SparseRows' values)."""
    seen, out = {}, []
    for _, W in list(drive.recurrent) + list(drive.feedforward):
        t = W.values if hasattr(W, "row_ptr") else W
        if id(t) not in seen:
            seen[id(t)] = len(out)
            out.append(t)
    return out, seen


class _Simulate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cx: Context, scale, x, n_weights, *rest):
        weights, phys = rest[:n_weights], rest[n_weights:]
        plan, p = cx.plan, cx.p
        _plan.fold(plan, scale.detach(), p)
        wants = 0
        for name, t in zip(PHYSIOLOGY, phys):
            if isinstance(t, torch.Tensor) and ctx.needs_input_grad[4 + n_weights + PHYSIOLOGY.index(name)]:
                wants |= WANT_BITS[name]
        v, g, counter, g_a, gating = cx.state
        g_init = g.clone() if wants & WANT_BITS["decay"] else None
        save = {"want_input": bool(wants & (WANT_BITS["decay"] | WANT_BITS["jump"]))}
        out = engine.run_forward(plan, p, x.detach().float(), v, g, counter, g_a, gating,
                                 probabilities=cx.probabilities, track=cx.track,
                                 track_b=cx.track_b, save=save)  # fmt: skip
        cx.out = out
        ctx.cx, ctx.save, ctx.wants, ctx.g_init = cx, save, wants, g_init
        ctx.n_weights = n_weights
        ctx.save_for_backward(scale, x, *weights)
        spikes = out["spikes"]
        prob = out.get("prob")
        if prob is None:
            prob = spikes.new_zeros(0)
        ctx.mark_non_differentiable(prob) if not cx.probabilities else None
        return spikes, prob

    @staticmethod
    def backward(ctx, grad_spikes, grad_prob):
        cx, save, wants = ctx.cx, ctx.save, ctx.wants
        plan, p = cx.plan, cx.p
        scale, x, *weights = ctx.saved_tensors
        device = plan.device
        B, T, N, C, Sp = plan.B, save["v"].shape[1], plan.N, plan.ch.C, plan.ch.Sp
        if grad_spikes is None:
            grad_spikes = torch.zeros((B, T, N), device=device)
        grad_spikes = grad_spikes.contiguous().float()
        net = plan.net(p)
        bw = _BackwardArgs()
        bw.T, bw.wants = T, wants
        flags = 0
        if p.n_ref is not None:
            flags |= _lib.F_REFRACTORY
        if p.mg_c is not None:
            flags |= _lib.F_MG_BLOCK
        if p.adapt is not None:
            flags |= _lib.F_ADAPT
        if p.spike_mode == "sample":
            flags |= _lib.F_SAMPLE
        if getattr(p, "current", False):  # current-based neurons (wiretorch_b200.current)
            flags |= _lib.F_CURRENT
        if cx.probabilities and grad_prob is not None and grad_prob.numel():
            flags |= _lib.F_PROB
            grad_prob = grad_prob.contiguous().float()
            bw.grad_prob = grad_prob.data_ptr()
        bw.flags = flags
        bw.grad_spikes = grad_spikes.data_ptr()
        bw.v_saved, bw.G_saved = save["v"].data_ptr(), save["G"].data_ptr()
        bw.spike_bits = save["spike_bits"].data_ptr()
        bw.held_bits = _lib.ptr(save.get("held_bits"))
        bw.a_saved = _lib.ptr(save.get("a"))
        bw.X_saved = _lib.ptr(save.get("X"))
        g_init = ctx.g_init
        bw.g_init = _lib.ptr(g_init)
        n_weights = ctx.n_weights
        need_scale = ctx.needs_input_grad[1]
        need_x = ctx.needs_input_grad[2] and plan.n_in > 0
        need_w = any(ctx.needs_input_grad[4 : 4 + n_weights])
        # the scale and weight gradients target by target (the adjoints written
        # target-major, each read once) wherever a target's slice of them fits on chip
        lib = _lib.lib()
        slice_trials = lib.wt_edge_grads_slice_trials(_lib.C.byref(net), T) if (need_scale or need_w) else 0
        target_major = slice_trials > 0 and not cx.recurrent and plan.n_edges > 0
        Q = QT = None
        if need_x or not target_major:
            Q = torch.empty((B, T, C, N), device=device)
            bw.Q = Q.data_ptr()
        if target_major:
            Tp = -(-T // 8) * 8
            QT = torch.empty((C, N, B, Tp), device=device)
            bw.QT = QT.data_ptr()
        shapes = {"E_syn": (B, Sp, N), "decay": (B, 2, Sp, N), "jump": (B, 2, Sp, N)}
        partial = {}
        for name, field in zip(PHYSIOLOGY, ("g_theta", "g_reset", "g_E_L", "g_C_m", "g_beta",
                                            "g_E_syn", "g_decay", "g_jump", "g_adapt",
                                            "g_adapt_decay", "g_E_adapt")):  # fmt: skip
            if wants & WANT_BITS[name]:
                alloc = torch.zeros if cx.recurrent else torch.empty  # added to step by step
                partial[name] = alloc(shapes.get(name, (B, N)), device=device)
                setattr(bw, field, partial[name].data_ptr())
        stream = _lib.C.c_void_p(_lib.stream_of(device))
        if cx.recurrent:
            _recurrent_scan(plan, net, bw, save, T, stream)
        else:
            with _lib.timed("wt_backward"):
                rc = _lib.lib().wt_backward(_lib.C.byref(net), _lib.C.byref(bw), stream)
            _lib.check(rc, "wt_backward")
            _lib.count_launches(1)

        t = plan.tensors
        g_scale = g_w = g_x = None
        if need_scale or need_w or need_x:
            eg = _EdgeArgs()
            eg.T = T
            eg.spike_bits = save["spike_bits"].data_ptr()
            xs = x.detach().float().contiguous()
            eg.x = xs.data_ptr() if plan.n_in else None
            eg.f_saved = _lib.ptr(save.get("f"))
            eg.Q = _lib.ptr(Q)
            eg.w_raw, eg.jf = t["w_raw"].data_ptr(), t["jf"].data_ptr()
            sc = scale.detach().float().contiguous()
            eg.scale = sc.data_ptr()
            eg.chunk_path = t["chunk_path"].data_ptr()
            if need_scale:
                g_scale = torch.zeros((plan.K, N), dtype=torch.float64, device=device)
                eg.g_scale = g_scale.data_ptr()
            if need_w:
                g_w = torch.zeros(max(plan.n_edges, 1), dtype=torch.float64, device=device)
                eg.g_w = g_w.data_ptr()
            if need_x:
                g_x = torch.empty(x.shape, device=device)
                eg.g_x = g_x.data_ptr()
            if need_scale or need_w:
                words = _lib.lib().wt_edge_grads_scratch_words(_lib.C.byref(net), T)
                _lib.check(0 if words >= 0 else 1, "wt_edge_grads_scratch_words")
                fired = torch.empty(words + 1, dtype=torch.int32, device=device)
                eg.fired, eg.work = fired.data_ptr(), fired[words:].data_ptr()
            if target_major:
                ie = _plan.in_edges(plan)
                eg.QT = QT.data_ptr()
                for name in ("in_ptr", "in_edge", "in_src", "in_path", "in_fcol"):
                    setattr(eg, name, _lib.ptr(ie.get(name)))
                n_src = N + plan.n_in
                slices = -(-B // slice_trials)
                # room for every source firing on one step in sixteen (625 Hz at 0.1 ms)
                ev_cap = min(B * T * n_src // 16 + 4096, 2**31 - 1)
                ev_start = torch.empty(n_src * (slices + 1), dtype=torch.int32, device=device)
                ev = torch.empty(ev_cap, dtype=torch.int32, device=device)
                in_acc = torch.empty(max(int(ie["in_edge"].numel()), 1), device=device)
                err = torch.zeros(1, dtype=torch.int32, device=device)
                eg.ev_start, eg.ev, eg.ev_cap = ev_start.data_ptr(), ev.data_ptr(), ev_cap
                eg.in_acc, eg.err = in_acc.data_ptr(), err.data_ptr()
            with _lib.timed("wt_edge_grads"):
                rc = _lib.lib().wt_edge_grads(_lib.C.byref(net), _lib.C.byref(eg), stream)
            _lib.check(rc, "wt_edge_grads")
            # the firing rows (recurrent, input), then the source-by-source kernel or the
            # event lists (count, scan, list) and the target-by-target kernel
            fired_kernels = 1 + int(plan.n_in > 0)
            _lib.count_launches(int(need_scale or need_w) * (fired_kernels + (4 if target_major else 1)) + int(need_x))
            if target_major:
                if engine.DEFER_CHECKS:
                    engine._defer_check(err, "wt_edge_grads")
                else:
                    engine.check_device(err, "wt_edge_grads")

        ctx.save = ctx.g_init = None  # release the saved run as soon as it is used
        grads_w = [None] * n_weights
        if need_w:
            grads_w = _dense_weight_grads(plan, cx.drive, weights, g_w, ctx.needs_input_grad[4:])
        grads_p = []
        for name in PHYSIOLOGY:
            if name not in partial:
                grads_p.append(None)
                continue
            part = partial[name]
            if name == "E_syn":
                grads_p.append(_to_types(plan, part.sum((0, 2))))
            elif name in ("decay", "jump"):
                grads_p.append(torch.stack([_to_types(plan, r) for r in part.sum((0, 3))]))
            else:
                grads_p.append(part.sum(0))
        return (None, None if g_scale is None else g_scale.float(), g_x, None, *grads_w, *grads_p)


def _to_types(plan, per_channel):
    """A per-channel vector ``(S',)`` as per synapse type ``(S,)`` (exact layout: same)."""
    out = per_channel.new_zeros(plan.ch.S)
    for c, members in enumerate(plan.ch.member):
        out[members[0]] = per_channel[c]
    return out


def _dense_weight_grads(plan, drive, weights, g_w, needs):
    """Per distinct weight tensor, its gradient: the per-edge gradients summed over the
    pathways (and input channels) that use it, scattered into its dense shape."""
    pathways = list(drive.recurrent) + list(drive.feedforward)
    tensors = [W.values if hasattr(W, "row_ptr") else W for _, W in pathways]
    segs = plan.tensors.get("_segments")
    out = []
    for i, W in enumerate(weights):
        if not needs[i]:
            out.append(None)
            continue
        sparse = hasattr(pathways[[id(t) for t in tensors].index(id(W))][1], "row_ptr")
        flat = torch.zeros(W.numel() if not sparse else W.shape[0], dtype=torch.float64, device=W.device)
        for k, c, base, n_e, rows_of_edge, cols in segs:
            if tensors[k] is not W:
                continue
            ge = g_w[base : base + n_e]
            if sparse:
                flat += ge
            else:
                flat.index_add_(0, rows_of_edge * W.shape[1] + cols, ge)
        out.append(flat.view(W.shape).to(W.dtype))
    return out


def _recurrent_scan(plan, net, bw, save, T, stream):
    """The reverse scan when gradients flow through the recurrent spikes: one step at a
    time, each step's input adjoints carried back along the recurrent edges to that
    step's source spikes (``wt_recurrent_carry``) before the step's membrane adjoint
    (``wt_backward`` over that step, its adjoint state kept between the steps)."""
    B, N, C, Sp = plan.B, plan.N, plan.ch.C, plan.ch.Sp
    device = plan.device
    adj = torch.zeros((B, 2 + 4 * Sp, N), device=device)
    Qt = torch.empty((C, N, B), device=device)
    R = torch.empty((B, N), device=device)
    rc = _CarryArgs()
    rc.T, rc.adj, rc.Qt, rc.R = T, adj.data_ptr(), Qt.data_ptr(), R.data_ptr()
    rc.f_saved = _lib.ptr(save.get("f"))
    bw.adj, bw.R = adj.data_ptr(), R.data_ptr()
    lib = _lib.lib()
    with _lib.timed("wt_backward"):
        for t in reversed(range(T)):
            rc.t = t
            _lib.check(lib.wt_recurrent_carry(_lib.C.byref(net), _lib.C.byref(rc), stream), "wt_recurrent_carry")
            bw.t_lo, bw.t_hi = t, t + 1
            _lib.check(lib.wt_backward(_lib.C.byref(net), _lib.C.byref(bw), stream), "wt_backward")
    _lib.count_launches(3 * T)


def simulate_with_grad(plan, v, g, x, drive, p, refractory, gating, adaptation,
                       probabilities, track, track_batch_idx):  # fmt: skip
    """``engine.simulate`` when gradients are wanted."""
    _plan.segments(plan)
    state = engine._prepare_state(plan, v, g, refractory, gating, adaptation, p)
    track_b = -1 if track_batch_idx is None else int(track_batch_idx)
    cx = Context(plan, p, drive, state, probabilities, track, track_b)
    cx.recurrent = bool(drive.recurrent_gradients and drive.recurrent)
    weights, _ = _unique_weights(drive)
    phys = [getattr(p, n) if getattr(p, n) is not None else torch.zeros(0) for n in PHYSIOLOGY]
    spikes, prob = _Simulate.apply(cx, drive.scale, x, len(weights), *weights, *phys)
    # The outputs hold the autograd graph, which holds ``cx``: take ``out`` off it so that
    # no reference cycle keeps a step's saved tensors alive after its backward pass.
    out, cx.out = cx.out, None
    v_k, g_k, counter, g_a, gating_k = state
    cx.state = None
    return engine._run(plan, out, v_k, g_k, counter, g_a, gating_k, p, track, refractory,
                       spikes=spikes, prob=prob if probabilities else None)  # fmt: skip
