"""The spike-train losses' filter and the van Rossum rate loss, on the engine's kernels.

``double_exponential`` has the signature and result of wiretorch's
``training_utils/filtering.py:28-48``: trains ``x`` ``(B, T, N)`` filtered first with the
rise and then with the decay exponential, continuing from carried state (which enters
undecayed at the first step); ``kernel_*[k] = exp(-k dt / tau)``, of which the filter
uses the per-step decay ``kernel[1]``. The reference computes it as a Toeplitz product
on the CPU and a Triton recursion on CUDA; here it is the ``wt_filter_forward`` /
``wt_filter_backward`` kernels (a parallel scan over T when the trains are few).

``VanRossumRateLoss`` is ``training_utils/losses.py:140-194``: the mean squared
difference of the filtered output and the filtered target rate (expected spikes per
step), carrying the filter state from chunk to chunk; both filters and the mean square
run fused in one kernel (``wt_van_rossum_forward``), the gradient in one more.
"""

from __future__ import annotations

import torch
from torch import nn

from wiretorch_b200 import _lib


def _step_decay(kernel: torch.Tensor) -> float:
    """``kernel[1]``, read from the device once per kernel tensor."""
    decay = getattr(kernel, "_wt_step_decay", None)
    if decay is None:
        decay = float(kernel[1]) if kernel.numel() > 1 else 0.0
        kernel._wt_step_decay = decay
    return decay


class _FilterArgs(_lib.C.Structure):
    _fields_ = [
        ("B", _lib.C.c_int32), ("T", _lib.C.c_int32), ("N", _lib.C.c_int32),
        ("x", _lib.P), ("x_bstride", _lib.C.c_int64), ("x_tstride", _lib.C.c_int64),
        ("carry_rise", _lib.P), ("carry_smooth", _lib.P),
        ("a_rise", _lib.C.c_float), ("a_decay", _lib.C.c_float),
        ("rise", _lib.P), ("smooth", _lib.P), ("last_rise", _lib.P), ("last_smooth", _lib.P),
    ]  # fmt: skip


class _FilterGradArgs(_lib.C.Structure):
    _fields_ = [
        ("B", _lib.C.c_int32), ("T", _lib.C.c_int32), ("N", _lib.C.c_int32),
        ("grad_smooth", _lib.P), ("grad_scale", _lib.C.c_float),
        ("a_rise", _lib.C.c_float), ("a_decay", _lib.C.c_float), ("grad_x", _lib.P),
    ]  # fmt: skip


def filter_forward(x, a_rise, a_decay, carried_rise=None, carried_smooth=None, rise=True):
    """``(rise, smooth, last_rise, last_smooth)``; ``x`` may broadcast over time
    (stride 0). ``rise`` False skips writing the rise train (None is returned)."""
    if not x.is_cuda:
        raise RuntimeError("wiretorch_b200 runs on CUDA tensors only (no CPU path)")
    B, T, N = x.shape
    if x.dtype != torch.float32:
        x = x.float()
    if x.stride(2) != 1:
        x = x.contiguous()
    out_r = torch.empty((B, T, N), device=x.device) if rise else None
    out_s = torch.empty((B, T, N), device=x.device)
    last_r = torch.empty((B, N), device=x.device)
    last_s = torch.empty((B, N), device=x.device)
    f = _FilterArgs()
    f.B, f.T, f.N = B, T, N
    f.x, f.x_bstride, f.x_tstride = x.data_ptr(), x.stride(0), x.stride(1)
    cr = None if carried_rise is None else carried_rise.reshape(B, N).float().contiguous()
    cs = None if carried_smooth is None else carried_smooth.reshape(B, N).float().contiguous()
    f.carry_rise, f.carry_smooth = _lib.ptr(cr), _lib.ptr(cs)
    f.a_rise, f.a_decay = a_rise, a_decay
    f.rise, f.smooth = _lib.ptr(out_r), out_s.data_ptr()
    f.last_rise, f.last_smooth = last_r.data_ptr(), last_s.data_ptr()
    with _lib.timed("wt_filter_forward"):
        rc = _lib.lib().wt_filter_forward(_lib.C.byref(f), _lib.C.c_void_p(_lib.stream_of(x.device)))
    _lib.check(rc, "wt_filter_forward")
    _lib.count_launches(1)
    return out_r, out_s, last_r, last_s


def filter_backward(grad_smooth, a_rise, a_decay, grad_scale=1.0):
    B, T, N = grad_smooth.shape
    grad_smooth = grad_smooth.float().contiguous()
    grad_x = torch.empty_like(grad_smooth)
    f = _FilterGradArgs()
    f.B, f.T, f.N = B, T, N
    f.grad_smooth, f.grad_scale = grad_smooth.data_ptr(), grad_scale
    f.a_rise, f.a_decay, f.grad_x = a_rise, a_decay, grad_x.data_ptr()
    with _lib.timed("wt_filter_backward"):
        rc = _lib.lib().wt_filter_backward(_lib.C.byref(f), _lib.C.c_void_p(_lib.stream_of(grad_smooth.device)))
    _lib.check(rc, "wt_filter_backward")
    _lib.count_launches(1)
    return grad_x


class _DoubleExponential(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, a_rise, a_decay, carried_rise, carried_smooth):
        rise, smooth, _, _ = filter_forward(x, a_rise, a_decay, carried_rise, carried_smooth)
        ctx.decays = (a_rise, a_decay)
        ctx.mark_non_differentiable(rise)
        return rise, smooth

    @staticmethod
    def backward(ctx, _grad_rise, grad_smooth):
        return filter_backward(grad_smooth, *ctx.decays), None, None, None, None


def double_exponential(x, kernel_rise, kernel_decay, carried_rise, carried_smooth):
    """Filter ``x`` ``(B, T, N)``; return ``(rise, smooth)`` (``filtering.py:28-48``).
    No gradient flows into the carried states."""
    return _DoubleExponential.apply(
        x, _step_decay(kernel_rise), _step_decay(kernel_decay),
        None if carried_rise is None else carried_rise.detach(),
        None if carried_smooth is None else carried_smooth.detach(),
    )  # fmt: skip


class _VanRossumArgs(_lib.C.Structure):
    _fields_ = [
        ("B", _lib.C.c_int32), ("T", _lib.C.c_int32), ("N", _lib.C.c_int32),
        ("x", _lib.P), ("x_bstride", _lib.C.c_int64), ("x_tstride", _lib.C.c_int64),
        ("y", _lib.P), ("y_bstride", _lib.C.c_int64), ("y_tstride", _lib.C.c_int64),
        ("carry", _lib.P), ("a_rise", _lib.C.c_float), ("a_decay", _lib.C.c_float),
        ("err", _lib.P), ("last", _lib.P), ("partial", _lib.P),
    ]  # fmt: skip


class _VanRossumGradArgs(_lib.C.Structure):
    _fields_ = [
        ("B", _lib.C.c_int32), ("T", _lib.C.c_int32), ("N", _lib.C.c_int32),
        ("err", _lib.P), ("grad_loss", _lib.P), ("scale", _lib.C.c_float),
        ("a_rise", _lib.C.c_float), ("a_decay", _lib.C.c_float), ("grad_x", _lib.P),
    ]  # fmt: skip


def _unit_neuron_stride(t):
    t = t if t.dtype == torch.float32 else t.float()
    return t if t.stride(2) == 1 else t.contiguous()


class _VanRossumRate(torch.autograd.Function):
    """mean((smooth(x) - smooth(y))^2) in one kernel; the backward in one more. The
    states after the chunk are left in ``state["last"]`` ``(4, B, N)``."""

    @staticmethod
    def forward(ctx, x, y, carry, a_rise, a_decay, state):
        if not x.is_cuda:
            raise RuntimeError("wiretorch_b200 runs on CUDA tensors only (no CPU path)")
        B, T, N = x.shape
        x, y = _unit_neuron_stride(x.detach()), _unit_neuron_stride(y.detach())
        dev = x.device
        err = torch.empty((B, T, N), device=dev)
        last = torch.empty((4, B, N), device=dev)
        partial = torch.empty((max(-(-B * N // 256), 1),), dtype=torch.float64, device=dev)
        a = _VanRossumArgs()
        a.B, a.T, a.N = B, T, N
        a.x, a.x_bstride, a.x_tstride = x.data_ptr(), x.stride(0), x.stride(1)
        a.y, a.y_bstride, a.y_tstride = y.data_ptr(), y.stride(0), y.stride(1)
        a.carry = _lib.ptr(carry)
        a.a_rise, a.a_decay = a_rise, a_decay
        a.err, a.last, a.partial = err.data_ptr(), last.data_ptr(), partial.data_ptr()
        with _lib.timed("wt_van_rossum_forward"):
            rc = _lib.lib().wt_van_rossum_forward(_lib.C.byref(a), _lib.C.c_void_p(_lib.stream_of(dev)))
        _lib.check(rc, "wt_van_rossum_forward")
        _lib.count_launches(1)
        state["last"] = last
        ctx.save_for_backward(err)
        ctx.decays = (a_rise, a_decay)
        return (partial.sum() / max(B * T * N, 1)).float()

    @staticmethod
    def backward(ctx, grad):
        (err,) = ctx.saved_tensors
        B, T, N = err.shape
        grad = grad.detach().float().reshape(1).contiguous()
        grad_x = torch.empty_like(err)
        a = _VanRossumGradArgs()
        a.B, a.T, a.N = B, T, N
        a.err, a.grad_loss, a.scale = err.data_ptr(), grad.data_ptr(), 2.0 / max(B * T * N, 1)
        a.a_rise, a.a_decay, a.grad_x = *ctx.decays, grad_x.data_ptr()
        with _lib.timed("wt_van_rossum_backward"):
            rc = _lib.lib().wt_van_rossum_backward(_lib.C.byref(a), _lib.C.c_void_p(_lib.stream_of(err.device)))
        _lib.check(rc, "wt_van_rossum_backward")
        _lib.count_launches(1)
        return grad_x, None, None, None, None, None


class VanRossumRateLoss(nn.Module):
    """Mean squared difference of the double-filtered output spikes and the filtered
    target rate (``training_utils/losses.py:31-194``), carrying the filter state across
    chunks. ``target_rate`` is expected spikes per step, ``(B, T, N)`` (any strides: a
    rate constant in time can be an expanded view). Both filters, the difference and its
    mean square run as one kernel (``wt_van_rossum_forward``), its gradient as another."""

    def __init__(self, tau_rise, tau_decay, dt, window_size, device="cuda"):
        super().__init__()
        t = torch.arange(window_size, dtype=torch.float32, device=device) * dt
        self.register_buffer("kernel_rise", torch.exp(-t / tau_rise))
        self.register_buffer("kernel_decay", torch.exp(-t / tau_decay))
        self.reset_state()

    def reset_state(self):
        self.prev_output_rise = self.prev_target_rise = None
        self.prev_output_smooth = self.prev_target_smooth = None

    def forward(self, target_rate, output_spikes=None, output_probabilities=None):
        signal = output_probabilities if output_probabilities is not None else output_spikes
        a_r, a_d = _step_decay(self.kernel_rise), _step_decay(self.kernel_decay)
        B, T, N = signal.shape
        carry = None
        if self.prev_output_rise is not None:
            parts = [self.prev_output_rise, self.prev_output_smooth, self.prev_target_rise,
                     self.prev_target_smooth]  # fmt: skip
            carry = torch.stack([q.detach().reshape(B, N).float() for q in parts]).contiguous()
        state = {}
        loss = _VanRossumRate.apply(signal, target_rate.expand(B, T, N), carry, a_r, a_d, state)
        last = state["last"]
        self.prev_output_rise, self.prev_output_smooth = last[0][:, None], last[1][:, None]
        self.prev_target_rise, self.prev_target_smooth = last[2][:, None], last[3][:, None]
        return loss
