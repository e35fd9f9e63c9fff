"""ctypes binding of the engine's C ABI (``include/wiretorch_b200.h``).

The structures mirror the header field for field. ``lib()`` loads
``_lib/libwiretorch_b200.so`` (built by ``wiretorch_b200.build``; the environment
variable ``WIRETORCH_B200_LIB`` names another build of the same sources) and raises if
it is missing: the engine has no other implementation to fall back on.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB = Path(os.environ.get("WIRETORCH_B200_LIB") or Path(__file__).parent / "_lib" / "libwiretorch_b200.so")
MAX_CHANNELS = 8
CHUNK_EDGES = 128
EVENT_BYTES = 16  # sizeof(WtEvent)

OK, ERR_ARGS, ERR_LAUNCH, ERR_BARRIER, ERR_EVENTS, ERR_FIXED_POINT, ERR_UNSUPPORTED, ERR_RANGE = range(8)
PHASES = 7  # WT_PHASES: the phases of a forward step that WtForward.phases records
ERRORS = {
    ERR_ARGS: "inconsistent arguments",
    ERR_LAUNCH: "kernel launch failed",
    ERR_BARRIER: "a grid barrier timed out",
    ERR_EVENTS: "an event list overflowed",
    ERR_FIXED_POINT: "a synaptic input exceeded the fixed-point range",
    ERR_UNSUPPORTED: "unsupported configuration",
    ERR_RANGE: "a device index outside its table (range check)",
}

F_REFRACTORY, F_MG_BLOCK, F_ADAPT, F_SAMPLE, F_GATED = 1, 2, 4, 8, 16
F_PARTITION = 1 << 9
F_STREAM = 1 << 10
F_CURRENT = 1 << 11
F_SAVE, F_TRACK, F_PROB, F_SAVE_INPUT = 32, 64, 128, 256

P = C.c_void_p
_f8 = C.c_float * MAX_CHANNELS
_i8 = C.c_int32 * MAX_CHANNELS


class WtNet(C.Structure):
    _fields_ = [
        ("B", C.c_int32), ("N", C.c_int32), ("n_in", C.c_int32),
        ("S", C.c_int32), ("C", C.c_int32),
        ("theta", P), ("U_reset", P), ("E_L", P), ("C_m", P), ("beta", P),
        ("n_ref", P), ("adapt", P), ("adapt_decay", P), ("E_adapt", P),
        ("decay_r", _f8), ("decay_d", _f8), ("jump_r", _f8), ("jump_d", _f8),
        ("E_syn", _f8), ("g_clip", _f8), ("mg_a", _f8), ("mg_lc", _f8),
        ("input_of", _i8), ("fx_inv", _f8),
        ("dt", C.c_float), ("surr_scale", C.c_float),
        ("src_slot", P), ("slot_chunk", P), ("src_chunk", P), ("chunk_desc", P), ("edge_col", P), ("edge_cw", P),
        ("n_slots", C.c_int32), ("n_chunks", C.c_int32), ("n_rec_edges", C.c_int64),
        ("slot_gate", P), ("slot_row", P), ("gate_params", P), ("gate_cols", P),
        ("R", C.c_int32), ("R_f", C.c_int32), ("N_src", C.c_int32),
        ("src_gate", P),
    ]  # fmt: skip


class WtForward(C.Structure):
    _fields_ = [
        ("T", C.c_int32), ("T_total", C.c_int32), ("t0", C.c_int32), ("flags", C.c_int32),
        ("v", P), ("g", P), ("counter", P), ("g_a", P), ("gating", P),
        ("x", P), ("noise", P), ("spikes", P), ("prob", P),
        ("v_saved", P), ("G_saved", P), ("spike_bits", P), ("held_bits", P),
        ("a_saved", P), ("f_saved", P), ("X_saved", P),
        ("track_v", P), ("track_I", P), ("track_g", P), ("track_a", P),
        ("track_b", C.c_int32),
        ("words", P), ("peer_words", P * 8), ("progress", P), ("peer_progress", P * 8),
        ("n_ranks", C.c_int32), ("rank", C.c_int32), ("word0", C.c_int32), ("epoch", C.c_uint32),
        ("amps", P), ("peer_amps", P * 8),
        ("push_src_chunk", P * 8), ("push_chunk_desc", P * 8), ("push_ev", P * 8),
        ("push_cap", C.c_longlong * 8), ("push_half", C.c_longlong * 8), ("push_count", P * 8),
        ("push_reserve", P), ("pull_ev", P), ("pull_off", C.c_longlong * 8), ("pull_half", C.c_longlong),
        ("pull_count", P),
        ("phases", P), ("phase_warps", C.c_int32),
    ]  # fmt: skip


class WtWorkspace(C.Structure):
    _fields_ = [
        ("X", P), ("ev", P), ("ev_count", P), ("barrier", P),
        ("err", P), ("ev_cap", C.c_int64), ("edges", P),
    ]  # fmt: skip


_lib = None


def lib() -> C.CDLL:
    """The engine's shared library (``RuntimeError`` if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise RuntimeError(
                f"{LIB} is missing: build it with `python -m wiretorch_b200.build` "
                "(the engine has no CPU or PyTorch fallback)"
            )
        _lib = C.CDLL(str(LIB))
        _lib.wt_last_error.restype = C.c_char_p
        _lib.wt_edge_grads_scratch_words.restype = C.c_int64
        _lib.wt_edge_grads_slice_trials.restype = C.c_int32
        for name in ("wt_forward", "wt_fold_weights", "wt_workspace_bytes", "wt_abi_version",
                     "wt_backward", "wt_edge_grads", "wt_filter_forward", "wt_filter_backward",
                     "wt_forward_noalloc", "wt_noalloc_error", "wt_van_rossum_forward",
                     "wt_van_rossum_backward", "wt_lowrank_product", "wt_lowrank_forward", "wt_recurrent_carry",
                     "wt_unpack_spikes", "wt_pack_spikes"):
            getattr(_lib, name).restype = C.c_int
    return _lib


#: Kernels this process has launched through the library (for the benchmark's count).
LAUNCHES = 0


def count_launches(n: int) -> None:
    global LAUNCHES
    LAUNCHES += n


#: When a dict, each launch through the library records CUDA events around itself on
#: the current stream under its kernel's name: ``{name: [(start, end), ...]}``.
TIMER = None


class timed:
    """Context manager: events around a launch (only while ``TIMER`` is a dict)."""

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        if TIMER is not None:
            import torch

            self.start = torch.cuda.Event(enable_timing=True)
            self.start.record()
        return self

    def __exit__(self, *exc):
        if TIMER is not None:
            import torch

            end = torch.cuda.Event(enable_timing=True)
            end.record()
            TIMER.setdefault(self.name, []).append((self.start, end))
        return False


def check(rc: int, what: str) -> None:
    if rc != OK:
        detail = lib().wt_last_error().decode()
        raise RuntimeError(f"{what}: {ERRORS.get(rc, rc)} ({detail})")


def ptr(t) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_of(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream
