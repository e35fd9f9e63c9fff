"""ORACLE — test infrastructure, not product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm import
this module, and only as the checker (or the timed CPU baseline). It drives
``cond_lif.c``, the C restatement of wiretorch's
``conductance/dynamics.py:146-237`` time loop (and of the current-based
``current/dynamics.py:116-205`` one), from a ``Drive`` and ``Physiology`` as
the reference's networks hand them to their engine (``network.py:889-909``): dense
``(n_rows, N)`` weights (or ``SparseRows``) are turned into CSR here with numpy,
independently of the engine's own conversion.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).parent
LIB = HERE / "_build" / "libwtoracle.so"

_f = C.POINTER(C.c_float)
_i32 = C.POINTER(C.c_int32)
_i64 = C.POINTER(C.c_int64)
_u8 = C.POINTER(C.c_uint8)


class _Pathway(C.Structure):
    _fields_ = [
        ("n_rows", C.c_int), ("rows", _i64), ("row_ptr", _i64), ("cols", _i32),
        ("w", _f), ("scale", _f), ("made", _u8), ("recurrent", C.c_int),
        ("gate", C.c_int), ("stp", C.c_int), ("saturates", C.c_int), ("start", C.c_int),
        ("n", C.c_int), ("c", C.c_float), ("d", C.c_float), ("U", C.c_float),
        ("d_D", C.c_float), ("d_F", C.c_float),
    ]  # fmt: skip


class _Net(C.Structure):
    _fields_ = [
        ("B", C.c_int), ("N", C.c_int), ("S", C.c_int), ("n_in", C.c_int), ("K", C.c_int),
        ("pathways", C.POINTER(_Pathway)),
        ("theta", _f), ("U_reset", _f), ("E_L", _f), ("C_m", _f), ("beta", _f),
        ("n_ref", _i32), ("adapt", _f), ("adapt_decay", _f), ("E_adapt", _f),
        ("E_syn", _f), ("g_clip", _f), ("decay", _f), ("jump", _f),
        ("mg_c", _f), ("mg_a", _f), ("dt", C.c_float), ("surr_scale", C.c_float),
        ("sample", C.c_int), ("R", C.c_int), ("current", C.c_int),
    ]  # fmt: skip


class _State(C.Structure):
    _fields_ = [("v", _f), ("g", _f), ("counter", _i32), ("g_a", _f), ("gating", _f)]


class _Out(C.Structure):
    _fields_ = [("spikes", _u8), ("v_track", _f), ("prob", _f)]


def build() -> Path:
    """Compile ``cond_lif.c`` (once)."""
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "cond_lif.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(str(build()))
        _lib.wto_simulate.restype = C.c_int
    return _lib


def _np(t, dtype=None):
    if t is None:
        return None
    if hasattr(t, "detach"):
        t = t.detach().cpu().numpy()
    a = np.asarray(t)
    return np.ascontiguousarray(a if dtype is None else a.astype(dtype))


def _ptr(a, ctype):
    return None if a is None else a.ctypes.data_as(ctype)


def csr_of(W) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``(row_ptr int64, cols int32, values float32)`` of a dense matrix or of a
    ``SparseRows``."""
    if hasattr(W, "row_ptr"):
        return _np(W.row_ptr, np.int64), _np(W.cols, np.int32), _np(W.values, np.float32)
    W = _np(W, np.float32)
    rows, cols = np.nonzero(W)
    row_ptr = np.zeros(W.shape[0] + 1, dtype=np.int64)
    np.add.at(row_ptr, rows + 1, 1)
    return np.cumsum(row_ptr), cols.astype(np.int32), W[rows, cols].astype(np.float32)


class _CurrentAsFields:
    """A current-based physiology (``current/dynamics.py:56-85``) in the fields the C
    structure holds: U_rest as E_L, R as C_m, the types' signs as E_syn, each type's
    current a decay component with a unit jump and no rise."""

    def __init__(self, p):
        sign = _np(p.sign, np.float32)
        S = sign.shape[0]
        self.theta, self.U_reset, self.beta = p.theta, p.U_reset, p.beta
        self.E_L, self.C_m, self.E_syn = p.U_rest, p.R, sign
        self.g_clip = np.full(S, np.inf, np.float32)
        self.decay = np.stack([np.zeros(S, np.float32), _np(p.decay, np.float32)])
        self.jump = np.stack([np.zeros(S, np.float32), np.ones(S, np.float32)])
        self.adapt, self.adapt_decay, self.E_adapt = p.adapt, p.adapt_decay, None
        self.mg_c = self.mg_a = None
        self.n_ref, self.dt, self.surr_scale, self.spike_mode = p.n_ref, np.float32(1.0), p.surr_scale, p.spike_mode


class Network:
    """A ``Drive`` + ``Physiology`` held as the oracle's C structures. A current-based
    physiology (one with ``sign`` and ``U_rest``) runs the current-based step; its state
    is then the currents ``(B, N, S)`` in place of the conductances."""

    def __init__(self, drive, p, B: int, n_in: int, csr_cache: dict | None = None):
        self.current = hasattr(p, "sign") and hasattr(p, "U_rest")
        if self.current:
            p = _CurrentAsFields(p)
        self.keep = []  # arrays the C structures point into
        made = _np(drive.made, np.uint8)
        scale = _np(drive.scale, np.float32)
        K, S = made.shape
        N = scale.shape[1]
        self.B, self.N, self.S, self.K, self.n_in = B, N, S, K, n_in
        csr_cache = {} if csr_cache is None else csr_cache
        paths = (_Pathway * max(K, 1))()
        pathways = [(r, W, True) for r, W in drive.recurrent]
        pathways += [(r, W, False) for r, W in drive.feedforward]
        gates = list(drive.gates) if drive.gates else [None] * K
        R = 0
        for k, (rows, W, recurrent) in enumerate(pathways):
            if id(W) not in csr_cache:
                csr_cache[id(W)] = csr_of(W)
            row_ptr, cols, vals = csr_cache[id(W)]
            rows = _np(rows, np.int64)
            sc = np.ascontiguousarray(scale[k])
            mk = np.ascontiguousarray(made[k])
            self.keep += [rows, row_ptr, cols, vals, sc, mk]
            pk = paths[k]
            pk.n_rows, pk.rows, pk.row_ptr = len(rows), _ptr(rows, _i64), _ptr(row_ptr, _i64)
            pk.cols, pk.w, pk.scale = _ptr(cols, _i32), _ptr(vals, _f), _ptr(sc, _f)
            pk.made, pk.recurrent = _ptr(mk, _u8), int(recurrent)
            gate = gates[k]
            if gate is not None:
                prm = _np(gate.params, np.float32)
                pk.gate, pk.stp, pk.saturates = 1, int(gate.stp), int(gate.saturates)
                pk.start, pk.n = int(gate.start), int(gate.n)
                pk.c, pk.d, pk.U, pk.d_D, pk.d_F = (float(v) for v in prm)
                R = max(R, gate.start + gate.width)
        self.R = R
        net = _Net()
        net.B, net.N, net.S, net.n_in, net.K = B, N, S, n_in, K
        net.pathways = paths
        self.paths = paths

        def arr(name, dtype=np.float32):
            a = _np(getattr(p, name, None), dtype)
            if a is not None:
                self.keep.append(a)
            return a

        for name in ("theta", "U_reset", "E_L", "C_m", "beta", "E_syn", "g_clip",
                     "decay", "jump", "adapt", "adapt_decay", "E_adapt", "mg_c", "mg_a"):  # fmt: skip
            setattr(net, name, _ptr(arr(name), _f))
        net.n_ref = _ptr(arr("n_ref", np.int32), _i32)
        net.dt = float(np.asarray(_np(p.dt)).reshape(-1)[0])
        net.surr_scale = float(np.asarray(_np(p.surr_scale)).reshape(-1)[0])
        net.sample = int(p.spike_mode == "sample")
        net.R = R
        net.current = int(self.current)
        self.net = net
        self.has_ref = p.n_ref is not None
        self.has_adapt = p.adapt is not None

    def simulate(self, x, v, g, refractory=None, gating=None, adaptation=None,
                 noise=None, track=True, probabilities=False) -> dict:  # fmt: skip
        """Run ``x.shape[1]`` steps; returns the new state and the outputs (numpy)."""
        x = _np(x, np.float32)
        B, T = x.shape[:2]
        assert B == self.B and x.shape[2] == self.n_in
        g = _np(g, np.float32)
        if self.current:  # the currents (B, N, S) as the decay component of (B, N, 2, S)
            g = np.stack([np.zeros_like(g), g], axis=2)
        st = {
            "v": _np(v, np.float32).copy(),
            "g": g.copy(),
            "refractory": None if not self.has_ref else (
                np.zeros((B, self.N), np.int32) if refractory is None
                else _np(refractory, np.int32).copy()),
            "adaptation": None if not self.has_adapt else (
                np.zeros((B, self.N), np.float32) if adaptation is None
                else _np(adaptation, np.float32).copy()),
            "gating": None if self.R == 0 else _np(gating, np.float32).copy(),
        }  # fmt: skip
        state = _State(
            _ptr(st["v"], _f), _ptr(st["g"], _f), _ptr(st["refractory"], _i32),
            _ptr(st["adaptation"], _f), _ptr(st["gating"], _f),
        )
        spikes = np.zeros((B, T, self.N), np.uint8)
        v_track = np.zeros((B, T, self.N), np.float32) if track else None
        prob = np.zeros((B, T, self.N), np.float32) if probabilities else None
        out = _Out(_ptr(spikes, _u8), _ptr(v_track, _f), _ptr(prob, _f))
        nz = _np(noise, np.float32) if noise is not None else None
        rc = lib().wto_simulate(C.byref(self.net), C.byref(state), _ptr(x, _f), T,
                                C.byref(out), _ptr(nz, _f))  # fmt: skip
        if rc:
            raise MemoryError("oracle: allocation failed")
        if self.current:
            st["g"] = np.ascontiguousarray(st["g"][:, :, 1])
        return dict(spikes=spikes.astype(bool), v_track=v_track, prob=prob, **st)


def set_threads(n: int) -> None:
    """OpenMP threads of the oracle (trials run in parallel)."""
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        C.CDLL("libgomp.so.1").omp_set_num_threads(int(n))
    except OSError:
        pass
