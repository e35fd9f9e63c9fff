"""Reading and writing the golden cases of ``tests/golden/*.npz``.

A case is one call of the engine: the network as the engine sees it (a ``Drive`` and a
``Physiology``), the input and state it starts from, and what wiretorch's own
implementation produced from them — the spike raster (bit-packed along the neuron
axis), the voltage after every step, the final state, and, for the gradient cases, the
gradients of ``sum(spikes * R)`` (plus ``sum(probabilities * R2)``) with respect to
every differentiable input of the engine. Cases that come from a recording of the
reference's own test suite also carry that recording (``rec.*``): its spike raster,
voltages and the state at every window start.

The configuration (``config_*``) and statistics (``statistics_*``) cases store their
weights as CSR rows (``SparseRows``) and their 0/1 inputs bit-packed (``x_bits``), and
record voltages every ``snap`` steps instead of every step. The loss cases
(``loss_*``) are plain arrays, read with ``numpy.load``.

``make_golden.py`` writes them; the tests read them with ``load``.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from wiretorch_b200.types import CurrentPhysiology, Drive, Gate, Physiology, SparseRows

GOLDEN = Path(__file__).parent / "golden"

PHYSIOLOGY_FIELDS = (
    "theta", "U_reset", "E_L", "C_m", "beta", "E_syn", "g_clip", "decay", "jump",
    "dt", "surr_scale", "n_ref", "mg_c", "mg_a", "adapt", "adapt_decay", "E_adapt",
)  # fmt: skip


#: The current-based family's physiology (``meta["family"] == "current"``).
CURRENT_FIELDS = ("theta", "U_reset", "beta", "U_rest", "R", "sign", "decay", "surr_scale", "n_ref",
                  "adapt", "adapt_decay")  # fmt: skip


def pack(spikes) -> np.ndarray:
    return np.packbits(np.asarray(spikes) > 0.5, axis=-1)


def unpack(bits, n) -> np.ndarray:
    return np.unpackbits(bits, axis=-1, count=n).astype(bool)


def _np(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def save(path: Path, *, drive, p, inputs: dict, outputs: dict, grads: dict,
         recorded: dict, meta: dict) -> None:  # fmt: skip
    """Write one case. ``drive`` and ``p`` are the reference's own objects (read by
    attribute); ``inputs``/``outputs``/``grads``/``recorded`` map names to arrays."""
    arrays = {}
    sources = {}  # id of a weight tensor -> index, so shared weights are stored once

    def source(W):
        if id(W) not in sources:
            i = sources[id(W)] = len(sources)
            if isinstance(W, SparseRows):  # CSR rows: the configuration-sized networks
                arrays[f"net.Wcsr.{i}.row_ptr"] = _np(W.row_ptr).astype(np.int64)
                arrays[f"net.Wcsr.{i}.cols"] = _np(W.cols).astype(np.int32)
                arrays[f"net.Wcsr.{i}.values"] = _np(W.values).astype(np.float32)
                arrays[f"net.Wcsr.{i}.n_targets"] = np.int64(W.n_targets)
            else:
                arrays[f"net.W.{i}"] = _np(W).astype(np.float32)
        return sources[id(W)]

    meta = dict(meta)
    meta["rec"] = []
    meta["ff"] = []
    for side, pathways in (("rec", drive.recurrent), ("ff", drive.feedforward)):
        for k, (rows, W) in enumerate(pathways):
            arrays[f"net.{side}_rows.{k}"] = _np(rows).astype(np.int64)
            meta[side].append(source(W))
    gates = []
    for k, gate in enumerate(drive.gates or []):
        if gate is None:
            gates.append(None)
        else:
            arrays[f"net.gate_params.{k}"] = _np(gate.params).astype(np.float32)
            gates.append(dict(stp=bool(gate.stp), saturates=bool(gate.saturates),
                              start=int(gate.start), n=int(gate.n)))  # fmt: skip
    meta["gates"] = gates
    meta["recurrent_gradients"] = bool(drive.recurrent_gradients)
    meta["spike_mode"] = p.spike_mode
    arrays["net.made"] = _np(drive.made).astype(bool)
    arrays["net.scale"] = _np(drive.scale).astype(np.float32)
    for name in CURRENT_FIELDS if meta.get("family") == "current" else PHYSIOLOGY_FIELDS:
        value = getattr(p, name)
        if value is not None:
            arrays[f"phys.{name}"] = _np(value)
    for prefix, group in (("in", inputs), ("out", outputs), ("grad", grads),
                          ("rec", recorded)):  # fmt: skip
        for key, value in group.items():
            if value is None:
                continue
            if key.startswith("x") and meta.get("x_bits"):  # 0/1 input trains, bit-packed
                a = _np(value)
                assert np.isin(a, (0.0, 1.0)).all()
                arrays[f"{prefix}.{key}.xbits"] = pack(a)
                arrays[f"{prefix}.{key}.xshape"] = np.array(a.shape, np.int64)
            elif key.endswith("spikes"):
                arrays[f"{prefix}.{key}.bits"] = pack(_np(value))
            else:
                arrays[f"{prefix}.{key}"] = _np(value)
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(path, **arrays)


def load(name: str, device="cpu"):
    """Read case ``name`` into ``(drive, p, data, meta)``: ``data`` maps the flat keys
    (``in.x``, ``out.spikes`` unpacked, ``grad.scale``, ...) to numpy arrays."""
    with np.load(GOLDEN / f"{name}.npz") as raw:
        arrays = {k: raw[k] for k in raw.files}
    meta = json.loads(str(arrays.pop("meta")))
    N = arrays["net.scale"].shape[1]

    def t(a, dtype=None):
        out = torch.from_numpy(np.ascontiguousarray(a)).to(device)
        return out if dtype is None else out.to(dtype)

    weights = {}

    def W(i):
        if i not in weights:
            if f"net.Wcsr.{i}.row_ptr" in arrays:
                weights[i] = SparseRows(t(arrays[f"net.Wcsr.{i}.row_ptr"]), t(arrays[f"net.Wcsr.{i}.cols"]),
                                        t(arrays[f"net.Wcsr.{i}.values"]),
                                        int(arrays[f"net.Wcsr.{i}.n_targets"]))  # fmt: skip
            else:
                weights[i] = t(arrays[f"net.W.{i}"])
        return weights[i]

    recurrent = [(t(arrays[f"net.rec_rows.{k}"]), W(i)) for k, i in enumerate(meta["rec"])]
    feedforward = [(t(arrays[f"net.ff_rows.{k}"]), W(i)) for k, i in enumerate(meta["ff"])]
    gates = []
    for k, g in enumerate(meta["gates"]):
        gates.append(None if g is None else Gate(t(arrays[f"net.gate_params.{k}"]), **g))
    drive = Drive(
        made=t(arrays["net.made"]),
        scale=t(arrays["net.scale"]),
        recurrent=recurrent,
        feedforward=feedforward,
        recurrent_gradients=meta["recurrent_gradients"],
        gates=gates,
    )
    phys = {}
    current = meta.get("family") == "current"
    for name in CURRENT_FIELDS if current else PHYSIOLOGY_FIELDS:
        key = f"phys.{name}"
        phys[name] = t(arrays[key]) if key in arrays else None
    p = (CurrentPhysiology if current else Physiology)(**phys, spike_mode=meta["spike_mode"])
    data = {}
    for key, value in arrays.items():
        if key.startswith(("net.", "phys.")) or key.endswith((".shape", ".xshape")):
            continue
        if key.endswith(".xbits"):
            shape = tuple(arrays[key.removesuffix(".xbits") + ".xshape"])
            data[key.removesuffix(".xbits")] = unpack(value, shape[-1]).astype(np.float32)
        elif key.endswith(".bits"):
            data[key.removesuffix(".bits")] = unpack(value, N)
        else:
            data[key] = value
    return drive, p, data, meta


KINDS = ("config_", "statistics_", "loss_", "current_", "curstats_")


def cases() -> list[str]:
    """The scenario cases (one engine call of a reference test network each)."""
    return sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith(KINDS))


def curstats_cases() -> list[str]:
    """The reference's at-scale statistics networks of the current-based family."""
    return sorted(p.stem for p in GOLDEN.glob("curstats_*.npz"))


def current_cases() -> list[str]:
    """The current-based family's scenario cases (``current_*``)."""
    return sorted(p.stem for p in GOLDEN.glob("current_*.npz"))


def config_cases() -> list[str]:
    """The benchmark configurations' networks run by the reference (``config_c*``)."""
    return sorted(p.stem for p in GOLDEN.glob("config_*.npz"))


def statistics_cases() -> list[str]:
    """The reference's at-scale statistics networks (``statistics_*``)."""
    return sorted(p.stem for p in GOLDEN.glob("statistics_*.npz"))


def first_divergence(a, b) -> int:
    """The first step (axis 1) at which two ``(B, T, N)`` rasters differ (T if none)."""
    diff = (np.asarray(a) != np.asarray(b)).any(axis=(0, 2))
    return int(np.argmax(diff)) if diff.any() else diff.shape[0]


def population_rates(spikes, types, dt_ms) -> np.ndarray:
    """Mean firing rate (Hz) of each cell type over trials, steps and its neurons."""
    rates = np.asarray(spikes, np.float64).mean(axis=(0, 1)) / (dt_ms / 1000.0)
    return np.array([rates[types == t].mean() for t in np.unique(types)])
