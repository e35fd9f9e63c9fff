"""Reading and writing the golden cases of ``tests/golden/*.npz``.

A case is one call of the engine: the network as the engine sees it (a ``Drive`` and a
``Physiology``), the input and state it starts from, and what wiretorch's own
implementation produced from them — the spike raster (bit-packed along the neuron
axis), the voltage after every step, the final state, and, for the gradient cases, the
gradients of ``sum(spikes * R)`` (plus ``sum(probabilities * R2)``) with respect to
every differentiable input of the engine. Cases that come from a recording of the
reference's own test suite also carry that recording (``rec.*``): its spike raster,
voltages and the state at every window start.

``make_golden.py`` writes them; the tests read them with ``load``.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from wiretorch_b200.types import Drive, Gate, Physiology

GOLDEN = Path(__file__).parent / "golden"

PHYSIOLOGY_FIELDS = (
    "theta", "U_reset", "E_L", "C_m", "beta", "E_syn", "g_clip", "decay", "jump",
    "dt", "surr_scale", "n_ref", "mg_c", "mg_a", "adapt", "adapt_decay", "E_adapt",
)  # fmt: skip


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
            sources[id(W)] = len(sources)
            arrays[f"net.W.{sources[id(W)]}"] = _np(W).astype(np.float32)
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
    for name in PHYSIOLOGY_FIELDS:
        value = getattr(p, name)
        if value is not None:
            arrays[f"phys.{name}"] = _np(value)
    for prefix, group in (("in", inputs), ("out", outputs), ("grad", grads),
                          ("rec", recorded)):  # fmt: skip
        for key, value in group.items():
            if value is None:
                continue
            if key.endswith("spikes"):
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
    for name in PHYSIOLOGY_FIELDS:
        key = f"phys.{name}"
        phys[name] = t(arrays[key]) if key in arrays else None
    p = Physiology(**phys, spike_mode=meta["spike_mode"])
    data = {}
    for key, value in arrays.items():
        if key.startswith(("net.", "phys.")) or key.endswith(".shape"):
            continue
        if key.endswith(".bits"):
            data[key.removesuffix(".bits")] = unpack(value, N)
        else:
            data[key] = value
    return drive, p, data, meta


def cases() -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob("*.npz"))
