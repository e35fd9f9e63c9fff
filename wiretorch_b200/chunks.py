"""The runners' data path: batches copied to the device while the previous chunk runs,
chunks staged back to the host, and spikes moved between the two as bits.

It keeps the interface of wiretorch's runner data path — ``to_device`` and ``Prefetcher``
(``snn_runners/chunks.py:19-70``, what ``SNNTrainer`` iterates, ``trainer.py:219``) and the
inference runner's staging of each chunk into reused pinned host buffers (``_Stager``,
``snn_runners/inference_runner.py:111-150``, here ``Stager``) — and changes the format in
which spikes cross the host link. The reference copies spike tensors whole: a byte per
spike for its bool datasets and outputs. Here a spike tensor of shape ``(..., n)`` travels
as ``PackedSpikes``: each row of n spikes in ceil(n / 8) bytes, spike i in bit i % 8 of
byte i / 8 (numpy's ``packbits(x, axis=-1, bitorder="little")``), an eighth of the bytes of
a bool tensor and a thirty-second of a float one. The library's kernels pack and unpack on
a CUDA device (``wt_pack_spikes``, ``wt_unpack_spikes``: one pass over the unpacked side
in HBM); host tensors — a dataset being written once in this format, a staged chunk being
read — are packed and unpacked with numpy.
"""

from __future__ import annotations

import ctypes as C
from concurrent.futures import Future

import numpy as np
import torch

from . import _lib

#: Data fields of a dataloader batch, besides the input spikes (the reference's names).
TARGET_FIELDS = ("target_spikes", "target_calcium", "target_rate")


class _SpikeBits(C.Structure):
    _fields_ = [("rows", C.c_int64), ("n", C.c_int32), ("kind", C.c_int32), ("bits", _lib.P),
                ("spikes", _lib.P), ("err", _lib.P)]  # fmt: skip


_F32, _U8 = 0, 1


def _kind(dtype: torch.dtype) -> int | None:
    return _F32 if dtype == torch.float32 else _U8 if dtype in (torch.bool, torch.uint8) else None


class PackedSpikes:
    """A spike tensor of shape ``(*lead, n)`` held as bits: ``bits`` (uint8, shape
    ``(*lead, ceil(n / 8))``) and ``n``. ``dtype`` is the tensor's own type, what
    ``unpack`` returns unless asked for another."""

    def __init__(self, bits: torch.Tensor, n: int, dtype: torch.dtype = torch.bool):
        if bits.dtype != torch.uint8 or bits.dim() < 1 or bits.shape[-1] != (n + 7) // 8:
            raise ValueError(f"bits must be uint8 of shape (..., {(n + 7) // 8}) for {n} spikes a row")
        self.bits, self.n, self.dtype = bits, int(n), dtype

    @property
    def shape(self) -> torch.Size:
        return torch.Size((*self.bits.shape[:-1], self.n))

    @property
    def device(self) -> torch.device:
        return self.bits.device

    @property
    def nbytes(self) -> int:
        return self.bits.numel()

    def to(self, device, non_blocking: bool = False) -> PackedSpikes:
        return PackedSpikes(self.bits.to(device, non_blocking=non_blocking), self.n, self.dtype)

    def pin_memory(self) -> PackedSpikes:
        return PackedSpikes(self.bits.pin_memory(), self.n, self.dtype)

    def unpack(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        """The spikes as a tensor of ``dtype`` (default: the packed tensor's), on the
        bits' device: 0 or 1."""
        dtype = dtype or self.dtype
        if self.bits.device.type != "cuda":
            flat = np.unpackbits(self.bits.contiguous().numpy(), axis=-1, count=self.n, bitorder="little")
            return torch.from_numpy(flat).to(dtype)
        kind = _kind(dtype)
        out = torch.empty(self.shape, dtype=dtype if kind is not None else torch.float32, device=self.device)
        a = _SpikeBits(out.numel() // max(self.n, 1) if self.n else 0, self.n, _F32 if kind is None else kind,
                       self.bits.contiguous().data_ptr(), out.data_ptr(), None)  # fmt: skip
        with _lib.timed("wt_unpack_spikes"):
            rc = _lib.lib().wt_unpack_spikes(C.byref(a), C.c_void_p(_lib.stream_of(self.device)))
        _lib.check(rc, "wt_unpack_spikes")
        _lib.count_launches(1)
        return out if kind is not None else out.to(dtype)


def pack_spikes(x: torch.Tensor, check: bool = True) -> PackedSpikes:
    """``x`` (0 or 1 along its last dimension, any dtype) as bits, on its own device.

    A spike is any value other than 0. With ``check``, a value other than 0 or 1 (a count
    of spikes in one step, which bits cannot hold) raises ``ValueError``; on a CUDA device
    the check reads the kernel's error word back (a host synchronisation)."""
    n = x.shape[-1] if x.dim() else 1
    lead = tuple(x.shape[:-1])
    if x.device.type != "cuda":
        a = x.detach().contiguous().numpy()
        if check and np.any((a != 0) & (a != 1)):
            raise ValueError("pack_spikes: values other than 0 and 1 (spike counts) cannot be held as bits")
        return PackedSpikes(torch.from_numpy(np.packbits(a != 0, axis=-1, bitorder="little")), n, x.dtype)
    src = x.detach()
    if _kind(src.dtype) is None:
        src = src.float()
    src = src.contiguous()
    bits = torch.empty((*lead, (n + 7) // 8), dtype=torch.uint8, device=x.device)
    err = torch.zeros(1, dtype=torch.int32, device=x.device) if check else None
    a = _SpikeBits(src.numel() // max(n, 1) if n else 0, n, _kind(src.dtype), bits.data_ptr(), src.data_ptr(),
                   _lib.ptr(err))  # fmt: skip
    with _lib.timed("wt_pack_spikes"):
        rc = _lib.lib().wt_pack_spikes(C.byref(a), C.c_void_p(_lib.stream_of(x.device)))
    _lib.check(rc, "wt_pack_spikes")
    _lib.count_launches(1)
    if check and int(err.item()):
        raise ValueError("pack_spikes: values other than 0 and 1 (spike counts) cannot be held as bits")
    return PackedSpikes(bits, n, x.dtype)


def _to(value, device):
    if isinstance(value, PackedSpikes):  # the bits cross, the device unpacks
        return value.to(device, non_blocking=True).unpack()
    return value.to(device, non_blocking=True)


def to_device(batch, device) -> dict[str, torch.Tensor | None]:
    """The batch's input spikes and targets on ``device`` (None where absent); fields held
    as ``PackedSpikes`` are copied as bits and unpacked there (on the current stream)."""
    out = {"input_spikes": _to(batch.input_spikes, device)}
    for name in TARGET_FIELDS:
        value = getattr(batch, name, None)
        out[name] = None if value is None else _to(value, device)
    return out


class Prefetcher:
    """Iterates over batches on the device, copying each one while the last one runs.

    On CUDA the next batch's host-to-device copy (and the unpacking of its packed
    spikes) is issued on a side stream as soon as the current batch is handed out, so it
    overlaps the current chunk's compute; pinned host batches make the copy asynchronous.
    Elsewhere it is ``to_device(next(batches))``.
    """

    _END = object()

    def __init__(self, batches, device):
        self.batches = batches
        self.device = device
        cuda = torch.device(device).type == "cuda" and torch.cuda.is_available()
        self.stream = torch.cuda.Stream(device) if cuda else None
        self._next = None

    def __iter__(self):
        return self

    def __next__(self) -> dict[str, torch.Tensor | None]:
        if self.stream is None:
            return to_device(next(self.batches), self.device)
        batch = self._next if self._next is not None else self._copy()
        if batch is self._END:
            raise StopIteration
        compute = torch.cuda.current_stream(self.device)
        compute.wait_stream(self.stream)
        for tensor in batch.values():
            if tensor is not None:  # made on the side stream, used on this one
                tensor.record_stream(compute)
        self._next = self._copy()
        return batch

    def _copy(self):
        try:
            batch = next(self.batches)
        except StopIteration:
            return self._END
        with torch.cuda.stream(self.stream):
            return to_device(batch, self.device)


class StagedChunk(Future):
    """A staged chunk: its host buffers, readable once the copies have landed. The
    consumer sets the result (any value) when done with them, which frees them for the
    next chunk."""

    def __init__(self, host: dict, done):
        super().__init__()
        self.host, self.done = host, done

    def _landed(self) -> None:
        if self.done is not None:
            self.done.synchronize()

    def arrays(self) -> dict[str, np.ndarray]:
        """Every tensor as a numpy array, spikes unpacked (what the reference's staging
        returns)."""
        self._landed()
        return {name: (t.unpack() if isinstance(t, PackedSpikes) else t).numpy() for name, t in self.host.items()}

    def packed(self) -> dict:
        """The host buffers as they are: spikes as ``PackedSpikes``, the rest tensors."""
        self._landed()
        return dict(self.host)


class Stager:
    """Copies a chunk's tensors to reused pinned host buffers without blocking; spike
    tensors are packed on the device first and cross as bits.

    ``stage(record)`` returns a ``StagedChunk``. A buffer is reused only once the previous
    chunk's consumer has finished with it (set its result), so at most one chunk is in
    flight while the next is simulated. Which tensors are spikes: bool tensors, and those
    named in ``spike_fields`` (float 0/1, for instance the engine's output).
    """

    def __init__(self, spike_fields: tuple[str, ...] = ()):
        self.spike_fields = set(spike_fields)
        self._buffers: dict[str, torch.Tensor] = {}
        self._pending: StagedChunk | None = None

    def _buffer(self, name: str, like: torch.Tensor) -> torch.Tensor:
        buf = self._buffers.get(name)
        if buf is None or buf.shape != like.shape or buf.dtype != like.dtype:
            buf = torch.empty(like.shape, dtype=like.dtype, pin_memory=like.is_cuda)
            self._buffers[name] = buf
        return buf

    def stage(self, record: dict[str, torch.Tensor]) -> StagedChunk:
        if self._pending is not None:
            self._pending.result()  # the previous chunk is done with the buffers
        host = {}
        for name, tensor in record.items():
            if tensor.is_cuda and (tensor.dtype == torch.bool or name in self.spike_fields):
                packed = pack_spikes(tensor, check=False)
                buf = self._buffer(name, packed.bits)
                buf.copy_(packed.bits, non_blocking=True)
                host[name] = PackedSpikes(buf, packed.n, tensor.dtype)
            else:
                buf = self._buffer(name, tensor)
                buf.copy_(tensor, non_blocking=True)
                host[name] = buf
        done = torch.cuda.Event() if any(t.is_cuda for t in record.values()) else None
        if done is not None:
            done.record()
        self._pending = StagedChunk(host, done)
        return self._pending

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        if self._pending is not None:
            self._pending.result()
