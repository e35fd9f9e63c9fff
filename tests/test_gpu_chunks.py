"""Spikes as bits on the GPU (``wt_pack_spikes`` / ``wt_unpack_spikes`` through the C ABI)
against numpy's ``packbits``/``unpackbits(..., bitorder="little")``, bit for bit: ragged
rows, empty tensors, unaligned buffers (the scalar path), spike counts refused; at the
full C5 input size the round trip bits -> spikes -> bits is the identity. Then the data
path built on them: ``Prefetcher`` over packed batches and ``Stager`` packing a chunk's
spikes before they cross to the host."""

import ctypes as C
from collections import namedtuple

import numpy as np
import pytest
import torch

from wiretorch_b200 import _lib
from wiretorch_b200.chunks import PackedSpikes, Prefetcher, Stager, _SpikeBits, pack_spikes

pytestmark = pytest.mark.gpu

SpikeData = namedtuple("SpikeData", ["input_spikes", "target_rate"])


def _random_bits(rows, n, seed):
    rng = np.random.default_rng(seed)
    bits = rng.integers(0, 256, size=(rows, (n + 7) // 8), dtype=np.uint8)
    if n % 8:  # the pad bits of a row's last byte are zero, as packbits writes them
        bits[:, -1] &= np.uint8((1 << (n % 8)) - 1)
    return bits


@pytest.mark.parametrize("rows,n", [(0, 5), (1, 1), (3, 7), (5, 8), (7, 13), (64, 64), (33, 1001), (4, 50000)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bool, torch.uint8])
def test_unpack_and_pack_match_numpy(rows, n, dtype):
    bits = _random_bits(rows, n, rows * 7 + n)
    dev = PackedSpikes(torch.from_numpy(bits).cuda(), n, dtype)
    x = dev.unpack()
    assert x.dtype == dtype and x.shape == (rows, n)
    ref = np.unpackbits(bits, axis=-1, count=n, bitorder="little")
    assert np.array_equal(x.cpu().to(torch.uint8).numpy(), ref)
    back = pack_spikes(x)
    assert torch.equal(back.bits.cpu(), torch.from_numpy(bits))


@pytest.mark.parametrize("kind,dtype,size", [(0, torch.float32, 4), (1, torch.uint8, 1)])
def test_unaligned_buffers_take_the_scalar_path(kind, dtype, size):
    """Spike buffers that start off the vector boundary (one element in) give the same
    bits and spikes."""
    rows, n = 9, 24  # rows of a multiple of 8: the vector path, were the base aligned
    bits = _random_bits(rows, n, 5)
    dbits = torch.from_numpy(bits).cuda()
    buf = torch.zeros(rows * n + 1, dtype=dtype, device="cuda")
    lib = _lib.lib()
    stream = C.c_void_p(_lib.stream_of(torch.device("cuda")))
    a = _SpikeBits(rows, n, kind, dbits.data_ptr(), buf.data_ptr() + size, None)
    _lib.check(lib.wt_unpack_spikes(C.byref(a), stream), "wt_unpack_spikes")
    ref = np.unpackbits(bits, axis=-1, count=n, bitorder="little").reshape(-1)
    assert np.array_equal(buf[1:].cpu().to(torch.uint8).numpy(), ref)
    assert int(buf[0]) == 0
    out = torch.zeros_like(dbits)
    a = _SpikeBits(rows, n, kind, out.data_ptr(), buf.data_ptr() + size, None)
    _lib.check(lib.wt_pack_spikes(C.byref(a), stream), "wt_pack_spikes")
    assert torch.equal(out, dbits)


def test_counts_are_refused_on_the_device():
    x = torch.zeros((3, 40), device="cuda")
    x[1, 17] = 2.0
    with pytest.raises(ValueError, match="counts"):
        pack_spikes(x)
    p = pack_spikes(x, check=False)
    assert float(p.unpack(torch.float32)[1, 17]) == 1.0


def test_bad_arguments_are_rejected():
    lib = _lib.lib()
    a = _SpikeBits(4, 10, 7, None, None, None)
    assert lib.wt_unpack_spikes(C.byref(a), None) == _lib.ERR_ARGS
    a = _SpikeBits(4, 10, 0, None, None, None)
    assert lib.wt_pack_spikes(C.byref(a), None) == _lib.ERR_ARGS


def test_round_trip_at_the_c5_input_size():
    """C5's input of one simulation (4 trials x 5,000 steps x 50,000 columns, 1e9
    spikes): bits -> float spikes -> bits is the identity, and the spike count is the
    bits' population count."""
    B, T, n = 4, 5000, 50000
    gen = torch.Generator(device="cuda").manual_seed(11)
    bits = torch.randint(0, 256, (B, T, n // 8), generator=gen, device="cuda", dtype=torch.int32).to(torch.uint8)
    x = PackedSpikes(bits, n, torch.float32).unpack()
    assert x.shape == (B, T, n)
    popcount = int(sum(((bits.int() >> k) & 1).sum() for k in range(8)))
    assert int(x.sum(dtype=torch.float64)) == popcount
    back = pack_spikes(x)
    assert torch.equal(back.bits, bits)


def test_prefetcher_over_packed_batches():
    """Packed pinned batches reach the device as the spikes they hold; the unpacking runs
    on the side stream, ordered before the compute stream's use."""
    gen = torch.Generator().manual_seed(3)
    originals, batches = [], []
    for _ in range(4):
        x = (torch.rand((8, 100, 333), generator=gen) < 0.05).float()
        originals.append(x)
        batches.append(SpikeData(pack_spikes(x).pin_memory(), None))
    got = list(Prefetcher(iter(batches), "cuda"))
    assert len(got) == 4
    for x, d in zip(originals, got):
        assert d["input_spikes"].dtype == torch.float32 and d["input_spikes"].is_cuda
        assert torch.equal(d["input_spikes"].cpu(), x)
        assert d["target_rate"] is None


def test_stager_packs_spikes_before_the_copy():
    gen = torch.Generator(device="cuda").manual_seed(4)
    out = torch.rand((4, 200, 1000), generator=gen, device="cuda") < 0.02
    v = torch.randn((4, 1000), generator=gen, device="cuda")
    rates = (torch.rand((4, 200, 1000), generator=gen, device="cuda") < 0.1).float()
    with Stager(spike_fields=("rates",)) as st:
        for _ in range(2):  # the buffers are reused for the second chunk
            chunk = st.stage({"output_spikes": out, "v": v, "rates": rates})
            packed = chunk.packed()
            assert isinstance(packed["output_spikes"], PackedSpikes)
            assert packed["output_spikes"].nbytes == out.numel() // 8
            arrays = chunk.arrays()
            chunk.set_result(None)
            assert np.array_equal(arrays["output_spikes"], out.cpu().numpy())
            assert np.array_equal(arrays["v"], v.cpu().numpy())
            assert np.array_equal(arrays["rates"], rates.cpu().numpy())
