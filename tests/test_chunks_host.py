"""The runners' data path on the host (no GPU): the bit format of ``PackedSpikes`` against
numpy's ``packbits(..., bitorder="little")``, and ``to_device`` / ``Prefetcher`` /
``Stager`` with the reference's batch layout (``snn_runners/chunks.py:19-70``,
``inference_runner.py:111-150``), on the CPU."""

from collections import namedtuple

import numpy as np
import pytest
import torch

from wiretorch_b200.chunks import PackedSpikes, Prefetcher, Stager, pack_spikes, to_device

SpikeData = namedtuple("SpikeData", ["input_spikes", "target_spikes"])


@pytest.mark.parametrize("n", [1, 7, 8, 9, 13, 64, 101])
@pytest.mark.parametrize("dtype", [torch.bool, torch.uint8, torch.float32])
def test_host_round_trip_and_bit_order(n, dtype):
    gen = torch.Generator().manual_seed(n)
    x = (torch.rand((3, 5, n), generator=gen) < 0.3).to(dtype)
    p = pack_spikes(x)
    assert p.bits.shape == (3, 5, (n + 7) // 8) and p.shape == x.shape and p.dtype == dtype
    ref = np.packbits(x.numpy() != 0, axis=-1, bitorder="little")
    assert np.array_equal(p.bits.numpy(), ref)
    # spike i of a row is bit i % 8 of byte i / 8
    row = x.reshape(-1, n)[0]
    if row.any():
        i = int(torch.nonzero(row).flatten()[0])
        assert (p.bits.reshape(-1, (n + 7) // 8)[0, i // 8] >> (i % 8)) & 1 == 1
    assert torch.equal(p.unpack(), x)
    assert torch.equal(p.unpack(torch.float32), x.float())


def test_counts_are_refused():
    x = torch.tensor([[0.0, 1.0, 2.0]])
    with pytest.raises(ValueError, match="counts"):
        pack_spikes(x)
    assert torch.equal(pack_spikes(x, check=False).unpack(torch.float32), torch.tensor([[0.0, 1.0, 1.0]]))


def test_empty_and_shape_checks():
    p = pack_spikes(torch.zeros((0, 10), dtype=torch.bool))
    assert p.bits.shape == (0, 2) and p.unpack().shape == (0, 10)
    with pytest.raises(ValueError):
        PackedSpikes(torch.zeros((2, 3), dtype=torch.uint8), 10)


def test_to_device_and_prefetcher_on_the_cpu():
    gen = torch.Generator().manual_seed(0)
    batches = []
    for _ in range(3):
        x = torch.rand((2, 4, 20), generator=gen) < 0.2
        y = torch.rand((2, 4, 6), generator=gen) < 0.5
        batches.append(SpikeData(pack_spikes(x), y))
    got = list(Prefetcher(iter(batches), "cpu"))
    assert len(got) == 3
    for b, d in zip(batches, got):
        assert torch.equal(d["input_spikes"], b.input_spikes.unpack())
        assert torch.equal(d["target_spikes"], b.target_spikes)
        assert d["target_rate"] is None
    d = to_device(batches[0], "cpu")
    assert d["input_spikes"].dtype == torch.bool


def test_stager_on_host_tensors():
    rec = {"output_spikes": torch.tensor([[True, False, True]]), "v": torch.tensor([1.0, 2.0])}
    with Stager() as st:
        chunk = st.stage(rec)
        arrays = chunk.arrays()
        chunk.set_result(None)
    assert np.array_equal(arrays["output_spikes"], rec["output_spikes"].numpy())
    assert np.array_equal(arrays["v"], rec["v"].numpy())
