"""The neuron partition's host side on the CPU: the blocks, and each rank's local network
(its targets' edges, sources kept global), checked in two gloo processes that together
must hold every edge of the network exactly once."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wiretorch_b200 import partition
from wiretorch_b200.testing import random_network


def test_blocks_are_whole_words_covering_the_neurons():
    for N, P in [(20000, 3), (100, 2), (1000, 8), (33, 2)]:
        b = partition.blocks(N, P)
        assert b[0][0] == 0 and b[-1][1] == N
        assert all(lo % 32 == 0 and lo < hi for lo, hi in b)
        assert all(b[r][1] == b[r + 1][0] for r in range(P - 1))
    with pytest.raises(ValueError):
        partition.blocks(40, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        drive, p, *_ = random_network(N=500, n_in=60, B=2, T=10, seed=3)
        n0, n1 = partition.blocks(500, world)[rank]
        d_loc, p_loc = partition.local_network(drive, p, n0, n1)
        # every local edge lands on this rank's block and matches the full weights
        total = torch.zeros(1, dtype=torch.int64)
        for (rows, W), (_, W_loc) in zip(drive.recurrent + drive.feedforward, d_loc.recurrent + d_loc.feedforward):
            if hasattr(W_loc, "row_ptr"):  # SparseRows
                dense = torch.zeros(W_loc.shape)
                counts = torch.diff(W_loc.row_ptr)
                r = torch.repeat_interleave(torch.arange(counts.numel()), counts)
                dense[r, W_loc.cols.long()] = W_loc.values
            else:
                dense = W_loc
            assert torch.equal(dense, W.detach()[:, n0:n1])
            total += int((dense != 0).sum())
        assert p_loc.theta.shape[0] == n1 - n0 and d_loc.scale.shape[1] == n1 - n0
        dist.all_reduce(total)
        full = sum(int((W != 0).sum()) for _, W in drive.recurrent + drive.feedforward)
        result[rank] = int(total) == full
    finally:
        dist.destroy_process_group()


def test_two_ranks_hold_every_edge_once():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), result), nprocs=world, start_method="spawn")
    assert dict(result) == {0: True, 1: True}


def test_sparse_rows_restriction():
    from wiretorch_b200 import configs

    cfg = configs.c1(B=1, T=5, device="cpu")
    W = cfg.drive.recurrent[0][1]
    n0, n1 = 320, 704
    W_loc = partition._restrict(W, n0, n1)
    dense = torch.zeros(W.shape)
    counts = torch.diff(W.row_ptr)
    r = torch.repeat_interleave(torch.arange(counts.numel()), counts)
    dense[r, W.cols.long()] = W.values
    loc = torch.zeros(W_loc.shape)
    counts = torch.diff(W_loc.row_ptr)
    r = torch.repeat_interleave(torch.arange(counts.numel()), counts)
    loc[r, W_loc.cols.long()] = W_loc.values
    assert torch.equal(loc, dense[:, n0:n1])


def _gating_rank_main(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from types import SimpleNamespace

        from wiretorch_b200 import configs
        from wiretorch_b200 import plan as P

        cfg = configs.c5(B=2, T=4, device="cpu", N=2000, mean_degree=100.0, lam=0.2)
        n0, n1 = partition.blocks(cfg.N, world)[rank]
        d_loc, p_loc = partition.local_network(cfg.drive, cfg.p, n0, n1)
        plan = P.build(d_loc, p_loc, cfg.B, cfg.n_in, "cpu", n_src=cfg.N)
        assert partition.owner_gates(plan)
        owner = partition.gating_owners(plan, world)
        # each depressing synapse's columns (u, then x) belong to the rank of its neuron
        cuts = [b[0] for b in partition.blocks(cfg.N, world)]
        for (rows, _), gate in zip(cfg.drive.recurrent, cfg.drive.gates):
            want = torch.tensor([sum(int(j) >= c for c in cuts[1:]) for j in rows])
            assert torch.equal(owner[gate.start : gate.start + gate.n], want)
            assert torch.equal(owner[gate.start + gate.n : gate.start + 2 * gate.n], want)
        assert int((owner >= 0).sum()) == plan.R
        # the gathered state takes every column from its owner
        truth = torch.arange(cfg.B * plan.R, dtype=torch.float32).reshape(cfg.B, plan.R)
        mine = torch.where(owner == rank, truth, torch.full_like(truth, -1.0))
        partition._gather_gating(SimpleNamespace(group=None, P=world, rank=rank), plan, mine)
        result[rank] = bool(torch.equal(mine, truth))
    finally:
        dist.destroy_process_group()


def test_owner_stepped_gating_gathered_from_the_owners():
    """Owner-stepped gates (every neuron of the C5 model owns one depressing slot): the
    column owners follow the blocks, and the gathered state is each owner's."""
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    mp.start_processes(_gating_rank_main, args=(world, _free_port(), result), nprocs=world, start_method="spawn")
    assert dict(result) == {0: True, 1: True}


def test_pushed_events_land_in_each_peers_own_layout():
    """A rank writes its pushed events and their counts into every peer's inbound area at
    that peer's offsets: with areas of different sizes (ranks with different chunk
    counts), each region and each counts slot lies inside the peer's own area."""
    from wiretorch_b200.partition import inbound_layout, push_pointers

    B, P = 4, 3
    chunks = [[10, 3, 7], [1, 50, 2], [4, 4, 100]]  # chunks[r][q]: source rank q's chunks on rank r
    layouts = [inbound_layout(chunks[r], B) for r in range(P)]
    sizes = [lay[3] + 2 * 8 * 4 for lay in layouts]
    bases = [10**9 * (r + 1) for r in range(P)]  # disjoint address ranges
    for q in range(P):
        ptr = push_pointers(q, bases, layouts)
        for r in range(P):
            lo, hi = bases[r], bases[r] + sizes[r]
            region_end = ptr["push_ev"][r] + (ptr["push_half"][r] + ptr["push_cap"][r]) * 16
            assert lo <= ptr["push_ev"][r] and region_end <= bases[r] + layouts[r][3]  # both parities
            assert ptr["push_cap"][r] == B * chunks[r][q]
            assert lo <= ptr["push_count"][r] and ptr["push_count"][r] + 16 * 4 <= hi
            assert ptr["push_count"][r] == bases[r] + layouts[r][3]
        assert ptr["pull_count"] == bases[q] + layouts[q][3]
