"""A neuron-partitioned run (two ranks, one GPU each: spike words exchanged by peer
stores inside the forward kernel) against the same network run on one GPU: the spikes
and the state (the gating state of a gated network too) must be identical (the
fixed-point synaptic sums do not depend on which rank adds what). Needs two GPUs;
skipped otherwise."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

NET = dict(N=3000, n_in=200, B=4, T=150, seed=7, tau_ref=2.0)


def _network(kind, device):
    """``(drive, p, x, v, g, kw, N, B)`` of the test network: a random one, or the C5
    model (gated pathways: short-term depression, replicated on every rank; NMDA) small."""
    if kind == "random":
        from wiretorch_b200.testing import random_network

        drive, p, x, v, g, kw = random_network(**NET, device=device)
        return drive, p, x, v, g, {"refractory": kw["refractory"]}, NET["N"], NET["B"]
    from wiretorch_b200 import configs

    cfg = configs.c5(B=3, T=300, device=device, N=4000, mean_degree=400.0, lam=0.05 * 250 ** (1 / 3),
                     w_e=3.0, w_in=30.0)  # fmt: skip
    v, g, kw = cfg.state()
    return cfg.drive, cfg.p, cfg.inputs(seed=3), v, g, kw, cfg.N, cfg.B


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, kind):
    from wiretorch_b200 import partition

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    part = None
    try:
        drive, p, x, v, g, kw, N, B = _network(kind, f"cuda:{rank}")
        part = partition.Partition(N, B)
        run = partition.simulate(part, v, g, x, drive, p, **kw)
        again = partition.simulate(part, v, g, x, drive, p, **kw)  # a new epoch
        torch.cuda.synchronize()
        same = bool(torch.equal(again.output, run.output))
        torch.save({"spikes": run.output.cpu(), "v": run.v.cpu(), "counter": run.refractory.cpu(),
                    "gating": None if run.gating is None else run.gating.cpu(),
                    "n0": part.n0, "n1": part.n1, "same": same}, f"{out_dir}/rank{rank}.pt")  # fmt: skip
        dist.barrier()
    finally:
        if part is not None:
            part.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["random", "c5"])
def test_partitioned_run_matches_one_gpu(tmp_path, kind):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from wiretorch_b200 import engine

    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path), kind), nprocs=2, start_method="spawn")
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(2)]
    assert all(q["same"] for q in parts)
    assert parts[0]["n1"] == parts[1]["n0"]
    drive, p, x, v, g, kw, N, B = _network(kind, "cuda:0")
    ref = engine.simulate(v, g, x, drive, p, **kw)
    spikes = torch.cat([q["spikes"] for q in parts], dim=2)
    assert float(spikes.sum()) > 100
    assert torch.equal(spikes, ref.output.cpu())
    assert torch.equal(torch.cat([q["v"] for q in parts], 1), ref.v.cpu())
    assert torch.equal(torch.cat([q["counter"] for q in parts], 1), ref.refractory.cpu())
    if ref.gating is not None:  # every rank holds the whole gating state, stepped alike
        for q in parts:
            assert torch.equal(q["gating"], ref.gating.cpu())
