"""Where a forward step's time goes: the per-warp phase stamps of the forward kernel
(``WtForward.phases``) over one engine call, summarised per phase.

    python tests/phase_times.py [c5|c2|c4] [--steps 100]
    python -m torch.distributed.run --nproc-per-node P tests/phase_times.py c5   # partitioned

Builds the configuration (C5 by default, pooled channels), runs 300 steps from rest
untimed, then one instrumented call of ``--steps`` steps (neuron-partitioned over the
ranks when run with several). Per rank it prints, averaged over the steps: the step's
length (start to start, the slowest warp), and for each phase the mean over warps of
its length and of its latest end relative to the step's start:

  emit    the next step's input columns emitted
  scatter the step's events scattered (the even warps, before their items)
  items   the warp's items updated and their spikes emitted
  late    the odd warps' scatter
  barrier the wait at the grid barrier
  exchange (partitioned runs) the progress wait, barrier and spike emission from the words

and the spread of the warps' ends of work within a step (median, 90th percentile, last).
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402

NAMES = ["emit", "scatter", "items", "late", "barrier", "exchange"]


def build(name):
    from wiretorch_b200 import configs

    if name == "c2":
        return configs.c2(B=64, T=500, device="cuda")
    if name == "c4":
        return configs.c4(B=32, T=10000, device="cuda")
    return configs.c5(B=4, T=5000, device="cuda")


def summary(stamps: np.ndarray) -> dict:
    """``stamps`` (T, warps, 7) ns; rows of warps that did not run are zero."""
    live = stamps[0, :, 0] > 0
    s = stamps[:, live].astype(np.float64)
    T = s.shape[0]
    start = s[:, :, 0].min(1)  # the step's start: its earliest warp
    step_len = np.diff(start).mean() / 1e3 if T > 1 else float("nan")
    out = {"warps": int(live.sum()), "step_us": step_len}
    for k, name in enumerate(NAMES):
        d = (s[:, :, k + 1] - s[:, :, k]) / 1e3
        out[name] = (d.mean(), (s[:, :, k + 1].max(1) - start).mean() / 1e3)
    # the spread of the warps' ends of work (late scatter done) within a step: median,
    # 90th percentile and last, from the step's start
    ends = (s[:, :, 4] - start[:, None]) / 1e3
    out["ends"] = tuple(np.percentile(ends, q, axis=1).mean() for q in (50, 90, 100))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("config", nargs="?", default="c5")
    ap.add_argument("--steps", type=int, default=100)
    args = ap.parse_args()
    from wiretorch_b200 import engine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    part = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        from wiretorch_b200 import partition

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    engine.POOL_SYNAPSES = True
    cfg = build(args.config)
    if world > 1:
        part = partition.Partition(cfg.N, cfg.B)
    x = cfg.inputs(T=300 + args.steps, seed=1)
    v, g, kw = cfg.state()

    def sim(v, g, x, kw):
        if part is not None:
            return partition.simulate(part, v, g, x, cfg.drive, cfg.p, **kw)
        return engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)

    with torch.no_grad():
        run = sim(v, g, x[:, :300].contiguous(), kw)
        engine.PHASE_RECORD = []
        run2 = sim(run.v, run.syn, x[:, 300:].contiguous(), cfg.carried(run))
        torch.cuda.synchronize()
    stamps = engine.PHASE_RECORD[0].cpu().numpy()
    engine.PHASE_RECORD = None
    res = summary(stamps)
    spikes = float(run2.output.sum()) / args.steps
    lines = [f"rank {rank}/{world} {args.config}: {res['warps']} warps, {res['step_us']:.1f} us per step, "
             f"{spikes:.0f} spikes per step (this rank's neurons)"]
    for name in NAMES:
        mean, end = res[name]
        lines.append(f"  {name:9s} {mean:8.2f} us per warp   latest end {end:8.2f} us into the step")
    p50, p90, last = res["ends"]
    lines.append(f"  warps' work ends (us into the step): median {p50:.2f}, 90th percentile {p90:.2f}, last {last:.2f}")
    text = "\n".join(lines)
    if part is not None:
        import torch.distributed as dist

        texts = [None] * world
        dist.all_gather_object(texts, text)
        if rank == 0:
            print("\n".join(texts))
        dist.barrier()
        part.close()
        dist.destroy_process_group()
    else:
        print(text)


if __name__ == "__main__":
    main()
