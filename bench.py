#!/usr/bin/env python
"""Benchmark of the conductance-LIF simulation hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

For N > 1 run one process per GPU (``torch.distributed.run``); ranks talk over NCCL.

Workload (``--config c2``, the default): BASELINE configuration 2 — 20,000 conductance
LIF neurons in 40 cell types, learnt per-type-pair scales, batch 64 per GPU, T=500 steps
of 0.1 ms, Poisson input. One step is one training step: the forward simulation through
the engine (``wiretorch_b200.engine.simulate``), the van Rossum rate loss (20 ms-filtered
output against filtered target rates), backpropagation through time to the 41x40 scales,
the gradients' all-reduce across ranks and an SGD update (gradient norm clipped at 1). Every rank simulates its own 64
trials (trial-batch sharding, weak scaling). Inputs are larger than L2.

``value``: neuron-steps per second of the whole job (trials x neurons x time steps of all
ranks / the slowest rank's device time). ``synaptic_events_per_s``: edges traversed by
recurrent spikes per second (counted on the device over one extra, untimed step and
multiplied by the steps timed), input events separately.
``roofline``: the dominant kernel's algorithmic bytes per launch / its CUDA-event
duration against the measured HBM copy bandwidth. ``e2e``: the same step fed from pinned
host memory (spike input as bytes, target rates), with the loss and gradient read back;
each step's input is copied on a second stream while the previous step computes.
``cpu_baseline``: the oracle (the C restatement of the reference's time loop) on a
bounded sample of the same network on the host cores. ``--impl reference`` times that
CPU implementation alone.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

DT = 0.1  # ms


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c2", choices=["c2", "c1", "c3", "c4", "c5"])
    ap.add_argument("--chunk", type=int, default=None,
                    help="c3 / c4 / c5: steps per engine call, the state carried over (default 250 / 1000 / 1000)")
    ap.add_argument("--partition", action="store_true",
                    help="c2 / c4 / c5 forward: the network's neurons partitioned over the ranks (strong scaling)")
    ap.add_argument("--recurrent-gradients", action="store_true",
                    help="c2: gradients through the recurrent spikes (Drive.recurrent_gradients)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=None, help="trials per GPU (default: the config's)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    return ap.parse_args()


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))  # fmt: skip
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def sum_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t)
    return float(t)


class Clocks:
    """nvidia-smi samples of this GPU's clocks and throttle reasons while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")  # fmt: skip

    def __init__(self, index):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        ident = str(self.index)
        try:  # the GPU's UUID: nvidia-smi does not see CUDA_VISIBLE_DEVICES
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={ident}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)  # fmt: skip
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        self.file.flush()
        rows = []
        with open(self.file.name) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        max_sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(max_sm) if max_sm else None,
                "reasons": reasons, "samples": len(rows)}  # fmt: skip


def measured_peak():
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------------------
# The workload
# ---------------------------------------------------------------------------------------


def build(args, rank, device):
    from wiretorch_b200 import configs, engine

    if args.config == "c2":
        cfg = configs.c2(B=args.batch or 64, T=500, seed=0, device=device)
        engine.POOL_SYNAPSES = True  # 41 synapse types with 2 distinct dynamics
        cfg.drive.recurrent_gradients = args.recurrent_gradients
    elif args.config in ("c3", "c4", "c5"):
        if args.config == "c3":
            cfg = configs.c3(B=args.batch or 256, T=2000, seed=0, device=device)
        elif args.config == "c4":
            cfg = configs.c4(B=args.batch or 32, T=10000, seed=0, device=device)
            engine.POOL_SYNAPSES = True
        else:
            cfg = configs.c5(B=args.batch or 4, T=5000, seed=0, device=device)
            engine.POOL_SYNAPSES = True  # the excitatory and the input AMPA share dynamics
        args.chunk = args.chunk or (250 if args.config == "c3" else 1000)
        cfg.extra["chunk"] = args.chunk
        return cfg, cfg.inputs(T=args.chunk, seed=1 + rank)  # one chunk of input, reused
    else:
        cfg = configs.c1(B=args.batch or 8, T=1000, seed=0, device=device)
    x = cfg.inputs(seed=1 + rank)
    return cfg, x


def make_step(cfg, world, train: bool):
    """``step(x, target) -> loss`` (or the spike count for a forward-only config)."""
    from wiretorch_b200 import configs, engine, filtering

    v0, g0, kw0 = cfg.state()
    if cfg.name in ("c3", "c4", "c5"):
        def forward_chunks(x, target=None):
            """The T steps as engine calls of x.shape[1] steps, the state carried over."""
            v, g, kw = v0, g0, kw0
            with torch.no_grad():
                for _ in range(cfg.T // x.shape[1]):
                    run = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
                    v, g, kw = run.v, run.syn, cfg.carried(run)
            return v.sum()

        return forward_chunks, None
    if not train:
        def forward(x, target=None):
            with torch.no_grad():
                run = engine.simulate(v0, g0, x, cfg.drive, cfg.p, **kw0)
            return run.output.sum()

        return forward, None
    log_sf = torch.zeros(cfg.extra["log_sf_shape"], device=x_device(cfg), requires_grad=True)
    loss_fn = filtering.VanRossumRateLoss(DT, 20.0, DT, cfg.T, device=x_device(cfg))
    lr = 1e-3

    def step(x, target):
        loss_fn.reset_state()
        cfg.drive.scale = configs.scale_from_log_sf(cfg, log_sf)
        run = engine.simulate(v0, g0, x, cfg.drive, cfg.p, **kw0)
        loss = loss_fn(target, output_spikes=run.output)
        log_sf.grad = None
        loss.backward()
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(log_sf.grad)
        with torch.no_grad():  # SGD with the gradient's norm clipped at 1 (no host read)
            grad = log_sf.grad
            log_sf.sub_(lr * grad * torch.clamp(1.0 / (grad.norm() + 1e-12), max=1.0))
        return loss

    return step, log_sf


def x_device(cfg):
    return cfg.drive.scale.device


def target_of(cfg):
    """Expected spikes per step of the target rates, constant in time: (B, T, N) view."""
    r = cfg.extra["target_rates"] * DT / 1000.0
    return r[:, None, :].expand(cfg.B, cfg.T, cfg.N)


def forward_bytes(cfg, plan, T, spikes_bits_saved: bool, fired_sources_edges: float):
    """Algorithmic bytes of one forward launch: per neuron-step the state read and written
    (v 8, conductances 16 per channel, refractory counter 2, adaptation 8), the spike bit,
    and with saving for the backward pass v 4, summed conductances 4 per channel and the
    spike and refractory bits; the input read (4 per input-step); 8 bytes (target,
    weight) per edge of every source that fired in at least one trial of a step; and the
    gating state (release probabilities, resources) read and written, 8 per column-step."""
    S = plan.ch.Sp
    per = 8 + 16 * S + 2 + 1 / 8
    if cfg.p.adapt is not None:
        per += 8
    if spikes_bits_saved:
        per += 4 + 4 * S + 2 / 8
    gating = cfg.B * T * cfg.extra["gating"].shape[1] * 8 if "gating" in cfg.extra else 0
    return cfg.B * T * cfg.N * per + cfg.B * T * cfg.n_in * 4 + fired_sources_edges * 8 + gating


def factorised_bytes(cfg, T):
    """Algorithmic bytes of one factorised launch of T steps: per neuron-step the state
    read and written (v 8, conductances 16 per channel, refractory counter 2), the spike
    bit and the input read (4); per step the factors U and V (N x 64 bf16 each)."""
    C = 2
    per = 8 + 16 * C + 2 + 1 / 8 + 4
    return cfg.B * T * cfg.N * per + T * 2 * cfg.N * 64 * 2


def fired_edges_once(cfg, spikes, x):
    """Sum over steps of the out-degrees of the sources (neurons, inputs) that fired in at
    least one trial: the edges the step must read at least once."""
    deg = cfg.out_degree.double()
    any_rec = (spikes > 0).any(0).double()  # (T, N)
    e = float((any_rec * deg[: cfg.N]).sum())
    any_in = (x != 0).any(0).double()
    e += float((any_in * deg[cfg.N :]).sum())
    return e


def cpu_baseline(cfg, seconds_target=15.0, threads=None):
    """The oracle on the host cores: a sample of trials and steps of the same network.
    Returns (neuron-steps/s, cores, sample description)."""
    from oracle import oracle

    threads = threads or os.cpu_count() or 1
    oracle.set_threads(threads)
    cpu = _to_cpu(cfg)
    B = min(cfg.B, threads)
    T = 20
    net = oracle.Network(cpu.drive, cpu.p, B, cfg.n_in)
    x = cfg.inputs(T=T, seed=99)[:B].cpu()
    v, g, kw = cpu.state()
    v, g = v[:B], g[:B]
    kw = {k: t[:B] for k, t in kw.items()}
    t0 = time.perf_counter()
    net.simulate(x, v, g, **kw, track=False)
    el = time.perf_counter() - t0
    # grow the sample towards the target duration (bounded)
    T2 = int(min(cfg.T, max(T, T * seconds_target / max(el, 1e-3))))
    x = cfg.inputs(T=T2, seed=99)[:B].cpu()
    t0 = time.perf_counter()
    net.simulate(x, v, g, **kw, track=False)
    el = time.perf_counter() - t0
    rate = B * T2 * cfg.N / el
    return rate, threads, f"{B} trials x {T2} steps of the {cfg.name} network, forward only ({el:.1f} s)"


def _to_cpu(cfg):
    import copy

    from wiretorch_b200.types import SparseRows

    c = copy.copy(cfg)
    d = copy.copy(cfg.drive)

    def mv(W):
        if isinstance(W, SparseRows):
            return SparseRows(W.row_ptr.cpu(), W.cols.cpu(), W.values.detach().cpu(), W.n_targets)
        return W.detach().cpu()

    d.recurrent = [(r.cpu(), mv(W)) for r, W in cfg.drive.recurrent]
    d.feedforward = [(r.cpu(), mv(W)) for r, W in cfg.drive.feedforward]
    d.made, d.scale = cfg.drive.made.cpu(), cfg.drive.scale.detach().cpu()
    p = copy.copy(cfg.p)
    for name in vars(p):
        val = getattr(p, name)
        if isinstance(val, torch.Tensor):
            setattr(p, name, val.detach().cpu())
    c.drive, c.p = d, p
    c.extra = {k: (t.cpu() if isinstance(t, torch.Tensor) else t) for k, t in cfg.extra.items()}
    c.out_degree = cfg.out_degree.cpu()
    c.rates_in = cfg.rates_in.cpu()
    return c


def run_reference(args, rank, world):
    """``--impl reference``: the CPU implementation (the oracle port of the reference's
    time loop) on the host cores; rank 0 only."""
    if rank != 0:
        return
    device = "cuda" if torch.cuda.is_available() else "cpu"
    cfg, _ = build(args, 0, device)
    for _ in range(max(args.warmup, 0)):
        pass
    rates = []
    for _ in range(max(args.steps, 1)):
        rate, cores, sample = cpu_baseline(cfg, seconds_target=max(5.0, 60.0 / max(args.steps, 1)))
        rates.append(rate)
    value = statistics.median(rates)
    line = {
        "impl": "reference", "metric": "neuron-steps/s", "value": value, "unit": "neuron-steps/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_of(args, cfg, world=1),
        "cpu_baseline": {"value": value, "unit": "neuron-steps/s", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "neuron-steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }  # fmt: skip
    print(json.dumps(line))


def config_of(args, cfg, world):
    c = {
        "workload": f"{cfg.name}: {cfg.N} neurons, {cfg.B} trials/GPU, {cfg.T} steps of 0.1 ms"
                    + (", forward + BPTT + van Rossum rate loss + SGD" if args.config == "c2" else ", forward")
                    + (f", factorised W = U V^T rank {cfg.extra.get('rank')}" if args.config == "c3" else "")
                    + (f", {cfg.extra.get('edges')} edges" if args.config in ("c4", "c5") else "")
                    + (f", {args.chunk} steps per call" if args.config in ("c3", "c4", "c5") else "")
                    + (", gradients through the recurrent spikes" if getattr(args, "recurrent_gradients", False) else ""),
        "global_batch": cfg.B * world, "seq_len": cfg.T, "parallelism": f"trial-batch x{world}",
        "l2": "inputs larger than L2 (spike input and state streams exceed 126 MB per step)",
    }  # fmt: skip
    return c


def main_partition(args, rank, world, local):
    """``--partition``: one network (c2, c4 or c5, forward only) with its neurons partitioned
    over the ranks, each step's spikes exchanged by peer stores inside the forward kernel.
    Total work is fixed as ranks are added (strong scaling)."""
    from wiretorch_b200 import _lib, partition

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg, x = build(args, 0, device)  # every rank: the same network and input
    part = partition.Partition(cfg.N, cfg.B)
    chunked = cfg.name in ("c4", "c5")

    def step():
        v, g, kw = cfg.state()
        with torch.no_grad():
            for _ in range(cfg.T // x.shape[1] if chunked else 1):
                run = partition.simulate(part, v, g, x, cfg.drive, cfg.p, **kw)
                v, g, kw = run.v, run.syn, cfg.carried(run)
        return run

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    _lib.TIMER = {}
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        start.record()
        for _ in range(args.steps):
            run = step()
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    timer, _lib.TIMER = _lib.TIMER, None
    elapsed_max = max_over_ranks(start.elapsed_time(end) / 1000.0, world)
    kernel = {k: sum(a.elapsed_time(b) for a, b in v) / len(v) for k, v in timer.items()}
    neuron_steps = cfg.B * cfg.N * cfg.T * args.steps  # the one network, whatever the ranks
    spikes = sum_over_ranks(float(run.output.sum()), world)
    if rank == 0:
        print(json.dumps({
            "metric": "neuron-steps/s", "value": neuron_steps / elapsed_max, "unit": "neuron-steps/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": elapsed_max / args.steps * 1000.0, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Poisson input, seeded connectome)",
            "config": {**config_of(args, cfg, world), "parallelism": f"neuron-partition x{world}",
                       "global_batch": cfg.B,
                       "workload": f"{cfg.name}: {cfg.N} neurons ({world} blocks), {cfg.B} trials, {cfg.T} steps "
                                   f"of 0.1 ms, forward, spikes exchanged each step by peer stores"},
            "mean_rate_hz": spikes / (cfg.B * cfg.N * x.shape[1]) / (DT / 1000.0),
            "kernel_ms": kernel, "clocks": clocks.summary(),
        }))  # fmt: skip
    barrier(world)
    part.close()


def main():
    args = parse()
    rank, world, local = dist_setup(args)
    if args.partition and args.impl != "reference":
        main_partition(args, rank, world, local)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    from wiretorch_b200 import _lib, engine

    # the forward's device error word is read behind the launches (no host
    # synchronisation per step); every run's word is checked before the results print
    engine.DEFER_CHECKS = True
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg, x = build(args, rank, device)
    train = args.config == "c2"
    step, log_sf = make_step(cfg, world, train)
    target = target_of(cfg) if train else None
    for _ in range(max(args.warmup, 3)):
        step(x, target)
    torch.cuda.synchronize()
    factorised = cfg.name == "c3"
    plan = None if factorised else engine.get_plan(cfg.drive, cfg.p, cfg.B, cfg.n_in, device)

    # ---- synaptic events: counted on the device over one untimed step (the counter's
    # atomics stay out of the timed region) ----
    edges = torch.zeros(2, dtype=torch.int64, device=device)
    if factorised:  # every spike reaches every neuron through W = U V^T
        with torch.no_grad():
            v0_, g0_, kw0_ = cfg.state()
            r0 = engine.simulate(v0_, g0_, x, cfg.drive, cfg.p, **kw0_)
        per_chunk = float(r0.output.sum()) * cfg.N, float((x != 0).sum())
        edges[0], edges[1] = int(per_chunk[0] * cfg.T / x.shape[1]), int(per_chunk[1] * cfg.T / x.shape[1])
    else:
        engine.EDGE_COUNTER = edges
        step(x, target)
        torch.cuda.synchronize()
        engine.EDGE_COUNTER = None

    # ---- timed region: K steps, device time, max over ranks ----
    _lib.TIMER = {}
    launches0 = _lib.LAUNCHES
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        start.record()
        for _ in range(args.steps):
            step(x, target)
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    launches = _lib.LAUNCHES - launches0
    timer, _lib.TIMER = _lib.TIMER, None
    elapsed = start.elapsed_time(end) / 1000.0
    elapsed_max = max_over_ranks(elapsed, world)
    K = args.steps
    neuron_steps = cfg.B * cfg.N * cfg.T * K * world
    rec_edges, in_edges = float(edges[0]) * K, float(edges[1]) * K  # one step counted
    rec_edges_all = sum_over_ranks(rec_edges, world)
    in_edges_all = sum_over_ranks(in_edges, world)
    clock = clocks.summary()

    # ---- the dominant kernel's roofline ----
    kernel_ms = {k: sum(s.elapsed_time(e) for s, e in v) / len(v) for k, v in timer.items()}
    kernel_total = {k: sum(s.elapsed_time(e) for s, e in v) for k, v in timer.items()}
    dominant = max(kernel_total, key=kernel_total.get)
    with torch.no_grad():
        from wiretorch_b200 import engine as eng

        v0, g0, kw0 = cfg.state()
        run = eng.simulate(v0, g0, x, cfg.drive, cfg.p, **kw0)
    if factorised:
        kname = "wt_lowrank_forward"
        fwd_bytes = factorised_bytes(cfg, x.shape[1])
        kdesc = "wt_lowrank_forward (persistent factorised step kernel, tcgen05 product per step)"
    else:
        kname = "wt_forward"
        fwd_bytes = forward_bytes(cfg, plan, x.shape[1], train, fired_edges_once(cfg, run.output, x))
        kdesc = "wt_forward (persistent forward step kernel)"
    peak, peak_kind = measured_peak()
    fwd_s = kernel_ms[kname] / 1000.0
    roofline = {
        "kernel": kdesc,
        "bound": "hbm", "achieved": fwd_bytes / fwd_s / 1e9, "peak": peak, "unit": "GB/s",
        "frac": fwd_bytes / fwd_s / 1e9 / peak, "peak_kind": peak_kind,
        "traffic": None, "algorithmic_bytes_per_launch": fwd_bytes,
        "launch_ms": kernel_ms[kname],
    }  # fmt: skip
    prof = ROOT / "profiles" / f"traffic_{args.config}.json"
    if prof.exists():
        info = json.loads(prof.read_text())
        per_ns = info.get("dram_bytes_per_neuron_step", {}).get(kname)
        if per_ns:  # measured DRAM bytes per neuron-step, scaled to this launch
            steps_per_launch = x.shape[1]
            roofline["traffic"] = per_ns * cfg.B * cfg.N * steps_per_launch
            roofline["traffic_source"] = str(prof.relative_to(ROOT))

    # ---- end to end from host buffers ----
    e2e = None
    if not args.no_e2e:
        x_host = (x.cpu() != 0).to(torch.uint8).pin_memory()
        tgt_host = cfg.extra["target_rates"].cpu().pin_memory() if train else None
        out_host = torch.empty(1 + (log_sf.numel() if train else 0), pin_memory=True)
        h2d = x_host.numel() + (tgt_host.numel() * 4 if train else 0)
        d2h = out_host.numel() * 4

        # Each step's input crosses from pinned host memory on a copy stream while the
        # previous step computes (the copy of step k + 1 overlaps step k); every copy lies
        # inside the timed region, between its two events.
        copy_stream = torch.cuda.Stream(device)
        main = torch.cuda.current_stream(device)

        def fetch(after):
            copy_stream.wait_event(after)
            with torch.cuda.stream(copy_stream):
                xd = x_host.to(device, non_blocking=True).float()
                r = tgt_host.to(device, non_blocking=True) * (DT / 1000.0) if train else None
                ready = torch.cuda.Event()
                ready.record(copy_stream)
            return xd, r, ready

        def e2e_step(inputs):
            xd, r, ready = inputs
            main.wait_event(ready)
            xd.record_stream(main)
            if train:
                r.record_stream(main)
                loss = step(xd, r[:, None, :].expand(cfg.B, cfg.T, cfg.N))
                res = torch.cat([loss.detach().reshape(1), log_sf.detach().reshape(-1)])
            else:
                res = step(xd).reshape(1).float()
            out_host.copy_(res, non_blocking=True)

        first = torch.cuda.Event()
        first.record(main)
        e2e_step(fetch(first))
        torch.cuda.synchronize()
        barrier(world)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        pending = fetch(s2)
        for k in range(K):
            inputs = pending
            if k + 1 < K:
                pending = fetch(inputs[2])  # the next step's input, behind this one's copy
            e2e_step(inputs)
        e2.record()
        torch.cuda.synchronize()
        e2e_el = max_over_ranks(s2.elapsed_time(e2) / 1000.0, world)
        e2e = {"value": neuron_steps / e2e_el, "unit": "neuron-steps/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": e2e_el / K * 1000.0}  # fmt: skip

    engine.check_errors()  # every deferred device error check of the runs above
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and not factorised:
        rate, cores, sample = cpu_baseline(cfg)
        cpu = {"value": rate, "unit": "neuron-steps/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": "neuron-steps/s", "value": neuron_steps / elapsed_max, "unit": "neuron-steps/s",
            "n_gpus": world, "steps": K, "warmup": max(args.warmup, 3),
            "ms_per_step": elapsed_max / K * 1000.0, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Poisson input, seeded connectome)",
            "config": config_of(args, cfg, world),
            "synaptic_events_per_s": rec_edges_all / elapsed_max,
            "input_events_per_s": in_edges_all / elapsed_max,
            "mean_rate_hz": float(run.output.mean()) / (DT / 1000.0),
            "roofline": roofline, "kernel_ms": kernel_ms, "gpu_launches": launches,
            "clocks": clock, "e2e": e2e, "cpu_baseline": cpu,
        }  # fmt: skip
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
