#!/usr/bin/env python
"""Benchmark of the conductance-LIF simulation hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5] [--impl ours|reference]

For N > 1 run one process per GPU (``torch.distributed.run``); ranks talk over NCCL.

Workload (``--config c5``, the default: the largest configuration): benchmark
configuration C5 — 1,000,000 conductance-LIF neurons with ~1B edges from a
distance-dependent model, AMPA + NMDA (Mg block) + GABA_A, short-term depression,
refractoriness, 4 trials, T=5,000 steps of 0.1 ms, forward, run as engine calls of 1,000
steps with the state carried. One step is one such 5,000-step simulation. At N = 1 it
runs on one GPU; at N > 1 the network's neurons are partitioned over the ranks (each
holds a block of neurons and every edge onto them) and every step's spikes cross between
the GPUs by peer stores inside the forward kernel: total work is fixed (strong scaling).

``--config c2``: configuration 2's training step — 20,000 neurons in 40 cell types,
learnt per-type-pair scales, 64 trials per GPU, T=500: forward through the engine
(``wiretorch_b200.engine.simulate``), the van Rossum rate loss (20 ms-filtered output
against filtered target rates), backpropagation through time to the 41x40 scales, the
gradients' all-reduce across ranks and an SGD update (gradient norm clipped at 1); every
rank simulates its own 64 trials (trial-batch sharding, weak scaling). ``--config c1 /
c3 / c4``: the other configurations, forward. ``--config c2c``: the current-based family
(``wiretorch_b200.current``) on configuration 2's network, forward.

``value``: neuron-steps per second of the whole job (trials x neurons x time steps of
the work all ranks did / the slowest rank's device time). ``synaptic_events_per_s``:
edges traversed by recurrent spikes per second (counted on the device over one extra,
untimed step and multiplied by the steps timed), input events separately.
``roofline``: the dominant kernel's algorithmic bytes per launch / its CUDA-event
duration against the measured HBM copy bandwidth. ``e2e``: the same step through the
public API fed from pinned host memory (the spike input as bits, unpacked on the
device by ``wiretorch_b200.chunks``, and the target rates for c2), each step's (or engine call's) input copied on a second stream while the
previous one computes, and its result (spike count, or loss and learnt parameters)
read back. ``cpu_baseline``: the oracle (the C restatement of the reference's time
loop) on a bounded sample of the same network on the host cores. ``--impl reference``
times that CPU implementation alone (and, for c1 / c2 / c2c where the reference's
package is installed under ``baseline/_ref``, the reference's own ``dynamics.simulate``
of the family).
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
    ap.add_argument("--config", default="c5", choices=["c5", "c2", "c1", "c3", "c4", "c2c"],
                    help="c2c: the current-based family on C2's network (forward)")
    ap.add_argument("--chunk", type=int, default=None,
                    help="c3 / c4 / c5: steps per engine call, the state carried over (default 250 / 1000 / 1000)")
    ap.add_argument("--partition", action="store_true",
                    help="the network's neurons partitioned over the ranks (strong scaling; "
                         "the default for c4 / c5 at N > 1)")
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
    elif args.config == "c2c":
        cfg = configs.c2_current(B=args.batch or 64, T=500, seed=0, device=device)
        engine.POOL_SYNAPSES = True  # 41 synapse types with 2 distinct (decay, sign) pairs
    else:
        cfg = configs.c1(B=args.batch or 8, T=1000, seed=0, device=device)
    x = cfg.inputs(seed=1 + rank)
    return cfg, x


def simulate_of(cfg):
    """The engine entry point of a configuration's family: ``wiretorch_b200.current`` for
    the current-based one (``c2c``), ``wiretorch_b200.engine`` otherwise."""
    from wiretorch_b200 import current, engine

    return current.simulate if cfg.name == "c2c" else engine.simulate


def plan_of(cfg, device):
    from wiretorch_b200 import current, engine

    if cfg.name == "c2c":
        return engine.get_plan(cfg.drive, current._fields(cfg.p), cfg.B, cfg.n_in, device)
    return engine.get_plan(cfg.drive, cfg.p, cfg.B, cfg.n_in, device)


def make_step(cfg, world, train: bool):
    """``step(x, target) -> result``: the loss (c2), or the final membrane state of a
    forward-only configuration (the state a caller would carry to the next run)."""
    from wiretorch_b200 import configs, engine, filtering

    v0, g0, kw0 = cfg.state()
    if cfg.name in ("c3", "c4", "c5"):
        def forward_chunks(x, target=None, fetch=None):
            """The T steps as engine calls of x.shape[1] steps, the state carried over;
            ``fetch`` (a ``Prefetcher``) gives each call's input (default: ``x`` for
            every call)."""
            v, g, kw = v0, g0, kw0
            with torch.no_grad():
                for i in range(cfg.T // x.shape[1]):
                    xi = x if fetch is None else fetch.get()
                    if fetch is not None:
                        fetch.prefetch()  # the next call's input, copied while this one runs
                    run = engine.simulate(v, g, xi, cfg.drive, cfg.p, **kw)
                    v, g, kw = run.v, run.syn, cfg.carried(run)
            return v

        return forward_chunks, None
    if not train:
        sim = simulate_of(cfg)

        def forward(x, target=None, fetch=None):
            xi = x if fetch is None else fetch.get()
            if fetch is not None:
                fetch.prefetch()
            with torch.no_grad():
                run = sim(v0, g0, xi, cfg.drive, cfg.p, **kw0)
            return run.v

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


class Prefetcher:
    """Inputs of successive engine calls copied from pinned host memory on a copy stream,
    one call ahead: ``get()`` returns the next call's device input (its copy ordered
    before the current stream's use of it) and starts the copy of the one after, so that
    it overlaps the call about to be launched."""

    def __init__(self, host_chunks, device, convert):
        self.host = host_chunks  # list of pinned host tensors, used in turn
        self.device = device
        self.convert = convert
        self.stream = torch.cuda.Stream(device)
        self.i = 0
        self.pending = None

    def _fetch(self):
        host = self.host[self.i % len(self.host)]
        self.i += 1
        with torch.cuda.stream(self.stream):  # into a fresh buffer: no wait on the compute
            dev = self.convert(host.to(self.device, non_blocking=True))
            ready = torch.cuda.Event()
            ready.record(self.stream)
        return dev, ready

    def start(self):
        self.pending = self._fetch()

    def get(self):
        dev, ready = self.pending
        main = torch.cuda.current_stream(self.device)
        main.wait_event(ready)
        dev.record_stream(main)
        self.pending = None
        return dev

    def prefetch(self):
        """Start the next copy (it runs beside the call that uses the current input)."""
        if self.pending is None:
            self.pending = self._fetch()


PACKED_NOTE = "spike input held on the host as bits (wiretorch_b200.chunks.PackedSpikes), unpacked on the device"


def packed_input(x):
    """One engine call's spike input as pinned host bits (the dataset format of
    ``wiretorch_b200.chunks``; packed once, outside the timed region) and the conversion
    the prefetcher applies on the device: ``wt_unpack_spikes`` into float32."""
    from wiretorch_b200.chunks import PackedSpikes, pack_spikes

    n = x.shape[-1]
    bits = pack_spikes(x.detach().cpu(), check=False).bits.pin_memory()
    return [bits], lambda b: PackedSpikes(b, n, torch.float32).unpack()


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
    # (the current-based family's channels have no rise component: 8 bytes each)
    per = 8 + (8 if cfg.name == "c2c" else 16) * S + 2 + 1 / 8
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
    B = cfg.B if cfg.B <= threads else threads * (cfg.B // threads)  # whole rounds of trials
    if _CPU_NET.get("cfg") is not cfg:  # the network on the host, built once per run
        cpu = _to_cpu(cfg)
        _CPU_NET.update(cfg=cfg, cpu=cpu, net=oracle.Network(cpu.drive, cpu.p, B, cfg.n_in))
    cpu, net = _CPU_NET["cpu"], _CPU_NET["net"]
    T = 20
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
    # the oracle runs a thread per trial, or with fewer trials than threads splits each
    # step's neurons over all of them
    return rate, threads, f"{B} trials x {T2} steps of the {cfg.name} network, forward only ({el:.1f} s)"


_CPU_NET: dict = {}


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
    """``--impl reference``: the CPU implementation of the path on the host cores, rank 0
    only: the oracle (the C restatement of the reference's time loop, forward only), each
    step a bounded sample of the configuration's trials and steps; for c1 / c2 / c2c also
    the reference's own ``dynamics.simulate`` when its package is installed under
    ``baseline/_ref`` (a bounded sample too; for c2 also its training step, forward +
    BPTT + loss, at a reduced number of steps)."""
    if rank != 0:
        return
    device = "cuda" if torch.cuda.is_available() else "cpu"
    cfg, _ = build(args, 0, device)
    per_step = max(5.0, 60.0 / max(args.steps, 1))
    for _ in range(max(args.warmup, 0)):  # warm-up: a short sample of the same run
        cpu_baseline(cfg, seconds_target=1.0)
    rates, cores, sample = [], 1, ""
    for _ in range(max(args.steps, 1)):
        rate, cores, sample = cpu_baseline(cfg, seconds_target=per_step)
        rates.append(rate)
    value = statistics.median(rates)
    line = {
        "impl": "reference", "metric": "neuron-steps/s", "value": value, "unit": "neuron-steps/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {**config_of(args, cfg, world=1),
                                        "workload": f"{cfg.name}: CPU forward simulation, sample: {sample}"},
        "cpu_baseline": {"value": value, "unit": "neuron-steps/s", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "neuron-steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }  # fmt: skip
    ref = reference_dynamics_baseline(args, cfg)
    if ref is not None:
        line["reference_dynamics"] = ref
    print(json.dumps(line))


def reference_dynamics_baseline(args, cfg):
    """The reference's own CPU path, ``conductance/dynamics.py:146-237`` ``simulate``,
    imported from ``baseline/_ref`` (its package installed there), on a bounded sample
    of the configuration with dense weights, as its networks hand them over; forward
    only. None where it does not apply; a note where it cannot run."""
    if cfg.name in ("c3", "c4", "c5"):
        dense = {"c3": "10 GB", "c4": "77 GB", "c5": "4 TB"}[cfg.name]
        return {"unavailable": f"the reference's dense weights for {cfg.name} ({dense}) do not fit on the host"}
    ref_dir = ROOT / "baseline" / "_ref"
    if not ref_dir.exists():
        return {"unavailable": "the reference package is not installed under baseline/_ref"}
    sys.path.insert(0, str(ref_dir))
    try:
        from wiretorch.network_simulators import network as ref_net

        if cfg.name == "c2c":  # the current-based family: current/dynamics.py
            from wiretorch.network_simulators.current import dynamics as ref_dyn
        else:
            from wiretorch.network_simulators.conductance import dynamics as ref_dyn
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"importing the reference failed: {type(e).__name__}: {e}"}
    cpu = _to_cpu(cfg)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    def dense_of(W):
        if not hasattr(W, "row_ptr"):
            return W
        n_rows, N = W.shape
        out = torch.zeros(n_rows, N)
        rows = torch.repeat_interleave(torch.arange(n_rows), W.row_ptr[1:] - W.row_ptr[:-1])
        out.index_put_((rows, W.cols.long()), W.values, accumulate=True)
        return out

    drive = ref_net.Drive(made=cpu.drive.made, scale=cpu.drive.scale,
                          recurrent=[(r, dense_of(W)) for r, W in cpu.drive.recurrent],
                          feedforward=[(r, dense_of(W)) for r, W in cpu.drive.feedforward])  # fmt: skip
    fields = ("theta", "U_reset", "E_L", "C_m", "beta", "E_syn", "g_clip", "decay", "jump", "dt",
              "surr_scale", "n_ref", "mg_c", "mg_a", "adapt", "adapt_decay", "E_adapt")  # fmt: skip
    if cfg.name == "c2c":
        fields = ("theta", "U_reset", "beta", "U_rest", "R", "sign", "decay", "surr_scale", "n_ref", "adapt",
                  "adapt_decay")  # fmt: skip
    p = ref_dyn.Physiology(**{f: getattr(cpu.p, f) for f in fields}, spike_mode=cpu.p.spike_mode)
    v, g, kw = cpu.state()

    def timed(T):
        x = cfg.inputs(T=T, seed=99).cpu()
        t0 = time.perf_counter()
        with torch.no_grad():
            ref_dyn.simulate(v, g, x, drive, p, **kw)
        return time.perf_counter() - t0

    timed(2)  # warm-up
    T = 5
    el = timed(T)
    T = int(min(cfg.T, max(T, T * 15.0 / max(el, 1e-3))))
    el = timed(T)
    out = {"value": cfg.B * cfg.N * T / el, "unit": "neuron-steps/s", "cores": threads,
           "kind": "reference", "sample": f"{cfg.B} trials x {T} steps of the {cfg.name} network, forward only, "
                                           f"dense weights ({el:.1f} s)"}  # fmt: skip
    if cfg.name == "c2":  # the benchmarked workload itself: forward + BPTT + loss, at reduced T
        try:
            from wiretorch.training_utils import losses as ref_losses
        except Exception as e:  # noqa: BLE001
            out["training"] = {"unavailable": f"importing the reference's losses failed: {type(e).__name__}: {e}"}
        else:
            out["training"] = _reference_training(ref_dyn, ref_losses, drive, p, cfg, cpu, v, g, kw, threads)
    return out


def _reference_training(ref_dyn, ref_losses, drive, p, cfg, cpu, v, g, kw, threads, seconds=15.0):
    """The reference's own C2 training step on the host cores at a reduced number of
    steps: its ``dynamics.simulate`` with autograd (dense weights), its
    ``VanRossumRateLoss`` (``training_utils/losses.py:140-194``) against the target rates,
    and the backward pass to the learnt per-type-pair log scales (the optimiser's step
    is negligible beside them)."""
    import copy

    B, N = cfg.B, cfg.N
    types = cpu.types.cpu()
    target = cpu.extra["target_rates"] * (DT / 1000.0)

    def timed(T):
        x = cfg.inputs(T=T, seed=99).cpu()
        log_sf = torch.zeros(cfg.extra["log_sf_shape"], requires_grad=True)
        d = copy.copy(drive)
        loss_fn = ref_losses.VanRossumRateLoss(DT, 20.0, DT, T)
        t0 = time.perf_counter()
        d.scale = torch.exp(log_sf)[:, types]
        run = ref_dyn.simulate(v, g, x, d, p, **kw)
        loss = loss_fn(target[:, None, :].expand(B, T, N), output_spikes=run.output)
        loss.backward()
        return time.perf_counter() - t0

    # (from rest the spikes depend on the scales from the third step on: a conductance step
    # uses the input a step later)
    timed(3)  # warm-up
    T = 4
    el = timed(T)
    T = int(min(cfg.T, max(T, T * seconds / max(el, 1e-3))))
    el = timed(T)
    return {"value": B * N * T / el, "unit": "neuron-steps/s", "cores": threads, "kind": "reference",
            "sample": f"{B} trials x {T} steps of the c2 network, forward + BPTT + van Rossum rate loss, dense "
                      f"weights, autograd ({el:.1f} s)"}  # fmt: skip


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


def local_out_degree(d_loc, n_src, n_in, device):
    """Per source (neurons, then input columns) its edges onto this rank's block."""
    deg = torch.zeros(n_src + n_in, dtype=torch.float64, device=device)
    for side, off in ((d_loc.recurrent, 0), (d_loc.feedforward, n_src)):
        for rows, W in side:
            deg.index_add_(0, rows.to(device) + off, torch.diff(W.row_ptr).double().to(device))
    return deg


def main_partition(args, rank, world, local):
    """The network's neurons partitioned over the ranks (c4 / c5 by default at N > 1, or
    ``--partition``), forward only, each step's spikes exchanged by peer stores inside
    the forward kernel. Total work is fixed as ranks are added (strong scaling)."""
    from wiretorch_b200 import _lib, engine, partition

    engine.DEFER_CHECKS = True
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg, x = build(args, 0, device)  # every rank: the same network and input
    part = partition.Partition(cfg.N, cfg.B)
    chunked = cfg.name in ("c4", "c5")
    calls = cfg.T // x.shape[1] if chunked else 1

    def step(fetch=None):
        v, g, kw = cfg.state()
        with torch.no_grad():
            for _ in range(calls):
                xi = x if fetch is None else fetch.get()
                run = partition.simulate(part, v, g, xi, cfg.drive, cfg.p, **kw)
                if fetch is not None:  # after the launch: the copy runs beside this call
                    fetch.prefetch()
                v, g, kw = run.v, run.syn, cfg.carried(run)
        return run

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # synaptic events of one untimed step, counted on the device (edges onto this block)
    edges = torch.zeros(2, dtype=torch.int64, device=device)
    engine.EDGE_COUNTER = edges
    step()
    torch.cuda.synchronize()
    engine.EDGE_COUNTER = None
    _lib.TIMER = {}
    launches0 = _lib.LAUNCHES
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        start.record()
        for _ in range(args.steps):
            run = step()
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    launches = _lib.LAUNCHES - launches0
    timer, _lib.TIMER = _lib.TIMER, None
    elapsed_max = max_over_ranks(start.elapsed_time(end) / 1000.0, world)
    kernel = {k: sum(a.elapsed_time(b) for a, b in v) / len(v) for k, v in timer.items()}
    K = args.steps
    neuron_steps = cfg.B * cfg.N * cfg.T * K  # the one network, whatever the ranks
    spikes = sum_over_ranks(float(run.output.sum()), world)
    rec_edges = sum_over_ranks(float(edges[0]) * K, world)
    in_edges = sum_over_ranks(float(edges[1]) * K, world)

    # ---- roofline of this rank's forward launch (its block's share of the bytes) ----
    key = next(k for k in partition._LOCAL if k[2] == part.rank)
    d_loc, p_loc, plan = partition._LOCAL[key]["local"]
    n_b = part.n1 - part.n0
    T = x.shape[1]
    per = 8 + 16 * plan.ch.Sp + 2 + 1 / 8 + (8 if cfg.p.adapt is not None else 0)
    gating = cfg.B * T * cfg.extra["gating"].shape[1] * 8 / world if "gating" in cfg.extra else 0
    edge_bytes = float(edges[0] + edges[1]) / calls * 8  # this block's edges, per trial-event
    fwd_bytes = cfg.B * T * n_b * per + cfg.B * T * cfg.n_in * 4 + edge_bytes + gating
    peak, peak_kind = measured_peak()
    launch_ms = max_over_ranks(kernel["wt_forward"], world)
    roofline = {
        "kernel": f"wt_forward (persistent forward step kernel, one of {world} neuron blocks)",
        "bound": "hbm", "achieved": fwd_bytes / (launch_ms / 1000) / 1e9, "peak": peak, "unit": "GB/s",
        "frac": fwd_bytes / (launch_ms / 1000) / 1e9 / peak, "peak_kind": peak_kind, "traffic": None,
        "algorithmic_bytes_per_launch": fwd_bytes, "launch_ms": launch_ms,
        "edges_counted": "per trial-event onto this rank's block (at C5's rates a source rarely fires in "
                         "two trials at one step)",
    }  # fmt: skip

    # ---- end to end: each call's input from pinned host memory, the block's state read back ----
    e2e = None
    if not args.no_e2e:
        x_host, unpack = packed_input(x)
        out_host = torch.empty((cfg.B, n_b), pin_memory=True)
        fetch = Prefetcher(x_host, device, unpack)
        fetch.start()
        out_host.copy_(step(fetch).v, non_blocking=True)
        torch.cuda.synchronize()
        barrier(world)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(K):
            out_host.copy_(step(fetch).v, non_blocking=True)
        e2.record()
        torch.cuda.synchronize()
        e2e_el = max_over_ranks(s2.elapsed_time(e2) / 1000.0, world)
        e2e = {"value": neuron_steps / e2e_el, "unit": "neuron-steps/s",
               "h2d_bytes_per_step": calls * x_host[0].numel(), "d2h_bytes_per_step": out_host.numel() * 4,
               "ms_per_step": e2e_el / K * 1000.0,
               "note": "every rank copies the replicated input; bytes are per rank", "input": PACKED_NOTE}  # fmt: skip
    engine.check_errors()
    if rank == 0:
        print(json.dumps({
            "metric": "neuron-steps/s", "value": neuron_steps / elapsed_max, "unit": "neuron-steps/s",
            "n_gpus": world, "steps": K, "warmup": max(args.warmup, 3),
            "ms_per_step": elapsed_max / K * 1000.0, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Poisson input, seeded connectome)",
            "config": {**config_of(args, cfg, world), "parallelism": f"neuron-partition x{world}",
                       "global_batch": cfg.B,
                       "workload": f"{cfg.name}: {cfg.N} neurons ({world} blocks), {cfg.B} trials, {cfg.T} steps "
                                   f"of 0.1 ms, forward, {calls} calls of {x.shape[1]} steps, "
                                   f"spikes exchanged each step by peer stores"},
            "synaptic_events_per_s": rec_edges / elapsed_max, "input_events_per_s": in_edges / elapsed_max,
            "mean_rate_hz": spikes / (cfg.B * cfg.N * x.shape[1]) / (DT / 1000.0),
            "roofline": roofline, "kernel_ms": kernel, "gpu_launches": launches,
            "clocks": clocks.summary(), "e2e": e2e, "cpu_baseline": None,
        }))  # fmt: skip
    barrier(world)
    part.close()


def main():
    args = parse()
    rank, world, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.partition or (world > 1 and args.config in ("c4", "c5")):
            main_partition(args, rank, world, local)
        else:
            main_single(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def main_single(args, rank, world, local):
    """One GPU per rank, each rank its own trials (weak scaling at N > 1)."""
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
    plan = None if factorised else plan_of(cfg, device)

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
    with torch.no_grad():
        v0, g0, kw0 = cfg.state()
        run = simulate_of(cfg)(v0, g0, x, cfg.drive, cfg.p, **kw0)
    if factorised:
        kname = "wt_lowrank_forward"
        fwd_bytes = factorised_bytes(cfg, x.shape[1])
        kdesc = "wt_lowrank_forward (persistent factorised step kernel, tcgen05 product per step)"
    else:
        kname = "wt_forward"
        fwd_bytes = forward_bytes(cfg, plan, x.shape[1], train, fired_edges_once(cfg, run.output, x))
        kdesc = "wt_forward (persistent forward step kernel)"
    mean_rate = float(run.output.mean()) / (DT / 1000.0)
    del run
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
        x_host, unpack = packed_input(x)
        calls = cfg.T // x.shape[1] if cfg.name in ("c3", "c4", "c5") else 1
        if train:
            e2e = e2e_training(cfg, step, log_sf, x_host[0], unpack, device, world, K, neuron_steps)
        else:
            fetch = Prefetcher(x_host, device, unpack)
            out_host = torch.empty((cfg.B, cfg.N), pin_memory=True)
            fetch.start()
            out_host.copy_(step(x, fetch=fetch), non_blocking=True)
            torch.cuda.synchronize()
            barrier(world)
            s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s2.record()
            for _ in range(K):  # the final membrane state of every step read back
                out_host.copy_(step(x, fetch=fetch), non_blocking=True)
            e2.record()
            torch.cuda.synchronize()
            e2e_el = max_over_ranks(s2.elapsed_time(e2) / 1000.0, world)
            e2e = {"value": neuron_steps / e2e_el, "unit": "neuron-steps/s",
                   "h2d_bytes_per_step": calls * x_host[0].numel(), "d2h_bytes_per_step": out_host.numel() * 4,
                   "ms_per_step": e2e_el / K * 1000.0, "input": PACKED_NOTE}  # fmt: skip

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
            "mean_rate_hz": mean_rate,
            "roofline": roofline, "kernel_ms": kernel_ms, "gpu_launches": launches,
            "clocks": clock, "e2e": e2e, "cpu_baseline": cpu,
        }  # fmt: skip
        print(json.dumps(line))


def e2e_training(cfg, step, log_sf, x_host, unpack, device, world, K, neuron_steps):
    """The c2 training step fed from pinned host memory (spike input as bits, unpacked on
    the device; target rates), the loss and the learnt scales read back every step; each
    step's input copied on a second stream while the previous step computes."""
    tgt_host = cfg.extra["target_rates"].cpu().pin_memory()
    out_host = torch.empty(1 + log_sf.numel(), pin_memory=True)
    h2d = x_host.numel() + tgt_host.numel() * 4
    d2h = out_host.numel() * 4
    fetch_x = Prefetcher([x_host], device, unpack)
    fetch_t = Prefetcher([tgt_host], device, lambda t: t * (DT / 1000.0))

    def e2e_step():
        xd, r = fetch_x.get(), fetch_t.get()
        fetch_x.prefetch()
        fetch_t.prefetch()
        loss = step(xd, r[:, None, :].expand(cfg.B, cfg.T, cfg.N))
        out_host.copy_(torch.cat([loss.detach().reshape(1), log_sf.detach().reshape(-1)]), non_blocking=True)

    fetch_x.start()
    fetch_t.start()
    e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(K):
        e2e_step()
    e2.record()
    torch.cuda.synchronize()
    e2e_el = max_over_ranks(s2.elapsed_time(e2) / 1000.0, world)
    return {"value": neuron_steps / e2e_el, "unit": "neuron-steps/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": e2e_el / K * 1000.0, "input": PACKED_NOTE}


if __name__ == "__main__":
    main()
