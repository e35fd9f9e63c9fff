"""Short, representative launches of the engine's kernels for profiling (ncu captures).

``python tests/profile_cases.py c2-active``: C2 (64 trials, pooled channels) run
450 steps from rest, then one 20-step call from that state with saving for the backward
pass, as in training. ``python tests/profile_cases.py c3-small``: C3 with 128
trials, 200 steps, then one 10-step call from that state. ``c5-small``: C5 at 250,000
neurons (4 trials, gated, pooled), 300 steps from rest, then one 20-step call;
``c5-full`` the same at C5's full size (1,000,000 neurons). In all the second launch of
the kernel is the one to capture (``-s 1 -c 1``).
"""

from __future__ import annotations

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402


def c2_active():
    from wiretorch_b200 import configs, engine

    cfg = configs.c2(B=64, T=500, device="cuda")
    engine.POOL_SYNAPSES = True
    x = cfg.inputs(seed=1)
    v, g, kw = cfg.state()
    with torch.no_grad():
        run = engine.simulate(v, g, x[:, :450], cfg.drive, cfg.p, **kw)
    log_sf = torch.zeros(cfg.extra["log_sf_shape"], device="cuda", requires_grad=True)
    cfg.drive.scale = configs.scale_from_log_sf(cfg, log_sf)
    run2 = engine.simulate(run.v, run.syn, x[:, 450:470].contiguous(), cfg.drive, cfg.p,
                           refractory=run.refractory)  # fmt: skip
    torch.cuda.synchronize()
    print(f"c2-active: {float(run2.output.sum()) / 20:.0f} spikes per step")


def c3_small():
    from wiretorch_b200 import configs, engine

    cfg = configs.c3(B=128, T=200, device="cuda")
    x = cfg.inputs(T=200, seed=1)
    v, g, kw = cfg.state()
    with torch.no_grad():
        run = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
        run2 = engine.simulate(run.v, run.syn, x[:, :10].contiguous(), cfg.drive, cfg.p,
                               refractory=run.refractory)  # fmt: skip
    torch.cuda.synchronize()
    print(f"c3-small: {float(run2.output.sum()):.0f} spikes in 10 steps")


def c5_small():
    from wiretorch_b200 import configs, engine

    # C5 at a quarter of the neurons (same out-degree, ~250M edges, ~3 GB of tables)
    cfg = configs.c5(B=4, T=320, device="cuda", N=250_000, lam=0.05 * 4 ** (1 / 3))
    engine.POOL_SYNAPSES = True
    x = cfg.inputs(T=320, seed=1)
    v, g, kw = cfg.state()
    with torch.no_grad():
        run = engine.simulate(v, g, x[:, :300].contiguous(), cfg.drive, cfg.p, **kw)
        run2 = engine.simulate(run.v, run.syn, x[:, 300:].contiguous(), cfg.drive, cfg.p, **cfg.carried(run))
    torch.cuda.synchronize()
    print(f"c5-small: {float(run2.output.sum()) / 20:.0f} spikes per step, {cfg.extra['edges']} edges")


def c5_full():
    from wiretorch_b200 import configs, engine

    # C5 as benchmarked (1,000,000 neurons, ~981M edges, 4 trials), pooled channels
    cfg = configs.c5(B=4, T=320, device="cuda")
    engine.POOL_SYNAPSES = True
    x = cfg.inputs(T=320, seed=1)
    v, g, kw = cfg.state()
    with torch.no_grad():
        run = engine.simulate(v, g, x[:, :300].contiguous(), cfg.drive, cfg.p, **kw)
        run2 = engine.simulate(run.v, run.syn, x[:, 300:].contiguous(), cfg.drive, cfg.p, **cfg.carried(run))
    torch.cuda.synchronize()
    print(f"c5-full: {float(run2.output.sum()) / 20:.0f} spikes per step, {cfg.extra['edges']} edges")


CASES = {"c2-active": c2_active, "c3-small": c3_small, "c5-small": c5_small, "c5-full": c5_full}

if __name__ == "__main__":
    CASES[sys.argv[1]]()
