"""Short, representative launches of the engine's kernels for profiling (ncu captures).

``python tests/profile_cases.py c2-active``: C2 (64 trials, pooled channels) run
450 steps from rest, then one 20-step call from that state with saving for the backward
pass, as in training. ``python tests/profile_cases.py c3-small``: C3 with 128
trials, 200 steps, then one 10-step call from that state. ``c5-small``: C5 at 250,000
neurons (4 trials, gated, pooled), 300 steps from rest, then one 20-step call;
``c5-full`` the same at C5's full size (1,000,000 neurons). In these the second launch
of the kernel is the one to capture (``-s 1 -c 1``). ``c2-step``: two C2 training steps
(every kernel of the second step is one to capture; ``c2-step-16`` with 16 trials, for
captures of many passes); ``c2-carry``: the per-step carry of
gradients through the recurrent spikes; ``c3-product``: the tensor-core product alone; ``misc``: one launch each of the
filter, fold, input-gradient, carry and product kernels.
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


def c2_step(B=64):
    """One C2 training step (64 trials, 500 steps, pooled channels): forward with saving,
    van Rossum rate loss, reverse scan, edge gradients to the per-pair scales, after one
    untimed step. Every kernel of the step launches once in the second step."""
    from wiretorch_b200 import configs, engine, filtering

    cfg = configs.c2(B=B, T=500, device="cuda")
    engine.POOL_SYNAPSES = True
    x = cfg.inputs(seed=1)
    v, g, kw = cfg.state()
    log_sf = torch.zeros(cfg.extra["log_sf_shape"], device="cuda", requires_grad=True)
    loss_fn = filtering.VanRossumRateLoss(0.1, 20.0, 0.1, cfg.T, device="cuda")
    target = (cfg.extra["target_rates"] * 1e-4)[:, None, :].expand(cfg.B, cfg.T, cfg.N)
    for _ in range(2):
        loss_fn.reset_state()
        cfg.drive.scale = configs.scale_from_log_sf(cfg, log_sf)
        run = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
        loss = loss_fn(target, output_spikes=run.output)
        log_sf.grad = None
        loss.backward()
    torch.cuda.synchronize()
    print(f"c2-step: loss {float(loss.detach()):.5f}, |grad| {float(log_sf.grad.norm()):.3e}")


def c2_carry():
    """C2 with gradients through the recurrent spikes (16 trials, 40 steps): the
    per-step carry kernel along the recurrent edges, 40 launches in the backward pass."""
    from wiretorch_b200 import configs, engine

    cfg = configs.c2(B=16, T=40, device="cuda")
    engine.POOL_SYNAPSES = True
    cfg.drive.recurrent_gradients = True
    x = cfg.inputs(seed=1)
    v, g, kw = cfg.state()
    log_sf = torch.zeros(cfg.extra["log_sf_shape"], device="cuda", requires_grad=True)
    cfg.drive.scale = configs.scale_from_log_sf(cfg, log_sf)
    run = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
    (run.output * torch.randn_like(run.output)).sum().backward()
    torch.cuda.synchronize()
    print(f"c2-carry: |grad| {float(log_sf.grad.norm()):.3e}")


def c3_product():
    """The tensor-core product of C3's factors: V (50,000 x 64) times P^T for 256 trials
    and two pathways (``wt_lowrank_product``), three launches."""
    from wiretorch_b200 import lowrank

    N, r, B = 50000, 64, 256
    gen = torch.Generator(device="cuda").manual_seed(0)
    V = (torch.randn(N, r, generator=gen, device="cuda") / N**0.5).to(torch.bfloat16)
    P = torch.randn(B, 2, r, generator=gen, device="cuda")  # two pathways (E, I)
    for _ in range(3):
        out = lowrank.product(V, P)
    torch.cuda.synchronize()
    print(f"c3-product: {tuple(out.shape)}")


def misc():
    """One launch each of the kernels outside the training step's main three: the
    double-exponential filter forward and backward on C2's output shape (64 x 500 x
    20,000), the weight fold of C2, the input gradient (C2 at 16 trials, 100 steps, the
    input requiring grad), the recurrent carry (``c2_carry``) and the factorised product
    (``c3_product``)."""
    from wiretorch_b200 import configs, engine, filtering

    gen = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.rand((64, 500, 20000), generator=gen, device="cuda") < 0.0015).float().requires_grad_(True)
    t = torch.arange(500, dtype=torch.float32, device="cuda") * 0.1
    rise, smooth = filtering.double_exponential(x, torch.exp(-t / 0.1), torch.exp(-t / 20.0), None, None)
    smooth.sum().backward()
    cfg = configs.c2(B=16, T=100, device="cuda")
    engine.POOL_SYNAPSES = True
    xi = cfg.inputs(seed=1).requires_grad_(True)
    v, g, kw = cfg.state()
    run = engine.simulate(v, g, xi, cfg.drive, cfg.p, **kw)  # folds the weights, saves for backward
    (run.output * torch.randn_like(run.output)).sum().backward()
    torch.cuda.synchronize()
    c2_carry()
    c3_product()
    print(f"misc: |dL/dx| {float(xi.grad.norm()):.3e}")


CASES = {"c2-active": c2_active, "misc": misc, "c3-small": c3_small, "c5-small": c5_small, "c5-full": c5_full,
         "c2-step": c2_step, "c2-step-16": lambda: c2_step(16), "c2-carry": c2_carry,
         "c3-product": c3_product}  # fmt: skip

if __name__ == "__main__":
    CASES[sys.argv[1]]()
