"""The engine at the benchmark configurations' scale, on the B200.

Three kinds of evidence, against the ``north_star`` acceptance bar (identical spike
rasters over the first 1,000 steps, fp32 traces within 1e-5 relative until the first
spike divergence, per-type firing rates within 1%, BPTT gradients within 1e-3):

* the reference's own runs (``tests/golden/config_*.npz``, made by its CPU dynamics):
  configuration 1 at its specified size (1,000 neurons, 8 trials, 1,000 steps) and
  configurations 2, 4 and 5 at 2,000 neurons, in free run from rest; the gradient of
  configuration 2's van Rossum rate loss with respect to its learnt per-type-pair log
  scales;
* the reference's at-scale statistics networks (``tests/golden/statistics_*.npz``),
  judged as the reference's ``tests/test_statistics.py:50-85`` judges its simulators;
* the oracle (``oracle/cond_lif.c``, itself pinned to the reference by
  ``tests/test_oracle_config_golden.py``) on configuration 2 at its full 20,000 neurons
  (4 trials, 500 steps, pooled channels as benchmarked: lockstep and free run) and on
  configurations 4 and 5 at a tenth of their neurons over 3,000 / 2,000 steps
  (per-type firing rates).
"""

import math

import numpy as np
import pytest
import torch

import golden_io
import lockstep
from oracle import oracle
from wiretorch_b200 import configs, engine
from wiretorch_b200.filtering import VanRossumRateLoss

pytestmark = pytest.mark.gpu

V_RTOL = 1e-5
RATE_RTOL = 0.01


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def _kw(d, prefix):
    return {k: _t(d[f"{prefix}{k}"]) for k in ("refractory", "gating", "adaptation") if f"{prefix}{k}" in d}


def engine_snapshots(drive, p, x, v, g, kw, snap, pool):
    """The engine's free run in ``snap``-step calls, the state carried: spikes, the
    voltage after every call, and the final run."""
    engine.POOL_SYNAPSES = pool
    spikes, v_snap = [], []
    try:
        with torch.no_grad():
            for start in range(0, x.shape[1], snap):
                run = engine.simulate(v, g, x[:, start : start + snap].contiguous(), drive, p, **kw)
                spikes.append(run.output.cpu().numpy() > 0.5)
                v, g = run.v, run.syn
                kw = {k: getattr(run, k) for k in kw}
                v_snap.append(v.cpu().numpy())
    finally:
        engine.POOL_SYNAPSES = False
    return np.concatenate(spikes, 1), np.stack(v_snap), run


# C2's 41 synapse types (one per cell type, as the reference's registry makes them) run
# pooled into their 2 distinct dynamics only: the kernels carry at most 8 channels.
FREE_RUNS = [pytest.param(name, pool, id=f"{name}-{'pooled' if pool else 'exact'}")
             for name in golden_io.config_cases() for pool in (False, True)
             if pool or name != "config_c2"]  # fmt: skip


@pytest.mark.parametrize("name,pool", FREE_RUNS)
def test_config_free_run_matches_the_reference(name, pool):
    """Identical spike rasters over every step (C1: all 1,000), voltages within 1e-5
    relative at every recorded step, the final state likewise."""
    drive, p, d, meta = golden_io.load(name, "cuda")
    x = _t(d["in.x"])
    spikes, v_snap, run = engine_snapshots(drive, p, x, _t(d["in.v"]), _t(d["in.g"]), _kw(d, "in."),
                                           meta["snap"], pool)  # fmt: skip
    ref = d["out.spikes"]
    first = golden_io.first_divergence(spikes, ref)
    for w in range(ref.shape[1] // meta["snap"]):
        if (w + 1) * meta["snap"] > first:
            break
        np.testing.assert_allclose(v_snap[w], d["out.v_snap"][w], rtol=V_RTOL, atol=0,
                                   err_msg=f"{name}: voltages after step {(w + 1) * meta['snap']}")  # fmt: skip
    assert first == ref.shape[1], f"{name}: rasters differ from step {first} of {ref.shape[1]}"
    assert int(ref.sum()) > 200
    np.testing.assert_allclose(run.v.cpu().numpy(), d["out.v"], rtol=V_RTOL, atol=0)
    g = run.syn.cpu().numpy()
    ref_g = d["out.g"]
    if pool:  # each pool's conductance sits at its first member type
        ch = engine.get_plan(drive, p, x.shape[0], x.shape[2], x.device, pool=True).ch
        g = np.stack([g[..., m[0]] for m in ch.member], -1)
        ref_g = np.stack([ref_g[..., list(m)].sum(-1) for m in ch.member], -1)
    np.testing.assert_allclose(g, ref_g, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("pool", [True], ids=["pooled"])
def test_config_c2_rate_loss_gradient_matches_the_reference(pool):
    """C2's training loss (van Rossum rate loss: 20 ms-filtered output spikes against
    the filtered target rates) and its gradient with respect to the learnt per-type-pair
    log scales, through ``grad_steps`` steps, within 1e-3 of the largest entry."""
    drive, p, d, meta = golden_io.load("config_c2", "cuda")
    T = meta["grad_steps"]
    types = _t(d["in.types"])
    log_sf = _t(d["in.log_sf"]).requires_grad_(True)
    drive.scale = torch.exp(log_sf)[:, types]
    B, N = d["in.v"].shape
    target = (_t(d["in.target_rates"]) * float(p.dt) / 1000.0)[:, None, :].expand(B, T, N)
    loss_fn = VanRossumRateLoss(float(p.dt), meta["tau_decay"], float(p.dt), T)
    engine.POOL_SYNAPSES = pool
    try:
        run = engine.simulate(_t(d["in.v"]), _t(d["in.g"]), _t(d["in.x"][:, :T]), drive, p, **_kw(d, "in."))
        loss = loss_fn(target, output_spikes=run.output)
        loss.backward()
    finally:
        engine.POOL_SYNAPSES = False
    assert float(run.output.detach().sum()) == float(d["grad.spikes_sum"])
    np.testing.assert_allclose(float(loss.detach()), float(d["grad.loss"]), rtol=1e-5)
    ref = d["grad.log_sf"]
    got = log_sf.grad.cpu().numpy()
    assert np.abs(ref).max() > 0
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err <= 1e-3, f"log_sf gradient differs by {err:.2e} of its largest entry"


def _statistics(name):
    drive, p, d, meta = golden_io.load(name, "cuda")
    A, B = meta["seeds"]
    x = _t(d[f"in.x_{A}"])
    spikes, _, _ = engine_snapshots(drive, p, x, _t(d["in.v"]), _t(d["in.g"]), _kw(d, "in."), meta["chunk"],
                                    pool=False)  # fmt: skip
    spikes = spikes[:, meta["burn_in"] :]
    types = d["in.types"]
    rates = spikes.mean(axis=(0, 1)) * 1000.0 / float(p.dt)
    pop = lambda r: np.array([r[types == t].mean() for t in np.unique(types)])  # noqa: E731
    ref, ref_b = pop(d[f"rec.rates_{A}"]), pop(d[f"rec.rates_{B}"])
    allowed = np.maximum(2 * np.abs(ref_b - ref), 0.02 * ref)
    return spikes, rates, pop, ref, allowed, d


def test_statistics_recurrent_matches_the_recording():
    """The reference's at-scale recurrent network (2,000 neurons, 3,000 steps): per-type
    rates as close to its GPU recording as its two recorded inputs are to each other
    (or 2%); rank agreement of the neurons' rates at least as good."""
    spikes, rates, pop, ref, allowed, d = _statistics("statistics_recurrent")
    assert np.all(np.abs(pop(rates) - ref) <= allowed), (pop(rates), ref, allowed)
    floor = np.corrcoef(d["rec.rates_0"], d["rec.rates_1"])[0, 1]
    assert np.corrcoef(rates, d["rec.rates_0"])[0, 1] >= floor - 0.01
    # against the reference's CPU run of the same input: per-type rates within 1%
    cpu = pop(d["out.spikes"].mean(axis=(0, 1)) * 1000.0)
    assert np.all(np.abs(pop(rates) - cpu) <= RATE_RTOL * cpu), (pop(rates), cpu)


def test_statistics_feedforward_matches_the_recording():
    """The reference's feedforward statistics network: spikes within 0.1% of its
    recording (the network is not chaotic)."""
    spikes, rates, pop, ref, allowed, d = _statistics("statistics_feedforward")
    mismatched = (spikes != d["rec.spikes"]).sum() / d["rec.spikes"].sum()
    assert mismatched < 1e-3, f"{mismatched:.2%} of spikes differ from the recording"
    assert (spikes != d["out.spikes"]).sum() / d["out.spikes"].sum() < 1e-3


# ---------------------------------------------------------------------------------------
# Full-size and tenth-size configurations against the oracle
# ---------------------------------------------------------------------------------------


def test_c2_full_size_pooled_against_oracle():
    """Configuration 2 at 20,000 neurons (4 trials, 500 steps), pooled channels as
    benchmarked: lockstep in 10-step windows (spikes exact, a flip within 1e-3 mV of
    threshold excused; voltages within 2e-4 mV; conductances within 1e-5 relative), and
    the free run's raster identical to the oracle's up to its first divergence, which
    must come from a neuron at threshold."""
    cfg = configs.c2(B=4, T=500, device="cuda")
    x = cfg.inputs(seed=1)
    v, g, kw = cfg.state()
    oracle.set_threads(4)
    net = oracle.Network(cfg.drive, cfg.p, cfg.B, cfg.n_in)
    windows = lockstep.oracle_windows(net, x, v, g, kw, 10)
    ch = engine.get_plan(cfg.drive, cfg.p, cfg.B, cfg.n_in, x.device, pool=True).ch
    pools = [list(m) for m in ch.member]

    def sim(v_, g_, x_, kw_):
        engine.POOL_SYNAPSES = True
        try:
            with torch.no_grad():
                return engine.simulate(v_, g_, x_, cfg.drive, cfg.p, track=True, **kw_)
        finally:
            engine.POOL_SYNAPSES = False

    excused, n_windows, dv, dg = lockstep.compare(sim, net, cfg.drive, cfg.p, x, v, g, kw, pools=pools,
                                                  oracle=windows)  # fmt: skip
    assert excused <= 0.01 * n_windows
    # free run from rest, one call of 500 steps
    spikes, _, _ = engine_snapshots(cfg.drive, cfg.p, x, v, g, kw, 500, pool=True)
    ref = windows[1]
    first = golden_io.first_divergence(spikes, ref)
    print(f"C2 full size: {int(ref.sum())} oracle spikes, free run identical for {first} of 500 steps, "
          f"{excused} excused windows of {n_windows}")  # fmt: skip
    if first < 500:  # the first flip must be a rounding at threshold
        b, n = np.argwhere(spikes[:, first] != ref[:, first])[0]
        v_enter = windows[2][b, first - 1, n] if first > 0 else float(v[b, n])
        assert abs(v_enter - float(cfg.p.theta[n])) < 1e-3, (first, b, n, v_enter)


def _tenth(name):
    if name == "c4":  # 13,900 neurons in 800 types, the same degree law
        return configs.c4(B=4, T=3000, device="cuda", N=13900, n_types=800), 3000
    # 100,000 neurons, the same expected out-degree (connection length x 10^(1/3))
    return configs.c5(B=4, T=2000, device="cuda", N=100_000, lam=0.05 * 10 ** (1 / 3)), 2000


@pytest.mark.parametrize("name", ["c4", "c5"])
def test_tenth_size_per_type_rates_against_oracle(name):
    """Configurations 4 and 5 at a tenth of their neurons: the per-type firing rates of
    the whole run within 1% of the oracle's (types: the excitatory, inhibitory and
    silent classes of C4's 800 cell types; C5's excitatory and inhibitory neurons),
    and the rasters identical up to the first divergence."""
    cfg, T = _tenth(name)
    engine.POOL_SYNAPSES = True
    x = cfg.inputs(T=T, seed=1)
    v, g, kw = cfg.state()
    try:
        with torch.no_grad():
            run = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
    finally:
        engine.POOL_SYNAPSES = False
    spikes = run.output.cpu().numpy() > 0.5
    oracle.set_threads(cfg.B)
    net = oracle.Network(cfg.drive, cfg.p, cfg.B, cfg.n_in)
    ref = net.simulate(x, v, g, **kw, track=False)["spikes"]
    first = golden_io.first_divergence(spikes, ref)
    if name == "c4":  # sign class of each neuron: 0 excitatory, 1 inhibitory, 2 silent
        rows_e = cfg.drive.recurrent[0][0].cpu().numpy()
        rows_i = cfg.drive.recurrent[1][0].cpu().numpy()
        types = np.full(cfg.N, 2)
        types[rows_e], types[rows_i] = 0, 1
    else:
        types = cfg.types.cpu().numpy()
    got = golden_io.population_rates(spikes, types, 0.1)
    want = golden_io.population_rates(ref, types, 0.1)
    print(f"{name} tenth: rasters identical for {first} of {T} steps; rates {got} Hz, oracle {want} Hz")
    assert want.min() > 0.5
    assert np.all(np.abs(got - want) <= RATE_RTOL * want), (got, want)


# ---------------------------------------------------------------------------------------
# The loss filter and the van Rossum rate loss against the reference
# ---------------------------------------------------------------------------------------


def test_filter_matches_the_reference_over_carried_chunks():
    """``double_exponential`` over three chunks with the state carried (as the van
    Rossum losses carry it), and the gradient of ``sum(smooth * R)`` per chunk, against
    the reference's own (``training_utils/filtering.py:28-73``)."""
    from wiretorch_b200.filtering import double_exponential

    with np.load(golden_io.GOLDEN / "loss_filter.npz") as z:
        d = {k: z[k] for k in z.files}
    T, dt = int(d["T"]), float(d["dt"])
    t = torch.arange(T, dtype=torch.float32, device="cuda") * dt
    k_r, k_d = torch.exp(-t / float(d["tau_rise"])), torch.exp(-t / float(d["tau_decay"]))
    def close(got, ref):
        # float32 recursions against the reference's Toeplitz products: the same sums in
        # another order, within 1e-5 relative plus 1e-6 of the largest magnitude (the
        # adjoint sums 60 terms of both signs, so single entries can cancel)
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6 * np.abs(ref).max())

    cr = cs = None
    for c in range(3):
        x = _t(d[f"x.{c}"]).requires_grad_(True)
        rise, smooth = double_exponential(x, k_r, k_d, cr, cs)
        (smooth * _t(d[f"R.{c}"])).sum().backward()
        close(rise.detach().cpu().numpy(), d[f"rise.{c}"])
        close(smooth.detach().cpu().numpy(), d[f"smooth.{c}"])
        close(x.grad.cpu().numpy(), d[f"grad_x.{c}"])
        cr, cs = rise[:, -1:].detach(), smooth[:, -1:].detach()


def test_van_rossum_rate_loss_matches_the_reference_over_carried_chunks():
    """``VanRossumRateLoss`` as C2 uses it (rise dt, decay 20 ms) over three chunks:
    each chunk's loss, its gradient with respect to the output spikes, and the carried
    filter state, against the reference's (``training_utils/losses.py:140-194``)."""
    with np.load(golden_io.GOLDEN / "loss_van_rossum.npz") as z:
        d = {k: z[k] for k in z.files}
    B, T, N, dt = int(d["B"]), int(d["T"]), int(d["N"]), float(d["dt"])
    loss_fn = VanRossumRateLoss(float(d["tau_rise"]), float(d["tau_decay"]), dt, T)
    target = _t(d["target_rate"])[:, None, :].expand(B, T, N)
    for c in range(3):
        s = _t(d[f"spikes.{c}"]).requires_grad_(True)
        loss = loss_fn(target, output_spikes=s)
        loss.backward()
        np.testing.assert_allclose(float(loss), float(d[f"loss.{c}"]), rtol=1e-5)
        g = s.grad.cpu().numpy()
        ref = d[f"grad_spikes.{c}"]
        assert np.abs(g - ref).max() <= 1e-4 * np.abs(ref).max()
        carried = torch.stack([loss_fn.prev_output_rise, loss_fn.prev_output_smooth, loss_fn.prev_target_rise,
                               loss_fn.prev_target_smooth]).cpu().numpy()  # fmt: skip
        # the state after up to 300 steps of a float32 recursion, against the reference's
        # Toeplitz products: the same sums rounded in another order
        np.testing.assert_allclose(carried, d[f"carried.{c}"], rtol=3e-5, atol=1e-7)
