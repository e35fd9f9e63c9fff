"""Generate the golden cases of ``tests/golden`` from wiretorch's own implementation.

    python tests/golden/make_golden.py [--reference PATH] [name ...]

Run where the reference wiretorch checkout is available (``--reference``, default the
``WIRETORCH_REFERENCE`` environment variable). It imports the reference's package
(``src/wiretorch``) and its test networks (``tests/networks.py``), builds each
scenario, and calls the reference's PyTorch dynamics,
``wiretorch.network_simulators.conductance.dynamics.simulate``
(``conductance/dynamics.py:146-237``), on the CPU with exactly the ``Drive`` and
``Physiology`` its network hands its engine (``network.py:889-909``). What it produced is
written with ``golden_io.save``: a free run with the voltage of every step and the final
state, and the gradients of a fixed random readout of the spikes with respect to every
differentiable input of the engine (scale, weights, input, physiology), backpropagated
through the first ``GRAD_STEPS`` steps. Scenarios recorded by the reference's own suite
(``tests/fixtures/*.npz``) carry that recording too, which pins the oracle to the
reference's golden vectors.

Three more kinds of case:

* ``config_c1`` ... ``config_c5``: the benchmark configurations' networks, built with
  ``wiretorch_b200.configs`` on the CPU (C1 at its full size; C2, C4 and C5 at 2,000
  neurons with the degrees lowered and the weights raised to keep them active), run
  through the reference's ``dynamics.simulate`` with its own ``Drive``/``Gate``/
  ``Physiology`` classes and dense weights; recorded: the spike raster, the voltage
  every ``SNAP`` steps and the final state. ``config_c2`` also records the gradient of
  the reference's ``VanRossumRateLoss`` (``training_utils/losses.py:140-194``) with
  respect to the learnt per-type-pair log scales, through ``GRAD_STEPS_C2`` steps.
* ``statistics_recurrent`` / ``statistics_feedforward``: the networks of the
  reference's at-scale statistics test (``tests/fixtures/generate.py``
  ``STATS_NETWORKS``, 2,000 and 1,000 neurons, 3,000 and 2,000 steps of 1 ms), their
  inputs, the firing rates (and feedforward spikes) recorded from the reference's GPU
  simulator in ``tests/fixtures/statistics.npz``, and a run of its CPU dynamics.
* ``current_*``: the reference's current-based test networks (``tests/networks.py``
  ``current_recurrent``, ``current_feedforward``, ``current_feedforward_probabilities``,
  and the recurrent one with a refractory period, short-term plasticity and adaptation)
  run through ``network_simulators/current/dynamics.py`` ``simulate``, with the
  reference suite's recordings (``tests/fixtures/current_*.npz``) where there are, and the
  gradients of a fixed readout with respect to the scale, the weights, the input and the
  learnable physiology.
* ``curstats_recurrent`` / ``curstats_feedforward``: the current-based networks of the
  reference's statistics test (``STATS_NETWORKS["current_*"]``, 2,000 and 1,000 neurons),
  their inputs, the rates (and feedforward spikes) recorded in
  ``tests/fixtures/statistics_current.npz``, and a run of the reference's current-based
  dynamics here.
* ``loss_filter`` / ``loss_van_rossum``: the reference's ``double_exponential``
  (``training_utils/filtering.py:28-73``, its CPU Toeplitz path) and
  ``VanRossumRateLoss`` over three chunks with the filter state carried, with the
  gradients of the outputs.
"""

from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).parent
sys.path.insert(0, str(HERE.parent))  # golden_io
sys.path.insert(0, str(HERE.parents[1]))  # wiretorch_b200

import golden_io  # noqa: E402

PHYS_GRADS = ("theta", "U_reset", "E_L", "C_m", "beta", "E_syn", "decay", "jump",
              "adapt", "adapt_decay", "E_adapt")  # fmt: skip
T_FREE = 200
WINDOW = 10  # steps between recorded states (the reference's lockstep window)
GRAD_STEPS = 100
READOUT_SEED = 7


def import_reference(path: Path):
    sys.path.insert(0, str(path / "src"))
    sys.path.insert(0, str(path / "tests"))
    import networks  # noqa: F401  (the reference's test networks)
    from wiretorch.network_simulators.conductance import dynamics  # noqa: F401

    return networks, dynamics


def readout(seed, shape):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.normal(size=shape).astype(np.float32))


def engine_inputs(model):
    """The state a network hands its engine (``network.py:896-909``)."""
    kw = {}
    if model.has_refractory:
        kw["refractory"] = model.refractory.clone()
    if model.n_gating:
        kw["gating"] = model.gating.clone()
    if model._adapting:
        kw["adaptation"] = model.adaptation.clone()
    return model.v.clone(), model._synaptic.clone(), kw


def free_run(dynamics, model, x, probabilities):
    """The whole input in ``WINDOW``-step calls (chunking does not change the run),
    recording the state entering each window for the lockstep tests."""
    drive, p = model._drive(), model._physiology()
    v, g, kw = engine_inputs(model)
    inputs = {"x": x, "v": v, "g": g, **kw}
    windows = {"v": [], "g": [], **{k: [] for k in kw}}
    spikes, v_track, prob = [], [], []
    with torch.no_grad():
        for start in range(0, x.shape[1], WINDOW):
            for key, value in (("v", v), ("g", g), *kw.items()):
                windows[key].append(value.clone())
            run = dynamics.simulate(
                v, g, x[:, start : start + WINDOW], drive, p,
                probabilities=probabilities, track=True, track_batch_idx=None, **kw,
            )  # fmt: skip
            spikes.append(run.output)
            v_track.append(run.tracked["v"])
            prob.append(run.probabilities)
            v, g = run.v, run.syn
            for key in kw:
                kw[key] = getattr(run, key)
        for key, value in (("v", v), ("g", g), *kw.items()):
            windows[key].append(value.clone())
    outputs = {
        "spikes": torch.cat(spikes, dim=1),
        "v_track": torch.cat(v_track, dim=1),
        "v": v,
        "g": g,
        "prob": torch.cat(prob, dim=1) if probabilities else None,
        **kw,
        **{f"win_{k}": torch.stack(vals) for k, vals in windows.items()},
    }
    return drive, p, inputs, outputs


def gradients(dynamics, model, x, probabilities):
    """Gradients of ``sum(spikes R) (+ sum(prob R2))`` over ``GRAD_STEPS`` steps with
    respect to the engine's inputs, all made leaves."""
    drive, p = model._drive(), model._physiology()
    v, g, kw = engine_inputs(model)
    x = x[:, :GRAD_STEPS].clone().requires_grad_(True)
    leaves = {"x": x}
    drive.scale = drive.scale.detach().clone().requires_grad_(True)
    leaves["scale"] = drive.scale
    made = {}

    def leaf(W):
        if id(W) not in made:
            made[id(W)] = W.detach().clone().requires_grad_(True)
        return made[id(W)]

    drive.recurrent = [(r, leaf(W)) for r, W in drive.recurrent]
    drive.feedforward = [(r, leaf(W)) for r, W in drive.feedforward]
    for name in PHYS_GRADS:
        value = getattr(p, name)
        if value is not None:
            value = value.detach().clone().requires_grad_(True)
            setattr(p, name, value)
            leaves[f"phys.{name}"] = value
    for name in ("g_clip", "dt", "surr_scale", "mg_c", "mg_a"):
        value = getattr(p, name)
        if value is not None:
            setattr(p, name, value.detach())
    run = dynamics.simulate(v, g, x, drive, p, probabilities=probabilities, **kw)
    loss = (run.output * readout(READOUT_SEED, run.output.shape)).sum()
    if probabilities:
        loss = loss + (run.probabilities * readout(READOUT_SEED + 2, run.output.shape)).sum()
    loss.backward()
    grads = {"loss": loss.detach()}
    for key, value in leaves.items():
        grads[key] = value.grad if value.grad is not None else torch.zeros_like(value)
    # Weight gradients, stored per weight tensor in the order save() numbers them.
    seen = {}
    for W in [W for _, W in drive.recurrent] + [W for _, W in drive.feedforward]:
        if id(W) not in seen:
            seen[id(W)] = len(seen)
            grads[f"W.{seen[id(W)]}"] = W.grad if W.grad is not None else torch.zeros_like(W)
    grads["spikes_sum"] = run.output.sum().detach()
    return grads


def recorded_fixture(reference: Path, name: str, state_key: str):
    with np.load(reference / "tests" / "fixtures" / f"{name}.npz") as data:
        raw = {k: data[k] for k in data.files}
    spikes = np.unpackbits(raw["spikes.bits"], axis=-1, count=int(raw["spikes.shape"][-1]))
    out = {
        "spikes": spikes.astype(bool),
        "voltages": raw["voltages"],
        "state_v": raw["state.v"],
        "state_g": raw[f"state.{state_key}"],
    }
    if "probabilities" in raw:
        out["probabilities"] = raw["probabilities"]
    return out


def scenario_cases(networks):
    """``name -> (build(batch) -> Built, probabilities, recorded fixture, state key)``."""
    rec, ff, SEED = networks.recurrent, networks.feedforward, networks.SEED
    learn_all = {
        "tau_mem": True, "theta": True, "U_reset": True, "E_L": True, "g_L": True,
        "tau_rise": True, "tau_decay": True, "E_syn": True, "g_bar": True,
    }  # fmt: skip
    learn_adapt = {
        "adapt": ["excitatory"], "tau_adapt": ["excitatory"], "E_adapt": True,
        "theta": True,
    }  # fmt: skip
    return {
        "recurrent_frozen": (lambda b: rec(b, SEED), False, "recurrent_frozen", "g"),
        "recurrent_scaling_factors": (
            lambda b: rec(b, SEED, scaling_factors=True), False,
            "recurrent_scaling_factors", "g",
        ),
        "feedforward_scaling_factors": (
            lambda b: ff(b, SEED), False, "feedforward_scaling_factors", "g_FF",
        ),
        "feedforward_probabilities": (
            lambda b: ff(b, SEED, probabilities=True), True,
            "feedforward_probabilities", "g_FF",
        ),
        "feedforward_learnt_weights": (
            lambda b: ff(b, SEED, learnt_weights=True), False,
            "feedforward_learnt_weights", "g_FF",
        ),
        "recurrent_refractory": (lambda b: rec(b, SEED, tau_ref=3.0), False, None, "g"),
        "recurrent_nmda": (lambda b: rec(b, SEED, mg=1.0), False, None, "g"),
        "recurrent_adaptation": (
            lambda b: rec(b, SEED, adapt=0.5, learn=learn_adapt), False, None, "g",
        ),
        "recurrent_stp": (lambda b: rec(b, SEED, stp=True), False, None, "g"),
        "recurrent_saturation": (lambda b: rec(b, SEED, saturation=0.3), False, None, "g"),
        "recurrent_learnt_physiology": (
            lambda b: rec(b, SEED, learn=learn_all, tau_ref=2.0), False, None, "g",
        ),
        "recurrent_learnt_weights": (
            lambda b: rec(b, SEED, learnt_weights=True), False, None, "g",
        ),
        "feedforward_features": (
            lambda b: ff(b, SEED, tau_ref=2.0, mg=1.0, adapt=0.3, stp=True), True,
            None, "g_FF",
        ),
    }  # fmt: skip


def make_scenario(name, spec, networks, dynamics, reference, batch=2, recurrent_gradients=False):
    build, probabilities, fixture, state_key = spec
    built = build(batch)
    model = built.model
    if recurrent_gradients:
        model.recurrent_gradients = True
    x = torch.from_numpy(built.input_spikes).float()[:, :T_FREE]
    drive, p, inputs, outputs = free_run(dynamics, model, x, probabilities)
    model.reset_state()
    grads = gradients(dynamics, model, x, probabilities)
    recorded = recorded_fixture(reference, fixture, state_key) if fixture else {}
    meta = dict(case=name, batch=batch, steps=T_FREE, grad_steps=GRAD_STEPS, window=WINDOW,
                readout_seed=READOUT_SEED, probabilities=probabilities,
                origin="reference tests/networks.py scenario")  # fmt: skip
    golden_io.save(HERE / f"{name}.npz", drive=drive, p=p, inputs=inputs,
                   outputs=outputs, grads=grads, recorded=recorded, meta=meta)  # fmt: skip
    s = outputs["spikes"]
    print(f"{name}: {int(s.sum())} spikes in {tuple(s.shape)}, loss {float(grads['loss']):.4f}")


# ---------------------------------------------------------------------------------------
# Configuration cases
# ---------------------------------------------------------------------------------------

SNAP = 50  # steps between recorded voltages
GRAD_STEPS_C2 = 150


def coalesced(W):
    """A ``SparseRows`` with each (row, target) pair once, duplicates summed in float32:
    the same numbers the dense matrix of the reference holds."""
    from wiretorch_b200.types import SparseRows

    n_rows, N = W.shape
    rows = torch.repeat_interleave(torch.arange(n_rows), W.row_ptr[1:] - W.row_ptr[:-1])
    sp = torch.sparse_coo_tensor(torch.stack([rows, W.cols.long()]), W.values.float(), (n_rows, N)).coalesce()
    r, c = sp.indices()
    row_ptr = torch.zeros(n_rows + 1, dtype=torch.int64)
    row_ptr[1:] = torch.cumsum(torch.bincount(r, minlength=n_rows), 0)
    return SparseRows(row_ptr, c.to(torch.int32), sp.values().contiguous(), N)


def dense_of(W):
    if not hasattr(W, "row_ptr"):
        return W
    n_rows, N = W.shape
    out = torch.zeros(n_rows, N)
    rows = torch.repeat_interleave(torch.arange(n_rows), W.row_ptr[1:] - W.row_ptr[:-1])
    out[rows, W.cols.long()] = W.values
    return out


def sparse_of(W):
    """A dense ``(n_rows, N)`` matrix as ``SparseRows`` (its non-zero entries)."""
    from wiretorch_b200.types import SparseRows

    W = W.detach().float()
    rows, cols = torch.nonzero(W, as_tuple=True)
    row_ptr = torch.zeros(W.shape[0] + 1, dtype=torch.int64)
    row_ptr[1:] = torch.cumsum(torch.bincount(rows, minlength=W.shape[0]), 0)
    return SparseRows(row_ptr, cols.to(torch.int32), W[rows, cols].contiguous(), W.shape[1])


def reference_objects(cfg):
    """The configuration's network as the reference's own ``Drive``, ``Gate`` and
    ``Physiology`` (dense weights), plus the same network with coalesced ``SparseRows``
    for saving."""
    from wiretorch.network_simulators import network as ref_net
    from wiretorch.network_simulators.conductance import dynamics as ref_dyn

    made = {}

    def co(W):
        if id(W) not in made:
            made[id(W)] = coalesced(W)
        return made[id(W)]

    rec = [(r, co(W)) for r, W in cfg.drive.recurrent]
    ff = [(r, co(W)) for r, W in cfg.drive.feedforward]
    dense = {}

    def de(W):
        if id(W) not in dense:
            dense[id(W)] = dense_of(W)
        return dense[id(W)]

    gates = [None if g is None else ref_net.Gate(g.params, g.stp, g.saturates, g.start, g.n)
             for g in (cfg.drive.gates or [])]  # fmt: skip
    ref_drive = ref_net.Drive(made=cfg.drive.made, scale=cfg.drive.scale,
                              recurrent=[(r, de(W)) for r, W in rec],
                              feedforward=[(r, de(W)) for r, W in ff], gates=gates)  # fmt: skip
    fields = {name: getattr(cfg.p, name) for name in golden_io.PHYSIOLOGY_FIELDS}
    ref_p = ref_dyn.Physiology(**fields, spike_mode=cfg.p.spike_mode)
    cfg.drive.recurrent, cfg.drive.feedforward = rec, ff
    return ref_drive, ref_p


def reference_free_run(dynamics, drive, p, x, v, g, kw, snap):
    """The reference's run of ``x`` in ``snap``-step calls (the state carried): spikes,
    the voltage after every call, and the final state."""
    spikes, v_snap = [], []
    kw = dict(kw)
    with torch.no_grad():
        for start in range(0, x.shape[1], snap):
            run = dynamics.simulate(v, g, x[:, start : start + snap], drive, p, **kw)
            spikes.append(run.output)
            v, g = run.v, run.syn
            for key in kw:
                kw[key] = getattr(run, key)
            v_snap.append(v.clone())
    return torch.cat(spikes, 1), torch.stack(v_snap), v, g, kw


def config_builders():
    from wiretorch_b200 import configs

    return {
        # C1 exactly as specified: 1,000 neurons, 8 trials, 1,000 steps
        "config_c1": (lambda: configs.c1(B=8, T=1000, device="cpu"), 1000),
        # C2's construction at 2,000 neurons: pair probabilities ~U(0, 0.05) (a tenth of
        # the degree), weights tripled, 200 inputs reaching each neuron with p 0.25 (half
        # the input count) at 0.7 of the weight: 8-15 Hz, as C2
        "config_c2": (lambda: configs.c2(B=2, T=400, device="cpu", N=2000, n_in=200, p_in=0.25,
                                         w_mu=-1.0 + math.log(3), w_mu_i=0.6 + math.log(3),
                                         w_in_mu=-0.5 + math.log(0.7)), 400),
        # C4's construction at 2,000 neurons in 200 types, mean out-degree 60: 4-9 Hz
        "config_c4": (lambda: configs.c4(B=2, T=600, device="cpu", N=2000, n_types=200, mean_degree=60.0), 600),
        # C5's construction (NMDA with Mg block, depression) at 2,000 neurons, mean
        # out-degree 60, connection length scaled with the density, weights 2.6-fold: 3-6 Hz
        "config_c5": (lambda: configs.c5(B=2, T=600, device="cpu", N=2000, mean_degree=60.0,
                                         lam=0.05 * 500 ** (1 / 3), w_e=1.2 * 2.6, w_in=30.0), 600),
    }  # fmt: skip


def make_config_case(name, build, T, dynamics):
    from wiretorch.training_utils.losses import VanRossumRateLoss

    torch.manual_seed(0)
    cfg = build()
    x = cfg.inputs(T=T, seed=1)
    v, g, kw = cfg.state()
    ref_drive, ref_p = reference_objects(cfg)
    spikes, v_snap, v_end, g_end, kw_end = reference_free_run(dynamics, ref_drive, ref_p, x, v, g, kw, SNAP)
    outputs = {"spikes": spikes, "v_snap": v_snap, "v": v_end, "g": g_end, **kw_end}
    grads = {}
    meta = dict(case=name, config=cfg.name, batch=cfg.B, steps=T, snap=SNAP, x_bits=True,
                n_in=cfg.n_in, origin="wiretorch_b200.configs network run by the reference's dynamics.simulate")  # fmt: skip
    inputs = {"x": x, "v": v, "g": g, **kw, "types": cfg.types}
    if name == "config_c2":
        # the learnt per-pair log scales, moved off zero, and the rate loss of C2
        log_sf = (0.2 * torch.randn(cfg.extra["log_sf_shape"], generator=torch.Generator().manual_seed(5)))
        log_sf.requires_grad_(True)
        ref_drive.scale = torch.exp(log_sf)[:, cfg.types]
        target = cfg.extra["target_rates"] * float(cfg.p.dt) / 1000.0
        loss_fn = VanRossumRateLoss(float(cfg.p.dt), 20.0, float(cfg.p.dt), GRAD_STEPS_C2)
        run = dynamics.simulate(v, g, x[:, :GRAD_STEPS_C2], ref_drive, ref_p, **kw)
        loss = loss_fn(target[:, None, :].expand(cfg.B, GRAD_STEPS_C2, cfg.N), output_spikes=run.output)
        loss.backward()
        grads = {"log_sf": log_sf.grad, "loss": loss.detach(), "spikes_sum": run.output.sum().detach()}
        inputs.update(log_sf=log_sf.detach(), target_rates=cfg.extra["target_rates"])
        meta.update(grad_steps=GRAD_STEPS_C2, tau_decay=20.0)
    cfg.drive.gates = cfg.drive.gates or []
    golden_io.save(HERE / f"{name}.npz", drive=cfg.drive, p=cfg.p, inputs=inputs, outputs=outputs,
                   grads=grads, recorded={}, meta=meta)  # fmt: skip
    rate = float(spikes.float().mean()) / (float(cfg.p.dt) / 1000.0)
    print(f"{name}: N={cfg.N}, {sum(int(W.cols.numel()) for W in {id(W): W for _, W in cfg.drive.recurrent}.values())} "
          f"recurrent edges, {int(spikes.sum())} spikes ({rate:.1f} Hz), {(HERE / f'{name}.npz').stat().st_size / 1e6:.2f} MB")


# ---------------------------------------------------------------------------------------
# The reference's at-scale statistics networks
# ---------------------------------------------------------------------------------------


def make_statistics_case(name, reference, networks, dynamics):
    """``statistics_<net>``: the network of the reference's ``STATS_NETWORKS[<net>]``
    with both recorded inputs and the rates its GPU simulator recorded."""
    sys.path.insert(0, str(reference / "tests" / "fixtures"))
    import generate  # the reference's fixture generator (its STATS_* constants)

    net = name.removeprefix("statistics_")
    builder, kwargs, n_steps = generate.STATS_NETWORKS[net]
    seeds = generate.STATS_INPUT_SEEDS
    builts = [builder(generate.STATS_BATCH, networks.SEED, n_steps=n_steps, input_seed=s, **kwargs) for s in seeds]
    model = builts[0].model
    drive, p = model._drive(), model._physiology()
    v, g, kw = engine_inputs(model)
    sparse = {}

    def sp(W):
        if id(W) not in sparse:
            sparse[id(W)] = sparse_of(W)
        return sparse[id(W)]

    from wiretorch_b200.types import Drive as WtDrive

    saved = WtDrive(made=drive.made, scale=drive.scale, recurrent=[(r, sp(W)) for r, W in drive.recurrent],
                    feedforward=[(r, sp(W)) for r, W in drive.feedforward], gates=list(drive.gates or []))  # fmt: skip
    xs = [torch.from_numpy(b.input_spikes).float() for b in builts]
    # the reference's CPU dynamics on the first input, 250-step calls as stats_run makes
    spikes, _, _, _, _ = reference_free_run(dynamics, drive, p, xs[0], v, g, kw, 250)
    with np.load(reference / "tests" / "fixtures" / "statistics.npz") as rec:
        recorded = {f"rates_{s}": rec[f"{net}.rates.{s}"] for s in seeds}
        recorded.update({f"population_rate_{s}": rec[f"{net}.population_rate.{s}"] for s in seeds})
        if f"{net}.spikes.bits" in rec.files:
            shape = tuple(rec[f"{net}.spikes.shape"])
            recorded["spikes"] = np.unpackbits(rec[f"{net}.spikes.bits"], axis=-1, count=shape[-1]).astype(bool)
    types = builts[0].structure["types"]
    inputs = {"v": v, "g": g, **kw, "types": torch.from_numpy(np.asarray(types))}
    for s, x in zip(seeds, xs):
        inputs[f"x_{s}"] = x
    meta = dict(case=name, batch=generate.STATS_BATCH, steps=n_steps, burn_in=generate.STATS_BURN_IN,
                chunk=250, seeds=list(seeds), x_bits=True, n_in=int(xs[0].shape[2]),
                origin=f"reference tests/fixtures/generate.py STATS_NETWORKS[{net!r}] and statistics.npz")  # fmt: skip
    golden_io.save(HERE / f"{name}.npz", drive=saved, p=p, inputs=inputs,
                   outputs={"spikes": spikes[:, generate.STATS_BURN_IN :]}, grads={}, recorded=recorded,
                   meta=meta)  # fmt: skip
    rates = spikes[:, generate.STATS_BURN_IN :].float().mean((0, 1)) * 1000.0
    print(f"{name}: CPU reference {float(rates.mean()):.2f} Hz, recorded {recorded[f'rates_{seeds[0]}'].mean():.2f} Hz, "
          f"{(HERE / f'{name}.npz').stat().st_size / 1e6:.2f} MB")


def make_current_statistics_case(name, reference, networks):
    """``curstats_<net>``: the current-based network of the reference's
    ``STATS_NETWORKS["current_<net>"]`` with both recorded inputs, the rates the
    reference recorded for it (``statistics_current.npz``, from its PyTorch
    current-based dynamics) and a run of the same dynamics here on the first input."""
    from wiretorch.network_simulators.current import dynamics as current_dynamics

    sys.path.insert(0, str(reference / "tests" / "fixtures"))
    import generate

    net = "current_" + name.removeprefix("curstats_")
    builder, kwargs, n_steps = generate.STATS_NETWORKS[net]
    seeds = generate.STATS_INPUT_SEEDS
    builts = [builder(generate.STATS_BATCH, networks.SEED, n_steps=n_steps, input_seed=s, **kwargs) for s in seeds]
    model = builts[0].model
    drive, p = model._drive(), model._physiology()
    v, I, kw = engine_inputs(model)
    sparse = {}

    def sp(W):
        if id(W) not in sparse:
            sparse[id(W)] = sparse_of(W)
        return sparse[id(W)]

    from wiretorch_b200.types import Drive as WtDrive

    saved = WtDrive(made=drive.made, scale=drive.scale, recurrent=[(r, sp(W)) for r, W in drive.recurrent],
                    feedforward=[(r, sp(W)) for r, W in drive.feedforward], gates=list(drive.gates or []),
                    recurrent_gradients=bool(drive.recurrent_gradients))  # fmt: skip
    xs = [torch.from_numpy(b.input_spikes).float() for b in builts]
    spikes, _, _, _, _ = reference_free_run(current_dynamics, drive, p, xs[0], v, I, kw, 250)
    with np.load(reference / "tests" / "fixtures" / "statistics_current.npz") as rec:
        recorded = {f"rates_{s}": rec[f"{net}.rates.{s}"] for s in seeds}
        recorded.update({f"population_rate_{s}": rec[f"{net}.population_rate.{s}"] for s in seeds})
        if f"{net}.spikes.bits" in rec.files:
            shape = tuple(rec[f"{net}.spikes.shape"])
            recorded["spikes"] = np.unpackbits(rec[f"{net}.spikes.bits"], axis=-1, count=shape[-1]).astype(bool)
    types = builts[0].structure["types"]
    inputs = {"v": v, "g": I, **kw, "types": torch.from_numpy(np.asarray(types))}
    for s, x in zip(seeds, xs):
        inputs[f"x_{s}"] = x
    meta = dict(case=name, batch=generate.STATS_BATCH, steps=n_steps, burn_in=generate.STATS_BURN_IN,
                chunk=250, seeds=list(seeds), x_bits=True, n_in=int(xs[0].shape[2]), family="current",
                dt=float(networks.DT),
                origin=f"reference tests/fixtures/generate.py STATS_NETWORKS[{net!r}] and statistics_current.npz")  # fmt: skip
    golden_io.save(HERE / f"{name}.npz", drive=saved, p=p, inputs=inputs,
                   outputs={"spikes": spikes[:, generate.STATS_BURN_IN :]}, grads={}, recorded=recorded,
                   meta=meta)  # fmt: skip
    rates = spikes[:, generate.STATS_BURN_IN :].float().mean((0, 1)) * 1000.0 / float(networks.DT)
    print(f"{name}: CPU reference {float(rates.mean()):.2f} Hz, recorded {recorded[f'rates_{seeds[0]}'].mean():.2f} Hz, "
          f"{(HERE / f'{name}.npz').stat().st_size / 1e6:.2f} MB")


# ---------------------------------------------------------------------------------------
# The loss filter and the van Rossum rate loss
# ---------------------------------------------------------------------------------------

LOSS_CHUNKS = 3


def make_loss_cases():
    """``loss_filter``: ``double_exponential`` of (B, T, N) trains over three chunks, the
    state carried as ``VanRossumLoss.smooth`` carries it, and the gradient of
    ``sum(smooth * R)`` per chunk; ``loss_van_rossum``: ``VanRossumRateLoss`` with C2's
    filter (rise dt, decay 20 ms) over three chunks, each chunk's loss and gradient with
    respect to the output spikes."""
    from wiretorch.training_utils.filtering import double_exponential
    from wiretorch.training_utils.losses import VanRossumRateLoss

    rng = np.random.default_rng(11)
    B, T, N, dt = 3, 60, 70, 0.1
    # filter: a mix of spikes and real values, rise 2 ms, decay 10 ms
    tau_r, tau_d = 2.0, 10.0
    t = torch.arange(T, dtype=torch.float32) * dt
    k_r, k_d = torch.exp(-t / tau_r), torch.exp(-t / tau_d)
    xs = [torch.from_numpy((rng.random((B, T, N)) < 0.05).astype(np.float32) + rng.normal(size=(B, T, N)).astype(np.float32) * 0.1)
          for _ in range(LOSS_CHUNKS)]  # fmt: skip
    Rs = [torch.from_numpy(rng.normal(size=(B, T, N)).astype(np.float32)) for _ in range(LOSS_CHUNKS)]
    arrays = dict(B=B, T=T, N=N, dt=dt, tau_rise=tau_r, tau_decay=tau_d)
    cr = cs = None
    for c in range(LOSS_CHUNKS):
        x = xs[c].clone().requires_grad_(True)
        rise, smooth = double_exponential(x, k_r, k_d, cr, cs)
        (smooth * Rs[c]).sum().backward()
        arrays.update({f"x.{c}": xs[c].numpy(), f"R.{c}": Rs[c].numpy(), f"rise.{c}": rise.detach().numpy(),
                       f"smooth.{c}": smooth.detach().numpy(), f"grad_x.{c}": x.grad.numpy()})  # fmt: skip
        cr, cs = rise[:, -1:].detach(), smooth[:, -1:].detach()
    np.savez_compressed(HERE / "loss_filter.npz", **arrays)
    # the van Rossum rate loss as the C2 training step uses it
    B, T, N = 4, 100, 90
    loss_fn = VanRossumRateLoss(dt, 20.0, dt, T)
    target = torch.from_numpy(rng.uniform(1.0, 30.0, (B, N)).astype(np.float32)) * dt / 1000.0
    arrays = dict(B=B, T=T, N=N, dt=dt, tau_rise=dt, tau_decay=20.0, target_rate=target.numpy())
    for c in range(LOSS_CHUNKS):
        s = torch.from_numpy((rng.random((B, T, N)) < 0.02).astype(np.float32)).requires_grad_(True)
        loss = loss_fn(target[:, None, :].expand(B, T, N), output_spikes=s)
        loss.backward()
        arrays.update({f"spikes.{c}": s.detach().numpy(), f"loss.{c}": loss.detach().numpy(),
                       f"grad_spikes.{c}": s.grad.numpy(),
                       f"carried.{c}": torch.stack([loss_fn.prev_output_rise, loss_fn.prev_output_smooth,
                                                    loss_fn.prev_target_rise, loss_fn.prev_target_smooth]).numpy()})  # fmt: skip
    np.savez_compressed(HERE / "loss_van_rossum.npz", **arrays)
    print("loss_filter, loss_van_rossum written")


def current_scenarios(networks):
    """The current-based family's cases: ``name -> (build(batch) -> Built, probabilities,
    recorded fixture)``, from the reference's ``tests/networks.py``."""
    SEED = networks.SEED
    return {
        "current_recurrent": (lambda b: networks.current_recurrent(b, SEED), False, "current_recurrent"),
        "current_feedforward": (lambda b: networks.current_feedforward(b, SEED), False, "current_feedforward"),
        "current_feedforward_probabilities": (
            lambda b: networks.current_feedforward_probabilities(b, SEED), True,
            "current_feedforward_probabilities",
        ),
        "current_recurrent_features": (
            lambda b: networks.current_recurrent(b, SEED, tau_ref=2.0, stp=True, adapt=0.3), False, None,
        ),
    }  # fmt: skip


CURRENT_PHYS_GRADS = ("theta", "U_reset", "beta", "U_rest", "R", "decay", "adapt", "adapt_decay")


def current_gradients(dynamics, model, x, probabilities):
    """Gradients of ``sum(spikes R) (+ sum(prob R2))`` over ``GRAD_STEPS`` steps of a
    current-based network with respect to its scale, weights, input and learnable
    physiology, through the recurrent spikes when the network's drive says so (the
    current-based networks' default)."""
    drive, p = model._drive(), model._physiology()
    v, I, kw = engine_inputs(model)
    x = x[:, :GRAD_STEPS].clone().requires_grad_(True)
    leaves = {"x": x}
    drive.scale = drive.scale.detach().clone().requires_grad_(True)
    leaves["scale"] = drive.scale
    made = {}

    def leaf(W):
        if id(W) not in made:
            made[id(W)] = W.detach().clone().requires_grad_(True)
        return made[id(W)]

    drive.recurrent = [(r, leaf(W)) for r, W in drive.recurrent]
    drive.feedforward = [(r, leaf(W)) for r, W in drive.feedforward]
    for name in ("sign", "surr_scale"):
        value = getattr(p, name)
        if isinstance(value, torch.Tensor):
            setattr(p, name, value.detach())
    for name in CURRENT_PHYS_GRADS:  # the learnable physiology, made leaves
        value = getattr(p, name)
        if isinstance(value, torch.Tensor):
            value = value.detach().clone().requires_grad_(True)
            setattr(p, name, value)
            leaves[f"phys.{name}"] = value
    run = dynamics.simulate(v, I, x, drive, p, probabilities=probabilities, **kw)
    loss = (run.output * readout(READOUT_SEED, run.output.shape)).sum()
    if probabilities:
        loss = loss + (run.probabilities * readout(READOUT_SEED + 2, run.output.shape)).sum()
    loss.backward()
    grads = {"loss": loss.detach()}
    for key, value in leaves.items():
        grads[key] = value.grad if value.grad is not None else torch.zeros_like(value)
    seen = {}
    for W in [W for _, W in drive.recurrent] + [W for _, W in drive.feedforward]:
        if id(W) not in seen:
            seen[id(W)] = len(seen)
            grads[f"W.{seen[id(W)]}"] = W.grad if W.grad is not None else torch.zeros_like(W)
    grads["spikes_sum"] = run.output.sum().detach()
    return grads


def make_current_case(name, spec, reference, batch=2):
    """A current-based network's free run through the reference's
    ``current/dynamics.py`` ``simulate``, with the reference suite's recording where it
    has one, and the gradients of a fixed readout of its first ``GRAD_STEPS`` steps."""
    from wiretorch.network_simulators.current import dynamics as current_dynamics

    build, probabilities, fixture = spec
    built = build(batch)
    x = torch.from_numpy(built.input_spikes).float()[:, :T_FREE]
    drive, p, inputs, outputs = free_run(current_dynamics, built.model, x, probabilities)
    built.model.reset_state()
    grads = current_gradients(current_dynamics, built.model, x, probabilities)
    recorded = recorded_fixture(reference, fixture, "I_syn") if fixture else {}
    meta = dict(case=name, batch=batch, steps=T_FREE, window=WINDOW, probabilities=probabilities,
                family="current", origin="reference tests/networks.py current-based network")  # fmt: skip
    meta.update(grad_steps=GRAD_STEPS, readout_seed=READOUT_SEED)
    golden_io.save(HERE / f"{name}.npz", drive=drive, p=p, inputs=inputs, outputs=outputs, grads=grads,
                   recorded=recorded, meta=meta)  # fmt: skip
    s = outputs["spikes"]
    print(f"{name}: {int(s.sum())} spikes in {tuple(s.shape)}, loss {float(grads['loss']):.4f}, "
          f"recurrent gradients {bool(drive.recurrent_gradients)}")  # fmt: skip


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("WIRETORCH_REFERENCE"))
    parser.add_argument("names", nargs="*")
    args = parser.parse_args()
    if not args.reference:
        sys.exit("give --reference (a wiretorch checkout) or WIRETORCH_REFERENCE")
    reference = Path(args.reference)
    torch.set_num_threads(1)
    networks, dynamics = import_reference(reference)
    cases = scenario_cases(networks)
    configs_ = config_builders()
    stats = ["statistics_recurrent", "statistics_feedforward"]
    current = current_scenarios(networks)
    curstats = ["curstats_recurrent", "curstats_feedforward"]
    todo = args.names or [*cases, "recurrent_gradients", *configs_, *stats, "loss", *current, *curstats]
    for name in todo:
        if name in current:
            make_current_case(name, current[name], reference)
        elif name in curstats:
            make_current_statistics_case(name, reference, networks)
        elif name in configs_:
            make_config_case(name, *configs_[name], dynamics)
        elif name in stats:
            make_statistics_case(name, reference, networks, dynamics)
        elif name == "loss":
            make_loss_cases()
        elif name == "recurrent_gradients":
            make_scenario(name, cases["recurrent_scaling_factors"][:2] + (None, "g"),
                          networks, dynamics, reference, recurrent_gradients=True)  # fmt: skip
        elif name in cases:
            make_scenario(name, cases[name], networks, dynamics, reference)
        else:
            sys.exit(f"unknown case {name}")


if __name__ == "__main__":
    main()
