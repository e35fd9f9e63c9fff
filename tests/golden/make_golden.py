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

The configuration cases (``config_c1`` ...) build their network with
``wiretorch_b200.configs`` and simulate it through the reference's public
``ConductanceLIFNetwork``.
"""

from __future__ import annotations

import argparse
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
    todo = args.names or [*cases, "recurrent_gradients"]
    for name in todo:
        if name == "recurrent_gradients":
            make_scenario(name, cases["recurrent_scaling_factors"][:2] + (None, "g"),
                          networks, dynamics, reference, recurrent_gradients=True)  # fmt: skip
        elif name in cases:
            make_scenario(name, cases[name], networks, dynamics, reference)
        else:
            sys.exit(f"unknown case {name}")


if __name__ == "__main__":
    main()
