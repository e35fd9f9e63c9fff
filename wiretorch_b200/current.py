"""The current-based LIF family on the engine's kernels: ``simulate`` with the signature
of wiretorch's ``network_simulators/current/engine.py:67-70``, run by the same persistent
forward kernel as the conductance family in its current-based mode (``WT_F_CURRENT``).

A wiretorch current-based network calls its engine through its ``_engine`` class
attribute (``current/network.py:67``); setting

    CurrentNetwork._engine = wiretorch_b200.current

routes it here. The step is the reference's (``current/dynamics.py:116-205``): the spike
from the voltage; each synapse type's current decays and takes this step's input (every
pathway's activation times its kernel, the scaling factor into each type it makes); the
adaptation current rises by the spike; and the voltage integrates
``v <- beta v + (1 - beta) (U_rest + R (sum_j sign_j I_j - I_a))`` and resets. The kernel
differs from its conductance mode in two places: the membrane update, and when a step's
input enters — here the same step's membrane sees it, so every warp scatters the step's
events first and a grid barrier completes them before the neurons update (the
conductance step reads them a step later). The synaptic input is summed in fixed point
over all pathways (order-independent), where the reference adds pathway after pathway in
float32.

With ``engine.POOL_SYNAPSES`` (``WIRETORCH_POOL_SYNAPSES=1``), synapse types of the same
decay and sign share a channel, as in the conductance family: the returned currents then
hold each pool's sum at its first member type.

The kernel reads the current-based parameters in the conductance fields of ``WtNet``
(``U_rest`` as ``E_L``, ``R`` as ``C_m``, the types' signs as ``E_syn``; each type a single
exponential). Gradients flow to the scales, the weights and the input (and, with
``Drive.recurrent_gradients``, the current-based networks' default, through the recurrent
spikes): the backward kernel's current-based adjoint, then the engine's edge gradients;
and to a learnt physiology (``theta``, ``U_reset``, ``U_rest``, ``R``, ``beta``, the
synaptic ``decay``, ``adapt``, ``adapt_decay``), from per-(trial, neuron) sums the
same reverse scan accumulates.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from wiretorch_b200 import engine, plan as _plan
from wiretorch_b200.types import Run


@dataclass
class _Fields:
    """A current-based ``Physiology`` in the fields the plan and the kernel read."""

    theta: torch.Tensor
    U_reset: torch.Tensor
    E_L: torch.Tensor  # U_rest
    C_m: torch.Tensor  # R
    beta: torch.Tensor
    E_syn: torch.Tensor  # sign
    g_clip: torch.Tensor
    decay: torch.Tensor  # (2, S): no rise, the current's decay
    jump: torch.Tensor  # (2, S): 0, 1
    surr_scale: torch.Tensor
    spike_mode: str
    n_ref: torch.Tensor | None
    adapt: torch.Tensor | None
    adapt_decay: torch.Tensor | None
    E_adapt: None = None
    mg_c: None = None
    mg_a: None = None
    dt: float = 1.0  # not used by the current-based step
    current: bool = True


_FIELDS: dict = {}
_SOURCE_FIELDS = ("theta", "U_reset", "U_rest", "R", "beta", "sign", "decay", "surr_scale", "n_ref", "adapt",
                  "adapt_decay")  # fmt: skip


def _fields(p) -> _Fields:
    """The fields of ``p``; the per-neuron tensors are ``p``'s own, so that gradients
    reach them, and the decays are stacked under autograd when they are learnt (then the
    fields are built afresh for every call, the stack being part of its graph)."""
    learnt = torch.is_grad_enabled() and p.decay.requires_grad
    # cached per physiology object and its very tensors (a field replaced is a new entry)
    parts = tuple(getattr(p, n) for n in _SOURCE_FIELDS)
    key = (id(p), *map(id, parts))
    hit = _FIELDS.get(key)
    if not learnt and hit is not None and all(a is b for a, b in zip(hit[0], (p, *parts))):
        return hit[1]
    S = p.sign.shape[0]
    dev = p.sign.device
    zeros = torch.zeros(S, device=dev)
    f = _Fields(
        theta=p.theta, U_reset=p.U_reset, E_L=p.U_rest, C_m=p.R, beta=p.beta,
        E_syn=p.sign.detach().float(), g_clip=torch.full((S,), float("inf"), device=dev),
        decay=torch.stack([zeros, p.decay.float() if learnt else p.decay.detach().float()]),
        jump=torch.stack([zeros, torch.ones(S, device=dev)]),
        surr_scale=p.surr_scale, spike_mode=p.spike_mode, n_ref=p.n_ref,
        adapt=p.adapt, adapt_decay=p.adapt_decay,
    )  # fmt: skip
    if not learnt:
        if len(_FIELDS) > 64:
            _FIELDS.clear()
        _FIELDS[key] = ((p, *parts), f)
    return f


#: Parameters of a current-based ``Physiology`` that may carry gradients.
PHYSIOLOGY = ("theta", "U_reset", "beta", "U_rest", "R", "decay", "adapt", "adapt_decay")


def simulate(
    v, I, x, drive, p, *, refractory=None, gating=None, adaptation=None,
    probabilities=False, track=False, track_batch_idx=None, retain=None,
) -> Run:  # fmt: skip
    """Simulate ``x.shape[1]`` steps from state ``(v, I)`` (``(B, N)``, ``(B, N, S)``) with
    input ``x`` ``(B, T, n_in)``: the reference's ``current/engine.py`` ``simulate``, same
    arguments and result (``Run.syn`` the currents ``(B, N, S)``; tracked ``v``, ``I``
    ``(Bt, T, N, S)`` after each step's input, and ``a``)."""
    if retain is not None:
        raise NotImplementedError("track_gradients retains a per-step autograd graph, which the kernels do not build")
    if not x.is_cuda:
        raise RuntimeError("wiretorch_b200 runs on CUDA tensors only (no CPU path)")
    weights = [W for _, W in drive.recurrent] + [W for _, W in drive.feedforward]
    learnt = [n for n in PHYSIOLOGY if isinstance(getattr(p, n, None), torch.Tensor) and getattr(p, n).requires_grad]
    if torch.is_grad_enabled() and getattr(p.sign, "requires_grad", False):
        raise NotImplementedError("current-based networks: the synapse types' signs are not learnable")
    grad = torch.is_grad_enabled() and (
        drive.scale.requires_grad or x.requires_grad or any(getattr(W, "requires_grad", False) for W in weights)
        or bool(learnt)
    )
    B, T, n_in = x.shape
    device = x.device
    f = _fields(p)
    plan = engine.get_plan(drive, f, B, n_in, device)  # pooled as engine.POOL_SYNAPSES says
    # the kernel's state (B, 2, S, N) seen as the conductance layout (B, N, 2, S): the
    # currents are the decay component, the rise component zero
    S = plan.ch.S  # synapse types (pooled into plan.ch.Sp channels by _internal_g)
    g = torch.zeros((B, v.shape[1], 2, S), device=device)
    g[:, :, 1] = I.detach().to(device, torch.float32)
    if grad:
        from wiretorch_b200 import autograd

        run = autograd.simulate_with_grad(plan, v, g, x, drive, f, refractory, gating, adaptation, probabilities,
                                          track, track_batch_idx)  # fmt: skip
        run.syn = run.syn[:, :, 1]
        if run.tracked is not None:
            run.tracked["I"] = run.tracked.pop("g")[..., 1, :]
            run.tracked.pop("I_leak", None)
        return run
    _plan.fold(plan, drive.scale)
    v_k, g_k, counter, g_a, gating_k = engine._prepare_state(plan, v, g, refractory, gating, adaptation, f)
    track_b = -1 if track_batch_idx is None else int(track_batch_idx)
    with torch.no_grad():
        out = engine.run_forward(plan, f, x.detach().float(), v_k, g_k, counter, g_a, gating_k,
                                 probabilities=probabilities, track=track, track_b=track_b)  # fmt: skip
    tracked = None
    if track:
        tracked = {"v": out["track_v"], "I": engine._external_tracked_g(plan, out["track_g"])[..., 1, :]}
        if "track_a" in out:
            tracked["a"] = out["track_a"]
    return Run(
        output=out["spikes"],
        v=v_k,
        syn=engine._external_g(plan, g_k)[:, :, 1],
        probabilities=out.get("prob"),
        tracked=tracked,
        refractory=counter if refractory is not None or p.n_ref is not None else None,
        gating=gating_k,
        adaptation=g_a,
    )
