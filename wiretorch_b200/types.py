"""The data the engine takes and returns, field for field as wiretorch names them.

A network hands the engine one ``Drive`` (its pathways' weights and kernel scales),
one ``Physiology`` (every parameter of the dynamics) and the state; the engine returns
a ``Run``. These mirror ``wiretorch.network_simulators.network.Drive`` / ``Gate`` /
``Run`` (``network_simulators/network.py:105-157, 160-183, 321-351``) and
``wiretorch.network_simulators.conductance.dynamics.Physiology``
(``conductance/dynamics.py:56-92``): the engine reads them by attribute, so the
reference's own objects are accepted unchanged, and these classes let a caller (and the
test suite) build them without the reference installed.

One addition: a recurrent or feedforward pathway may give its weights as a
``SparseRows`` (CSR rows over the targets) instead of a dense ``(n_rows, N)`` matrix, for
connectomes whose dense weights would not fit (the reference holds them dense).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class SparseRows:
    """A pathway's weights as CSR rows: row ``r`` (the pathway's ``r``-th source)
    reaches targets ``cols[row_ptr[r]:row_ptr[r+1]]`` with weights ``values[...]``.

    ``row_ptr`` ``(n_rows + 1,)`` int64, ``cols`` ``(E,)`` int32, ``values`` ``(E,)``
    float32, on the simulation device; ``n_targets`` is ``N``. Pathways of one source
    cell type share the same object, as they share the dense tensor in the reference.
    """

    row_ptr: torch.Tensor
    cols: torch.Tensor
    values: torch.Tensor
    n_targets: int

    @property
    def shape(self) -> tuple[int, int]:
        return (self.row_ptr.numel() - 1, self.n_targets)

    @property
    def requires_grad(self) -> bool:
        return self.values.requires_grad


@dataclass(frozen=True)
class Gate:
    """A pathway's presynaptic dynamics over its ``n`` source rows
    (``network_simulators/network.py:160-183``).

    ``params`` ``(5,)``: the saturation ``c``, the per-step decay of the receptors'
    gating, the release probability at rest ``U``, and the per-step decays of the
    resources' deficit and of the facilitation. Its columns of the gating state
    ``(B, R)``, from ``start``: with ``stp`` the release probabilities ``u`` then the
    resources ``x`` (``n`` each), then if it ``saturates`` the receptors' gating.
    """

    params: torch.Tensor
    stp: bool
    saturates: bool
    start: int
    n: int

    @property
    def width(self) -> int:
        return self.n * (2 * self.stp + self.saturates)

    @property
    def columns(self) -> slice:
        return slice(self.start, self.start + self.width)


@dataclass
class Drive:
    """The synaptic drive of one forward call (``network_simulators/network.py:105``).

    ``made`` ``(K, S)`` bool: the synapse types each pathway makes; ``scale`` ``(K, N)``
    multiplies its kernel per target neuron. Recurrent pathways come first; each is
    ``(rows, W)``: its source neurons (rows of the network's own output, or input
    columns for a feedforward pathway) and their ``(n_rows, N)`` weights (dense, or a
    ``SparseRows``). ``gates`` per pathway: its ``Gate`` or None.
    """

    made: torch.Tensor
    scale: torch.Tensor
    recurrent: list = field(default_factory=list)
    feedforward: list = field(default_factory=list)
    differentiable_inputs: slice | None = None
    recurrent_gradients: bool = False
    gates: list = field(default_factory=list)

    def gate(self, k: int):
        return self.gates[k] if self.gates else None

    @property
    def gated(self) -> bool:
        return any(g is not None for g in self.gates)


@dataclass
class Physiology:
    """Every parameter of the dynamics (``conductance/dynamics.py:56-92``).

    Per neuron ``(N,)``: ``theta``, ``U_reset``, ``E_L``, ``C_m``, ``beta`` (the leak's
    per-step decay); per synapse type ``(S,)``: ``E_syn``, ``g_clip``; ``decay`` and
    ``jump`` ``(2, S)``: per-step decay and per-unit-input jump of the rise and decay
    components. ``n_ref`` ``(N,)`` int32 refractory periods in steps (None: none);
    ``mg_c``, ``mg_a`` ``(S,)`` the Mg block (None: none); ``adapt``, ``adapt_decay``,
    ``E_adapt`` ``(N,)`` the adaptation (None: none adapts).
    """

    theta: torch.Tensor
    U_reset: torch.Tensor
    E_L: torch.Tensor
    C_m: torch.Tensor
    beta: torch.Tensor
    E_syn: torch.Tensor
    g_clip: torch.Tensor
    decay: torch.Tensor
    jump: torch.Tensor
    dt: torch.Tensor
    surr_scale: torch.Tensor
    spike_mode: str = "deterministic"
    storage_dtype: torch.dtype = torch.float32
    n_ref: torch.Tensor | None = None
    mg_c: torch.Tensor | None = None
    mg_a: torch.Tensor | None = None
    adapt: torch.Tensor | None = None
    adapt_decay: torch.Tensor | None = None
    E_adapt: torch.Tensor | None = None


@dataclass
class CurrentPhysiology:
    """Every parameter of the current-based dynamics (``current/dynamics.py:56-85``).

    Per neuron ``(N,)``: ``theta``, ``U_reset``, ``beta`` (the leak's per-step decay),
    ``U_rest`` (the voltage the leak relaxes to), ``R`` (the membrane resistance); per
    synapse type ``(S,)``: ``sign`` (+1 or -1) and ``decay`` (the current's per-step
    decay). ``n_ref`` ``(N,)`` int32 refractory periods in steps (None: none); ``adapt``,
    ``adapt_decay`` ``(N,)`` the adaptation current's rise per spike and decay (None:
    none adapts).
    """

    theta: torch.Tensor
    U_reset: torch.Tensor
    beta: torch.Tensor
    U_rest: torch.Tensor
    R: torch.Tensor
    sign: torch.Tensor
    decay: torch.Tensor
    surr_scale: torch.Tensor
    spike_mode: str = "deterministic"
    storage_dtype: torch.dtype = torch.float32
    n_ref: torch.Tensor | None = None
    adapt: torch.Tensor | None = None
    adapt_decay: torch.Tensor | None = None


@dataclass
class Run:
    """What a simulation produced (``network_simulators/network.py:321-351``).

    ``output`` ``(B, T, N)`` spikes; ``v`` ``(B, N)`` and ``syn`` ``(B, N, 2, S)`` the
    state after the last step; ``refractory`` the steps of refractory period left,
    ``gating`` the presynaptic pathways' state, ``adaptation`` the adaptation
    conductances; ``tracked`` per-step variables when tracking.
    """

    output: torch.Tensor
    v: torch.Tensor
    syn: torch.Tensor
    probabilities: torch.Tensor | None = None
    tracked: dict | None = None
    refractory: torch.Tensor | None = None
    gating: torch.Tensor | None = None
    adaptation: torch.Tensor | None = None

    @property
    def spikes(self) -> torch.Tensor:
        return self.output

    @property
    def g(self) -> torch.Tensor:
        return self.syn


#: The physiology that can be learnt, in the order the backward kernel reports it
#: (``conductance/engine.py:190-193``).
PHYSIOLOGY = (
    "theta", "U_reset", "E_L", "C_m", "beta", "E_syn", "decay", "jump",
    "adapt", "adapt_decay", "E_adapt",
)  # fmt: skip
