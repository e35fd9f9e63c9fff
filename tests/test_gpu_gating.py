"""Gated sources stepped through their resolved gating give exactly the results of
walking their slots.

A gated source that owns one slot is stepped by the forward kernel from the per-source
table ``src_gate`` (its gate and row, resolved once per neuron group); a warp holding a
source with several slots walks every slot as before (``emit``). Both must produce the
same spikes, state, gating state and saved factors, bit for bit: the synaptic sums are
fixed point, so the order in which events land does not matter. Checked on the C5
model (short-term depression on both recurrent pathways) as built, and with a third
pathway (depression and receptor saturation) from 200 of its excitatory neurons, whose
sources then own two gated slots each.
"""

import math

import pytest
import torch

from wiretorch_b200 import configs, engine
from wiretorch_b200.types import Gate, SparseRows

pytestmark = pytest.mark.gpu


def _c5_small():
    return configs.c5(B=3, T=120, device="cuda", N=4000, mean_degree=400.0, lam=0.05 * 250 ** (1 / 3),
                      w_e=3.0, w_in=30.0)  # fmt: skip


def _doubled(cfg, n=200):
    """``cfg`` with a third recurrent pathway: the first ``n`` excitatory sources again,
    half their weights, AMPA only, with depression (U 0.5) and saturation."""
    d = cfg.drive
    rows_e, W_e = d.recurrent[0]
    end = int(W_e.row_ptr[n])
    W2 = SparseRows(W_e.row_ptr[: n + 1].clone(), W_e.cols[:end].clone(), 0.5 * W_e.values[:end], W_e.n_targets)
    dev = rows_e.device
    made = torch.cat([d.made[:2], torch.tensor([[1, 0, 0, 0]], dtype=torch.bool, device=dev), d.made[2:]])
    scale = torch.cat([d.scale[:2], torch.ones(1, cfg.N, device=dev), d.scale[2:]])
    R0 = cfg.extra["gating"].shape[1]
    params = torch.tensor([0.8, math.exp(-0.1 / 5.0), 0.5, math.exp(-0.1 / 300.0), 0.0], device=dev)
    gates = [d.gates[0], d.gates[1], Gate(params, stp=True, saturates=True, start=R0, n=n), None]
    d.recurrent = [d.recurrent[0], d.recurrent[1], (rows_e[:n].clone(), W2)]
    d.made, d.scale, d.gates = made, scale, gates
    extra = torch.empty((cfg.B, 3 * n), device=dev)
    extra[:, :n], extra[:, n : 2 * n], extra[:, 2 * n :] = 0.5, 1.0, 0.0
    cfg.extra["gating"] = torch.cat([cfg.extra["gating"], extra], 1)
    return cfg


def _run(cfg, x, walk, grad=False):
    """One forward (and, with ``grad``, the gradient of the summed spikes' filtered
    trace with respect to the pathway scales), with the gate table, or without it
    (``walk``: every gated source walks its slots)."""
    scale = cfg.drive.scale.detach().clone().requires_grad_(grad)
    cfg.drive.scale = scale
    plan = engine.get_plan(cfg.drive, cfg.p, cfg.B, cfg.n_in, x.device)
    table = plan.tensors.pop("src_gate") if walk else None
    try:
        v, g, kw = cfg.state()
        if grad:
            run = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
            assert engine.get_plan(cfg.drive, cfg.p, cfg.B, cfg.n_in, x.device) is plan
            (run.output * torch.linspace(0.0, 1.0, run.output.shape[1], device=x.device)[None, :, None]).sum().backward()
            cfg.drive.scale = scale.detach()
            return run, scale.grad
        with torch.no_grad():
            return engine.simulate(v, g, x, cfg.drive, cfg.p, **kw), None
    finally:
        if table is not None:
            plan.tensors["src_gate"] = table


@pytest.mark.parametrize("doubled", [False, True], ids=["single-slot", "two-slot"])
def test_resolved_gating_matches_walking_the_slots(doubled):
    cfg = _c5_small()
    if doubled:
        cfg = _doubled(cfg)
    x = cfg.inputs(seed=5)
    table = engine.get_plan(cfg.drive, cfg.p, cfg.B, cfg.n_in, x.device).tensors["src_gate"]
    assert int((table[:, 0] == -2).sum()) == (200 if doubled else 0)
    assert int((table[:, 0] >= 0).sum()) == cfg.N - (200 if doubled else 0)
    fast, _ = _run(cfg, x, walk=False)
    slow, _ = _run(cfg, x, walk=True)
    assert float(fast.output.sum()) > 20  # the network is active
    for name in ("output", "v", "syn", "gating", "refractory"):
        a, b = getattr(fast, name), getattr(slow, name)
        assert torch.equal(a, b), name
    # the third pathway's synapses depress and saturate
    if doubled:
        R0 = cfg.extra["gating"].shape[1] - 600
        assert float(fast.gating[:, R0 + 200 : R0 + 400].min()) < 0.99
        assert float(fast.gating[:, R0 + 400 :].max()) > 0.0


def test_resolved_gating_gradients_match():
    """Saved gating factors (training runs) are the same: so are the scale gradients."""
    cfg = _doubled(_c5_small())
    x = cfg.inputs(seed=6)[:, :60].contiguous()
    fast, g_fast = _run(cfg, x, walk=False, grad=True)
    slow, g_slow = _run(cfg, x, walk=True, grad=True)
    assert torch.equal(fast.output, slow.output)
    assert g_fast is not None and float(g_fast.abs().sum()) > 0
    torch.testing.assert_close(g_fast, g_slow, rtol=1e-5, atol=1e-6 * float(g_slow.abs().max()))

