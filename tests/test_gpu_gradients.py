"""Surrogate gradients of the engine against wiretorch's own (golden cases), on the B200.

The loss is the reference suite's fixed random readout of the spikes,
``sum(spikes * R)`` (plus ``sum(probabilities * R2)`` where the network outputs them),
over the first ``grad_steps`` steps (``tests/harness.py:145-156`` of the reference).
Every differentiable input of the engine is a leaf: the kernel scales ``(K, N)``, the
weights, the input, and the learnt physiology; each gradient must match the reference's
to 1e-3 of its largest entry (the reference allows its own CUDA kernels 2e-3,
``tests/test_gradients.py:19``). Weight gradients are compared on the weights' non-zero
entries (see ``wiretorch_b200.autograd``).
"""

import numpy as np
import pytest
import torch

import golden_io
from wiretorch_b200 import engine
from wiretorch_b200.types import PHYSIOLOGY

pytestmark = pytest.mark.gpu

TOL = 1e-3
CASES = golden_io.cases()


def readout(seed, shape):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.normal(size=shape).astype(np.float32)).cuda()


def _leaf(t):
    return t.detach().clone().requires_grad_(True)


def engine_gradients(name, recurrent=None):
    drive, p, d, meta = golden_io.load(name, "cuda")
    if recurrent is not None:
        drive.recurrent_gradients = recurrent
    T = meta["grad_steps"]
    x = _leaf(torch.from_numpy(d["in.x"][:, :T]).cuda())
    drive.scale = _leaf(drive.scale)
    made = {}

    def leaf_w(W):
        if id(W) not in made:
            made[id(W)] = _leaf(W)
        return made[id(W)]

    drive.recurrent = [(r, leaf_w(W)) for r, W in drive.recurrent]
    drive.feedforward = [(r, leaf_w(W)) for r, W in drive.feedforward]
    phys = {}
    for name_ in PHYSIOLOGY:
        if getattr(p, name_) is not None:
            phys[name_] = _leaf(getattr(p, name_))
            setattr(p, name_, phys[name_])
    kw = {}
    for key in ("refractory", "gating", "adaptation"):
        if f"in.{key}" in d:
            kw[key] = torch.from_numpy(d[f"in.{key}"]).cuda()
    v = torch.from_numpy(d["in.v"]).cuda()
    g = torch.from_numpy(d["in.g"]).cuda()
    run = engine.simulate(v, g, x, drive, p, probabilities=meta["probabilities"], **kw)
    loss = (run.output * readout(meta["readout_seed"], run.output.shape)).sum()
    if meta["probabilities"]:
        loss = loss + (run.probabilities * readout(meta["readout_seed"] + 2, run.output.shape)).sum()
    loss.backward()
    grads = {"x": x.grad, "scale": drive.scale.grad}
    for key, t in phys.items():
        grads[f"phys.{key}"] = t.grad
    seen = []
    for W in [W for _, W in drive.recurrent] + [W for _, W in drive.feedforward]:
        if all(W is not s for s in seen):
            grads[f"W.{len(seen)}"] = W.grad
            seen.append(W)
    masks = {f"W.{i}": (W.detach() != 0).cpu().numpy() for i, W in enumerate(seen)}
    return float(loss), run.output, grads, d, masks


@pytest.mark.parametrize("name", CASES)
def test_gradients_match_reference(name):
    loss, spikes, grads, d, masks = engine_gradients(name)
    T = spikes.shape[1]
    np.testing.assert_array_equal(spikes.detach().cpu().numpy() > 0.5, d["out.spikes"][:, :T])
    np.testing.assert_allclose(loss, float(d["grad.loss"]), rtol=1e-4, atol=1e-4)
    for key, got in grads.items():
        expected = d[f"grad.{key}"]
        if got is None:
            assert np.abs(expected).max() == 0, f"{key}: no gradient, expected one"
            continue
        got = got.detach().cpu().numpy()
        if key.startswith("W."):
            got, expected = got[masks[key]], expected[masks[key]]
        scale = max(float(np.abs(expected).max()), 1e-12)
        np.testing.assert_allclose(got, expected, rtol=0, atol=TOL * scale, err_msg=key)


def test_recurrent_carry_matters():
    """The recurrent case's gradients without the carry along the recurrent edges miss
    the reference's by far more than the tolerance: the carry is what makes them match."""
    _, _, grads, d, masks = engine_gradients("recurrent_gradients", recurrent=False)
    worst = 0.0
    for key, got in grads.items():
        if got is None or key.startswith("W."):
            continue
        expected = d[f"grad.{key}"]
        scale = max(float(np.abs(expected).max()), 1e-12)
        worst = max(worst, float(np.abs(got.detach().cpu().numpy() - expected).max()) / scale)
    assert worst > 10 * TOL
