"""The current-based family (``wiretorch_b200.current``, the forward kernel's
``WT_F_CURRENT`` mode) against the reference's own current-based dynamics
(``network_simulators/current/dynamics.py``) on its test networks (golden cases
``current_*``; three of them also match the reference suite's recordings), on the B200.

* **Lockstep**: restart from every recorded window state and take the window's steps;
  spikes must match exactly (a neuron within 1e-4 of threshold excused, at most 1% of
  trial-windows), voltages within 1e-5 plus 1e-6 relative and currents within 1e-5
  relative.
* **Free run**: the whole 200-step input from the initial state gives exactly the
  recorded spike raster.
* **Gradients**: of the reference suite's fixed random readout of the spikes (plus the
  probabilities where the network outputs them) over the first 100 steps, with respect
  to the scales, the weights, the input and the learnable physiology, each within 1e-3 of
  its largest entry; through the recurrent spikes where the network's drive asks (the
  family's default).

Voltages are in the family's natural units (reset 0, threshold 1): 1e-5 is a hundred-
thousandth of the reset-to-threshold gap; the relative 1e-6 (eight float32 ulps) covers
strongly inhibited neurons far below reset, where over 200 steps of free run the two
summation orders drift by a few ulps. The kernel sums a step's synaptic input over all
pathways in fixed point; the reference adds pathway after pathway in float32.
"""

import numpy as np
import pytest
import torch

import golden_io
from wiretorch_b200 import current, engine

pytestmark = pytest.mark.gpu

CASES = golden_io.current_cases()
THRESHOLD_MARGIN = 1e-4
V_ATOL, V_RTOL = 1e-5, 1e-6
I_RTOL, I_ATOL = 1e-5, 1e-6


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _kw(d, prefix, w=None):
    out = {}
    for key in ("refractory", "gating", "adaptation"):
        name = f"{prefix}{key}"
        if name in d:
            out[key] = _t(d[name] if w is None else d[name][w])
    return out


def _run(drive, p, meta, x, v, I, kw):
    with torch.no_grad():
        return current.simulate(_t(v), _t(I), _t(x), drive, p, **kw, probabilities=meta["probabilities"],
                                track=True, track_batch_idx=None)  # fmt: skip


def test_cases_exist():
    assert len(CASES) >= 4, CASES


@pytest.mark.parametrize("name", CASES)
def test_lockstep(name):
    drive, p, d, meta = golden_io.load(name, "cuda")
    x = d["in.x"]
    W, B = meta["window"], x.shape[0]
    theta = p.theta.cpu().numpy()
    excused = 0
    for w, start in enumerate(range(0, x.shape[1], W)):
        stop = start + W
        run = _run(drive, p, meta, x[:, start:stop], d["out.win_v"][w], d["out.win_g"][w], _kw(d, "out.win_", w))
        spikes = run.output.cpu().numpy() > 0.5
        ok = np.ones(B, bool)
        diff = spikes != d["out.spikes"][:, start:stop]
        if diff.any():
            v_enter = np.concatenate([d["out.win_v"][w][:, None], d["out.v_track"][:, start : stop - 1]], 1)
            for b, t, n in zip(*np.nonzero(diff)):
                if ok[b]:
                    margin = abs(v_enter[b, t, n] - theta[n])
                    assert margin < THRESHOLD_MARGIN, (w, b, t, n, margin)
                    ok[b] = False
                    excused += 1
        np.testing.assert_allclose(run.tracked["v"].cpu().numpy()[ok], d["out.v_track"][ok, start:stop],
                                   rtol=V_RTOL, atol=V_ATOL, err_msg=f"window {w}")  # fmt: skip
        np.testing.assert_allclose(run.syn.cpu().numpy()[ok], d["out.win_g"][w + 1][ok], rtol=I_RTOL, atol=I_ATOL,
                                   err_msg=f"window {w}")  # fmt: skip
        for key in ("refractory", "gating", "adaptation"):
            if f"out.win_{key}" in d and getattr(run, key) is not None:
                np.testing.assert_allclose(getattr(run, key).cpu().numpy()[ok], d[f"out.win_{key}"][w + 1][ok],
                                           rtol=1e-5, atol=1e-6, err_msg=f"{key}, window {w}")  # fmt: skip
        if meta["probabilities"]:
            np.testing.assert_allclose(run.probabilities.cpu().numpy()[ok], d["out.prob"][ok, start:stop], rtol=0,
                                       atol=1e-5)  # fmt: skip
    assert excused <= 0.01 * (x.shape[1] // W) * B


@pytest.mark.parametrize("name", CASES)
def test_free_run_is_spike_exact(name):
    drive, p, d, meta = golden_io.load(name, "cuda")
    run = _run(drive, p, meta, d["in.x"], d["in.v"], d["in.g"], _kw(d, "in."))
    spikes = run.output.cpu().numpy() > 0.5
    differs = (spikes != d["out.spikes"]).any(axis=(0, 2))
    assert not differs.any(), f"first divergence at step {int(np.argmax(differs))}"
    np.testing.assert_allclose(run.tracked["v"].cpu().numpy(), d["out.v_track"], rtol=V_RTOL, atol=V_ATOL)
    if "rec.spikes" in d:  # the reference suite's own recording
        assert (spikes == d["rec.spikes"]).all()


@pytest.mark.parametrize("name", CASES)
def test_pooled_free_run_is_spike_exact(name):
    """Synapse types of one decay and sign pooled into a channel (as the benchmark runs):
    the same raster, and the final currents summed over each pool."""
    drive, p, d, meta = golden_io.load(name, "cuda")
    engine.POOL_SYNAPSES = True
    try:
        run = _run(drive, p, meta, d["in.x"], d["in.v"], d["in.g"], _kw(d, "in."))
        plan = engine.get_plan(drive, current._fields(p), d["in.x"].shape[0], d["in.x"].shape[2], "cuda")
    finally:
        engine.POOL_SYNAPSES = False
    spikes = run.output.cpu().numpy() > 0.5
    differs = (spikes != d["out.spikes"]).any(axis=(0, 2))
    assert not differs.any(), f"first divergence at step {int(np.argmax(differs))}"
    np.testing.assert_allclose(run.tracked["v"].cpu().numpy(), d["out.v_track"], rtol=V_RTOL, atol=V_ATOL)
    got, want = run.syn.cpu().numpy(), d["out.g"]
    for members in plan.ch.member:
        np.testing.assert_allclose(got[..., members[0]], want[..., members].sum(-1), rtol=I_RTOL, atol=I_ATOL)


def test_tracked_currents_and_chunking():
    """The tracked currents are the state after each step's input (the last equals the
    final state), and a run split into two calls equals one call."""
    drive, p, d, meta = golden_io.load("current_recurrent", "cuda")
    x = d["in.x"]
    whole = _run(drive, p, meta, x, d["in.v"], d["in.g"], {})
    np.testing.assert_array_equal(whole.tracked["I"][:, -1].cpu().numpy(), whole.syn.cpu().numpy())
    first = _run(drive, p, meta, x[:, :70], d["in.v"], d["in.g"], {})
    second = _run(drive, p, meta, x[:, 70:], first.v.cpu().numpy(), first.syn.cpu().numpy(), {})
    assert torch.equal(torch.cat([first.output, second.output], 1), whole.output)
    assert torch.equal(second.v, whole.v)


def test_learnt_signs_are_refused():
    drive, p, d, meta = golden_io.load("current_feedforward", "cuda")
    p.sign = p.sign.clone().float().requires_grad_(True)
    with pytest.raises(NotImplementedError, match="signs"):
        current.simulate(_t(d["in.v"]), _t(d["in.g"]), _t(d["in.x"]), drive, p)


# ---- gradients: the reference's autograd through current/dynamics.py (golden cases) ----

TOL = 1e-3  # of each gradient's largest entry, as for the conductance family


def _readout(seed, shape):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.normal(size=shape).astype(np.float32)).cuda()


def _leaf(t):
    return t.detach().clone().requires_grad_(True)


PHYS = ("theta", "U_reset", "beta", "U_rest", "R", "decay", "adapt", "adapt_decay")


def _engine_gradients(name, recurrent=None, physiology=False):
    drive, p, d, meta = golden_io.load(name, "cuda")
    if recurrent is not None:
        drive.recurrent_gradients = recurrent
    phys = {}
    if physiology:  # the learnable physiology as leaves
        for key in PHYS:
            if getattr(p, key) is not None:
                phys[key] = _leaf(getattr(p, key))
                setattr(p, key, phys[key])
    T = meta["grad_steps"]
    x = _leaf(_t(d["in.x"][:, :T]))
    drive.scale = _leaf(drive.scale)
    made = {}

    def leaf_w(W):
        if id(W) not in made:
            made[id(W)] = _leaf(W)
        return made[id(W)]

    drive.recurrent = [(r, leaf_w(W)) for r, W in drive.recurrent]
    drive.feedforward = [(r, leaf_w(W)) for r, W in drive.feedforward]
    run = current.simulate(_t(d["in.v"]), _t(d["in.g"]), x, drive, p, probabilities=meta["probabilities"],
                           **_kw(d, "in."))  # fmt: skip
    loss = (run.output * _readout(meta["readout_seed"], run.output.shape)).sum()
    if meta["probabilities"]:
        loss = loss + (run.probabilities * _readout(meta["readout_seed"] + 2, run.output.shape)).sum()
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


def _worst(grads, d, masks, weights=True):
    worst = {}
    for key, got in grads.items():
        expected = d[f"grad.{key}"]
        if got is None:
            worst[key] = 0.0 if np.abs(expected).max() == 0 else np.inf
            continue
        got = got.detach().cpu().numpy()
        if key.startswith("W."):
            if not weights:
                continue
            got, expected = got[masks[key]], expected[masks[key]]
        scale = max(float(np.abs(expected).max()), 1e-12)
        worst[key] = float(np.abs(got - expected).max()) / scale
    return worst


@pytest.mark.parametrize("name", CASES)
def test_gradients_match_reference(name):
    """Scale, weight and input gradients of a fixed readout of the spikes (through the
    recurrent spikes where the network's drive asks, the current-based default)."""
    loss, spikes, grads, d, masks = _engine_gradients(name)
    T = spikes.shape[1]
    np.testing.assert_array_equal(spikes.detach().cpu().numpy() > 0.5, d["out.spikes"][:, :T])
    np.testing.assert_allclose(loss, float(d["grad.loss"]), rtol=1e-4, atol=1e-4)
    worst = _worst(grads, d, masks)
    assert all(w <= TOL for w in worst.values()), worst


@pytest.mark.parametrize("name", CASES)
def test_physiology_gradients_match_reference(name):
    """With every learnable parameter of the physiology a leaf (threshold, reset, U_rest,
    R, the leak's and the synapses' decays, the adaptation's rise and decay): all
    gradients within 1e-3 of their largest entry."""
    loss, spikes, grads, d, masks = _engine_gradients(name, physiology=True)
    np.testing.assert_allclose(loss, float(d["grad.loss"]), rtol=1e-4, atol=1e-4)
    worst = _worst(grads, d, masks)
    assert any(k.startswith("phys.") for k in worst)
    assert all(w <= TOL for w in worst.values()), worst


def test_recurrent_carry_matters():
    """Without the carry along the recurrent edges the recurrent network's gradients
    miss the reference's by far more than the tolerance."""
    _, _, grads, d, masks = _engine_gradients("current_recurrent", recurrent=False)
    assert max(_worst(grads, d, masks, weights=False).values()) > 10 * TOL


def test_specialised_kernels_match_the_generic_one():
    """Current-based runs with a refractory period take kernels with the mode compiled in
    (forward, and forward saving for the backward pass); tracking sends the same run
    through the generic kernel. All three give identical spikes and state, bit for bit."""
    drive, p, d, meta = golden_io.load("current_recurrent", "cuda")
    p.n_ref = torch.full_like(p.theta, 20, dtype=torch.int32)
    kw = {"refractory": torch.zeros(p.theta.shape[0], dtype=torch.int32, device="cuda").expand(2, -1).contiguous()}
    x, v, I = _t(d["in.x"]), _t(d["in.v"]), _t(d["in.g"])
    with torch.no_grad():
        fast = current.simulate(v, I, x, drive, p, **kw)
        generic = current.simulate(v, I, x, drive, p, **kw, track=True)
    drive.scale = drive.scale.clone().requires_grad_(True)  # saving for the backward pass
    saving = current.simulate(v, I, x, drive, p, **kw)
    saving.output.sum().backward()
    assert float(fast.output.sum()) > 20
    for run in (generic, saving):
        for name in ("output", "v", "syn", "refractory"):
            assert torch.equal(getattr(fast, name).detach(), getattr(run, name).detach()), name
    assert drive.scale.grad is not None and torch.isfinite(drive.scale.grad).all()


@pytest.mark.parametrize("name", golden_io.curstats_cases())
def test_statistics_scale_rates_match_reference(name):
    """The reference's current-based statistics networks (2,000 and 1,000 neurons, 2,500 /
    1,500 steps after the burn-in, 250-step calls with the state carried): per-type
    population rates within the reference's own tolerance (twice the spread between its
    two recorded inputs, at least 2%) of its recording and of its CPU run."""
    drive, p, d, meta = golden_io.load(name, "cuda")
    A, B = meta["seeds"]
    x = _t(d[f"in.x_{A}"])
    v, I = _t(d["in.v"]), _t(d["in.g"])
    kw = {k: _t(d[f"in.{k}"]) for k in ("refractory", "gating", "adaptation") if f"in.{k}" in d}
    out = []
    with torch.no_grad():
        for start in range(0, x.shape[1], meta["chunk"]):
            run = current.simulate(v, I, x[:, start : start + meta["chunk"]], drive, p, **kw)
            out.append(run.output)
            v, I = run.v, run.syn
            kw = {k: getattr(run, k) for k in kw}
    spikes = torch.cat(out, 1)[:, meta["burn_in"] :].cpu().numpy() > 0.5
    types = d["in.types"]
    means = golden_io.population_rates(spikes, types, meta["dt"])
    ref = np.array([d[f"rec.rates_{A}"][types == t].mean() for t in np.unique(types)])
    ref_b = np.array([d[f"rec.rates_{B}"][types == t].mean() for t in np.unique(types)])
    allowed = np.maximum(2 * np.abs(ref_b - ref), 0.02 * ref)
    assert np.all(np.abs(means - ref) <= allowed), (means, ref, allowed)
    cpu = golden_io.population_rates(d["out.spikes"], types, meta["dt"])
    assert np.all(np.abs(means - cpu) <= allowed), (means, cpu, allowed)
