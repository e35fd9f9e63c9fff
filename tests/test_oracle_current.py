"""The oracle's current-based step (``cond_lif.c`` with ``current`` set, restating
``network_simulators/current/dynamics.py:116-205``) against the reference's own runs of
its current-based test networks (golden cases ``current_*``; three also match the
reference suite's recordings): the spike raster exactly, voltages within 1e-5 (natural
units, threshold 1) and the final currents within 1e-5 relative. Both of the oracle's
schedules (whole trials per thread, and each step's neurons over all threads) are run."""

import numpy as np
import pytest

import golden_io
from oracle import oracle

CASES = golden_io.current_cases()


@pytest.mark.parametrize("threads", [1, 4])
@pytest.mark.parametrize("name", CASES)
def test_oracle_free_run_matches_reference(name, threads):
    drive, p, d, meta = golden_io.load(name)
    oracle.set_threads(threads)
    try:
        net = oracle.Network(drive, p, d["in.x"].shape[0], d["in.x"].shape[2])
        kw = {k: d[f"in.{k}"] for k in ("refractory", "gating", "adaptation") if f"in.{k}" in d}
        out = net.simulate(d["in.x"], d["in.v"], d["in.g"], probabilities=meta["probabilities"], **kw)
    finally:
        oracle.set_threads(1)
    differs = (out["spikes"] != d["out.spikes"]).any(axis=(0, 2))
    assert not differs.any(), f"first divergence at step {int(np.argmax(differs))}"
    np.testing.assert_allclose(out["v_track"], d["out.v_track"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(out["g"], d["out.g"], rtol=1e-5, atol=1e-6)
    if meta["probabilities"]:
        np.testing.assert_allclose(out["prob"], d["out.prob"], rtol=0, atol=1e-5)
    if "rec.spikes" in d:
        assert (out["spikes"] == d["rec.spikes"]).all()


def test_c2c_configuration_at_a_tenth():
    """The current-based C2 configuration (``configs.c2_current``) at a tenth of its
    neurons with the same in-degrees: each cell type's synapse type carries the type's
    sign and time constant, the state is the currents (B, N, S), and the oracle's
    current-based step fires it in the benchmark's range (a few Hz, not silent, not
    saturated)."""
    from wiretorch_b200 import configs

    cfg = configs.c2_current(B=2, T=500, device="cpu", N=2000, p_max=0.5)
    v, I, kw = cfg.state()
    S = cfg.drive.made.shape[1]
    assert I.shape == (2, 2000, S) and v.shape == (2, 2000)
    assert set(cfg.p.sign.tolist()) == {1.0, -1.0} and float(cfg.p.sign[-1]) == 1.0
    exc = cfg.p.sign > 0
    np.testing.assert_allclose(cfg.p.decay[exc].numpy(), np.exp(-0.1 / 5.0), rtol=1e-6)
    np.testing.assert_allclose(cfg.p.decay[~exc].numpy(), np.exp(-0.1 / 10.0), rtol=1e-6)
    net = oracle.Network(cfg.drive, cfg.p, cfg.B, cfg.n_in)
    out = net.simulate(cfg.inputs(seed=1), v, I, **kw, track=False)
    rate = out["spikes"].mean() / 1e-4
    assert 1.0 < rate < 30.0, rate


def test_field_mapping_follows_the_physiology():
    """The current-based physiology as the kernel's fields: U_rest as E_L, R as C_m, the
    signs as E_syn, each type a decay component with a unit jump; cached per physiology
    and its tensors, so that a field replaced on the same object is seen."""
    import torch

    from wiretorch_b200 import current
    from wiretorch_b200.types import CurrentPhysiology

    N = 4
    p = CurrentPhysiology(theta=torch.ones(N), U_reset=torch.zeros(N), beta=torch.full((N,), 0.9),
                          U_rest=torch.full((N,), 0.1), R=torch.full((N,), 2.0), sign=torch.tensor([1.0, -1.0]),
                          decay=torch.tensor([0.9, 0.8]), surr_scale=torch.tensor(5.0))  # fmt: skip
    f = current._fields(p)
    assert f.E_L is p.U_rest and f.C_m is p.R and f.beta is p.beta and f.current
    assert torch.equal(f.E_syn, p.sign) and torch.equal(f.decay[1], p.decay) and not f.decay[0].any()
    assert torch.equal(f.jump, torch.tensor([[0.0, 0.0], [1.0, 1.0]]))
    assert current._fields(p) is f
    p.theta = torch.full((N,), 2.0)
    assert current._fields(p).theta is p.theta
