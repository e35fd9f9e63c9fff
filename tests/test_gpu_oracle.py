"""The engine against the oracle on networks larger than the golden cases.

The golden networks (150 neurons) fit one thread block; these span many blocks of the
persistent kernel, so they exercise its grid barrier and the events and accumulators
shared between blocks. Lockstep against the oracle (``lockstep.compare``), with every
feature of the time step, in the exact and the pooled channel layouts.
"""

import pytest
import torch

import lockstep
from oracle import oracle
from wiretorch_b200 import engine
from wiretorch_b200.testing import random_network

pytestmark = pytest.mark.gpu

FEATURES = {
    "plain": {},
    "refractory": {"tau_ref": 2.0},
    "nmda": {"mg": 1.0},
    "adaptation": {"adapt": 0.4},
    "everything": {"tau_ref": 3.0, "mg": 1.2, "adapt": 0.3},
}


def _sim(drive, p, pool):
    def run(v, g, x, kw):
        engine.POOL_SYNAPSES = pool
        try:
            with torch.no_grad():
                return engine.simulate(v, g, x, drive, p, track=True, **kw)
        finally:
            engine.POOL_SYNAPSES = False

    return run


@pytest.mark.parametrize("pool", [False, True], ids=["exact", "pooled"])
@pytest.mark.parametrize("feature", FEATURES)
@pytest.mark.parametrize("N,B", [(700, 3), (3000, 4)])
def test_lockstep_against_oracle(N, B, feature, pool):
    drive, p, x, v, g, kw = random_network(N=N, n_in=200, B=B, T=120, seed=N + B,
                                           device="cuda", **FEATURES[feature])  # fmt: skip
    net = oracle.Network(drive, p, B, x.shape[2])
    excused, windows, dv, dg = lockstep.compare(_sim(drive, p, pool), net, drive, p, x, v, g, kw)
    assert excused <= 0.01 * windows, f"{excused} near-threshold flips in {windows} trial-windows"


def _c5_small():
    """The C5 model (NMDA with Mg block, short-term depression on both recurrent
    pathways, distance-dependent connectivity) at 4,000 neurons and ~390 edges each."""
    from wiretorch_b200 import configs

    return configs.c5(B=3, T=120, device="cuda", N=4000, mean_degree=400.0, lam=0.05 * 250 ** (1 / 3),
                      w_e=3.0, w_in=30.0)  # fmt: skip


@pytest.mark.parametrize("pool", [False, True], ids=["exact", "pooled"])
def test_c5_model_lockstep_against_oracle(pool):
    cfg = _c5_small()
    x = cfg.inputs(seed=3)
    v, g, kw = cfg.state()
    net = oracle.Network(cfg.drive, cfg.p, cfg.B, cfg.n_in)
    # pooled: the excitatory and the input AMPA types share one channel
    ch = engine.get_plan(cfg.drive, cfg.p, cfg.B, cfg.n_in, x.device, pool=pool).ch
    assert ch.pooled == pool
    pools = [list(m) for m in ch.member] if ch.pooled else None
    excused, windows, dv, dg = lockstep.compare(_sim(cfg.drive, cfg.p, pool), net, cfg.drive, cfg.p, x, v, g, kw,
                                                pools=pools)  # fmt: skip
    assert excused <= 0.01 * windows, f"{excused} near-threshold flips in {windows} trial-windows"
    with torch.no_grad():
        run = engine.simulate(v, g, x, cfg.drive, cfg.p, **kw)
    assert float(run.output.sum()) > 20  # the network is active
    n_e = cfg.drive.gates[0].n
    assert float(run.gating[:, n_e : 2 * n_e].min()) < 0.99  # and its excitatory synapses depress


def _streamed(drive, p, x, v, g, kw, stream):
    engine.FORCE_STREAM = stream
    try:
        with torch.no_grad():
            return engine.simulate(v, g, x, drive, p, **kw)
    finally:
        engine.FORCE_STREAM = False


@pytest.mark.parametrize("feature", ["refractory", "everything"])
@pytest.mark.parametrize("N", [3000, 1001])
def test_streamed_state_gives_the_same_run(N, feature):
    """The state streamed through shared memory every step (the path of networks too
    large to keep it on chip) gives the very run of the state kept on chip, bit for bit,
    and matches the oracle in lockstep."""
    drive, p, x, v, g, kw = random_network(N=N, n_in=200, B=3, T=80, seed=N, device="cuda", **FEATURES[feature])
    on_chip = _streamed(drive, p, x, v, g, kw, False)
    streamed = _streamed(drive, p, x, v, g, kw, True)
    assert float(on_chip.output.sum()) > 0
    assert torch.equal(on_chip.output, streamed.output)
    assert torch.equal(on_chip.v, streamed.v)
    assert torch.equal(on_chip.syn, streamed.syn)
    net = oracle.Network(drive, p, x.shape[0], x.shape[2])

    def sim(v_, g_, x_, kw_):
        engine.FORCE_STREAM = True
        try:
            with torch.no_grad():
                return engine.simulate(v_, g_, x_, drive, p, track=True, **kw_)
        finally:
            engine.FORCE_STREAM = False

    excused, windows, dv, dg = lockstep.compare(sim, net, drive, p, x, v, g, kw)
    assert excused <= 0.01 * windows
