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
