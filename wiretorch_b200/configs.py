"""Seeded synthetic networks of the benchmark configurations, built as wiretorch's
networks hand them to their engine: a ``Drive`` (weights as ``SparseRows``), a
``Physiology`` and the state at rest.

The configurations (the benchmark specification's five) leave some physiology open; the
values chosen here are fixed once and named in each builder (leak conductance, input
weights), chosen so that neurons fire at a few to a few tens of Hz. Synapses with
``tau_rise = 0`` are single exponentials: ``conductance_kernel`` gives them jumps
``(-g_bar, +g_bar)`` and a rise decay of 0, so an input reaches the membrane one step
after it arrives (as in the reference).

Connectivity is generated with torch on the given device from a seeded generator (the
same seed gives the same network on the same kind of device). Cell types occupy
contiguous index ranges.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from wiretorch_b200.types import Drive, Physiology, SparseRows


@dataclass
class Config:
    """A built configuration: the engine's inputs plus what the benchmark needs."""

    name: str
    drive: Drive
    p: Physiology
    B: int
    T: int
    N: int
    n_in: int
    rates_in: torch.Tensor  # (n_in,) Hz of the Poisson inputs
    types: torch.Tensor  # (N,) cell type of each neuron
    n_types: int
    out_degree: torch.Tensor  # (N + n_in,) edges of each source (recurrent + input)
    extra: dict = field(default_factory=dict)

    def state(self):
        """``(v, g, kw)`` at rest: voltages at reset, conductances zero (and the gating
        state of a gated network at its rest values)."""
        dev = self.drive.scale.device
        current = hasattr(self.p, "sign")  # current-based: the currents (B, N, S)
        S = (self.p.sign if current else self.p.E_syn).shape[0]
        v = self.p.U_reset.expand(self.B, self.N).clone()
        if current:
            g = torch.zeros((self.B, S, self.N), device=dev).permute(0, 2, 1)
        else:
            g = torch.zeros((self.B, 2, S, self.N), device=dev).permute(0, 3, 1, 2)
        kw = {"refractory": torch.zeros((self.B, self.N), dtype=torch.int32, device=dev)}
        if self.p.adapt is not None:
            kw["adaptation"] = torch.zeros((self.B, self.N), device=dev)
        if "gating" in self.extra:
            kw["gating"] = self.extra["gating"].clone()
        return v, g, kw

    def carried(self, run):
        """The state keywords of the next engine call after ``run``."""
        kw = {"refractory": run.refractory}
        if run.adaptation is not None:
            kw["adaptation"] = run.adaptation
        if "gating" in self.extra:
            kw["gating"] = run.gating
        return kw

    def inputs(self, T=None, seed=1, generator_device=None):
        """Poisson input spikes ``(B, T, n_in)`` float32 (seeded)."""
        T = self.T if T is None else T
        dev = self.drive.scale.device
        gen = torch.Generator(device=dev).manual_seed(seed)
        dt = float(self.p.dt) if hasattr(self.p, "dt") else self.extra["dt"]  # (current-based: in extra)
        p = (self.rates_in * dt / 1000.0).to(dev)
        return (torch.rand((self.B, T, self.n_in), generator=gen, device=dev) < p).float()


def _kernel(tau_rise, tau_decay, g_bar):
    """``conductance_kernel`` (conductance/synapses.py:70-87): jumps of the rise and decay
    components per unit input, the difference of exponentials peaking at ``g_bar``."""
    r = tau_rise / tau_decay
    peak = torch.where(r > 0, r ** (r / (1 - r)) - r ** (1 / (1 - r)), torch.ones_like(r))
    return torch.stack([-g_bar, g_bar]) / peak


def _csr_from_edges(src, dst, w, n_rows, n_targets):
    order = torch.argsort(src * n_targets + dst, stable=True)
    src, dst, w = src[order], dst[order], w[order]
    row_ptr = torch.zeros(n_rows + 1, dtype=torch.int64, device=src.device)
    row_ptr[1:] = torch.cumsum(torch.bincount(src, minlength=n_rows), 0)
    return SparseRows(row_ptr, dst.to(torch.int32), w.float().contiguous(), n_targets)


def _block_edges(gen, rows, cols, p, device):
    """Bernoulli(p) edges between index ranges ``rows`` and ``cols`` (half-open pairs)."""
    r0, r1 = rows
    c0, c1 = cols
    nr, nc = r1 - r0, c1 - c0
    if nr == 0 or nc == 0 or p <= 0:
        e = torch.zeros(0, dtype=torch.int64, device=device)
        return e, e
    mask = torch.rand((nr, nc), generator=gen, device=device) < p
    nz = mask.nonzero()
    return nz[:, 0] + r0, nz[:, 1] + c0


def _physiology(N, types_e, dt, S_params, device, tau_mem=20.0, theta=-50.0, U_reset=-65.0,
                E_L=-70.0, g_L=10.0, tau_ref=2.0):  # fmt: skip
    """Per-neuron tables (all neurons alike) and per-synapse tables from ``S_params``:
    list of (tau_rise, tau_decay, E_syn, g_bar)."""
    f = lambda v: torch.tensor(v, dtype=torch.float32, device=device)  # noqa: E731
    dtt = f(dt)
    tr = f([s[0] for s in S_params])
    td = f([s[1] for s in S_params])
    gb = f([s[3] for s in S_params])
    decay_r = torch.where(tr > 0, torch.exp(-dtt / tr.clamp(min=1e-30)), torch.zeros_like(tr))
    ones = torch.ones(N, device=device)
    return Physiology(
        theta=ones * theta, U_reset=ones * U_reset, E_L=ones * E_L,
        C_m=ones * (tau_mem * g_L), beta=torch.exp(-dtt / (ones * tau_mem)),
        E_syn=f([s[2] for s in S_params]),
        g_clip=torch.full((len(S_params),), float("inf"), device=device),
        decay=torch.stack([decay_r, torch.exp(-dtt / td)]),
        jump=_kernel(tr, td, gb), dt=dtt, surr_scale=f(10.0),
        n_ref=torch.full((N,), int(round(tau_ref / dt)), dtype=torch.int32, device=device),
    )  # fmt: skip


def c1(B=8, T=1000, seed=0, device="cuda", w_in=15.0, g_L=10.0):
    """Conductance LIF, N=1000 (800 E / 200 I), Erdos-Renyi p=0.1, log-normal weights
    (mu=-1, sigma=1, nS) signed by presynaptic type, tau_m=20 ms, E_L=-70, V_th=-50,
    V_reset=-65 mV, refractory 2 ms, E_exc=0 / E_inh=-80 mV, tau_syn 5 / 10 ms, dt=0.1 ms,
    T=1000, batch 8, one independent 10 Hz Poisson input per neuron; forward only.
    Chosen here: g_L = 10 nS, input weight 15 nS (rates of 2-3 Hz; with equal E and I
    weight distributions the network runs away above ~18 nS)."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    N, NE = 1000, 800
    src, dst = _block_edges(gen, (0, N), (0, N), 0.1, dev)
    keep = src != dst
    src, dst = src[keep], dst[keep]
    w = torch.exp(-1.0 + torch.randn(src.numel(), generator=gen, device=dev))
    e = src < NE
    W_e = _csr_from_edges(src[e], dst[e], w[e], NE, N)
    W_i = _csr_from_edges(src[~e] - NE, dst[~e], w[~e], N - NE, N)
    ar = torch.arange(N, device=dev)
    W_in = _csr_from_edges(ar, ar, torch.full((N,), w_in, device=dev), N, N)
    # synapse types: 0 AMPA (E), 1 GABA (I), 2 AMPA (input)
    S_params = [(0.0, 5.0, 0.0, 1.0), (0.0, 10.0, -80.0, 1.0), (0.0, 5.0, 0.0, 1.0)]
    made = torch.eye(3, dtype=torch.bool, device=dev)
    drive = Drive(made=made, scale=torch.ones(3, N, device=dev),
                  recurrent=[(ar[:NE], W_e), (ar[NE:], W_i)],
                  feedforward=[(ar, W_in)])  # fmt: skip
    p = _physiology(N, None, 0.1, S_params, dev, g_L=g_L)
    types = (ar >= NE).to(torch.int64)
    out_deg = torch.cat([torch.bincount(src, minlength=N), torch.ones(N, dtype=torch.int64, device=dev)])
    return Config("c1", drive, p, B, T, N, N, torch.full((N,), 10.0, device=dev), types, 2, out_deg)


def c2(B=64, T=500, seed=0, device="cuda", n_in=2000, p_in=0.05, w_mu=-1.0, w_mu_i=0.6,
       w_in_mu=-0.5, g_L=10.0, n_types=40, frac_e_types=0.75, N=20000, p_max=0.05):  # fmt: skip
    """N=20,000 neurons in 40 synthetic cell types (type sizes multinomial; 75% of the types
    excitatory), per-type-pair connection probability ~U(0, 0.05), log-normal per-synapse
    weights (sigma=1, nS; mu=w_mu from excitatory types, w_mu_i = w_mu + ln 5 from
    inhibitory ones, so that inhibition balances the 3:1 excitatory majority), learnt
    per-type-pair scale, dt=0.1 ms, T=500, batch 64,
    Poisson inputs at 5-20 Hz (``n_in`` inputs, each reaching a neuron with probability
    ``p_in``, log-normal weights mu=w_in_mu). Physiology as ``c1`` (g_L = 10 nS). At
    these values the network fires at 10-15 Hz.

    Every cell type makes its own synapse type, as the reference's synapse registry does
    (one per source cell type and synapse name): 30 AMPA-like (tau 5 ms, E 0 mV), 10
    GABA-like (tau 10 ms, E -80 mV), and the inputs' AMPA. ``extra["log_sf_shape"]``:
    the learnt per-pair log scale, (41 source types, 40 target types).

    ``N`` and ``p_max`` (pair probabilities ~ U(0, p_max)) make smaller networks of the
    same construction, for tests."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    rng = np.random.default_rng(seed)
    sizes = rng.multinomial(N, np.full(n_types, 1.0 / n_types))
    starts = np.concatenate([[0], np.cumsum(sizes)])
    n_e_types = int(round(frac_e_types * n_types))
    p_pair = rng.uniform(0.0, p_max, (n_types, n_types))
    rows_l, pathways = [], []
    srcs, dsts = [], []
    for a in range(n_types):
        s_a, d_a = [], []
        for b in range(n_types):
            s, d = _block_edges(gen, (starts[a], starts[a + 1]), (starts[b], starts[b + 1]),
                                float(p_pair[a, b]), dev)  # fmt: skip
            s_a.append(s)
            d_a.append(d)
        s_a, d_a = torch.cat(s_a), torch.cat(d_a)
        keep = s_a != d_a
        srcs.append(s_a[keep])
        dsts.append(d_a[keep])
    out_deg = torch.zeros(N + n_in, dtype=torch.int64, device=dev)
    for a in range(n_types):
        s_a, d_a = srcs[a], dsts[a]
        mu = w_mu if a < n_e_types else w_mu_i
        w = torch.exp(mu + torch.randn(s_a.numel(), generator=gen, device=dev))
        rows = torch.arange(starts[a], starts[a + 1], device=dev)
        pathways.append((rows, _csr_from_edges(s_a - starts[a], d_a, w, int(sizes[a]), N)))
        out_deg[starts[a] : starts[a + 1]] = torch.bincount(s_a - starts[a], minlength=int(sizes[a]))
    s_in, d_in = _block_edges(gen, (0, n_in), (0, N), p_in, dev)
    w_in = torch.exp(w_in_mu + torch.randn(s_in.numel(), generator=gen, device=dev))
    W_in = _csr_from_edges(s_in, d_in, w_in, n_in, N)
    out_deg[N:] = torch.bincount(s_in, minlength=n_in)
    S = n_types + 1
    S_params = [(0.0, 5.0, 0.0, 1.0) if a < n_e_types else (0.0, 10.0, -80.0, 1.0)
                for a in range(n_types)] + [(0.0, 5.0, 0.0, 1.0)]  # fmt: skip
    made = torch.eye(S, dtype=torch.bool, device=dev)
    types = torch.repeat_interleave(torch.arange(n_types, device=dev),
                                    torch.tensor(sizes, device=dev))  # fmt: skip
    drive = Drive(made=made, scale=torch.ones(S, N, device=dev), recurrent=pathways,
                  feedforward=[(torch.arange(n_in, device=dev), W_in)])  # fmt: skip
    p = _physiology(N, None, 0.1, S_params, dev, g_L=g_L)
    rates = torch.from_numpy(rng.uniform(5.0, 20.0, n_in).astype(np.float32)).to(dev)
    cfg = Config("c2", drive, p, B, T, N, n_in, rates, types, n_types, out_deg)
    cfg.extra["log_sf_shape"] = (S, n_types)
    cfg.extra["target_rates"] = torch.from_numpy(
        rng.uniform(1.0, 30.0, (B, N)).astype(np.float32)).to(dev)  # fmt: skip
    return cfg


def c2_current(B=64, T=500, seed=0, device="cuda", w_scale=0.15, N=20000, p_max=0.05, **kw):
    """The current-based family on C2's network: the same 40-type connectome, weights
    (times ``w_scale``, as current jumps) and Poisson input as ``c2``, with current-based
    neurons in the family's natural units (``current/dynamics.py``; reset 0, threshold 1,
    U_rest 0, R 1, tau_m 20 ms, refractory 2 ms, surrogate scale 10); each cell type's
    synapse type signed by the type (+1 excitatory, -1 inhibitory; the input +1) and
    decaying with its C2 time constant (5 or 10 ms). Forward only in the benchmark. At the
    chosen ``w_scale`` the network fires at 5-10 Hz."""
    from wiretorch_b200.types import CurrentPhysiology

    base = c2(B=B, T=T, seed=seed, device=device, N=N, p_max=p_max, **kw)
    dev = base.drive.scale.device
    d = base.drive

    def scaled(W):
        return type(W)(W.row_ptr, W.cols, W.values * w_scale, W.n_targets)

    drive = Drive(made=d.made, scale=d.scale, recurrent=[(r, scaled(W)) for r, W in d.recurrent],
                  feedforward=[(r, scaled(W)) for r, W in d.feedforward])  # fmt: skip
    S = d.made.shape[1]
    n_types = base.n_types
    n_e_types = sum(1 for a in range(n_types) if float(base.p.E_syn[a]) == 0.0)
    sign = torch.tensor([1.0 if a < n_e_types else -1.0 for a in range(n_types)] + [1.0], device=dev)
    tau_s = torch.tensor([5.0 if a < n_e_types else 10.0 for a in range(n_types)] + [5.0], device=dev)
    dt = 0.1
    ones = torch.ones(base.N, device=dev)
    p = CurrentPhysiology(
        theta=ones.clone(), U_reset=torch.zeros(base.N, device=dev), beta=ones * math.exp(-dt / 20.0),
        U_rest=torch.zeros(base.N, device=dev), R=ones.clone(), sign=sign, decay=torch.exp(-dt / tau_s),
        surr_scale=torch.tensor(10.0, device=dev), n_ref=torch.full((base.N,), 20, dtype=torch.int32, device=dev),
    )  # fmt: skip
    assert S == sign.numel()
    cfg = Config("c2c", drive, p, B, T, base.N, base.n_in, base.rates_in, base.types, n_types, base.out_degree)
    cfg.extra["dt"] = dt
    return cfg


def scale_from_log_sf(cfg: Config, log_sf: torch.Tensor) -> torch.Tensor:
    """The kernel scale ``(K, N)`` of learnt per-pair log scales ``(K, n_types)``: each
    pathway's factor for each target neuron's type (network.py:816-854 ``_drive``)."""
    return torch.exp(log_sf)[:, cfg.types]


def synaptic_events(cfg: Config, spikes: torch.Tensor, x: torch.Tensor | None = None) -> tuple[int, int]:
    """``(recurrent, input)`` synaptic events of a run: every recurrent spike times its
    neuron's out-degree, and every non-zero input times its input's out-degree."""
    deg = cfg.out_degree.to(spikes.device).double()
    rec = int((spikes.double().sum((0, 1)) * deg[: cfg.N]).sum())
    inp = 0
    if x is not None:
        inp = int(((x != 0).double().sum((0, 1)) * deg[cfg.N :]).sum())
    return rec, inp


def c3(B=256, T=2000, seed=0, device="cuda", rank=64, w_in=15.0, g_L=10.0):
    """Factorised-weight network: N=50,000 conductance-LIF neurons, recurrent weights
    W = U V^T of rank 64 with U and V ~ N(0, 1/sqrt(N)) in bf16, a sign mask per
    presynaptic neuron (80% excitatory: their row of W drives the excitatory synapse
    type, the rest the inhibitory one), batch 256, dt=0.1 ms, T=2,000, one 10 Hz Poisson
    input per neuron; forward only. Physiology as ``c1`` (g_L = 10 nS, input weight
    15 nS). The factors as specified give weights of order 8 / N nS, so the recurrent
    drive is weak next to the input."""
    from wiretorch_b200.lowrank import LowRank

    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    N = 50000
    sd = 1.0 / math.sqrt(N)
    U = (torch.randn(N, rank, generator=gen, device=dev) * sd).to(torch.bfloat16)
    V = (torch.randn(N, rank, generator=gen, device=dev) * sd).to(torch.bfloat16)
    exc = torch.rand(N, generator=gen, device=dev) < 0.8
    rows_e, rows_i = torch.nonzero(exc).flatten(), torch.nonzero(~exc).flatten()
    ar = torch.arange(N, device=dev)
    W_in = SparseRows(torch.arange(N + 1, device=dev), ar.to(torch.int32), torch.full((N,), w_in, device=dev), N)
    S_params = [(0.0, 5.0, 0.0, 1.0), (0.0, 10.0, -80.0, 1.0)]
    made = torch.tensor([[1, 0], [0, 1], [1, 0]], dtype=torch.bool, device=dev)
    drive = Drive(made=made, scale=torch.ones(3, N, device=dev),
                  recurrent=[(rows_e, LowRank(U[rows_e], V)), (rows_i, LowRank(U[rows_i], V))],
                  feedforward=[(ar, W_in)])  # fmt: skip
    p = _physiology(N, None, 0.1, S_params, dev, g_L=g_L)
    types = (~exc).to(torch.int64)
    out_deg = torch.cat([torch.full((N,), N, dtype=torch.int64, device=dev), torch.ones(N, dtype=torch.int64, device=dev)])
    cfg = Config("c3", drive, p, B, T, N, N, torch.full((N,), 10.0, device=dev), types, 2, out_deg)
    cfg.extra["rank"] = rank
    return cfg


def c4(B=32, T=10000, seed=0, device="cuda", N=139000, n_types=8000, mean_degree=360.0,
       degree_sigma=1.2, g_unit=0.7, g_inh=3.0, w_in=20.0, adapt=0.5):  # fmt: skip
    """Fly-scale synthetic connectome: N=139,000 neurons in 8,000 cell types (type sizes
    multinomial), ~50M directed edges with log-normal out-degree (mean 360, sigma 1.2) and
    targets drawn in proportion to a log-normal in-degree propensity (same law), integer
    synapse counts geometric(p=0.2) clipped to 2,000, a transmitter sign per cell type
    (60% excitatory, 35% inhibitory, 5% none: those make no synapses), conductance LIF
    with spike-rate adaptation (excitatory neurons) and refractoriness, dt=0.1 ms,
    T=10,000, batch 32, Poisson drive at 15 Hz to a random 5% of neurons; forward only.

    Chosen here: a synapse's conductance is ``g_unit`` nS per count (``g_inh`` times that
    for inhibitory sources) times a per-cell-type-pair scale ~ LogNormal(0, 0.5), folded
    into the weights, so the network's two pathways are its excitatory and inhibitory
    sources (the 8,000 types live in the weights, not in 8,000 pathways of (K, N) scales);
    adaptation ``adapt`` nS per spike decaying with 200 ms, E_adapt -90 mV; the driven
    neurons' input weight ``w_in`` nS. Physiology otherwise as ``c1``. At these values the
    network fires at 5-10 Hz (the oracle at a tenth of the size: 13,900 neurons)."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    rng = np.random.default_rng(seed)
    sizes = rng.multinomial(N, np.full(n_types, 1.0 / n_types))
    types = torch.repeat_interleave(torch.arange(n_types, device=dev), torch.tensor(sizes, device=dev))
    u = rng.random(n_types)
    sign_t = torch.tensor(np.where(u < 0.60, 1, np.where(u < 0.95, -1, 0)), device=dev)
    sign = sign_t[types]
    mu = math.log(mean_degree) - degree_sigma**2 / 2
    out_deg = torch.exp(mu + degree_sigma * torch.randn(N, generator=gen, device=dev)).round().long()
    out_deg = torch.where(sign != 0, out_deg.clamp(max=N - 1), torch.zeros_like(out_deg))
    propensity = torch.exp(degree_sigma * torch.randn(N, generator=gen, device=dev))
    cdf = torch.cumsum(propensity.double(), 0)
    cdf = cdf / cdf[-1]
    src = torch.repeat_interleave(torch.arange(N, device=dev), out_deg)
    dst = torch.searchsorted(cdf, torch.rand(src.numel(), generator=gen, device=dev, dtype=torch.float64))
    dst = dst.clamp(max=N - 1)
    key = torch.unique(src * N + dst)  # one edge per ordered pair, no self-connections
    src, dst = key // N, key % N
    keep = src != dst
    src, dst = src[keep], dst[keep]
    count = torch.clamp(torch.floor(torch.log(torch.rand(src.numel(), generator=gen, device=dev))
                                    / math.log(0.8)) + 1, max=2000)  # fmt: skip
    pair = torch.exp(0.5 * torch.randn(n_types * n_types // 64 + 1, generator=gen, device=dev))
    pair_idx = (types[src] * n_types + types[dst]) % pair.numel()
    w = count * g_unit * pair[pair_idx] * torch.where(sign[src] < 0, g_inh, 1.0)
    exc = sign[src] > 0
    rows_e = torch.nonzero(sign > 0).flatten()
    rows_i = torch.nonzero(sign < 0).flatten()
    # row index of each source within its pathway
    pos = torch.full((N,), -1, dtype=torch.int64, device=dev)
    pos[rows_e] = torch.arange(rows_e.numel(), device=dev)
    pos[rows_i] = torch.arange(rows_i.numel(), device=dev)
    W_e = _csr_from_edges(pos[src[exc]], dst[exc], w[exc], rows_e.numel(), N)
    W_i = _csr_from_edges(pos[src[~exc]], dst[~exc], w[~exc], rows_i.numel(), N)
    n_in = max(1, int(round(0.05 * N)))
    driven = torch.randperm(N, generator=gen, device=dev)[:n_in]
    W_in = _csr_from_edges(torch.arange(n_in, device=dev), driven, torch.full((n_in,), w_in, device=dev), n_in, N)
    S_params = [(0.0, 5.0, 0.0, 1.0), (0.0, 10.0, -80.0, 1.0), (0.0, 5.0, 0.0, 1.0)]
    made = torch.eye(3, dtype=torch.bool, device=dev)
    drive = Drive(made=made, scale=torch.ones(3, N, device=dev),
                  recurrent=[(rows_e, W_e), (rows_i, W_i)],
                  feedforward=[(torch.arange(n_in, device=dev), W_in)])  # fmt: skip
    p = _physiology(N, None, 0.1, S_params, dev)
    p.adapt = torch.where(sign > 0, adapt, 0.0).float()
    p.adapt_decay = torch.full((N,), math.exp(-0.1 / 200.0), device=dev)
    p.E_adapt = torch.full((N,), -90.0, device=dev)
    deg = torch.zeros(N + n_in, dtype=torch.int64, device=dev)
    deg[:N] = torch.bincount(src, minlength=N)
    deg[N:] = 1
    cfg = Config("c4", drive, p, B, T, N, n_in, torch.full((n_in,), 15.0, device=dev), types, n_types, deg)
    cfg.extra["edges"] = int(src.numel())
    return cfg


def _distance_edges(gen, pos, mean_degree, lam, dev, batch=20000):
    """Edges of a distance-dependent random graph on neurons at ``pos`` (N, 3) in the
    unit cube: every source draws ~Poisson(mean_degree) targets at distances ~
    Gamma(3, lam) (the law of 0.5 exp(-d / lam) p(d) over a uniform 3-d density) in
    uniform directions; points outside the cube are reflected back at its faces (so the
    mean out-degree stays ``mean_degree`` near the faces too), and each point picks a
    random neuron of its grid cell (cells of ~4 neurons); empty cells and
    self-connections are dropped."""
    N = pos.shape[0]
    G = max(1, round((N / 4.0) ** (1.0 / 3.0)))
    cell = (pos * G).long().clamp(max=G - 1)
    cid = (cell[:, 0] * G + cell[:, 1]) * G + cell[:, 2]
    order = torch.argsort(cid, stable=True)
    sorted_cid = cid[order]
    starts = torch.searchsorted(sorted_cid, torch.arange(G**3, device=dev))
    counts = torch.bincount(cid, minlength=G**3)
    srcs, dsts = [], []
    for j0 in range(0, N, batch):
        j1 = min(N, j0 + batch)
        k = torch.poisson(torch.full((j1 - j0,), float(mean_degree), device=dev), generator=gen).long()
        src = torch.repeat_interleave(torch.arange(j0, j1, device=dev), k)
        m = src.numel()
        d = -lam * torch.log(torch.rand((m, 3), generator=gen, device=dev).clamp(min=1e-12)).sum(1)  # Gamma(3, lam)
        u = torch.randn((m, 3), generator=gen, device=dev)
        pt = pos[src] + u / u.norm(dim=1, keepdim=True).clamp(min=1e-12) * d[:, None]
        pt = torch.remainder(pt, 2.0)
        pt = torch.where(pt > 1.0, 2.0 - pt, pt)  # reflection at the faces
        c = (pt * G).long().clamp(min=0, max=G - 1)
        tc = (c[:, 0] * G + c[:, 1]) * G + c[:, 2]
        n_in_cell = counts[tc]
        ok = n_in_cell > 0
        src, tc, n_in_cell = src[ok], tc[ok], n_in_cell[ok]
        pick = (torch.rand(src.numel(), generator=gen, device=dev) * n_in_cell).long().clamp(max=n_in_cell - 1)
        dst = order[starts[tc] + pick]
        keep = dst != src
        srcs.append(src[keep])
        dsts.append(dst[keep])
    return torch.cat(srcs), torch.cat(dsts)


def c5(B=4, T=5000, seed=0, device="cuda", N=1_000_000, mean_degree=1000.0, lam=0.05, w_e=1.2, g_inh=12.0,
       nmda=0.1, U=0.2, tau_rec=200.0, w_in=20.0):  # fmt: skip
    """1,000,000-neuron synthetic connectome: neurons uniform in the unit cube, ~1B edges
    from a distance-dependent model (connection probability 0.5 exp(-d / 0.05), out-degree
    capped at a mean of 1,000: every source draws ~Poisson(1000) targets at distances ~
    Gamma(3, 0.05), see ``_distance_edges``; the uncapped model would give
    0.5 * 8 pi 0.05^3 * N ~ 1,570 edges per neuron), 80/20 E/I, log-normal weights (sigma 1,
    mean ``w_e`` nS excitatory, ``g_inh`` times that inhibitory), conductance LIF with
    AMPA + NMDA (Mg block, 1 mM; NMDA weight ``nmda`` of AMPA's) from excitatory sources
    and GABA_A from inhibitory ones, short-term depression on both (U=0.2, tau_rec=200 ms,
    no facilitation), refractoriness, dt=0.1 ms, T=5,000, batch 4, 15 Hz Poisson input to
    5% of the neurons (weight ``w_in`` nS); forward only, made for the neuron partition.
    Chosen here: the weights and the input (the specification leaves them open). At these
    values the network fires at ~2 Hz in irregular population bursts (the oracle at
    20,000 neurons with the same degree); ``w_e`` 0.6 with ``g_inh`` 3 runs away to
    200 Hz."""
    from wiretorch_b200.types import Gate

    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    pos = torch.rand((N, 3), generator=gen, device=dev)
    exc_n = torch.rand(N, generator=gen, device=dev) < 0.8
    src, dst = _distance_edges(gen, pos, mean_degree, lam, dev)
    w = torch.exp(math.log(w_e) - 0.5 + torch.randn(src.numel(), generator=gen, device=dev))
    e = exc_n[src]
    w = torch.where(e, w, w * g_inh)
    rows_e, rows_i = torch.nonzero(exc_n).flatten(), torch.nonzero(~exc_n).flatten()
    row_of = torch.empty(N, dtype=torch.int64, device=dev)
    row_of[rows_e] = torch.arange(rows_e.numel(), device=dev)
    row_of[rows_i] = torch.arange(rows_i.numel(), device=dev)
    W_e = _csr_from_edges(row_of[src[e]], dst[e], w[e], rows_e.numel(), N)
    W_i = _csr_from_edges(row_of[src[~e]], dst[~e], w[~e], rows_i.numel(), N)
    n_edges = int(src.numel())
    out_deg = torch.bincount(src, minlength=N)
    del src, dst, w, e
    n_in = max(1, int(round(0.05 * N)))
    driven = torch.randperm(N, generator=gen, device=dev)[:n_in]
    W_in = _csr_from_edges(torch.arange(n_in, device=dev), driven, torch.full((n_in,), w_in, device=dev), n_in, N)
    # synapse types: 0 AMPA (E), 1 NMDA (E), 2 GABA_A (I), 3 AMPA (input)
    S_params = [(0.0, 5.0, 0.0, 1.0), (2.0, 100.0, 0.0, nmda), (0.0, 10.0, -80.0, 1.0), (0.0, 5.0, 0.0, 1.0)]
    made = torch.tensor([[1, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1]], dtype=torch.bool, device=dev)
    d_D = math.exp(-0.1 / tau_rec)
    params = torch.tensor([0.0, 0.0, U, d_D, 0.0], device=dev)
    n_e, n_i = rows_e.numel(), rows_i.numel()
    gates = [Gate(params, stp=True, saturates=False, start=0, n=n_e),
             Gate(params, stp=True, saturates=False, start=2 * n_e, n=n_i), None]  # fmt: skip
    drive = Drive(made=made, scale=torch.ones(3, N, device=dev), recurrent=[(rows_e, W_e), (rows_i, W_i)],
                  feedforward=[(torch.arange(n_in, device=dev), W_in)], gates=gates)  # fmt: skip
    p = _physiology(N, None, 0.1, S_params, dev)
    p.mg_c = torch.tensor([0.0, 1.0 / 3.57, 0.0, 0.0], device=dev)
    p.mg_a = torch.full((4,), 0.062, device=dev)
    deg = torch.cat([out_deg, torch.ones(n_in, dtype=torch.int64, device=dev)])
    cfg = Config("c5", drive, p, B, T, N, n_in, torch.full((n_in,), 15.0, device=dev),
                 (~exc_n).long(), 2, deg)  # fmt: skip
    cfg.extra["edges"] = n_edges
    R = 2 * (n_e + n_i)
    gating = torch.empty((B, R), device=dev)
    gating[:, : n_e] = U
    gating[:, n_e : 2 * n_e] = 1.0
    gating[:, 2 * n_e : 2 * n_e + n_i] = U
    gating[:, 2 * n_e + n_i :] = 1.0
    cfg.extra["gating"] = gating  # release probabilities at U, resources full
    return cfg
