"""Small seeded networks for smoke checks and tests, built as the reference's networks
hand them to their engine (a ``Drive`` and a ``Physiology``).

``random_network`` is a conductance-based LIF network of excitatory and inhibitory
neurons with Erdos-Renyi recurrent connectivity, log-normal weights and Poisson input,
with the physiology of the reference's test networks (``tests/networks.py:63-83`` of
wiretorch: E/I cells, AMPA/NMDA/GABA_A synapse types). Options add its features:
refractory periods, a Mg block, adaptation.
"""

from __future__ import annotations

import numpy as np
import torch

from wiretorch_b200.types import Drive, Physiology


def _kernel(tau_rise, tau_decay, g_bar):
    """Jumps of the rise and decay components per unit input, normalised so the
    difference of exponentials peaks at ``g_bar`` (``conductance/synapses.py:70-87``)."""
    r = tau_rise / tau_decay
    peak = r ** (r / (1 - r)) - r ** (1 / (1 - r))
    return torch.stack([-g_bar, g_bar]) / peak


def random_network(N=300, n_in=100, B=2, T=100, seed=0, dt=1.0, tau_ref=None, mg=None,
                   adapt=None, device="cpu"):  # fmt: skip
    """``(drive, p, x, v, g, kw)`` of a seeded network and its input."""
    rng = np.random.default_rng(seed)
    types = (rng.random(N) < 0.2).astype(np.int64)  # 0 excitatory, 1 inhibitory
    w_mean = np.where(types == 0, 0.3, 1.8)
    p_conn = np.where(types == 0, 0.15, 0.3) * 150 / N
    W = rng.lognormal(np.log(w_mean)[:, None] - 0.35, 0.83, (N, N))
    W *= rng.random((N, N)) < p_conn[:, None]
    W_ff = rng.lognormal(np.log(0.18) - 0.35, 0.83, (n_in, N)) * (rng.random((n_in, N)) < 0.3 * 80 / n_in)
    x = (rng.random((B, T, n_in)) < 0.01 * dt).astype(np.float32)
    f = lambda a: torch.tensor(np.asarray(a, dtype=np.float32), device=device)  # noqa: E731
    rows_e = torch.tensor(np.flatnonzero(types == 0), device=device)
    rows_i = torch.tensor(np.flatnonzero(types == 1), device=device)
    # synapse types: 0 AMPA(E), 1 NMDA(E), 2 GABA_A(I), 3 AMPA(input), 4 NMDA(input)
    tau_rise = f([0.1, 10.0, 0.5, 0.1, 10.0])
    tau_decay = f([5.0, 60.0, 6.0, 5.0, 70.0])
    g_bar = f([4.0, 0.5, 8.0, 6.0, 0.1])
    made = torch.tensor([[1, 1, 0, 0, 0], [0, 0, 1, 0, 0], [0, 0, 0, 1, 1]], dtype=torch.bool,
                        device=device)  # fmt: skip
    drive = Drive(
        made=made,
        scale=torch.ones(3, N, device=device),
        recurrent=[(rows_e, f(W[types == 0])), (rows_i, f(W[types == 1]))],
        feedforward=[(torch.arange(n_in, device=device), f(W_ff))],
    )
    tau_mem = np.where(types == 0, 85.0, 50.0)
    g_L = np.where(types == 0, 1.35, 0.9)
    dtt = torch.tensor(dt, device=device)
    p = Physiology(
        theta=f(np.where(types == 0, -38.0, -45.0)),
        U_reset=f(np.full(N, -60.0)),
        E_L=f(np.full(N, -60.0)),
        C_m=f(tau_mem * g_L),
        beta=torch.exp(-dtt / f(tau_mem)),
        E_syn=f([0.0, 0.0, -70.0, 0.0, 0.0]),
        g_clip=f([40.0, 4.0, 80.0, 40.0, 4.0]),
        decay=torch.exp(-dtt / torch.stack([tau_rise, tau_decay])),
        jump=_kernel(tau_rise, tau_decay, g_bar),
        dt=dtt,
        surr_scale=torch.tensor(5.0, device=device),
    )
    if tau_ref is not None:
        p.n_ref = torch.full((N,), int(round(tau_ref / dt)), dtype=torch.int32, device=device)
    if mg is not None:
        p.mg_c = f([0.0, mg / 3.57, 0.0, 0.0, mg / 3.57])
        p.mg_a = f([0.062] * 5)
    if adapt is not None:
        p.adapt = f(np.where(types == 0, adapt, 0.0))
        p.adapt_decay = f(np.exp(-dt / np.full(N, 200.0)))
        p.E_adapt = f(np.full(N, -90.0))
    v = torch.full((B, N), -60.0, device=device)
    g = torch.zeros((B, 2, 5, N), device=device).permute(0, 3, 1, 2)
    kw = {"refractory": torch.zeros((B, N), dtype=torch.int32, device=device)}
    if adapt is not None:
        kw["adaptation"] = torch.zeros((B, N), device=device)
    return drive, p, torch.from_numpy(x).to(device), v, g, kw


def lowrank_network(N=300, B=130, T=60, rank=32, seed=0, dt=0.5, double_exp=False, device="cpu"):
    """A seeded factorised network: excitatory and inhibitory sources with recurrent
    weights ``W = U V^T`` (non-negative factors, rank ``rank``), one Poisson input column
    per neuron. Returns ``(drive_lowrank, drive_dense, p, x, v, g, kw)``: the same network
    with ``LowRank`` weights and with the assembled dense ones."""
    from wiretorch_b200.lowrank import LowRank
    from wiretorch_b200.types import SparseRows

    rng = np.random.default_rng(seed)
    f = lambda a: torch.tensor(np.asarray(a, dtype=np.float32), device=device)  # noqa: E731
    exc = rng.random(N) < 0.8
    rows_e = torch.tensor(np.flatnonzero(exc), device=device)
    rows_i = torch.tensor(np.flatnonzero(~exc), device=device)
    V = f(np.abs(rng.normal(0, 1, (N, rank))) / np.sqrt(rank))
    U = f(np.abs(rng.normal(0, 1, (N, rank))) / np.sqrt(rank) * (4.0 / N))
    lr_e, lr_i = LowRank(U[rows_e], V), LowRank(U[rows_i] * 3.0, V)
    ar = torch.arange(N + 1, device=device)
    w_in = SparseRows(ar, ar[:-1].to(torch.int32), f(rng.uniform(8.0, 14.0, N)), N)
    # synapse types: 0 excitatory, 1 inhibitory (single exponentials unless double_exp)
    tau_rise = f([2.0, 0.0]) if double_exp else f([0.0, 0.0])
    tau_decay = f([5.0, 10.0])
    dtt = torch.tensor(dt, device=device)
    decay_r = torch.where(tau_rise > 0, torch.exp(-dtt / tau_rise.clamp(min=1e-6)), torch.zeros_like(tau_rise))
    decay = torch.stack([decay_r, torch.exp(-dtt / tau_decay)])
    jump = torch.stack([-torch.ones(2, device=device), torch.ones(2, device=device)])
    made = torch.tensor([[1, 0], [0, 1], [1, 0]], dtype=torch.bool, device=device)
    scale = torch.ones(3, N, device=device)
    drive_lr = Drive(made=made, scale=scale, recurrent=[(rows_e, lr_e), (rows_i, lr_i)],
                     feedforward=[(torch.arange(N, device=device), w_in)])  # fmt: skip
    drive_dense = Drive(made=made, scale=scale, recurrent=[(rows_e, lr_e.dense()), (rows_i, lr_i.dense())],
                        feedforward=[(torch.arange(N, device=device), w_in)])  # fmt: skip
    p = Physiology(
        theta=f(np.full(N, -50.0)), U_reset=f(np.full(N, -65.0)), E_L=f(np.full(N, -70.0)),
        C_m=f(np.full(N, 200.0)), beta=torch.exp(-dtt / 20.0) * torch.ones(N, device=device),
        E_syn=f([0.0, -80.0]), g_clip=f([float("inf")] * 2), decay=decay, jump=jump, dt=dtt,
        surr_scale=torch.tensor(10.0, device=device),
    )  # fmt: skip
    p.n_ref = torch.full((N,), int(round(2.0 / dt)), dtype=torch.int32, device=device)
    x = (torch.from_numpy(rng.random((B, T, N))) < 40.0 * dt / 1000.0).float().to(device)
    v = torch.full((B, N), -65.0, device=device) + f(rng.uniform(0, 14, (B, N)))
    g = torch.zeros((B, 2, 2, N), device=device).permute(0, 3, 1, 2)
    kw = {"refractory": torch.zeros((B, N), dtype=torch.int32, device=device)}
    return drive_lr, drive_dense, p, x, v, g, kw
