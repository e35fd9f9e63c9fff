"""The engine's host-side tables (``wiretorch_b200.plan``) describe the reference's drive.

Built on the CPU from the golden cases' ``Drive``s, the slots, chunks and folded edges
must reproduce, for any set of active sources, every channel's input exactly as the
reference computes it: ``sum_k made_k * scale_k * (pre_k @ W_k)`` per synapse type
(``conductance/dynamics.py:95-100, 204-208``). No GPU involved: the chunks are walked
in Python.
"""

import numpy as np
import pytest
import torch

import golden_io
from wiretorch_b200 import plan as P
from wiretorch_b200._lib import CHUNK_EDGES


def _walk(plan, pre_rec, pre_ff):
    """Input channels of one trial from the plan's tables: (C, N) float64."""
    t = plan.tensors
    N = plan.N
    X = np.zeros((plan.ch.C, N))
    src_slot = t["src_slot"].numpy()
    slot_chunk = t["slot_chunk"].numpy()
    np.testing.assert_array_equal(t["src_chunk"].numpy(), slot_chunk[src_slot])
    desc = t["chunk_desc"].numpy()
    begin, length = desc & ((1 << 56) - 1), desc >> 56
    cols = t["edge_col"].numpy().astype(np.int64) & 0xFFFFFFFF
    w = P.edge_weights(plan).numpy().astype(np.float64)
    assert (t["edge_cw"].numpy() & 0xFFFFFFFF == cols).all()
    values = np.concatenate([pre_rec, pre_ff])
    for j in np.nonzero(values)[0]:
        for slot in range(src_slot[j], src_slot[j + 1]):
            for chunk in range(slot_chunk[slot], slot_chunk[slot + 1]):
                assert 0 < length[chunk] <= CHUNK_EDGES
                e = slice(begin[chunk], begin[chunk] + length[chunk])
                np.add.at(X, (cols[e] >> 27, cols[e] & 0x7FFFFFF), values[j] * w[e])
    return X / np.asarray(plan.fx_scale.double())[:, None]


def _reference_input(drive, p, pre_rec, pre_ff):
    """Per synapse type s: sum_k made[k, s] * jump_d[s] * scale_k * (pre_k @ W_k)."""
    made = drive.made.numpy()
    scale = drive.scale.double().numpy()
    jd = p.jump[1].double().numpy()
    N, S = scale.shape[1], made.shape[1]
    out = np.zeros((S, N))
    paths = [(r, W, pre_rec) for r, W in drive.recurrent]
    paths += [(r, W, pre_ff) for r, W in drive.feedforward]
    for k, (rows, W, pre) in enumerate(paths):
        a = pre[rows.numpy()] @ W.double().numpy()
        for s in range(S):
            if made[k, s]:
                out[s] += jd[s] * scale[k] * a
    return out


@pytest.mark.parametrize("pool", [False, True])
@pytest.mark.parametrize("name", ["recurrent_scaling_factors", "feedforward_learnt_weights",
                                  "recurrent_stp", "recurrent_saturation"])  # fmt: skip
def test_plan_reproduces_the_drive(name, pool):
    drive, p, d, meta = golden_io.load(name)
    n_in = d["in.x"].shape[2]
    plan = P.build(drive, p, 2, n_in, "cpu", pool=pool)
    P.fold(plan, drive.scale)
    rng = np.random.default_rng(0)
    N = plan.N
    pre_rec = (rng.random(N) < 0.2).astype(np.float64)
    pre_ff = rng.random(n_in) * (rng.random(n_in) < 0.3)
    X = _walk(plan, pre_rec, pre_ff)
    expected = _reference_input(drive, p, pre_rec, pre_ff)
    ch = plan.ch
    for c, members in enumerate(ch.member):
        total = sum(expected[s] for s in members)
        if ch.input_of[c] < 0:
            assert np.abs(total).max() == 0
            continue
        # channel c's decay component receives jump_d * X
        got = ch.jump_d[c] * X[ch.input_of[c]]
        np.testing.assert_allclose(got, total, rtol=1e-6, atol=1e-9)


def test_pooling_merges_identical_types():
    """Two source cell types whose synapse types share every dynamic parameter pool
    into one channel; distinct ones stay apart."""
    drive, p, d, meta = golden_io.load("recurrent_frozen")
    exact = P.build(drive, p, 2, d["in.x"].shape[2], "cpu", pool=False)
    assert exact.ch.Sp == drive.made.shape[1]
    pooled = P.build(drive, p, 2, d["in.x"].shape[2], "cpu", pool=True)
    assert pooled.ch.Sp <= exact.ch.Sp
    for members in pooled.ch.member:
        keys = {(float(p.decay[0, s]), float(p.decay[1, s]), float(p.E_syn[s])) for s in members}
        assert len(keys) == 1


def test_chunks_split_long_rows():
    """A source with more than CHUNK_EDGES targets gets several chunks, each at most
    CHUNK_EDGES long, covering its row once."""
    from wiretorch_b200.types import Drive, Physiology

    N = 700
    W = torch.zeros(3, N)
    W[0] = 1.0
    W[1, :5] = 2.0
    drive = Drive(made=torch.ones(1, 1, dtype=torch.bool), scale=torch.ones(1, N),
                  recurrent=[(torch.tensor([0, 3, 9]), W)])  # fmt: skip
    one = torch.ones(N)
    p = Physiology(theta=one, U_reset=one, E_L=one, C_m=one, beta=one * 0.5,
                   E_syn=torch.zeros(1), g_clip=torch.full((1,), float("inf")),
                   decay=torch.full((2, 1), 0.5), jump=torch.tensor([[-1.0], [1.0]]),
                   dt=torch.tensor(1.0), surr_scale=torch.tensor(1.0))  # fmt: skip
    plan = P.build(drive, p, 1, 0, "cpu")
    t = plan.tensors
    assert plan.n_chunks == -(-N // CHUNK_EDGES) + 1
    lens = t["chunk_len"][t["slot_chunk"][0] : t["slot_chunk"][1]]
    assert int(lens.sum()) == N and int(lens.max()) <= CHUNK_EDGES


@pytest.mark.parametrize("max_edges", [1, 7, 200, 1 << 26])
def test_edge_runs_cover_every_edge_once(max_edges):
    """The bounded runs of edges (used for the fixed-point bounds) visit every edge once,
    with its chunk's pathway, whatever the run size."""
    drive, p, d, meta = golden_io.load("recurrent_frozen")
    plan = P.build(drive, p, 2, d["in.x"].shape[2], "cpu", pool=False)
    seen = torch.full((plan.n_edges,), -1, dtype=torch.int64)
    count = torch.zeros(plan.n_edges, dtype=torch.int64)
    for pos, path in P._edge_runs(plan, max_edges=max_edges):
        seen[pos] = path
        count.index_add_(0, pos, torch.ones_like(pos))
    assert bool((count == 1).all())
    t = plan.tensors
    for q in range(plan.n_chunks):
        b, n = int(t["chunk_begin"][q]), int(t["chunk_len"][q])
        assert bool((seen[b : b + n] == int(t["chunk_path"][q])).all())


def test_source_gate_table_resolves_single_slots():
    """``src_gate``: a source with one slot carries that slot's gate and row; a source
    with several carries -2; one without slots, -1 (the C5 model at 2,000 neurons, and
    the same with 100 of its excitatory sources in a second gated pathway)."""
    from wiretorch_b200 import configs
    from wiretorch_b200.types import Gate, SparseRows

    cfg = configs.c5(B=2, T=10, device="cpu", N=2000, mean_degree=100.0, lam=0.2)
    d = cfg.drive
    rows_e, W_e = d.recurrent[0]
    n = 100
    end = int(W_e.row_ptr[n])
    d.recurrent = [*d.recurrent, (rows_e[:n].clone(), SparseRows(W_e.row_ptr[: n + 1], W_e.cols[:end],
                                                                 W_e.values[:end], W_e.n_targets))]  # fmt: skip
    d.made = torch.cat([d.made[:2], d.made[:1], d.made[2:]])
    d.scale = torch.cat([d.scale[:2], d.scale[:1], d.scale[2:]])
    R0 = max(g.start + g.width for g in d.gates if g is not None)
    d.gates = [d.gates[0], d.gates[1], Gate(d.gates[0].params, True, True, R0, n), None]
    plan = P.build(d, cfg.p, cfg.B, cfg.n_in, "cpu")
    t = plan.tensors
    table = t["src_gate"].numpy()
    src_slot, slot_gate, slot_row = t["src_slot"].numpy(), t["slot_gate"].numpy(), t["slot_row"].numpy()
    assert table.shape == (cfg.N + cfg.n_in, 2)
    for j in range(cfg.N + cfg.n_in):
        s0, ns = src_slot[j], src_slot[j + 1] - src_slot[j]
        if ns == 1:
            assert tuple(table[j]) == (slot_gate[s0], slot_row[s0])
        else:
            assert table[j, 0] == (-2 if ns > 1 else -1)
    assert (table[:, 0] == -2).sum() == n
    assert (table[cfg.N :, 0] == -1).all()  # the input columns are ungated
