"""From the reference's ``Drive`` and ``Physiology`` to the tables the kernels read.

The reference hands its engine, per forward call, one ``Drive``: ``K`` pathways (one per
source cell type and input side, recurrent first), each its source rows and their
dense ``(n_rows, N)`` weights, the synapse types each makes (``made`` ``(K, S)``) and a
per-target kernel scale (``scale`` ``(K, N)``); a pathway's activation
``a_k = pre_k @ W_k`` enters every synapse type it makes as
``g += a_k * jump * scale_k`` (``conductance/dynamics.py:95-100, 204-208``).

The kernels see the same thing event by event:

* **Channels.** The conductance state carries ``S'`` channels per neuron, each with a
  rise and a decay component. By default a channel is a synapse type (``S' = S``,
  exact). Its *input channel* is the set of pathways that make it: types made by the
  same pathways (one source cell type's AMPA and NMDA, say) share one input
  accumulator ``X_c``, and ``g_type += jump_type * X_c``.
  With ``pool=True``, synapse types whose dynamics are identical (decays, reversal
  potential, Mg block; no clip, and jumps ``(-J, +J)`` as ``conductance_kernel`` makes
  them) are pooled into one channel: its conductance is the sum of theirs, which the
  membrane only ever reads summed (exact when nothing clips: the per-type sums are
  non-negative), and each pathway's weights carry its type's ``J``. A network of 40
  excitatory cell types then carries 2 channels (excitatory, inhibitory), not 40.
  The state the engine returns holds each pool's conductance at its first member type
  and zeros at the others; reading such a state back sums it into the pool again.
* **Edges.** Every pathway's weights become CSR rows over its targets with the kernel
  scale folded in: ``w_e = W[r, n] * scale_k[n] * jf_k,c``, once per input channel
  ``c`` the pathway feeds (``jf`` is 1, or the pooled ``J``). The input accumulators are
  64-bit fixed point: weights are stored times ``2^s_c``, with ``s_c`` chosen from the
  largest possible input of the channel (every in-edge of a neuron at once) with
  ``2^20`` to spare for spike amplitudes and scale drift.
* **Slots and chunks.** A source (a neuron, or an input column) has one slot per
  pathway it belongs to (several for the short-term-plasticity or saturation splits of
  one cell type); each slot's edges are cut into chunks of at most ``CHUNK_EDGES``,
  the unit of work of the scatter, so that hubs with thousands of targets do not
  serialise a warp.
"""

from __future__ import annotations

import math
import weakref
from dataclasses import dataclass, field

import torch

from wiretorch_b200 import _lib
from wiretorch_b200._lib import CHUNK_EDGES, MAX_CHANNELS

#: Headroom of the fixed-point input accumulators, in powers of two, above the largest
#: input a channel can receive from unit spikes at the weights seen when the plan was
#: built (for input values, facilitation and learnt scales).
FIXED_POINT_HEADROOM = 20


def _csr(W, device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(row_ptr int64, cols int32, values float32)`` of dense weights (or SparseRows)."""
    if hasattr(W, "row_ptr"):
        return (W.row_ptr.to(device, torch.int64), W.cols.to(device, torch.int32),
                W.values.detach().to(device, torch.float32))  # fmt: skip
    W = W.detach().to(device, torch.float32)
    nz = W.nonzero()
    rows, cols = nz[:, 0], nz[:, 1]
    counts = torch.bincount(rows, minlength=W.shape[0])
    row_ptr = torch.zeros(W.shape[0] + 1, dtype=torch.int64, device=device)
    row_ptr[1:] = torch.cumsum(counts, 0)
    return row_ptr, cols.to(torch.int32), W[rows, cols].contiguous()


# Weight structure is cached per weight tensor: fixed and scaling-factor pathways hand
# the engine the same cached tensors every call (network.py:754-764).
_CSR_CACHE: dict = {}


def csr_of(W, device):
    key = W.values if hasattr(W, "row_ptr") else W
    version = getattr(key, "_version", 0)
    hit = _CSR_CACHE.get(id(key))
    if (hit is not None and hit[0]() is key and hit[1] == version
            and hit[2][0].device == torch.device(device)):  # fmt: skip
        return hit[2]
    out = _csr(W, device)
    if len(_CSR_CACHE) > 256:
        for k in [k for k, v in _CSR_CACHE.items() if v[0]() is None]:
            del _CSR_CACHE[k]
    _CSR_CACHE[id(key)] = (weakref.ref(key), version, out)
    return out


@dataclass
class Channels:
    """How the ``S`` synapse types map onto the kernel's channels."""

    S: int  # synapse types of the API state
    Sp: int  # channels the kernel carries
    C: int  # input channels
    member: list  # per channel: the synapse types it holds
    input_of: list  # per channel: its input channel (-1: no input)
    jump_r: list
    jump_d: list
    jf: torch.Tensor  # (K, C) float32: weight factor of pathway k into input channel c
    pooled: bool


def _channels(made: torch.Tensor, p, pool: bool) -> Channels:
    """Exact per-type channels, or pooled ones (see the module docstring)."""
    made = made.detach().cpu().bool()
    K, S = made.shape
    jr = p.jump[0].detach().cpu().float()
    jd = p.jump[1].detach().cpu().float()
    members: list[list[int]] = []
    if pool and not any(_requires_grad(getattr(p, n)) for n in ("E_syn", "decay", "jump")):
        keys = {}
        dr = p.decay[0].detach().cpu().float()
        dd = p.decay[1].detach().cpu().float()
        E = p.E_syn.detach().cpu().float()
        clip = p.g_clip.detach().cpu().float()
        mgc = p.mg_c.detach().cpu().float() if p.mg_c is not None else torch.zeros(S)
        mga = p.mg_a.detach().cpu().float() if p.mg_a is not None else torch.zeros(S)
        for s in range(S):
            # a double exponential (jump_r = -jump_d), or a single one (no rise: the
            # current-based family's currents)
            single = float(dr[s]) == 0.0 and float(jr[s]) == 0.0
            poolable = bool(torch.isinf(clip[s])) and (float(jr[s]) == -float(jd[s]) or single)
            key = (
                (float(dr[s]), float(dd[s]), float(E[s]), float(mgc[s]), float(mga[s]))
                if poolable
                else ("alone", s)
            )
            if key not in keys:
                keys[key] = len(members)
                members.append([])
            members[keys[key]].append(s)
    else:
        members = [[s] for s in range(S)]
    pooled = any(len(m) > 1 for m in members)
    Sp = len(members)
    if pooled:
        C = Sp
        input_of = [c if bool(made[:, m].any()) else -1 for c, m in enumerate(members)]
        jf = torch.zeros((K, C))
        for c, m in enumerate(members):
            for s in m:
                jf[:, c] += made[:, s].float() * jd[s]
        jump_r = [-1.0] * Sp
        jump_d = [1.0] * Sp
    else:
        columns: dict[tuple, int] = {}
        input_of = []
        for m in members:
            col = tuple(made[:, m[0]].tolist())
            if not any(col):
                input_of.append(-1)
                continue
            if col not in columns:
                columns[col] = len(columns)
            input_of.append(columns[col])
        C = max(len(columns), 1)
        jf = torch.zeros((K, C))
        for col, c in columns.items():
            jf[:, c] = torch.tensor(col, dtype=torch.float32)
        jump_r = [float(jr[m[0]]) for m in members]
        jump_d = [float(jd[m[0]]) for m in members]
    return Channels(S, Sp, C, members, input_of, jump_r, jump_d, jf, pooled)


def _requires_grad(t) -> bool:
    return isinstance(t, torch.Tensor) and t.requires_grad


@dataclass
class Plan:
    """Everything the kernels need that does not change from call to call (``net``),
    plus the per-call folded weights."""

    B: int
    N: int
    n_in: int
    K: int
    K_rec: int
    ch: Channels
    device: torch.device
    tensors: dict = field(default_factory=dict)  # device tables the WtNet points into
    fx_scale: torch.Tensor | None = None  # (C,) 2^s_c, on the device
    fx_exp: list = field(default_factory=list)
    n_slots: int = 0
    n_chunks: int = 0
    n_rec_edges: int = 0
    n_edges: int = 0
    R: int = 0
    R_f: int = 0
    gated: bool = False
    gate_f_cols: list = field(default_factory=list)  # per pathway: saved-factor column, -1
    N_src: int = 0  # neurons that are sources (N, or every rank's in a partitioned run)

    def net_for_fold(self) -> _lib.WtNet:
        """A ``WtNet`` with the structure only (enough for ``wt_fold_weights``)."""
        n = _lib.WtNet()
        n.B, n.N, n.n_in, n.S, n.C = self.B, self.N, self.n_in, self.ch.Sp, self.ch.C
        t = self.tensors
        n.src_slot, n.slot_chunk = t["src_slot"].data_ptr(), t["slot_chunk"].data_ptr()
        n.src_chunk = t["src_chunk"].data_ptr()
        n.chunk_desc = t["chunk_desc"].data_ptr()
        n.edge_col = t["edge_col"].data_ptr()
        n.n_slots, n.n_chunks = self.n_slots, self.n_chunks
        n.N_src = self.N_src or self.N
        one = t.setdefault("_one", torch.ones(1, device=self.device))
        n.theta = n.U_reset = n.E_L = n.C_m = n.beta = one.data_ptr()
        return n

    def net(self, p) -> _lib.WtNet:
        """The ``WtNet`` of this plan with physiology ``p`` (pointers into tensors that
        the caller keeps alive)."""
        n = _lib.WtNet()
        n.B, n.N, n.n_in, n.S, n.C = self.B, self.N, self.n_in, self.ch.Sp, self.ch.C
        keep = self.tensors.setdefault("_phys", {})
        for name in ("theta", "U_reset", "E_L", "C_m", "beta", "adapt", "adapt_decay", "E_adapt"):
            t = getattr(p, name)
            if t is not None:
                t = t.detach().to(self.device, torch.float32).contiguous()
                keep[name] = t
                setattr(n, name, t.data_ptr())
        if p.n_ref is not None:
            t = p.n_ref.to(self.device, torch.int32).contiguous()
            keep["n_ref"] = t
            n.n_ref = t.data_ptr()
        dr = p.decay[0].detach().cpu().float()
        dd = p.decay[1].detach().cpu().float()
        E = p.E_syn.detach().cpu().float()
        clip = p.g_clip.detach().cpu().float()
        for c, members in enumerate(self.ch.member):
            s = members[0]
            n.decay_r[c], n.decay_d[c] = float(dr[s]), float(dd[s])
            n.jump_r[c], n.jump_d[c] = self.ch.jump_r[c], self.ch.jump_d[c]
            n.E_syn[c], n.g_clip[c] = float(E[s]), float(clip[s])
            if p.mg_c is not None:
                mg_c = float(p.mg_c[s])
                n.mg_a[c] = float(p.mg_a[s])
                n.mg_lc[c] = math.log(mg_c) if mg_c > 0 else -math.inf
            else:
                n.mg_a[c], n.mg_lc[c] = 0.0, -math.inf
            n.input_of[c] = self.ch.input_of[c]
        for c in range(self.ch.C):
            n.fx_inv[c] = 2.0 ** (-self.fx_exp[c])
        n.dt = float(p.dt)
        n.surr_scale = float(p.surr_scale)
        t = self.tensors
        n.src_slot, n.slot_chunk = t["src_slot"].data_ptr(), t["slot_chunk"].data_ptr()
        n.src_chunk = t["src_chunk"].data_ptr()
        n.chunk_desc = t["chunk_desc"].data_ptr()
        n.edge_col, n.edge_cw = t["edge_col"].data_ptr(), t["edge_cw"].data_ptr()
        n.n_slots, n.n_chunks = self.n_slots, self.n_chunks
        n.n_rec_edges = self.n_rec_edges
        if self.gated:
            n.slot_gate, n.slot_row = t["slot_gate"].data_ptr(), t["slot_row"].data_ptr()
            n.gate_params, n.gate_cols = t["gate_params"].data_ptr(), t["gate_cols"].data_ptr()
            if "src_gate" in t:  # without it the kernel walks every gated source's slots
                n.src_gate = t["src_gate"].data_ptr()
        n.R, n.R_f = self.R, self.R_f
        n.N_src = self.N_src or self.N
        return n


def build(drive, p, B: int, n_in: int, device, pool: bool = False, n_src: int | None = None) -> Plan:
    """Compile the structure of ``drive`` (weights are folded per call: ``fold``).
    ``n_src``: the neurons that are sources, when they are not the N targets (one rank of
    a neuron-partitioned run: its targets, every rank's neurons as sources)."""
    device = torch.device(device)
    N = int(drive.scale.shape[1])
    N_src = N if n_src is None else int(n_src)
    pathways = [(r, W, True) for r, W in drive.recurrent]
    pathways += [(r, W, False) for r, W in drive.feedforward]
    K = len(pathways)
    ch = _channels(drive.made, p, pool)
    if ch.Sp > MAX_CHANNELS or ch.C > MAX_CHANNELS:
        raise NotImplementedError(
            f"{ch.Sp} synapse channels ({ch.C} input channels): the kernels carry at most "
            f"{MAX_CHANNELS}; pool synapse types with identical dynamics (pool=True)"
        )
    plan = Plan(B=B, N=N, n_in=n_in, K=K, K_rec=len(drive.recurrent), ch=ch, device=device)

    # Segments (pathway k, input channel c) of the edge arrays.
    seg_cols, seg_vals, seg_base, seg_of = [], [], [], []  # seg_of[k] = [(c, base)]
    csrs = []
    base = 0
    for k, (rows, W, _) in enumerate(pathways):
        row_ptr, cols, vals = csr_of(W, device)
        csrs.append(row_ptr)
        segs = []
        for c in range(ch.C):
            if float(ch.jf[k, c]) == 0.0:
                continue
            seg_cols.append(cols.to(torch.int64) | (c << 27))
            seg_vals.append(vals)
            segs.append((c, base))
            base += int(cols.numel())
        seg_of.append(segs)
    plan.n_edges = base
    # the recurrent pathways' segments come first in the edge arrays
    plan.n_rec_edges = sum(int(csrs[k][-1]) * len(seg_of[k]) for k in range(len(drive.recurrent)))
    plan.seg_meta = [(k, c, b0, int(csrs[k][-1])) for k, segs in enumerate(seg_of) for c, b0 in segs]
    plan.csr_row_ptr = csrs
    edge_col = (torch.cat(seg_cols).to(torch.int32) if seg_cols
                else torch.zeros(1, dtype=torch.int32, device=device))  # fmt: skip
    w_raw = torch.cat(seg_vals) if seg_vals else torch.zeros(1, device=device)

    # Slots: (pathway, row), ordered by source (neurons, then input columns) and pathway.
    src_l, path_l, row_l = [], [], []
    for k, (rows, W, rec) in enumerate(pathways):
        rows = rows.to(device, torch.int64)
        src_l.append(rows if rec else rows + N_src)
        path_l.append(torch.full_like(rows, k))
        row_l.append(torch.arange(rows.numel(), device=device))
    if src_l:
        src, path, row = torch.cat(src_l), torch.cat(path_l), torch.cat(row_l)
    else:
        src = path = row = torch.zeros(0, dtype=torch.int64, device=device)
    order = torch.argsort(src * max(K, 1) + path)
    src, path, row = src[order], path[order], row[order]
    plan.N_src = N_src
    plan.path_sources = src_l  # per pathway: the source of each of its rows
    n_src = N_src + n_in
    src_slot = torch.zeros(n_src + 1, dtype=torch.int64, device=device)
    src_slot[1:] = torch.cumsum(torch.bincount(src, minlength=n_src), 0)
    plan.n_slots = int(src.numel())

    # Chunks of every (slot, segment), in slot order.
    pair_slot, pair_begin, pair_len, pair_path = [], [], [], []
    for k in range(K):
        mine = (path == k).nonzero().flatten()
        if mine.numel() == 0 or not seg_of[k]:
            continue
        r = row[mine]
        row_ptr = csrs[k]
        start, length = row_ptr[r], row_ptr[r + 1] - row_ptr[r]
        for c, b0 in seg_of[k]:
            pair_slot.append(mine)
            pair_begin.append(start + b0)
            pair_len.append(length)
            pair_path.append(torch.full_like(mine, k))
    if pair_slot:
        ps, pb, pl, pp = (torch.cat(v) for v in (pair_slot, pair_begin, pair_len, pair_path))
        o = torch.argsort(ps, stable=True)
        ps, pb, pl, pp = ps[o], pb[o], pl[o], pp[o]
        nchunk = (pl + CHUNK_EDGES - 1) // CHUNK_EDGES
        total = int(nchunk.sum())
        owner = torch.repeat_interleave(torch.arange(ps.numel(), device=device), nchunk)
        first = torch.cumsum(nchunk, 0) - nchunk
        within = torch.arange(total, device=device) - first[owner]
        chunk_begin = pb[owner] + within * CHUNK_EDGES
        chunk_len = torch.clamp(pl[owner] - within * CHUNK_EDGES, max=CHUNK_EDGES)
        chunk_path = pp[owner]
        per_slot = torch.zeros(plan.n_slots, dtype=torch.int64, device=device)
        per_slot.index_add_(0, ps, nchunk)
    else:
        total = 0
        chunk_begin = torch.zeros(1, dtype=torch.int64, device=device)
        chunk_len = torch.zeros(1, dtype=torch.int64, device=device)
        chunk_path = torch.zeros(1, dtype=torch.int64, device=device)
        per_slot = torch.zeros(plan.n_slots, dtype=torch.int64, device=device)
    slot_chunk = torch.zeros(plan.n_slots + 1, dtype=torch.int64, device=device)
    slot_chunk[1:] = torch.cumsum(per_slot, 0)
    plan.n_chunks = total
    if total >= 2**31 or plan.n_edges >= 2**62:
        raise NotImplementedError("more than 2^31 chunks")

    # Presynaptic gating: one gate per gated pathway.
    gates = list(drive.gates) if drive.gates else [None] * K
    gate_index, params, cols, f_cols, R_f = {}, [], [], [], 0
    for k, gate in enumerate(gates):
        if gate is None:
            f_cols.append(-1)
            continue
        gate_index[k] = len(params)
        params.append(gate.params.detach().to(device, torch.float32).reshape(5))
        stp_col = gate.start if gate.stp else -1
        sat_col = gate.start + 2 * gate.n * int(gate.stp) if gate.saturates else -1
        cols.append([stp_col, gate.n, sat_col, R_f])
        f_cols.append(R_f)
        R_f += gate.n
    plan.gated = bool(gate_index)
    plan.R_f = R_f
    plan.gate_f_cols = f_cols
    t = plan.tensors
    if plan.gated:
        lookup = torch.full((K,), -1, dtype=torch.int64)
        for k, g in gate_index.items():
            lookup[k] = g
        t["slot_gate"] = lookup.to(device)[path].to(torch.int32).contiguous()
        t["slot_row"] = row.to(torch.int32).contiguous()
        t["gate_params"] = torch.stack(params).contiguous()
        t["gate_cols"] = torch.tensor(cols, dtype=torch.int32, device=device).contiguous()
        plan.R = max(g.start + g.width for g in gates if g is not None)
        # per source: (gate, row) of its one slot, gate -1 when ungated or slotless,
        # -2 when it owns several slots
        n_slots_of = src_slot[1:] - src_slot[:-1]
        src_gate = torch.full((n_src, 2), -1, dtype=torch.int32, device=device)
        one = (n_slots_of == 1).nonzero().flatten()
        first = src_slot[:-1][one]
        src_gate[one, 0] = t["slot_gate"][first]
        src_gate[one, 1] = t["slot_row"][first]
        src_gate[n_slots_of > 1, 0] = -2
        t["src_gate"] = src_gate.contiguous()

    t["src_slot"] = src_slot.to(torch.int32).contiguous()
    t["slot_chunk"] = slot_chunk.to(torch.int32).contiguous()
    # a source's chunks are contiguous (its slots are, and so are their chunks)
    t["src_chunk"] = slot_chunk[src_slot].to(torch.int32).contiguous()
    t["chunk_desc"] = (chunk_begin | (chunk_len.to(torch.int64) << 56)).contiguous()
    t["chunk_len"] = chunk_len.to(torch.int32).contiguous()  # for the host-side walks
    t["chunk_begin"] = chunk_begin.contiguous()
    t["chunk_path"] = chunk_path.to(torch.int32).contiguous()
    t["edge_col"] = edge_col.contiguous()
    t["w_raw"] = w_raw.contiguous()
    t["slot_path"] = path.to(torch.int32).contiguous()
    t["slot_src"] = src.to(torch.int32).contiguous()
    t["jf"] = ch.jf.to(device).contiguous()
    return plan


def segments(plan: Plan) -> list:
    """Per (pathway, input channel) segment of the edge arrays: ``(k, c, base, n_edges,
    row of each edge, target of each edge)``, for scattering edge gradients back into
    the pathways' dense weights."""
    t = plan.tensors
    if "_segments" not in t:
        out = []
        for k, c, base, n_e in plan.seg_meta:
            row_ptr = plan.csr_row_ptr[k]
            rows = torch.repeat_interleave(torch.arange(row_ptr.numel() - 1, device=plan.device),
                                           row_ptr[1:] - row_ptr[:-1])  # fmt: skip
            cols = (t["edge_col"][base : base + n_e].to(torch.int64) & 0x7FFFFFF)
            out.append((k, c, base, n_e, rows, cols))
        t["_segments"] = out
    return t["_segments"]


def in_edges(plan: Plan) -> dict:
    """The in-edges of every target, for the target-by-target edge gradients: ``in_ptr``
    (N + 1) and per in-edge (ordered by target, then pathway and channel, then edge) its
    edge ``in_edge``, source ``in_src``, pathway and input channel ``in_path`` (k 8 + c)
    and — in gated networks — its gating factor's column of the saved factors
    ``in_fcol`` (-1: ungated); int32 each, built once per plan."""
    t = plan.tensors
    if "_in_edges" not in t:
        dev = plan.device
        E = max(plan.n_edges, 0)
        e_l, j_l, k_l, n_l, f_l = [], [], [], [], []
        for k, c, base, n_e, rows, cols in segments(plan):
            e_l.append(torch.arange(base, base + n_e, device=dev))
            j_l.append(plan.path_sources[k][rows])
            k_l.append(torch.full((n_e,), k * 8 + c, dtype=torch.int64, device=dev))
            n_l.append(cols)
            fc = plan.gate_f_cols[k] if plan.gated and k < len(plan.gate_f_cols) else -1
            f_l.append(rows + fc if fc >= 0 else torch.full((n_e,), -1, dtype=torch.int64, device=dev))
        if E and e_l:
            e, j, kk, n, f = (torch.cat(v) for v in (e_l, j_l, k_l, n_l, f_l))
            # edge order already (segments in order of their base); then stably by target
            # and pathway
            order = torch.argsort(n * (8 * max(plan.K, 1)) + kk, stable=True)
            e, j, kk, n, f = e[order], j[order], kk[order], n[order], f[order]
        else:
            e = j = kk = n = f = torch.zeros(0, dtype=torch.int64, device=dev)
        in_ptr = torch.zeros(plan.N + 1, dtype=torch.int64, device=dev)
        in_ptr[1:] = torch.cumsum(torch.bincount(n, minlength=plan.N), 0)
        out = {"in_ptr": in_ptr, "in_edge": e, "in_src": j, "in_path": kk}
        if plan.gated:
            out["in_fcol"] = f
        t["_in_edges"] = {name: v.to(torch.int32).contiguous() for name, v in out.items()}
    return t["_in_edges"]


def edge_pathway(plan: Plan) -> torch.Tensor:
    """The pathway of every edge (int64)."""
    e = torch.zeros(max(plan.n_edges, 1), dtype=torch.int64, device=plan.device)
    for pos, path in _edge_runs(plan):
        e[pos] = path
    return e


def _edge_runs(plan: Plan, max_edges: int = 1 << 26):
    """``(positions, pathways)`` (int64) of the edges of consecutive runs of chunks, about
    ``max_edges`` edges a run: bounded temporaries, whatever the network's size."""
    t = plan.tensors
    if not plan.n_chunks:
        return
    lens_all = t["chunk_len"].to(torch.int64)
    ends = torch.cumsum(lens_all, 0)
    # chunk boundaries of the runs: every chunk holds at most WT_CHUNK_EDGES edges
    cuts = torch.searchsorted(ends, torch.arange(max_edges, int(ends[-1]) + max_edges, max_edges,
                                                 device=ends.device), right=True).tolist()  # fmt: skip
    q0 = 0
    for q1 in cuts:
        q1 = min(max(q1, q0 + 1), plan.n_chunks)
        if q1 <= q0:
            continue
        lens = lens_all[q0:q1]
        idx = torch.repeat_interleave(torch.arange(q0, q1, device=plan.device), lens)
        within = torch.arange(idx.numel(), device=plan.device) - (torch.cumsum(lens, 0) - lens)[idx - q0]
        yield t["chunk_begin"][idx] + within, t["chunk_path"][idx].to(torch.int64)
        q0 = q1
        if q0 >= plan.n_chunks:
            break


def fold(plan: Plan, scale: torch.Tensor, p=None) -> None:
    """The folded edges of this call's ``scale``: ``edge_cw`` packs each edge's target
    word with the bits of ``w * scale[k, col] * jf[k, c] * 2^s_c`` — the
    ``wt_fold_weights`` kernel on CUDA (torch on the CPU, for the tests of the tables)."""
    t = plan.tensors
    src = scale
    if (p is None and "edge_cw" in t and t.get("_scale_src") is src
            and t.get("_scale_version") == src._version):  # fmt: skip
        return  # the same scale tensor, unchanged since the last fold: the edges hold it
    scale = scale.detach().to(plan.device, torch.float32).contiguous()
    if plan.fx_scale is None:
        _choose_fixed_point(plan, scale)
    if plan.n_edges == 0:
        t["edge_cw"] = torch.zeros(1, dtype=torch.int64, device=plan.device)
        return
    if plan.device.type != "cuda":
        k = edge_pathway(plan)
        packed = t["edge_col"].to(torch.int64) & 0xFFFFFFFF
        col, c = packed & 0x7FFFFFF, packed >> 27
        w = (t["w_raw"] * scale[k, col] * t["jf"][k, c] * plan.fx_scale[c]).contiguous()
        t["edge_cw"] = packed | (w.view(torch.int32).to(torch.int64) << 32)
        return
    if "edge_cw" not in t:
        t["edge_cw"] = torch.empty(plan.n_edges, dtype=torch.int64, device=plan.device)
    net = plan.net(p) if p is not None else plan.net_for_fold()
    with _lib.timed("wt_fold_weights"):
        rc = _lib.lib().wt_fold_weights(
            _lib.C.byref(net), _lib.C.c_void_p(t["w_raw"].data_ptr()),
            _lib.C.c_void_p(t["chunk_path"].data_ptr()), _lib.C.c_void_p(scale.data_ptr()),
            _lib.C.c_void_p(t["jf"].data_ptr()), _lib.C.c_void_p(plan.fx_scale.data_ptr()),
            _lib.C.c_void_p(t["edge_cw"].data_ptr()), _lib.C.c_void_p(_lib.stream_of(plan.device)),
        )
    _lib.check(rc, "wt_fold_weights")
    _lib.count_launches(1)
    plan.tensors["_scale"] = scale  # alive until the kernel has read it
    # held, so that its identity cannot pass to another tensor; its version counter
    # shows an in-place change
    t["_scale_src"], t["_scale_version"] = src, src._version


def edge_weights(plan: Plan) -> torch.Tensor:
    """The folded weights of ``edge_cw`` (float32), for inspection and tests."""
    return (plan.tensors["edge_cw"] >> 32).to(torch.int32).view(torch.float32)


def _choose_fixed_point(plan: Plan, scale: torch.Tensor) -> None:
    """Per input channel, the power of two its weights are stored at: the largest input
    a neuron's channel can get (all its in-edges at once) times 2^FIXED_POINT_HEADROOM
    stays below 2^62. Reads one small tensor back from the device, once per plan."""
    t = plan.tensors
    if plan.n_edges == 0:
        plan.fx_exp = [0] * plan.ch.C
        plan.fx_scale = torch.ones(plan.ch.C, device=plan.device)
        return
    bound = torch.zeros(plan.ch.C * plan.N, device=plan.device, dtype=torch.float64)
    for pos, k in _edge_runs(plan):
        packed = t["edge_col"][pos].to(torch.int64) & 0xFFFFFFFF
        col, c = packed & 0x7FFFFFF, packed >> 27
        w = t["w_raw"][pos] * scale[k, col] * t["jf"][k, c]
        bound.index_add_(0, c * plan.N + col, w.abs().double())
    bound = bound.view(plan.ch.C, plan.N).amax(1).cpu()
    exps = []
    for b in bound.tolist():
        b = max(b, 2.0**-30)
        exps.append(max(min(62 - FIXED_POINT_HEADROOM - math.ceil(math.log2(b)), 60), -60))
    plan.fx_exp = exps
    plan.fx_scale = torch.tensor([2.0**e for e in exps], device=plan.device, dtype=torch.float32)
