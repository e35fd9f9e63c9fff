"""Neuron-partitioned runs: the network's neurons cut into blocks, one block per rank
(one process per GPU), every rank simulating its block for all trials.

A rank holds the state of its neurons and every edge that ends on them (its sources are
all ranks' neurons and the input columns). Each step the forward kernel of every rank
writes the spike words of its neurons (32 neurons of one trial per 32-bit word) into the
replicated spike words of every rank — peer stores over NVLink into buffers mapped with
CUDA IPC, no collective call — then publishes its progress into every rank's progress
slots; once all ranks have published the step, each rank emits the events of every
source from the words into its own targets. The next step's scatter and update follow,
so the exchange of step t + 1's spikes costs one wait per step (``WT_F_PARTITION``).

Blocks are whole 32-neuron words. The inputs ``x`` are replicated on every rank, and so
is the gating state of gated pathways. When every neuron owns at most one slot (one
pathway), a neuron's gate is stepped by the rank that owns the neuron alone, which
writes the factor of each of its spikes beside the spike words (``amps``, peer stores
like the words); after the call the ranks gather the gating state, each column from the
rank that stepped it (``_gather_gating``). Otherwise every rank steps every source's
gates alike from the words. Input columns' gates are stepped on every rank (the inputs
are replicated). The run is forward only (no saving for a backward pass). The
fixed-point synaptic sums make a partitioned run's spikes identical to a one-GPU run's.
"""

from __future__ import annotations

import copy

import torch


def blocks(N: int, P: int) -> list[tuple[int, int]]:
    """The neurons ``[n0, n1)`` of each of P ranks: contiguous runs of whole 32-neuron
    words, as even as the words allow."""
    words = -(-N // 32)
    if words < P:
        raise ValueError(f"{N} neurons are fewer than one 32-neuron word for each of {P} ranks")
    cuts = [words * r // P for r in range(P + 1)]
    return [(cuts[r] * 32, min(N, cuts[r + 1] * 32)) for r in range(P)]


def _restrict(W, n0: int, n1: int):
    """The columns ``[n0, n1)`` of a pathway's weights (dense or ``SparseRows``), as
    ``SparseRows`` with targets renumbered from 0."""
    from wiretorch_b200.types import SparseRows

    if isinstance(W, SparseRows):
        cols = W.cols.long()
        keep = (cols >= n0) & (cols < n1)
        counts = torch.diff(W.row_ptr)
        rows = torch.repeat_interleave(torch.arange(counts.numel(), device=cols.device), counts)
        rows = rows[keep]
        row_ptr = torch.zeros_like(W.row_ptr)
        row_ptr[1:] = torch.cumsum(torch.bincount(rows, minlength=counts.numel()), 0)
        return SparseRows(row_ptr, (cols[keep] - n0).to(torch.int32), W.values.detach()[keep].contiguous(), n1 - n0)
    return W.detach()[:, n0:n1].contiguous()


def local_network(drive, p, n0: int, n1: int):
    """``(drive, p)`` of the rank holding neurons ``[n0, n1)``: every pathway's edges onto
    those neurons (sources keep their global indices), the per-target scales and the
    per-neuron physiology of the block."""
    d = copy.copy(drive)
    d.recurrent = [(rows, _restrict(W, n0, n1)) for rows, W in drive.recurrent]
    d.feedforward = [(rows, _restrict(W, n0, n1)) for rows, W in drive.feedforward]
    d.scale = drive.scale.detach()[:, n0:n1].contiguous()
    q = copy.copy(p)
    for name in ("theta", "U_reset", "E_L", "C_m", "beta", "n_ref", "adapt", "adapt_decay", "E_adapt"):
        t = getattr(p, name, None)
        if isinstance(t, torch.Tensor) and t.dim() == 1 and t.numel() == drive.scale.shape[1]:
            setattr(q, name, t.detach()[n0:n1].contiguous())
    return d, q


def _cuda(result):
    """The values of a cuda-python runtime call, raising on its error code."""
    from cuda.bindings import runtime as rt

    err, *vals = result
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"CUDA runtime: {rt.cudaGetErrorString(err)[1].decode()}")
    return vals[0] if len(vals) == 1 else vals


class Partition:
    """This rank's block and the buffers shared with the other ranks (``group``: a
    ``torch.distributed`` group of one process per GPU, any backend; used on the host
    only, to exchange the buffers' CUDA IPC handles). The shared buffers are a
    ``cudaMalloc`` of their own, so that their IPC handle is their allocation's; call
    ``close`` on every rank, after a barrier, when the runs are over."""

    def __init__(self, N: int, B: int, group=None):
        import torch.distributed as dist
        from cuda.bindings import runtime as rt

        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.P > 8:
            raise NotImplementedError("at most 8 ranks")
        self.N, self.B = N, B
        self.n0, self.n1 = blocks(N, self.P)[self.rank]
        self.words_src = -(-N // 32)
        words_bytes = -(-(2 * B * self.words_src * 4) // 256) * 256
        amps_off = words_bytes + 256  # after the progress slots (8 x 8 bytes)
        total = amps_off + 2 * B * self.words_src * 32 * 4
        self._allocs, self._opened = [], []
        bases = self._shared(total)
        self._base = self._allocs[0]
        self.peer_words = bases
        self.peer_progress = [b + words_bytes for b in bases]
        self.peer_amps = [b + amps_off for b in bases]
        self.words, self.progress = bases[self.rank], bases[self.rank] + words_bytes
        self.epoch = 0
        self._push = {}  # per local plan: the tables and areas of pushed events
        dist.barrier(group=group)

    def _shared(self, nbytes: int) -> list:
        """A zeroed ``cudaMalloc`` of ``nbytes`` on every rank (collective), mapped into the
        others with CUDA IPC: the base address of every rank's, as this rank sees it."""
        import torch.distributed as dist
        from cuda.bindings import runtime as rt

        torch.cuda.synchronize()
        base = _cuda(rt.cudaMalloc(max(int(nbytes), 256)))
        _cuda(rt.cudaMemset(base, 0, max(int(nbytes), 256)))
        _cuda(rt.cudaDeviceSynchronize())
        self._allocs.append(base)
        handle = _cuda(rt.cudaIpcGetMemHandle(base))
        handles = [None] * self.P
        dist.all_gather_object(handles, bytes(handle.reserved), group=self.group)
        bases = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                bases.append(int(base))
                continue
            h = rt.cudaIpcMemHandle_t()
            h.reserved = hb
            peer = _cuda(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess))
            self._opened.append(peer)
            bases.append(int(peer))
        return bases

    def push_tables(self, plan) -> dict:
        """What a rank that pushes its events needs (collective, once per local plan):
        every rank's chunk range of every neuron and chunk descriptors (local copies), and
        an inbound event area on every rank with a region per source rank (sized for each
        source rank's neurons' chunks there, every trial) and inbound counts."""
        import torch.distributed as dist

        key = id(plan)
        if key in self._push:
            return self._push[key]
        t = plan.tensors
        dev = plan.device
        N_src = plan.N_src
        sc = t["src_chunk"][: N_src + 1].contiguous()
        n_chunks = int(sc[-1])
        cd = t["chunk_desc"][:n_chunks].contiguous()
        P = self.P
        sizes = [None] * P
        dist.all_gather_object(sizes, n_chunks, group=self.group)
        # every rank's tables, through the host (any backend)
        scs = [None] * P
        dist.all_gather_object(scs, sc.cpu(), group=self.group)
        cds = [None] * P
        dist.all_gather_object(cds, cd.cpu(), group=self.group)
        src_chunk = [x.to(dev) for x in scs]
        chunk_desc = [(x if x.numel() else torch.zeros(1, dtype=torch.int64)).to(dev) for x in cds]
        # this rank's inbound area: a region per source rank q (its neurons' chunks here)
        mine = inbound_layout([int(sc[n1] - sc[n0]) for n0, n1 in blocks(self.N, P)], self.B)
        bases = self._shared(mine[3] + 2 * 8 * 4)
        layout = [None] * P  # every rank's regions and where its inbound counts sit
        dist.all_gather_object(layout, mine, group=self.group)
        reserve = torch.zeros(2 * 8, dtype=torch.int32, device=dev)
        tables = {"src_chunk": src_chunk, "chunk_desc": chunk_desc, "reserve": reserve,
                  **push_pointers(self.rank, bases, layout)}  # fmt: skip
        self._push[key] = tables
        return tables

    def fill(self, run, plan=None) -> None:
        """The partition's fields of a ``WtForward`` for the next call (a new epoch); the
        amplitude buffers too when ``plan``'s gates are stepped by their owners."""
        self.epoch += 1
        run.words, run.progress = self.words, self.progress
        for r in range(self.P):
            run.peer_words[r] = self.peer_words[r]
            run.peer_progress[r] = self.peer_progress[r]
        run.n_ranks, run.rank, run.word0, run.epoch = self.P, self.rank, self.n0 // 32, self.epoch
        if plan is not None and owner_gates(plan):
            run.amps = self.peer_amps[self.rank]
            for r in range(self.P):
                run.peer_amps[r] = self.peer_amps[r]
        if plan is not None and PUSH and (not plan.gated or owner_gates(plan)):
            tb = self.push_tables(plan)
            for r in range(self.P):
                run.push_src_chunk[r] = tb["src_chunk"][r].data_ptr()
                run.push_chunk_desc[r] = tb["chunk_desc"][r].data_ptr()
                run.push_ev[r], run.push_cap[r] = tb["push_ev"][r], tb["push_cap"][r]
                run.push_half[r], run.push_count[r] = tb["push_half"][r], tb["push_count"][r]
                run.pull_off[r] = tb["pull_off"][r]
            tb["reserve"].zero_()  # every call starts with no reservation (even after a failed one)
            run.push_reserve = tb["reserve"].data_ptr()
            run.pull_ev, run.pull_half, run.pull_count = tb["pull_ev"], tb["pull_half"], tb["pull_count"]

    def close(self) -> None:
        from cuda.bindings import runtime as rt

        for peer in self._opened:
            _cuda(rt.cudaIpcCloseMemHandle(peer))
        self._opened = []
        for base in self._allocs:
            _cuda(rt.cudaFree(base))
        self._allocs, self._base, self._push = [], None, {}


def inbound_layout(chunks_of_ranks: list, B: int) -> tuple:
    """A rank's inbound event area: per source rank q the room for its neurons' chunks
    here (``chunks_of_ranks[q]``) in every trial, the regions' starts, one step parity's
    events, and the byte offset of the inbound counts ([2][8] uint32) after both
    parities' events."""
    caps = [B * int(c) for c in chunks_of_ranks]
    offs = [0]
    for c in caps[:-1]:
        offs.append(offs[-1] + c)
    half = sum(caps)
    counts_off = -(-(2 * half * 16) // 256) * 256
    return caps, offs, half, counts_off


def push_pointers(rank: int, bases: list, layouts: list) -> dict:
    """Where rank ``rank`` writes and reads pushed events, from every rank's area base (as
    this rank sees it) and every rank's ``inbound_layout``: its region of each rank r's
    area (events), that region's room, r's parity stride, and r's inbound counts — each
    at r's own offsets — and its own area."""
    caps, offs, half, counts_off = layouts[rank]
    P = len(bases)
    return {"push_ev": [bases[r] + layouts[r][1][rank] * 16 for r in range(P)],
            "push_cap": [layouts[r][0][rank] for r in range(P)],
            "push_half": [layouts[r][2] for r in range(P)],
            "push_count": [bases[r] + layouts[r][3] for r in range(P)],
            "pull_ev": bases[rank], "pull_off": offs, "pull_half": half,
            "pull_count": bases[rank] + counts_off}  # fmt: skip


#: Ranks push their events straight into every rank's inbound area (one grid barrier a
#: step) where the network has no gating or its owners step the gates; False: the spike
#: words are published and every rank walks them (two more grid barriers a step).
PUSH = True


def owner_gates(plan) -> bool:
    """Whether each neuron's gate can be stepped by the rank that owns the neuron alone:
    a gated network with the per-source gate table in which no neuron owns several
    slots (a spike then carries one factor)."""
    t = plan.tensors
    if not plan.gated or "src_gate" not in t:
        return False
    if "_owner_gates" not in t:
        t["_owner_gates"] = not bool((t["src_gate"][: plan.N_src, 0] == -2).any())
    return t["_owner_gates"]


def gating_owners(plan, P: int) -> torch.Tensor:
    """``(R,)`` int64: per column of the gating state, the rank that steps it in an
    owner-stepped run (the rank holding the column's source neuron), or -1 for the
    columns every rank steps alike (input columns' gates, unused columns)."""
    t = plan.tensors
    if "_gating_owners" not in t:
        R = plan.R
        owner = torch.full((R,), -1, dtype=torch.int64, device=plan.device)
        sg = t["src_gate"][: plan.N_src].long()
        j = (sg[:, 0] >= 0).nonzero().flatten()
        if j.numel():
            gate, row = sg[j, 0], sg[j, 1]
            cols = t["gate_cols"].long()[gate]  # (k, 4): u column, rows, saturation column, -
            cuts = torch.tensor([b[0] for b in blocks(plan.N_src, P)[1:]], device=plan.device)
            rank = torch.bucketize(j, cuts, right=True)
            stp, sat = cols[:, 0] >= 0, cols[:, 2] >= 0
            owner[(cols[:, 0] + row)[stp]] = rank[stp]
            owner[(cols[:, 0] + cols[:, 1] + row)[stp]] = rank[stp]
            owner[(cols[:, 2] + row)[sat]] = rank[sat]
        t["_gating_owners"] = owner
    return t["_gating_owners"]


def _gather_gating(part, plan, gating) -> None:
    """After an owner-stepped run: every rank's gating state made whole, in place — each
    column taken from the rank that stepped it (the others' copies of it are stale)."""
    import torch.distributed as dist

    owner = gating_owners(plan, part.P)
    if owner.numel() < gating.shape[1]:  # columns past the gates' own: nobody's
        owner = torch.cat([owner, owner.new_full((gating.shape[1] - owner.numel(),), -1)])
    on_gpu = dist.get_backend(part.group) == "nccl"
    mine = gating if on_gpu else gating.cpu()
    parts = [torch.empty_like(mine) for _ in range(part.P)]
    dist.all_gather(parts, mine.contiguous(), group=part.group)
    stacked = torch.stack(parts)  # (P, B, R)
    src = torch.where(owner < 0, part.rank, owner).to(stacked.device)
    whole = stacked[src, :, torch.arange(owner.numel(), device=stacked.device)]  # (R, B)
    gating.copy_(whole.t())


_LOCAL: dict = {}


def simulate(part: Partition, v, g, x, drive, p, *, refractory=None, gating=None, adaptation=None, pool=None):
    """This rank's block of a neuron-partitioned forward run: ``engine.simulate`` for the
    neurons ``[part.n0, part.n1)`` of the network ``(drive, p)`` (all ranks call it with
    the full network and input, and the full state or their block's own, as a previous
    call returned it). Returns the block's ``Run`` (spikes ``(B, T, n1 - n0)``, its
    state). Synchronises the device and the ranks once per call."""
    from wiretorch_b200 import engine, plan as _plan

    if not x.is_cuda:
        raise RuntimeError("wiretorch_b200 runs on CUDA tensors only (no CPU path)")
    n0, n1 = part.n0, part.n1
    key = (id(drive), id(p), part.rank, part.P, x.shape[0], x.shape[2])
    cached = _LOCAL.get(key)
    if cached is None or cached["drive"] is not drive or cached["p"] is not p:
        d_loc, p_loc = local_network(drive, p, n0, n1)
        pool_ = engine.POOL_SYNAPSES if pool is None else pool
        plan = _plan.build(d_loc, p_loc, x.shape[0], x.shape[2], x.device, pool=pool_, n_src=part.N)
        # the network objects are held, so that their ids cannot pass to others
        cached = _LOCAL[key] = {"drive": drive, "p": p, "local": (d_loc, p_loc, plan),
                                "scale": drive.scale, "version": drive.scale._version}  # fmt: skip
    d_loc, p_loc, plan = cached["local"]
    if cached["scale"] is not drive.scale or cached["version"] != drive.scale._version:
        d_loc.scale = drive.scale.detach()[:, n0:n1].contiguous()  # a new per-target scale
        cached["scale"], cached["version"] = drive.scale, drive.scale._version
    _plan.fold(plan, d_loc.scale)
    local = v.shape[1] == n1 - n0 != part.N  # the block's own state (a previous call's Run)
    cut = (lambda t: t) if local else (lambda t: None if t is None else t[:, n0:n1])  # noqa: E731
    # the gating state is whole on every rank (owner-stepped columns gathered after the run)
    v_k, g_k, counter, g_a, gating_k = engine._prepare_state(plan, cut(v), cut(g), cut(refractory), gating,
                                                             cut(adaptation), p_loc)  # fmt: skip
    # All ranks' kernels start together (their exchange waits are bounded), and none
    # starts before every rank's previous call has finished reading the shared words.
    import torch.distributed as dist

    torch.cuda.synchronize()
    dist.barrier(group=part.group)
    with torch.no_grad():
        out = engine.run_forward(plan, p_loc, x.detach().float(), v_k, g_k, counter, g_a, gating_k, part=part)
    if gating_k is not None and owner_gates(plan):
        _gather_gating(part, plan, gating_k)
    return engine._run(plan, out, v_k, g_k, counter, g_a, gating_k, p_loc, False, refractory)
