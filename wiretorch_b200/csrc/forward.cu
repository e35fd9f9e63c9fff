// The forward pass: one persistent cooperative kernel integrates T steps of the
// conductance-based LIF network (the time step of wiretorch's
// conductance/dynamics.py:146-237, which its Triton kernels scan_forward,
// compact_spikes and recurrent_step implement on CUDA).
//
// Work is cut into warp items: 32 consecutive neurons of one trial. The items, ordered
// neuron group by group and trial by trial within a group, are split into equal
// contiguous runs, one per warp of the grid, for the whole launch; a warp keeps its
// current group's constants in registers. When the warps' state fits in shared memory
// ("resident") it is read from HBM once at the start and written back once at the end;
// otherwise it streams through HBM every step. Every step, each warp stages its items'
// inputs (and streamed state) through a ring of shared-memory slots with asynchronous
// copies issued several items ahead, so that a warp keeps kilobytes of loads in flight
// while it computes. A channel whose rise component does not decay (a single-exponential
// synapse, tau_rise = 0) keeps no rise state: its rise is jump_r X of the previous step.
//
// Work per step t, over the whole grid, with one grid barrier between steps:
//
//   scatter (all warps): the events of step t — each a (trial, chunk of at most
//     WT_CHUNK_EDGES edges of one source's CSR row) — into X_t, the per
//     (input channel, trial, neuron) fixed-point accumulators: 64-bit integer
//     reductions, so the sum, and every result, is independent of the order in
//     which events land (bit-for-bit reproducible). The events were emitted during
//     step t - 1, so the reductions are issued first and drain while the warps go on.
//   update (every item of the warp, coalesced over neurons):
//     g_t = decay g_{t-1} + jump X_{t-1}           (completes the previous step's input)
//     s_t = H(v_t - theta) (1 - held)               (or escape noise)
//     v_{t+1} = exponential-Euler membrane step, reset where s_t or held
//     counters, adaptation; spikes, saved tensors, tracked variables
//     s_{t+1} from v_{t+1}: the spikes of the NEXT step are known already, so their
//     events are emitted now — one step of pipelining that lets the next step's
//     synaptic scatter run in the same phase as this step's membrane update.
//     Input columns likewise emit x_{t+1}'s non-zero entries.
//   Data that crosses blocks within the kernel (event lists, accumulators) is read
//   with L2-only loads: an SM's L1 is not coherent with the other SMs' writes.
//
// A presynaptic pathway with gating (short-term plasticity, receptor saturation:
// network.py:186-223) steps its state when its source's spike (or input) of the next
// step is known, and scales the events by the factor.
#include <algorithm>

#include "common.cuh"

namespace wt {

// Geometry of a launch, chosen by the host (see geometry_for).
struct Geometry {
    long long W;                  // warp items: groups x B
    int groups, Np;               // 32-neuron groups; accumulator row stride (N rounded up to 32)
    int resident;                 // state in shared memory
    int ks;                       // state words per item
    int w_cnt, w_ga, w_gd, w_gr;  // word offsets: counter, adaptation, decay, rise
    int max_items;                // most items of one warp
    int D;                        // ring slots per warp (copies issued D items ahead)
    int slot_rows, warp_rows;     // 128-byte rows of a ring slot, of a warp's shared memory
};

namespace {

// Asynchronous global -> shared copies (cp.async), grouped per thread. The 16-byte form
// reads through L2 only (data written by other SMs); the 4-byte form is used for data
// this SM alone writes.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most `pending` of this thread's groups are in flight.
__device__ __forceinline__ void cp_async_wait(int pending) {
    switch (pending) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
        case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    }
}

// One step of a slot's gating state for one trial (network.py:186-223) with the source's
// spike (or input) `s`: release probability u and resources x (short-term plasticity,
// `stp`), bound fraction a (receptor saturation, `sat`), in place. Returns the factor of
// the source's input. prm: the gate's (c, d, U, d_D, d_F).
__device__ __forceinline__ float gate_math(const float *prm, bool stp, bool sat, float &u, float &x, float &a,
                                           float s) {
    float f = 1.0f;
    if (stp) {
        const float U = prm[2], d_D = prm[3], d_F = prm[4];
        x = 1.0f - (1.0f - x) * d_D;
        u = U + (u - U) * d_F;
        const float r = u * x;
        f = r / U;
        x = x - s * r;
        u = u + s * U * (1.0f - u);
    }
    if (sat) {
        const float c = prm[0], d = prm[1];
        const float g = a * d;
        const float closed = 1.0f - g;
        f = stp ? fminf(c * f * closed, closed) : c * closed;
        a = fminf(g + s * f, 1.0f);
    }
    return f;
}

// Presynaptic gating of one slot for one trial: steps the state in the trial's gating
// row with `s` and returns the factor.
__device__ float gate_step(const WtNet &net, float *gating_b, int gate, int row, float s) {
    const int u_col = net.gate_cols[4 * gate + 0];
    const int n = net.gate_cols[4 * gate + 1];
    const int sat_col = net.gate_cols[4 * gate + 2];
    float u = 0.0f, x = 0.0f, a = 0.0f;
    if (u_col >= 0) {
        u = gating_b[u_col + row];
        x = gating_b[u_col + n + row];
    }
    if (sat_col >= 0) a = gating_b[sat_col + row];
    const float f = gate_math(net.gate_params + 5 * gate, u_col >= 0, sat_col >= 0, u, x, a, s);
    if (u_col >= 0) {
        gating_b[u_col + row] = u;
        gating_b[u_col + n + row] = x;
    }
    if (sat_col >= 0) gating_b[sat_col + row] = a;
    return f;
}

// The gating of a source that owns at most one slot (WtNet.src_gate), resolved once:
// its gate (-1: none, -2: several slots, walked by `emit`), the columns of its state in
// a trial's gating row (-1: not kept) and of its saved factor, the gate's parameters.
struct SrcGate {
    int gate, u_off, x_off, a_off, f_off;
    float prm[5];
};

__device__ __forceinline__ SrcGate src_gate_of(const WtNet &net, int j) {
    SrcGate G;
    const int2 gr = reinterpret_cast<const int2 *>(net.src_gate)[j];
    G.gate = gr.x;
    G.u_off = G.x_off = G.a_off = G.f_off = -1;
#pragma unroll
    for (int i = 0; i < 5; i++) G.prm[i] = 0.0f;
    if (gr.x >= 0) {
        const int4 cl = reinterpret_cast<const int4 *>(net.gate_cols)[gr.x];
        if (cl.x >= 0) {
            G.u_off = cl.x + gr.y;
            G.x_off = cl.x + cl.y + gr.y;
        }
        if (cl.z >= 0) G.a_off = cl.z + gr.y;
        G.f_off = cl.w + gr.y;
#pragma unroll
        for (int i = 0; i < 5; i++) G.prm[i] = net.gate_params[5 * gr.x + i];
    }
    return G;
}

__device__ __forceinline__ SrcGate no_gate() {
    SrcGate G;
    G.gate = -1;
    G.u_off = G.x_off = G.a_off = G.f_off = -1;
#pragma unroll
    for (int i = 0; i < 5; i++) G.prm[i] = 0.0f;
    return G;
}

// All 32 lanes call this together. Lane proposes source `j` of trial `b` whose spike
// (or input value) at step `step` is `value`; appends one event per chunk of each of
// its slots to that step's list, stepping the slots' gating first.
__device__ void emit(const WtNet &net, const WtForward &run, const WtWorkspace &ws, int step,
                     bool valid, int b, int j, float value, bool gated, int lane) {
    int s0 = 0, ns = 0;
    if (valid && (value != 0.0f || gated)) {
        s0 = net.src_slot[j];
        ns = net.src_slot[j + 1] - s0;
    }
    const int rounds = __reduce_max_sync(kFull, ns);
    const bool save = run.flags & WT_F_SAVE;
    const int t_abs = run.t0 + step;
    for (int k = 0; k < rounds; k++) {
        int cnt = 0, c0 = 0;
        float amp = value;
        if (k < ns) {
            const int slot = s0 + k;
            if (gated) {
                const int gate = net.slot_gate[slot];
                if (gate >= 0) {
                    const int row = net.slot_row[slot];
                    const float f = gate_step(net, run.gating + (size_t)b * net.R, gate, row, value);
                    amp = value * f;
                    if (save)
                        run.f_saved[((size_t)b * run.T_total + t_abs) * net.R_f +
                                    net.gate_cols[4 * gate + 3] + row] = f;
                }
            }
            if (value != 0.0f) {
                c0 = net.slot_chunk[slot];
                cnt = net.slot_chunk[slot + 1] - c0;
            }
        }
        const int incl = warp_inclusive_sum(cnt, lane);
        const int total = __shfl_sync(kFull, incl, 31);
        if (total == 0) continue;
        unsigned base = 0;
        if (lane == 31) base = atomicAdd(&ws.ev_count[step], (unsigned)total);
        base = __shfl_sync(kFull, base, 31);
        const long long off = (long long)base + incl - cnt;
        const bool fits = off + cnt <= ws.ev_cap;  // per lane; no early exit before the
        if (!fits && cnt) set_error(ws.err, WT_ERR_EVENTS);  // next round's collectives
        if (fits) {
            WtEvent *evs = ws.ev + (size_t)(step & 1) * ws.ev_cap;
            for (int q = 0; q < cnt; q++) {
                const long long d = net.chunk_desc[c0 + q];
                WtEvent e;
                e.edge = d & ((1LL << 56) - 1);
                e.trial_len = ((uint32_t)b << 8) | (uint32_t)((unsigned long long)d >> 56);
                e.amp = amp;
                evs[off + q] = e;
            }
        }
    }
}

// Emission of ungated sources: a source's chunks are contiguous (src_chunk), so the warp
// reserves room for all its lanes' events with one atomic, then writes each spiking
// lane's events with all 32 lanes. `on`: the lane's source fires with `value`.
// A source's chunks are [c0, c0 + cnt) (its src_chunk range, which the caller has loaded).
__device__ __forceinline__ void emit_fast(const WtNet &net, const WtWorkspace &ws, int step, bool on, int b,
                                          int c0, int cnt, float value, int lane) {
    unsigned m = __ballot_sync(kFull, on);
    if (!m) return;
    if (!on) cnt = 0;
    const int incl = warp_inclusive_sum(cnt, lane);
    const int total = __shfl_sync(kFull, incl, 31);
    if (total == 0) return;
    unsigned base = 0;
    if (lane == 31) base = atomicAdd(&ws.ev_count[step], (unsigned)total);
    base = __shfl_sync(kFull, base, 31);
    int4 *evs = reinterpret_cast<int4 *>(ws.ev + (size_t)(step & 1) * ws.ev_cap);
    while (m) {
        const int l = __ffs(m) - 1;
        m &= m - 1;
        const int lc0 = __shfl_sync(kFull, c0, l), lcnt = __shfl_sync(kFull, cnt, l);
        const long long off = (long long)base + __shfl_sync(kFull, incl, l) - lcnt;
        const int amp = __float_as_int(__shfl_sync(kFull, value, l));
        for (int q = lane; q < lcnt; q += 32) {
            if (off + q >= ws.ev_cap) {
                set_error(ws.err, WT_ERR_EVENTS);
                break;
            }
            const unsigned long long d = (unsigned long long)net.chunk_desc[lc0 + q];
            evs[off + q] = make_int4((int)(unsigned)d, (int)(unsigned)((d >> 32) & 0xffffffu),
                                     (int)(((unsigned)b << 8) | (unsigned)(d >> 56)), amp);
        }
    }
}

// The spike of a neuron entering a step: deterministic threshold, or escape noise;
// none while refractory. Returns s and sets held.
__device__ __forceinline__ float spike_of(float v, float theta, int counter, float u, int flags,
                                          float k, float &held) {
    held = ((flags & WT_F_REFRACTORY) && counter > 0) ? 1.0f : 0.0f;
    float s;
    if (flags & WT_F_SAMPLE)
        s = u < sigmoid(k * (v - theta)) ? 1.0f : 0.0f;
    else
        s = (v - theta) > 0.0f ? 1.0f : 0.0f;
    if (flags & WT_F_REFRACTORY) s = s * (1.0f - held);
    return s;
}

static_assert(WT_CHUNK_EDGES <= 128, "a chunk's edges take at most four per lane");
// Feature bits of a specialised kernel: the refractory period, saving for the backward
// pass, the Mg block, presynaptic gating, adaptation and one rank of a neuron partition
// known at compile time; everything else (escape noise, probabilities, tracking, saved
// input) in the generic variant, tested at run time.
constexpr int kRef = 1, kSave = 2, kGeneric = 4, kMg = 8, kGate = 16, kAdapt = 32, kPart = 64, kCur = 128;

// Warps per block of the forward kernel (one block per SM): 24 for the specialised
// kernels of up to four channels (80 registers a thread, as good as no spill), WT_GATE_WARPS
// for those with the Mg block, gating, adaptation or a partition, 16 for the others (up
// to 128 registers).
#ifndef WT_GATE_WARPS
#define WT_GATE_WARPS 24
#endif
#ifndef WT_PLAIN_WARPS
#define WT_PLAIN_WARPS 24
#endif
template <int S, int FEAT>
constexpr int warps_of() {
    return ((FEAT & kGeneric) == 0 && S <= 4) ? ((FEAT & (kMg | kGate | kAdapt | kPart)) ? WT_GATE_WARPS : WT_PLAIN_WARPS)
                                              : 16;
}
#ifndef WT_MAX_RING
#define WT_MAX_RING 4
#endif
constexpr int kMaxRing = WT_MAX_RING;     // deepest ring of staged items


// A warp's position in its run of items: neuron group g, trial b, and the trial's row
// offsets in the (B, N) state, the (B, Np) accumulators and the (B, T_total, N) outputs.
struct Cursor {
    int g, b;
    size_t bN, bNp, bTN;
    __device__ void next(int B, int N, int Np, size_t TN) {
        if (++b == B) {
            b = 0;
            ++g;
            bN = bNp = bTN = 0;
        } else {
            bN += N;
            bNp += Np;
            bTN += TN;
        }
    }
};

// A neuron's constants (conductance/dynamics.py:116-143): the leak's rate from its decay
// beta, and g_L = C_m rate.
struct NeuronConsts {
    float theta, U_reset, E_L, Cm, rate, g_L, adapt, a_decay, E_a;
    int n_ref;
    int c0, cnt;  // the neuron's chunks (as a source)
};

template <int S, int FEAT>
__global__ void __launch_bounds__(warps_of<S, FEAT>() * 32, 1) forward_kernel(const WtNet net, const WtForward run,
                                                             const WtWorkspace ws, const Geometry geo) {
    extern __shared__ __align__(16) float smem[];
    constexpr bool GEN = FEAT & kGeneric;
    const int flags = run.flags;
    const bool REF = GEN ? (flags & WT_F_REFRACTORY) != 0 : (FEAT & kRef) != 0;
    const bool SAVE = GEN ? (flags & WT_F_SAVE) != 0 : (FEAT & kSave) != 0;
    const bool ADAPT = GEN ? (flags & WT_F_ADAPT) != 0 : (FEAT & kAdapt) != 0;
    const bool MG = GEN ? (flags & WT_F_MG_BLOCK) != 0 : (FEAT & kMg) != 0;
    const bool SAMPLE = GEN && (flags & WT_F_SAMPLE);
    const bool gated = GEN ? (flags & WT_F_GATED) != 0 : (FEAT & kGate) != 0;
    const bool PROB = GEN && (flags & WT_F_PROB);
    const bool TRACK = GEN && (flags & WT_F_TRACK);
    const bool SAVE_IN = GEN && (flags & WT_F_SAVE_INPUT);
    const bool PART = GEN ? (flags & WT_F_PARTITION) != 0 : (FEAT & kPart) != 0;
    // current-based neurons: a step's input enters the currents the same step's membrane
    // update uses, so every warp scatters first and a grid barrier completes X_t before
    // the items read it (the conductance step uses the input a step later)
    const bool CUR = GEN ? (flags & WT_F_CURRENT) != 0 : (FEAT & kCur) != 0;

    const int B = net.B, N = net.N, n_in = net.n_in, C = net.C, T = run.T, Np = geo.Np;
    const int Nsrc = net.N_src > 0 ? net.N_src : N;  // neuron sources (all ranks' when partitioned)
    const int words_src = (Nsrc + 31) >> 5;
    const int Ip = (n_in + 31) & ~31;
    const long long itemsI = (long long)B * Ip;
    const long long nthreads = (long long)gridDim.x * blockDim.x;
    const long long gtid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const long long warp0 = gtid - lane;
    const long long gwarp = gtid >> 5, nwarps = nthreads >> 5;
    const size_t BNp = (size_t)B * Np;
    const size_t TN = (size_t)run.T_total * N;  // one trial's (T, N) plane
    const int words = (N + 31) >> 5;
    const float dt = net.dt, ksur = net.surr_scale;
    const bool RES = geo.resident;
    const int D = geo.D, ks = geo.ks, w_cnt = geo.w_cnt, w_ga = geo.w_ga, w_gd = geo.w_gd;
    const int slot_words = geo.slot_rows * 32;
    GridBarrier bar(ws.barrier, gridDim.x);
    // instrumented runs: lane 0 of each warp stamps the end of each phase of a step
    unsigned long long *const phases =
        (run.phases && gwarp < run.phase_warps) ? run.phases + (size_t)gwarp * WT_PHASES : nullptr;
    const size_t phase_row = (size_t)run.phase_warps * WT_PHASES;
    auto stamp = [&](int t, int k) {
        if (phases && lane == 0) {
            unsigned long long g;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g));
            phases[(size_t)t * phase_row + k] = g;
        }
    };

    // Per channel: the input channel feeding it, that input's fixed-point scale, and the
    // state word of its rise component (-1: it does not decay and keeps none).
    int in_c[S], rw[S];
    float fx_c[S];
    {
        int r = 0;
#pragma unroll
        for (int c = 0; c < S; c++) {
            in_c[c] = net.input_of[c];
            fx_c[c] = in_c[c] >= 0 ? net.fx_inv[in_c[c]] : 0.0f;
            rw[c] = net.decay_r[c] != 0.0f ? geo.w_gr + r++ : -1;
        }
    }

    // This warp's items, and its shared memory: resident state [item][word][lane], then
    // the ring of D slots, each [input channel int64 x 32][streamed state word x 32].
    const long long lo = geo.W * gwarp / nwarps, hi = geo.W * (gwarp + 1) / nwarps;
    const int nitems = (int)(hi - lo);
    Cursor start;
    start.g = (int)(lo / B);
    start.b = (int)(lo % B);
    start.bN = (size_t)start.b * N;
    start.bNp = (size_t)start.b * Np;
    start.bTN = (size_t)start.b * TN;
    float *wsm = smem + (size_t)(threadIdx.x >> 5) * geo.warp_rows * 32;
    float *ring = wsm + (RES ? (size_t)geo.max_items * ks * 32 : 0);
    // a lane's 16-byte pieces of an item's accumulator rows: piece k = lane + 32 i covers
    // channel k / 16, neurons 2 (k % 16) and 2 (k % 16) + 1 of the group
    const size_t x_goff = (size_t)(lane >> 4) * BNp + (lane & 15) * 2;
    const int x_soff = (lane >> 4) * 64 + (lane & 15) * 4;

    auto consts_of = [&](int n) {
        NeuronConsts k{};
        k.Cm = 1.0f;
        if (n < N) {
            k.theta = net.theta[n];
            k.U_reset = net.U_reset[n];
            k.E_L = net.E_L[n];
            k.Cm = net.C_m[n];
            k.rate = -log1pf(net.beta[n] - 1.0f) / dt;
            k.g_L = CUR ? net.beta[n] : k.Cm * k.rate;  // current-based: the leak's decay beta
            k.n_ref = REF ? net.n_ref[n] : 0;
            k.c0 = net.src_chunk[n];
            k.cnt = net.src_chunk[n + 1] - k.c0;
            if (ADAPT) {
                k.adapt = net.adapt[n];
                k.a_decay = net.adapt_decay[n];
                k.E_a = CUR ? 0.0f : net.E_adapt[n];
            }
        }
        return k;
    };
    // Stage item j (at cursor q) into ring slot `wr`: the previous step's input of its C
    // channels (when `with_x`), and its state when streamed. One copy group per call.
    auto issue = [&](int j, const Cursor &q, int wr, const unsigned long long *Xsrc, bool with_x) {
        if (j < nitems) {
            float *slot = ring + wr * slot_words;
            if (with_x) {
                const unsigned long long *src = Xsrc + q.bNp + (size_t)q.g * 32 + x_goff;
                float *dst = slot + x_soff;
                for (int k = lane; k < C * 16; k += 32, src += 2 * BNp, dst += 128) cp_async16(dst, src);
            }
            const int n = q.g * 32 + lane;
            if (!RES && n < N) {
                const size_t o = q.bN + n;
                const float *g_b = run.g + q.bN * 2 * S + n;
                float *st = slot + 2 * C * 32 + lane;
                cp_async4(st, run.v + o);
                if (REF) cp_async4(st + w_cnt * 32, run.counter + o);
                if (ADAPT) cp_async4(st + w_ga * 32, run.g_a + o);
#pragma unroll
                for (int c = 0; c < S; c++) {
                    cp_async4(st + (w_gd + c) * 32, g_b + (size_t)(S + c) * N);
                    if (rw[c] >= 0) cp_async4(st + rw[c] * 32, g_b + (size_t)c * N);
                }
            }
        }
        cp_async_commit();
    };
    // a neuron's spike (its chunk range known), or an input column's value
    auto emit_neuron = [&](int step, bool valid, int b, int j, const NeuronConsts &k, float value) {
        if (gated)
            emit(net, run, ws, step, valid, b, j, value, true, lane);
        else
            emit_fast(net, ws, step, valid && value != 0.0f, b, k.c0, k.cnt, value, lane);
    };
    // A gated source j through its resolved gating (src_gate): the state of its one slot
    // stepped in place, then its events emitted with the factor; a source with several
    // slots in the warp sends the warp through `emit`.
    // One step of a resolved gate G (G.gate >= 0) for trial b with the source's value of
    // `step`; returns the factor.
    auto step_gate = [&](const SrcGate &G, int step, int b, float value) -> float {
        float *gb = run.gating + (size_t)b * net.R;
        float u = 0.0f, x = 0.0f, a = 0.0f;
        if (G.u_off >= 0) {
            u = gb[G.u_off];
            x = gb[G.x_off];
        }
        if (G.a_off >= 0) a = gb[G.a_off];
        const float f = gate_math(G.prm, G.u_off >= 0, G.a_off >= 0, u, x, a, value);
        if (G.u_off >= 0) {
            gb[G.u_off] = u;
            gb[G.x_off] = x;
        }
        if (G.a_off >= 0) gb[G.a_off] = a;
        if (SAVE) run.f_saved[((size_t)b * run.T_total + run.t0 + step) * net.R_f + G.f_off] = f;
        return f;
    };
    auto emit_src = [&](int step, bool valid, int b, int j, float value) {
        const SrcGate G = valid ? src_gate_of(net, j) : no_gate();
        if (__any_sync(kFull, G.gate == -2)) {
            emit(net, run, ws, step, valid, b, j, value, true, lane);
            return;
        }
        float amp = value;
        if (valid && G.gate >= 0) amp = value * step_gate(G, step, b, value);
        const bool on = valid && value != 0.0f;
        int c0 = 0, cnt = 0;
        if (on) {
            c0 = net.src_chunk[j];
            cnt = net.src_chunk[j + 1] - c0;
        }
        emit_fast(net, ws, step, on, b, c0, cnt, amp, lane);
    };
    const bool GSRC = gated && net.src_gate != nullptr;
    // Owner-stepped gates: a partitioned gated run whose neurons each own at most one slot
    // (the host checks, and passes the amplitude buffers only then). The rank that owns a
    // neuron alone steps its gate and writes its spike's factor into every rank's replica
    // of the amplitudes (2, B, words_src * 32), beside the spike words; the exchange reads
    // the factors back instead of stepping every source's gates on every rank.
    const bool OG = PART && GSRC && run.amps != nullptr;
    const size_t amp_row = (size_t)words_src * 32;
    auto publish_amp = [&](int step, int b, int jg, bool on, float amp) {
        if (on) {
            const size_t ai = ((size_t)(step & 1) * B + b) * amp_row + jg;
            for (int r = 0; r < run.n_ranks; r++) run.peer_amps[r][ai] = amp;
        }
    };
    auto emit_input = [&](int step, bool valid, int b, int j, float value) {
        if (GSRC) {
            emit_src(step, valid, b, j, value);
        } else if (gated) {
            emit(net, run, ws, step, valid, b, j, value, true, lane);
        } else {
            const bool on = valid && value != 0.0f;
            int c0 = 0, cnt = 0;
            if (on) {
                c0 = net.src_chunk[j];
                cnt = net.src_chunk[j + 1] - c0;
            }
            emit_fast(net, ws, step, on, b, c0, cnt, value, lane);
        }
    };

    // A partitioned run: the warp's spike word of `step` (32 neurons of trial b) into every
    // rank's replica of the words (this rank's among them).
    auto publish = [&](int step, int b, int g, float s) {
        const unsigned word = __ballot_sync(kFull, s > 0.0f);
        if (lane == 0) {
            const size_t wi = ((size_t)(step & 1) * B + b) * words_src + run.word0 + g;
            for (int r = 0; r < run.n_ranks; r++) run.peer_words[r][wi] = word;
        }
    };
    // A rank that pushes its events (PUSH): the warp's sources jg (this rank's neurons,
    // global indices) that fire at `step` with `amp` get their events onto every rank r's
    // targets written straight into r's inbound area: one reservation per warp and rank
    // (this rank's local counter), all 32 lanes writing each firing source's chunks.
    const bool PUSH = PART && run.push_reserve != nullptr;
    // the edges of the network (partitioned runs check every event's edges against them)
    long long n_edges_all = 0;
    if (PART && net.n_chunks > 0) {
        const unsigned long long d = (unsigned long long)net.chunk_desc[net.n_chunks - 1];
        n_edges_all = (long long)(d & ((1ull << 56) - 1)) + (long long)(d >> 56);
    }
    auto push = [&](int step, int b, int jg, bool on, float amp) {
        unsigned firing = __ballot_sync(kFull, on);
        const int P = run.n_ranks, par = step & 1;
        // one firing source at a time, its ranks across the lanes: lane r < P finds the
        // source's chunks on rank r and reserves room for them there, then the lanes write
        // all of the source's events on all ranks at once (three dependent round trips a
        // source, whatever the number of ranks)
        while (firing) {
            const int l = __ffs(firing) - 1;
            firing &= firing - 1;
            const int j = __shfl_sync(kFull, jg, l);
            const int bl = __shfl_sync(kFull, b, l);
            const int a = __float_as_int(__shfl_sync(kFull, amp, l));
            if (j < 0 || j >= Nsrc) {  // range checks of the pushed events: a record, no access
                if (lane == 0) set_error(ws.err, WT_ERR_RANGE | (1 << 8));
                continue;
            }
            int c0 = 0, cnt = 0;
            if (lane < P) {
                const int32_t *sc = run.push_src_chunk[lane];
                c0 = sc[j];
                cnt = sc[j + 1] - c0;
                if (cnt < 0 || c0 < 0 || c0 + cnt > sc[Nsrc]) {
                    set_error(ws.err, WT_ERR_RANGE | (2 << 8));
                    cnt = 0;
                }
            }
            unsigned base = 0;
            if (cnt > 0) base = atomicAdd(run.push_reserve + par * 8 + lane, (unsigned)cnt);
            const int incl = warp_inclusive_sum(cnt, lane);
            const int total = __shfl_sync(kFull, incl, 31);
            for (int i0 = 0; i0 < total; i0 += 32) {
                const int i = i0 + lane;  // event i of the source: rank r, its chunk k there
                int r = 0;
#pragma unroll
                for (int q = 0; q < 8; q++) r += q < P && __shfl_sync(kFull, incl, q) <= i;
                const int rr = min(r, 7);
                const int k = i - (__shfl_sync(kFull, incl, rr) - __shfl_sync(kFull, cnt, rr));
                const int cr = __shfl_sync(kFull, c0, rr);
                const long long off = (long long)__shfl_sync(kFull, base, rr) + k;
                if (i >= total) continue;
                if (off >= run.push_cap[rr]) {
                    set_error(ws.err, WT_ERR_EVENTS);
                    continue;
                }
                const unsigned long long d = (unsigned long long)run.push_chunk_desc[rr][cr + k];
                int4 *evs = reinterpret_cast<int4 *>(run.push_ev[rr] + (size_t)par * run.push_half[rr]);
                evs[off] = make_int4((int)(unsigned)d, (int)(unsigned)((d >> 32) & 0xffffffu),
                                     (int)(((unsigned)bl << 8) | (unsigned)(d >> 56)), a);
            }
        }
    };
    // ... and once every rank has published `step`, the events of that step of every
    // source from the words. The step's grid barrier is fused with the exchange of
    // progress (GridBarrier::sync_progress: the last block to arrive writes this rank's
    // progress slot, (epoch << 32) | step + 1, into every rank and waits, bounded, for
    // every rank's, before it releases the grid). Leaves after a second grid barrier;
    // false when an error ended the run.
    auto exchange = [&](int step) -> bool {
        const unsigned long long mine = ((unsigned long long)run.epoch << 32) | (unsigned)(step + 1);
        if (PUSH)  // the events are in place: the barrier publishes their counts with the progress
            return bar.sync_progress(ws.err, run.peer_progress, run.rank, run.progress, run.n_ranks, mine,
                                     run.push_reserve, run.push_count, step & 1);
        if (!bar.sync_progress(ws.err, run.peer_progress, run.rank, run.progress, run.n_ranks, mine)) return false;
        const uint32_t *wsrc = run.words + (size_t)(step & 1) * B * words_src;
        const long long n_words = (long long)B * words_src;
        // a warp takes 32 words at once (one per lane) and walks the ones with a spike;
        // with replicated gates it walks them all (every source's gates step)
        for (long long base = gwarp * 32; base < n_words; base += nwarps * 32) {
            const long long mine = base + lane;
            const unsigned my_word = mine < n_words ? __ldcg(wsrc + mine) : 0u;  // written by the ranks: L2
            unsigned todo = __ballot_sync(kFull, (gated && !OG) ? mine < n_words : my_word != 0u);
            while (todo) {
                const int l = __ffs(todo) - 1;
                todo &= todo - 1;
                const long long it = base + l;
                const unsigned word = __shfl_sync(kFull, my_word, l);
                const int b = (int)(it / words_src), w = (int)(it % words_src);
                const int j = w * 32 + lane;
                const bool on = (word >> lane) & 1u;
                if (gated && !OG) {  // every source's gates step, on every rank alike (replicated state)
                    if (GSRC)
                        emit_src(step, j < Nsrc, b, j, on ? 1.0f : 0.0f);
                    else
                        emit(net, run, ws, step, j < Nsrc, b, j, on ? 1.0f : 0.0f, true, lane);
                    continue;
                }
                int c0 = 0, cnt = 0;
                float amp = 1.0f;
                if (on) {
                    c0 = net.src_chunk[j];
                    cnt = net.src_chunk[j + 1] - c0;
                    if (OG) amp = __ldcg(run.amps + ((size_t)(step & 1) * B + b) * amp_row + j);  // the owner's factor
                }
                emit_fast(net, ws, step, on, b, c0, cnt, amp, lane);
            }
        }
        return bar.sync(ws.err);
    };

    // Phase 0: empty accumulators and event counts; resident state.
    for (long long i = gtid; i < 2LL * C * (long long)BNp; i += nthreads) ws.X[i] = 0ull;
    for (long long i = gtid; i <= T; i += nthreads) ws.ev_count[i] = 0u;
    if (RES) {
        Cursor q = start;
        float *rp = wsm + lane;
        for (int j = 0; j < nitems; j++, q.next(B, N, Np, TN), rp += ks * 32) {
            const int n = q.g * 32 + lane;
            if (n >= N) continue;
            const size_t o = q.bN + n;
            const float *g_b = run.g + q.bN * 2 * S + n;
            rp[0] = run.v[o];
            if (REF) rp[w_cnt * 32] = __int_as_float(run.counter[o]);
            if (ADAPT) rp[w_ga * 32] = run.g_a[o];
#pragma unroll
            for (int c = 0; c < S; c++) {
                rp[(w_gd + c) * 32] = g_b[(size_t)(S + c) * N];
                if (rw[c] >= 0) rp[rw[c] * 32] = g_b[(size_t)c * N];
            }
        }
    }
    if (!bar.sync(ws.err)) return;

    const int sflags = (REF ? WT_F_REFRACTORY : 0) | (SAMPLE ? WT_F_SAMPLE : 0);
    // Emit step 0's events: the spikes of the state entering the run, and x at t0.
    {
        Cursor q = start;
        int g_k = -1;
        NeuronConsts k{};
        const float *rp = wsm + lane;
        for (int j = 0; j < nitems; j++, q.next(B, N, Np, TN), rp += ks * 32) {
            const int n = q.g * 32 + lane;
            const bool valid = n < N;
            if (q.g != g_k) {
                k = consts_of(n);
                g_k = q.g;
            }
            float s = 0.0f;
            if (valid) {
                const size_t o = q.bN + n;
                const float v = RES ? rp[0] : run.v[o];
                const int cnt = REF ? (RES ? __float_as_int(rp[w_cnt * 32]) : run.counter[o]) : 0;
                const float u01 = SAMPLE ? run.noise[q.bTN + (size_t)run.t0 * N + n] : 0.0f;
                float held;
                s = spike_of(v, k.theta, cnt, u01, sflags, ksur, held);
            }
            if (PART) {
                float amp = s;
                const int jg = run.word0 * 32 + n;
                if (OG) {
                    const SrcGate G = valid ? src_gate_of(net, jg) : no_gate();
                    if (G.gate == -2) set_error(ws.err, WT_ERR_UNSUPPORTED);
                    if (valid && G.gate >= 0) amp = s * step_gate(G, 0, q.b, s);
                    if (!PUSH) publish_amp(0, q.b, jg, valid && s != 0.0f, amp);
                }
                if (PUSH)
                    push(0, q.b, jg, valid && s != 0.0f, amp);
                else
                    publish(0, q.b, q.g, s);
            } else {
                emit_neuron(0, valid, q.b, n, k, s);
            }
        }
    }
    for (long long base = warp0; base < itemsI; base += nthreads) {
        const unsigned i = (unsigned)(base + lane);  // B x Ip < 2^32 (checked by the host)
        const int b = (int)(i / (unsigned)Ip), c = (int)(i - (unsigned)b * Ip);
        const bool valid = c < n_in;
        const float xv = valid ? run.x[((size_t)b * run.T_total + run.t0) * n_in + c] : 0.0f;
        emit_input(0, valid, b, Nsrc + c, xv);
    }
    // The input columns this lane emits each step (one per warp-iteration of the grid
    // over B x Ip) are loaded a step ahead, so that the emission does not wait for them.
    constexpr int kXAhead = 4;
    float x_ahead[kXAhead];
    // ... and, in gated networks, whether any of those columns has a gated slot (the
    // columns are the same every step): the others emit without the gate table
    bool x_gated[kXAhead];
#pragma unroll
    for (int r = 0; r < kXAhead; r++) {
        x_gated[r] = false;
        const long long base = warp0 + (long long)r * nthreads;
        if (GSRC && base < itemsI) {
            const unsigned i = (unsigned)(base + lane);
            const int b = (int)(i / (unsigned)Ip), c = (int)(i - (unsigned)b * Ip);
            const bool g = c < n_in && net.src_gate[2 * (Nsrc + c)] != -1;
            x_gated[r] = __any_sync(kFull, g);
        }
    }
    auto load_x = [&](int step_abs) {
#pragma unroll
        for (int r = 0; r < kXAhead; r++) {
            const long long base = warp0 + (long long)r * nthreads;
            x_ahead[r] = 0.0f;
            if (base < itemsI && step_abs < run.t0 + T) {
                const unsigned i = (unsigned)(base + lane);
                const int b = (int)(i / (unsigned)Ip), c = (int)(i - (unsigned)b * Ip);
                if (c < n_in) x_ahead[r] = __ldcs(run.x + ((size_t)b * run.T_total + step_abs) * n_in + c);
            }
        }
    };
    load_x(run.t0 + 1);
    if (PART) {  // the barrier orders every thread's stores to the ranks before the progress
        if (!exchange(0)) return;
    } else if (!bar.sync(ws.err)) {
        return;
    }

    for (int t = 0; t < T; t++) {
        const int t_abs = run.t0 + t;
        const bool emit_next = t + 1 < T;
        const bool has_x = CUR || t > 0;
        // the input the items complete their state with: X_{t-1}, or X_t (current-based)
        unsigned long long *Xprev = ws.X + (size_t)((t + (CUR ? 0 : 1)) & 1) * C * BNp;
        stamp(t, 0);
        // The first D items' copies go out now and land while the warp scatters (after
        // the scatter's barrier when the items read this step's input).
        Cursor qi = start;
        int wr = 0;
        auto issue_first = [&]() {
            for (int d = 0; d < D; d++) {
                issue(d, qi, wr, Xprev, has_x);
                qi.next(B, N, Np, TN);
                if (++wr == D) wr = 0;
            }
        };
        if (!CUR) issue_first();

        // ---------------- the input columns of the next step ----------------
        if (emit_next) {
            int r = 0;
            for (long long base = warp0; base < itemsI; base += nthreads, r++) {
                const unsigned i = (unsigned)(base + lane);
                const int b = (int)(i / (unsigned)Ip), c = (int)(i - (unsigned)b * Ip);
                const bool valid = c < n_in;
                float xv = 0.0f;
                bool xg = true;
#pragma unroll
                for (int q = 0; q < kXAhead; q++)
                    if (q == r) {
                        xv = x_ahead[q];
                        xg = x_gated[q];
                    }
                if (r >= kXAhead && valid) xv = run.x[((size_t)b * run.T_total + t_abs + 1) * n_in + c];
                if (GSRC && !xg) {  // ungated columns of a gated network
                    const bool on = valid && xv != 0.0f;
                    int c0 = 0, cnt = 0;
                    if (on) {
                        c0 = net.src_chunk[Nsrc + c];
                        cnt = net.src_chunk[Nsrc + c + 1] - c0;
                    }
                    emit_fast(net, ws, t + 1, on, b, c0, cnt, xv, lane);
                } else {
                    emit_input(t + 1, valid, b, Nsrc + c, xv);
                }
            }
            load_x(t_abs + 2);  // the next step's, landing while this step runs
        }

        // ---------------- scatter the events of step t into X_t ----------------
        // Step t's events were emitted during step t - 1 and X_t's buffer emptied then.
        // The events go round the warps; a warp reads up to 32 of its events at once (one
        // per lane, from L2: other blocks wrote them), then walks them one by one, loading
        // the next event's edges before it issues the current one's reductions.
        // Scatter and update of a step touch different buffers (X_t and the events of t;
        // X_{t-1} and the events of t + 1), so half the warps of a block scatter before
        // their items and half after: the reductions drain while the other half computes.
        auto scatter = [&]() {
            const long long n_local = min((long long)*reinterpret_cast<volatile unsigned *>(&ws.ev_count[t]),
                                          (long long)ws.ev_cap);  // never above: one event per (trial, chunk)
            const WtEvent *evs = ws.ev + (size_t)(t & 1) * ws.ev_cap;
            // a pushing rank's events of step t: its own list (the input columns), then the
            // region of each rank in its inbound area, counts published with the progress
            // (a count is never above its region's room; clamped all the same, so that no
            // read leaves the area)
            // (each rank's count read once, into registers: the lanes then find their
            // event's region without a load per rank)
            int pr[8];
            long long count = n_local;
#pragma unroll
            for (int r = 0; r < 8; r++) {
                pr[r] = 0;
                if (PUSH && r < run.n_ranks) {
                    const long long room =
                        (r + 1 < run.n_ranks ? run.pull_off[r + 1] : run.pull_half) - run.pull_off[r];
                    pr[r] = (int)min((long long)__ldcg(run.pull_count + (t & 1) * 8 + r), room);
                    count += pr[r];
                }
            }
            const WtEvent *pull = PUSH ? run.pull_ev + (size_t)(t & 1) * run.pull_half : nullptr;
            unsigned long long *X = ws.X + (size_t)(t & 1) * C * BNp;
            for (long long base = gwarp; base < count; base += nwarps * 32) {
                // lane k holds event base + k nwarps: the events go round the warps
                int4 raw = make_int4(0, 0, 0, 0);
                const long long mine = base + lane * nwarps;
                if (mine < n_local) {
                    raw = __ldcg(reinterpret_cast<const int4 *>(evs + mine));
                } else if (mine < count) {
                    long long m = mine - n_local, off = -1;
#pragma unroll
                    for (int r = 0; r < 8; r++) {
                        if (off < 0 && m < pr[r]) off = run.pull_off[r] + m;
                        if (off < 0) m -= pr[r];
                    }
                    if (off >= 0) raw = __ldcg(reinterpret_cast<const int4 *>(pull + off));
                }
                const int ne = (int)min(32LL, (count - base + nwarps - 1) / nwarps);
                unsigned long long cw[4], cw_n[4];
                auto load = [&](int e, unsigned long long *dst) {
                    const unsigned x = __shfl_sync(kFull, raw.x, e), y = __shfl_sync(kFull, raw.y, e);
                    int len = __shfl_sync(kFull, raw.z, e) & 255;
                    const long long e0 = ((long long)y << 32) | x;
                    if (PART && (e0 < 0 || e0 + len > n_edges_all || len > WT_CHUNK_EDGES)) {
                        if (lane == 0) set_error(ws.err, WT_ERR_RANGE | (3 << 8));
                        len = 0;
                    }
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int q = lane + 32 * u;
                        dst[u] = q < len ? __ldg(net.edge_cw + e0 + q) : 0ull;
                    }
                };
                load(0, cw_n);
                for (int e = 0; e < ne; e++) {
                    const unsigned bl = (unsigned)__shfl_sync(kFull, raw.z, e);
                    const float amp = __int_as_float(__shfl_sync(kFull, raw.w, e));
                    int len = (int)(bl & 255u);
#pragma unroll
                    for (int u = 0; u < 4; u++) cw[u] = cw_n[u];
                    if (e + 1 < ne) load(e + 1, cw_n);
                    if (PART && ((int)(bl >> 8) >= B || len > WT_CHUNK_EDGES)) {
                        if (lane == 0) set_error(ws.err, WT_ERR_RANGE | (4 << 8));
                        len = 0;
                    }
                    unsigned long long *Xb = X + (size_t)(bl >> 8) * Np;
                    if (ws.edges) {  // counting edges (instrumented runs)
                        const unsigned x = __shfl_sync(kFull, raw.x, e), y = __shfl_sync(kFull, raw.y, e);
                        if (lane == 0)
                            atomicAdd(ws.edges + ((((long long)y << 32) | x) >= net.n_rec_edges),
                                      (unsigned long long)len);
                    }
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        if (lane + 32 * u >= len) break;
                        const uint32_t col = (uint32_t)cw[u];
                        const float prod = __uint_as_float((uint32_t)(cw[u] >> 32)) * amp;
                        if (fabsf(prod) >= 0x1p62f) {
                            set_error(ws.err, WT_ERR_FIXED_POINT);
                            continue;
                        }
                        if (PART && ((int)(col & 0x7ffffffu) >= N || (int)(col >> 27) >= C)) {
                            set_error(ws.err, WT_ERR_RANGE | (5 << 8));
                            continue;
                        }
                        atomicAdd(Xb + (size_t)(col >> 27) * BNp + (col & 0x7ffffffu),
                                  (unsigned long long)__float2ll_rn(prod));
                    }
                }
            }
        };
        stamp(t, 1);
        const bool scatter_late = !CUR && ((threadIdx.x >> 5) & 1);
        if (!scatter_late) scatter();
        if (CUR) {
            if (!bar.sync(ws.err)) return;
            issue_first();
        }
        stamp(t, 2);

        // ---------------- the neurons: step t, and the spikes of step t + 1 ----------------
        Cursor q = start;
        int g_k = -1, rd = 0;
        NeuronConsts k{};
        // gated runs with resolved gating: the group's sources' gates (kg), and whether
        // one of them owns several slots (then the warp walks them in `emit`)
        const bool GN = GSRC && (!PART || OG);
        SrcGate kg = no_gate();
        bool gmulti = false;
        float *rp = wsm + lane;
        const size_t tN = (size_t)t_abs * N;
        for (int j = 0; j < nitems; j++) {
            const int b = q.b;
            const int n = q.g * 32 + lane;
            const bool valid = n < N;
            if (q.g != g_k) {
                k = consts_of(n);
                g_k = q.g;
                if (GN) {
                    kg = valid ? src_gate_of(net, PART ? run.word0 * 32 + n : n) : no_gate();
                    gmulti = __any_sync(kFull, kg.gate == -2);
                    if (OG && gmulti && lane == 0) set_error(ws.err, WT_ERR_UNSUPPORTED);
                }
            }
            // item j's slot: wait for its copies (this lane's, then the warp's)
            cp_async_wait(D - 1);
            __syncwarp();
            const float *slot = ring + rd * slot_words;
            const long long *sx = reinterpret_cast<const long long *>(slot) + lane;
            float xin[S];
#pragma unroll
            for (int c = 0; c < S; c++) xin[c] = (has_x && in_c[c] >= 0) ? __ll2float_rn(sx[in_c[c] * 32]) * fx_c[c] : 0.0f;
            float xall[GEN ? WT_MAX_CHANNELS : 1];
            if (SAVE_IN && has_x)
                for (int c = 0; c < C; c++) xall[c] = __ll2float_rn(sx[c * 32]) * net.fx_inv[c];
            // the item's state: resident, or staged in its slot, words 32 floats apart
            const float *src = RES ? rp : slot + 2 * C * 32 + lane;
            const float v = src[0];
            int cnt = REF ? __float_as_int(src[w_cnt * 32]) : 0;
            float ga = ADAPT ? src[w_ga * 32] : 0.0f;
            float gr[S], gd[S];
#pragma unroll
            for (int c = 0; c < S; c++) {
                gd[c] = src[(w_gd + c) * 32];
                gr[c] = rw[c] >= 0 ? src[rw[c] * 32] : 0.0f;
            }
            __syncwarp();  // the slot is free: stage item j + D into it
            issue(j + D, qi, wr, Xprev, has_x);
            qi.next(B, N, Np, TN);
            if (++wr == D) wr = 0;
            if (++rd == D) rd = 0;
            // the gating state the spike of step t + 1 steps: loaded now, used after the
            // membrane update
            const bool gstep = GN && emit_next && !gmulti && valid && kg.gate >= 0;
            float *gb = run.gating + (size_t)b * net.R;
            float gu = 0.0f, gx = 0.0f, gsa = 0.0f;
            if (gstep) {
                if (kg.u_off >= 0) {
                    gu = gb[kg.u_off];
                    gx = gb[kg.x_off];
                }
                if (kg.a_off >= 0) gsa = gb[kg.a_off];
            }

            const size_t o = q.bN + n;
            const size_t out = q.bTN + tN + n;
            float s = 0.0f, held = 0.0f, s_next = 0.0f;
            if (valid) {
                float *g_b = run.g + q.bN * 2 * S + n;
                if (!has_x) {  // a rise that does not decay is known only entering the run
#pragma unroll
                    for (int c = 0; c < S; c++)
                        if (rw[c] < 0) gr[c] = g_b[(size_t)c * N];
                } else {  // the input of step t - 1 completes g_t
#pragma unroll
                    for (int c = 0; c < S; c++) {
                        gr[c] = gr[c] * net.decay_r[c];
                        gd[c] = gd[c] * net.decay_d[c];
                        if (in_c[c] >= 0) {
                            gr[c] = gr[c] + net.jump_r[c] * xin[c];
                            gd[c] = gd[c] + net.jump_d[c] * xin[c];
                        }
                    }
                    unsigned long long *xz = Xprev + q.bNp + n;
                    for (int c = 0; c < C; c++, xz += BNp) *xz = 0ull;
                    const int t_in = CUR ? t_abs : t_abs - 1;  // the step whose input this is
                    if (SAVE_IN)
                        for (int c = 0; c < C; c++)
                            run.X_saved[(((size_t)b * run.T_total + t_in) * C + c) * N + n] = xall[c];
                    if (TRACK && (run.track_b < 0 || run.track_b == b)) {
                        const int bt = run.track_b < 0 ? b : 0;
                        float *tg = run.track_g + (((size_t)bt * run.T_total + t_in) * N + n) * 2 * S;
#pragma unroll
                        for (int c = 0; c < S; c++) {
                            tg[c] = gr[c];
                            tg[S + c] = gd[c];
                        }
                    }
                }
                const float u01 = SAMPLE ? run.noise[out] : 0.0f;
                s = spike_of(v, k.theta, cnt, u01, sflags, ksur, held);
                const float rr = fmaxf(s, held);
                float Gt[S];
                float I_leak = 0.0f, v_next, ga_in = ga;
                if (CUR) {
                    // current-based membrane (current/dynamics.py:116-125, 180-183), float32,
                    // in its order: the adaptation current rises by the spike first, then
                    // v' = (beta v + (1 - beta)(U_rest + R (sum_j sign_j I_j - I_a)))(1 - r) + U r
                    ga_in = ga;  // I_a{t}, saved for the backward pass
                    if (ADAPT) ga = ga * k.a_decay + k.adapt * s;
                    float Isyn = 0.0f;
#pragma unroll
                    for (int c = 0; c < S; c++) Isyn = Isyn + gd[c] * net.E_syn[c];
                    if (ADAPT) Isyn = Isyn - ga;
                    const float beta = k.g_L;
                    v_next = (beta * v + (1.0f - beta) * (k.E_L + k.Cm * Isyn)) * (1.0f - rr) + k.U_reset * rr;
                } else {
                    // membrane (conductance/dynamics.py:116-143), float32, in its order
                    float G = 0.0f, Isum = 0.0f;
#pragma unroll
                    for (int c = 0; c < S; c++) {
                        float gs = gr[c] + gd[c];
                        gs = fminf(fmaxf(gs, 0.0f), net.g_clip[c]);
                        // a channel without the block (mg_lc -inf) multiplies by sigmoid(+inf) = 1
                        if (MG && net.mg_lc[c] != -INFINITY) gs = gs * sigmoid(net.mg_a[c] * v - net.mg_lc[c]);
                        Gt[c] = gs;
                    }
#pragma unroll
                    for (int c = 0; c < S; c++) G = G + Gt[c];
#pragma unroll
                    for (int c = 0; c < S; c++) Isum = Isum + Gt[c] * (v - net.E_syn[c]);
                    I_leak = k.g_L * (v - k.E_L);
                    float J = Isum + I_leak;
                    if (ADAPT) {
                        G = G + ga;
                        J = J + ga * (v - k.E_a);
                    }
                    const float xx = dt * k.rate + dt * G / k.Cm;
                    const float step = -expm1f(-xx) / (k.g_L + G);
                    v_next = (v - step * J) * (1.0f - rr) + k.U_reset * rr;
                }
                if (SAVE) {
                    run.v_saved[out] = v;
                    float *Gs = run.G_saved + (q.bTN + tN) * S + n;
                    // (current-based: the currents after the step's input, and the
                    // adaptation current entering the step)
#pragma unroll
                    for (int c = 0; c < S; c++) Gs[(size_t)c * N] = CUR ? gd[c] : gr[c] + gd[c];
                    if (ADAPT) run.a_saved[out] = CUR ? ga_in : ga;
                }
                if (REF) {
                    const int c1 = cnt - 1;
                    cnt = s > 0.0f ? k.n_ref : (c1 > 0 ? c1 : 0);
                }
                if (ADAPT && !CUR) ga = ga * k.a_decay + k.adapt * s;
                run.spikes[out] = s;
                if (PROB) {
                    const float p = sigmoid(ksur * (v - k.theta));
                    run.prob[out] = REF ? p * (1.0f - held) : p;
                }
                if (TRACK && (run.track_b < 0 || run.track_b == b)) {
                    const int bt = run.track_b < 0 ? b : 0;
                    const size_t to = ((size_t)bt * run.T_total + t_abs) * N + n;
                    run.track_v[to] = v_next;
                    if (!CUR) {  // (current-based: the currents are the tracked channels)
                        float *tI = run.track_I + to * (S + 1);
#pragma unroll
                        for (int c = 0; c < S; c++) tI[c] = Gt[c] * (v - net.E_syn[c]);
                        tI[S] = I_leak;
                    }
                    if (ADAPT) run.track_a[to] = ga;
                }
                // the state entering step t + 1 (g: before this step's input)
                if (RES) {
                    rp[0] = v_next;
                    if (REF) rp[w_cnt * 32] = __int_as_float(cnt);
                    if (ADAPT) rp[w_ga * 32] = ga;
#pragma unroll
                    for (int c = 0; c < S; c++) {
                        rp[(w_gd + c) * 32] = gd[c];
                        if (rw[c] >= 0) rp[rw[c] * 32] = gr[c];
                    }
                } else {
                    run.v[o] = v_next;
                    if (REF) run.counter[o] = cnt;
                    if (ADAPT) run.g_a[o] = ga;
#pragma unroll
                    for (int c = 0; c < S; c++) {
                        g_b[(size_t)(S + c) * N] = gd[c];
                        if (rw[c] >= 0) g_b[(size_t)c * N] = gr[c];
                    }
                }
                if (emit_next) {
                    float h2;
                    const float u2 = SAMPLE ? run.noise[out + N] : 0.0f;
                    s_next = spike_of(v_next, k.theta, cnt, u2, sflags, ksur, h2);
                }
            }
            if (SAVE) {
                const unsigned sb = __ballot_sync(kFull, s > 0.0f);
                const unsigned hb = __ballot_sync(kFull, held > 0.0f);
                if (lane == 0) {  // lane 0 holds the word's first neuron
                    const size_t w = ((size_t)b * run.T_total + t_abs) * words + q.g;
                    run.spike_bits[w] = sb;
                    if (REF) run.held_bits[w] = hb;
                }
            }
            if (emit_next) {
                if (PART) {
                    float amp = s_next;
                    if (OG) {
                        if (gstep) {
                            const float f = gate_math(net.gate_params + 5 * kg.gate, kg.u_off >= 0, kg.a_off >= 0, gu, gx, gsa, s_next);
                            if (kg.u_off >= 0) {
                                gb[kg.u_off] = gu;
                                gb[kg.x_off] = gx;
                            }
                            if (kg.a_off >= 0) gb[kg.a_off] = gsa;
                            amp = s_next * f;
                        }
                        if (!PUSH) publish_amp(t + 1, b, run.word0 * 32 + n, valid && s_next != 0.0f, amp);
                    }
                    if (PUSH)
                        push(t + 1, b, run.word0 * 32 + n, valid && s_next != 0.0f, amp);
                    else
                        publish(t + 1, b, q.g, s_next);
                } else if (GN && !gmulti) {
                    float amp = s_next;
                    if (gstep) {
                        const float f = gate_math(net.gate_params + 5 * kg.gate, kg.u_off >= 0, kg.a_off >= 0, gu, gx, gsa, s_next);
                        if (kg.u_off >= 0) {
                            gb[kg.u_off] = gu;
                            gb[kg.x_off] = gx;
                        }
                        if (kg.a_off >= 0) gb[kg.a_off] = gsa;
                        if (SAVE) run.f_saved[((size_t)b * run.T_total + t_abs + 1) * net.R_f + kg.f_off] = f;
                        amp = s_next * f;
                    }
                    emit_fast(net, ws, t + 1, valid && s_next != 0.0f, b, k.c0, k.cnt, amp, lane);
                } else {
                    emit_neuron(t + 1, valid, b, n, k, s_next);
                }
            }
            q.next(B, N, Np, TN);
            rp += ks * 32;
        }
        cp_async_wait(0);  // the last (empty) groups
        stamp(t, 3);
        if (scatter_late) scatter();
        stamp(t, 4);
        if (PART && emit_next) {  // the step's barrier is the exchange's
            stamp(t, 5);
            if (!exchange(t + 1)) return;
        } else {
            if (!bar.sync(ws.err)) return;
            stamp(t, 5);
        }
        stamp(t, 6);
    }

    // The input of the last step completes the conductances the run leaves; resident
    // state goes back to HBM.
    if (T > 0) {
        const int t_last = run.t0 + T - 1;
        const unsigned long long *Xl = ws.X + (size_t)((T - 1) & 1) * C * BNp;
        Cursor q = start;
        const float *rp = wsm + lane;
        for (int j = 0; j < nitems; j++, q.next(B, N, Np, TN), rp += ks * 32) {
            const int b = q.b;
            const int n = q.g * 32 + lane;
            if (n >= N) continue;
            const size_t o = q.bN + n;
            const size_t xo = q.bNp + n;
            float *g_b = run.g + q.bN * 2 * S + n;
            float gr[S], gd[S];
#pragma unroll
            for (int c = 0; c < S; c++) {
                if (CUR) {  // the currents already hold the last step's input
                    gd[c] = RES ? rp[(w_gd + c) * 32] : g_b[(size_t)(S + c) * N];
                    gr[c] = (RES && rw[c] >= 0) ? rp[rw[c] * 32] : g_b[(size_t)c * N];
                    g_b[(size_t)c * N] = gr[c];
                    g_b[(size_t)(S + c) * N] = gd[c];
                    continue;
                }
                gd[c] = (RES ? rp[(w_gd + c) * 32] : g_b[(size_t)(S + c) * N]) * net.decay_d[c];
                if (rw[c] >= 0)
                    gr[c] = (RES ? rp[rw[c] * 32] : g_b[(size_t)c * N]) * net.decay_r[c];
                else
                    gr[c] = (T > 1 ? 0.0f : g_b[(size_t)c * N]) * net.decay_r[c];
                if (in_c[c] >= 0) {
                    const float xi = __ll2float_rn((long long)__ldcg(Xl + (size_t)in_c[c] * BNp + xo)) * fx_c[c];
                    gr[c] = gr[c] + net.jump_r[c] * xi;
                    gd[c] = gd[c] + net.jump_d[c] * xi;
                }
                g_b[(size_t)c * N] = gr[c];
                g_b[(size_t)(S + c) * N] = gd[c];
            }
            if (SAVE_IN && !CUR)
                for (int c = 0; c < C; c++)
                    run.X_saved[(((size_t)b * run.T_total + t_last) * C + c) * N + n] =
                        __ll2float_rn((long long)__ldcg(Xl + (size_t)c * BNp + xo)) * net.fx_inv[c];
            if (TRACK && !CUR && (run.track_b < 0 || run.track_b == b)) {
                const int bt = run.track_b < 0 ? b : 0;
                float *tg = run.track_g + (((size_t)bt * run.T_total + t_last) * N + n) * 2 * S;
#pragma unroll
                for (int c = 0; c < S; c++) {
                    tg[c] = gr[c];
                    tg[S + c] = gd[c];
                }
            }
            if (RES) {
                run.v[o] = rp[0];
                if (REF) run.counter[o] = __float_as_int(rp[w_cnt * 32]);
                if (ADAPT) run.g_a[o] = rp[w_ga * 32];
            }
        }
    }
}

}  // namespace

// The launch geometry: one block of warps_of<S, FEAT>() warps per SM (fewer blocks when there are
// fewer items than warps); state resident in shared memory when every warp's share fits
// beside a ring of at least two slots, else streamed with the deepest ring that fits.
// Cached per device, kernel and shape.
struct GeoKey {
    const void *kernel;
    int dev, B, N, C, n_rise, feat;
    bool operator==(const GeoKey &o) const {
        return kernel == o.kernel && dev == o.dev && B == o.B && N == o.N && C == o.C && n_rise == o.n_rise &&
               feat == o.feat;
    }
};

template <int S, int FEAT>
static cudaError_t geometry_for(const WtNet &net, int flags, Geometry &geo, int &grid, size_t &dyn) {
    static GeoKey keys[64];
    static Geometry geos[64];
    static int grids[64];
    static size_t dyns[64];
    static int n_cached = 0;
    constexpr int NW = warps_of<S, FEAT>();
    const void *kern = (const void *)forward_kernel<S, FEAT>;
    int dev = 0;
    cudaGetDevice(&dev);
    int n_rise = 0;
    for (int c = 0; c < S; c++) n_rise += net.decay_r[c] != 0.0f;
    const bool REF = flags & WT_F_REFRACTORY, ADAPT = flags & WT_F_ADAPT;
    const bool STREAM = flags & WT_F_STREAM;
    const GeoKey key{kern, dev, net.B, net.N, net.C, n_rise, REF * 2 + ADAPT + 4 * STREAM};
    for (int i = 0; i < n_cached; i++)
        if (keys[i] == key) {
            geo = geos[i];
            grid = grids[i];
            dyn = dyns[i];
            return cudaSuccess;
        }
    int sms = 0, optin = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, forward_kernel<S, FEAT>);
    if (e != cudaSuccess) return e;
    const long long max_dyn = optin - (long long)attr.sharedSizeBytes;
    e = cudaFuncSetAttribute(forward_kernel<S, FEAT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_dyn);
    if (e != cudaSuccess) return e;
    Geometry g{};
    g.groups = (net.N + 31) / 32;
    g.Np = g.groups * 32;
    g.W = (long long)g.groups * net.B;
    g.w_cnt = 1;
    g.w_ga = 1 + REF;
    g.w_gd = 1 + REF + ADAPT;
    g.w_gr = g.w_gd + S;
    g.ks = g.w_gr + n_rise;
    const long long blocks = std::min<long long>(sms, (g.W + NW - 1) / NW);
    const long long nw = blocks * NW;
    g.max_items = (int)((g.W + nw - 1) / nw);
    const long long x_rows = 2LL * net.C;  // a slot's int64 inputs, in 128-byte rows
    g.D = 0;
    for (int D = kMaxRing; D >= 2 && !g.D && !STREAM; D--) {  // resident, with at least two slots
        const long long rows = (long long)g.max_items * g.ks + D * x_rows;
        if (rows * 128 * NW <= max_dyn) {
            g.resident = 1;
            g.D = D;
            g.slot_rows = (int)x_rows;
            g.warp_rows = (int)rows;
        }
    }
    for (int D = kMaxRing; D >= 1 && !g.D; D--) {  // streamed
        const long long rows = D * (x_rows + g.ks);
        if (rows * 128 * NW <= max_dyn) {
            g.resident = 0;
            g.D = D;
            g.slot_rows = (int)(x_rows + g.ks);
            g.warp_rows = (int)rows;
        }
    }
    if (!g.D) return cudaErrorInvalidConfiguration;
    const size_t d = (size_t)g.warp_rows * 128 * NW;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, forward_kernel<S, FEAT>, NW * 32, d);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    geo = g;
    grid = (int)blocks;
    dyn = d;
    if (n_cached < 64) {
        keys[n_cached] = key;
        geos[n_cached] = geo;
        grids[n_cached] = grid;
        dyns[n_cached] = dyn;
        n_cached++;
    }
    return cudaSuccess;
}

template <int S, int FEAT>
static cudaError_t launch_sf(const WtNet &net, const WtForward &run, const WtWorkspace &ws, cudaStream_t st) {
    Geometry geo;
    int grid = 1;
    size_t dyn = 0;
    cudaError_t e = geometry_for<S, FEAT>(net, run.flags, geo, grid, dyn);
    if (e != cudaSuccess) return e;
    WtNet n = net;
    WtForward r = run;
    WtWorkspace w = ws;
    void *args[] = {&n, &r, &w, &geo};
    return cudaLaunchCooperativeKernel((const void *)forward_kernel<S, FEAT>, dim3(grid), dim3(warps_of<S, FEAT>() * 32), args, dyn,
                                       st);
}

// The specialised kernels cover the common runs (up to four channels; refractory period
// and saving as given; no other feature); everything else runs the generic kernel.
template <int S>
static cudaError_t launch_s(const WtNet &net, const WtForward &run, const WtWorkspace &ws, cudaStream_t st) {
    const int generic = WT_F_SAMPLE | WT_F_PROB | WT_F_TRACK | WT_F_SAVE_INPUT;
    const int feat = ((run.flags & WT_F_REFRACTORY) ? kRef : 0) | ((run.flags & WT_F_SAVE) ? kSave : 0) |
                     ((run.flags & WT_F_MG_BLOCK) ? kMg : 0) | ((run.flags & WT_F_GATED) ? kGate : 0) |
                     ((run.flags & WT_F_ADAPT) ? kAdapt : 0) | ((run.flags & WT_F_PARTITION) ? kPart : 0) |
                     ((run.flags & WT_F_CURRENT) ? kCur : 0);
    // the Mg block, gating and adaptation are specialised for forward runs with a
    // refractory period (the large simulations' cases: Mg block and gating in any
    // combination, or adaptation alone), and so are the ranks of a neuron partition;
    // other combinations with them run the generic kernel
    const int extra = feat & (kMg | kGate | kAdapt | kPart);
    if (S > 4 || (run.flags & generic) || (extra && (feat & (kRef | kSave)) != kRef) ||
        ((extra & kAdapt) && (extra & ~kPart) != kAdapt))
        return launch_sf<S, kGeneric>(net, run, ws, st);
    if (feat & kCur) {  // current-based neurons: forward runs with a refractory period
        switch (feat) {
            case kRef | kCur: return launch_sf<S, kRef | kCur>(net, run, ws, st);
            case kRef | kSave | kCur: return launch_sf<S, kRef | kSave | kCur>(net, run, ws, st);
            default: return launch_sf<S, kGeneric>(net, run, ws, st);
        }
    }
    if (feat & kPart) {
        switch (feat) {
            case kRef | kPart: return launch_sf<S, kRef | kPart>(net, run, ws, st);
            case kRef | kAdapt | kPart: return launch_sf<S, kRef | kAdapt | kPart>(net, run, ws, st);
            case kRef | kMg | kGate | kPart: return launch_sf<S, kRef | kMg | kGate | kPart>(net, run, ws, st);
            default: return launch_sf<S, kGeneric>(net, run, ws, st);
        }
    }
    switch (feat) {
        case 0: return launch_sf<S, 0>(net, run, ws, st);
        case kRef: return launch_sf<S, kRef>(net, run, ws, st);
        case kSave: return launch_sf<S, kSave>(net, run, ws, st);
        case kRef | kSave: return launch_sf<S, kRef | kSave>(net, run, ws, st);
        case kRef | kMg: return launch_sf<S, kRef | kMg>(net, run, ws, st);
        case kRef | kGate: return launch_sf<S, kRef | kGate>(net, run, ws, st);
        case kRef | kAdapt: return launch_sf<S, kRef | kAdapt>(net, run, ws, st);
        default: return launch_sf<S, kRef | kMg | kGate>(net, run, ws, st);
    }
}

// The 128-byte-aligned accumulator row stride the kernel uses for X.
long long forward_x_row(int N) { return (long long)((N + 31) / 32) * 32; }

cudaError_t launch_forward_s(const WtNet &net, const WtForward &run, const WtWorkspace &ws, cudaStream_t st,
                             int /*unused*/) {
    switch (net.S) {
        case 1: return launch_s<1>(net, run, ws, st);
        case 2: return launch_s<2>(net, run, ws, st);
        case 3: return launch_s<3>(net, run, ws, st);
        case 4: return launch_s<4>(net, run, ws, st);
        case 5: return launch_s<5>(net, run, ws, st);
        case 6: return launch_s<6>(net, run, ws, st);
        case 7: return launch_s<7>(net, run, ws, st);
        case 8: return launch_s<8>(net, run, ws, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace wt
