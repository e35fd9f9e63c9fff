// The forward pass: one persistent cooperative kernel integrates T steps of the
// conductance-based LIF network (the time step of wiretorch's
// conductance/dynamics.py:146-237, which its Triton kernels scan_forward,
// compact_spikes and recurrent_step implement on CUDA).
//
// Work per step t, over the whole grid, with one grid barrier between steps:
//
//   phase A (each (trial, neuron), coalesced over neurons):
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
//   phase B (all warps): scatter the events of step t — each a (trial, chunk of at
//     most WT_CHUNK_EDGES edges of one source's CSR row) — into X_t, the per
//     (input channel, trial, neuron) fixed-point accumulators: 64-bit integer
//     reductions, so the sum, and every result, is independent of the order in
//     which events land (bit-for-bit reproducible).
//
// A presynaptic pathway with gating (short-term plasticity, receptor saturation:
// network.py:186-223) steps its state when its source's spike (or input) of the next
// step is known, and scales the events by the factor.
#include "common.cuh"

namespace wt {
namespace {

struct Tables {
    // per-channel constants, copied to shared memory at launch
    float dr[WT_MAX_CHANNELS], dd[WT_MAX_CHANNELS], jr[WT_MAX_CHANNELS], jd[WT_MAX_CHANNELS];
    float E[WT_MAX_CHANNELS], clip[WT_MAX_CHANNELS], mga[WT_MAX_CHANNELS], mglc[WT_MAX_CHANNELS];
    float fx_inv[WT_MAX_CHANNELS];
    int in[WT_MAX_CHANNELS];
};

// Presynaptic gating of one slot for one trial (network.py:186-223): steps the state
// with the source's spike (or input) `s` and returns the factor of its input.
__device__ float gate_step(const WtNet &net, float *gating_b, int gate, int row, float s) {
    const float *prm = net.gate_params + 5 * gate;
    const int u_col = net.gate_cols[4 * gate + 0];
    const int n = net.gate_cols[4 * gate + 1];
    const int sat_col = net.gate_cols[4 * gate + 2];
    float f = 1.0f;
    bool have = false;
    if (u_col >= 0) {
        const float U = prm[2], d_D = prm[3], d_F = prm[4];
        float u = gating_b[u_col + row], x = gating_b[u_col + n + row];
        x = 1.0f - (1.0f - x) * d_D;
        u = U + (u - U) * d_F;
        const float r = u * x;
        f = r / U;
        have = true;
        x = x - s * r;
        u = u + s * U * (1.0f - u);
        gating_b[u_col + row] = u;
        gating_b[u_col + n + row] = x;
    }
    if (sat_col >= 0) {
        const float c = prm[0], d = prm[1];
        const float g = gating_b[sat_col + row] * d;
        const float closed = 1.0f - g;
        f = have ? fminf(c * f * closed, closed) : c * closed;
        gating_b[sat_col + row] = fminf(g + s * f, 1.0f);
    }
    return f;
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
            uint32_t *items = ws.ev_item + (size_t)(step & 1) * ws.ev_cap;
            float *amps = ws.ev_amp + (size_t)(step & 1) * ws.ev_cap;
            const uint32_t key = (uint32_t)b * (uint32_t)net.n_chunks;
            for (int q = 0; q < cnt; q++) {
                items[off + q] = key + (uint32_t)(c0 + q);
                amps[off + q] = amp;
            }
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

template <int S>
__global__ void __launch_bounds__(kBlock) forward_kernel(const WtNet net, const WtForward run,
                                                        const WtWorkspace ws) {
    __shared__ Tables tab;
    if (threadIdx.x < WT_MAX_CHANNELS) {
        const int c = threadIdx.x;
        tab.dr[c] = net.decay_r[c];
        tab.dd[c] = net.decay_d[c];
        tab.jr[c] = net.jump_r[c];
        tab.jd[c] = net.jump_d[c];
        tab.E[c] = net.E_syn[c];
        tab.clip[c] = net.g_clip[c];
        tab.mga[c] = net.mg_a[c];
        tab.mglc[c] = net.mg_lc[c];
        tab.fx_inv[c] = net.fx_inv[c];
        tab.in[c] = net.input_of[c];
    }
    __syncthreads();

    const int B = net.B, N = net.N, n_in = net.n_in, C = net.C, T = run.T;
    const int flags = run.flags;
    const bool gated = flags & WT_F_GATED;
    const int Np = (N + 31) & ~31, Ip = (n_in + 31) & ~31;  // padded: a warp = one word
    const long long itemsN = (long long)B * Np, itemsI = (long long)B * Ip;
    const long long nthreads = (long long)gridDim.x * blockDim.x;
    const long long gtid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const long long warp0 = gtid - lane;
    const long long gwarp = gtid >> 5, nwarps = nthreads >> 5;
    const size_t BN = (size_t)B * N;
    const int words = Np >> 5;
    const float dt = net.dt, ksur = net.surr_scale;
    GridBarrier bar(ws.barrier, gridDim.x);

    // Phase 0: empty accumulators and event counts.
    for (long long i = gtid; i < 2LL * C * (long long)BN; i += nthreads) ws.X[i] = 0ull;
    for (long long i = gtid; i <= T; i += nthreads) ws.ev_count[i] = 0u;
    if (!bar.sync(ws.err)) return;

    // Emit step 0's events: the spikes of the state entering the run, and x at t0.
    for (long long base = warp0; base < itemsN; base += nthreads) {
        const long long i = base + lane;
        const int b = (int)(i / Np), n = (int)(i % Np);
        const bool valid = n < N;
        float s = 0.0f;
        if (valid) {
            const size_t o = (size_t)b * N + n;
            float held;
            const int cnt = (flags & WT_F_REFRACTORY) ? run.counter[o] : 0;
            const float u = (flags & WT_F_SAMPLE) ? run.noise[((size_t)b * run.T_total + run.t0) * N + n] : 0.0f;
            s = spike_of(run.v[o], net.theta[n], cnt, u, flags, ksur, held);
        }
        emit(net, run, ws, 0, valid, b, n, s, gated, lane);
    }
    for (long long base = warp0; base < itemsI; base += nthreads) {
        const long long i = base + lane;
        const int b = (int)(i / Ip), c = (int)(i % Ip);
        const bool valid = c < n_in;
        const float xv = valid ? run.x[((size_t)b * run.T_total + run.t0) * n_in + c] : 0.0f;
        emit(net, run, ws, 0, valid, b, N + c, xv, gated, lane);
    }
    if (!bar.sync(ws.err)) return;

    for (int t = 0; t < T; t++) {
        const int t_abs = run.t0 + t;
        const bool emit_next = t + 1 < T;
        // ---------------- phase A: the neurons ----------------
        for (long long base = warp0; base < itemsN; base += nthreads) {
            const long long i = base + lane;
            const int b = (int)(i / Np), n = (int)(i % Np);
            const bool valid = n < N;
            float s = 0.0f, held = 0.0f, s_next = 0.0f;
            if (valid) {
                const size_t o = (size_t)b * N + n;
                float v = run.v[o];
                float gr[S], gd[S];
                float *g_b = run.g + (size_t)b * 2 * S * N + n;
#pragma unroll
                for (int c = 0; c < S; c++) {
                    gr[c] = g_b[(size_t)c * N];
                    gd[c] = g_b[(size_t)(S + c) * N];
                }
                if (t > 0) {  // the input of step t - 1 completes g_t
                    const unsigned long long *Xp = ws.X + (size_t)((t - 1) & 1) * C * BN + o;
#pragma unroll
                    for (int c = 0; c < S; c++) {
                        gr[c] = gr[c] * tab.dr[c];
                        gd[c] = gd[c] * tab.dd[c];
                        const int in = tab.in[c];
                        if (in >= 0) {
                            const float xin =
                                __ll2float_rn((long long)__ldcg(Xp + (size_t)in * BN)) * tab.fx_inv[in];
                            gr[c] = gr[c] + tab.jr[c] * xin;
                            gd[c] = gd[c] + tab.jd[c] * xin;
                        }
                    }
                    unsigned long long *Xz = ws.X + (size_t)((t - 1) & 1) * C * BN + o;
                    for (int c = 0; c < C; c++) {
                        if (flags & WT_F_SAVE_INPUT)
                            run.X_saved[(((size_t)b * run.T_total + t_abs - 1) * C + c) * N + n] =
                                __ll2float_rn((long long)__ldcg(Xz + (size_t)c * BN)) * tab.fx_inv[c];
                        Xz[(size_t)c * BN] = 0ull;
                    }
                    if ((flags & WT_F_TRACK) && (run.track_b < 0 || run.track_b == b)) {
                        const int bt = run.track_b < 0 ? b : 0;
                        float *tg = run.track_g + (((size_t)bt * run.T_total + t_abs - 1) * N + n) * 2 * S;
#pragma unroll
                        for (int c = 0; c < S; c++) {
                            tg[c] = gr[c];
                            tg[S + c] = gd[c];
                        }
                    }
                }
                int cnt = (flags & WT_F_REFRACTORY) ? run.counter[o] : 0;
                const float theta = net.theta[n];
                const float u = (flags & WT_F_SAMPLE) ? run.noise[((size_t)b * run.T_total + t_abs) * N + n] : 0.0f;
                s = spike_of(v, theta, cnt, u, flags, ksur, held);
                // membrane (conductance/dynamics.py:116-143), float32, in its order
                float Gt[S];
                float G = 0.0f, Isum = 0.0f;
#pragma unroll
                for (int c = 0; c < S; c++) {
                    float gs = gr[c] + gd[c];
                    gs = fminf(fmaxf(gs, 0.0f), tab.clip[c]);
                    if (flags & WT_F_MG_BLOCK) gs = gs * sigmoid(tab.mga[c] * v - tab.mglc[c]);
                    Gt[c] = gs;
                }
#pragma unroll
                for (int c = 0; c < S; c++) G = G + Gt[c];
#pragma unroll
                for (int c = 0; c < S; c++) Isum = Isum + Gt[c] * (v - tab.E[c]);
                const float Cm = net.C_m[n];
                const float rate = -log1pf(net.beta[n] - 1.0f) / dt;
                const float g_L = Cm * rate;
                const float I_leak = g_L * (v - net.E_L[n]);
                float J = Isum + I_leak;
                float ga = 0.0f;
                if (flags & WT_F_ADAPT) {
                    ga = run.g_a[o];
                    G = G + ga;
                    J = J + ga * (v - net.E_adapt[n]);
                }
                const float xx = dt * rate + dt * G / Cm;
                const float step = -expm1f(-xx) / (g_L + G);
                const float r = fmaxf(s, held);
                const float U_reset = net.U_reset[n];
                const float v_next = (v - step * J) * (1.0f - r) + U_reset * r;

                if (flags & WT_F_SAVE) {
                    const size_t so = ((size_t)b * run.T_total + t_abs) * N + n;
                    run.v_saved[so] = v;
                    float *Gs = run.G_saved + ((size_t)b * run.T_total + t_abs) * S * N + n;
#pragma unroll
                    for (int c = 0; c < S; c++) Gs[(size_t)c * N] = gr[c] + gd[c];
                    if (flags & WT_F_ADAPT) run.a_saved[so] = ga;
                }
                if (flags & WT_F_REFRACTORY) {
                    const int c1 = cnt - 1;
                    cnt = s > 0.0f ? net.n_ref[n] : (c1 > 0 ? c1 : 0);
                    run.counter[o] = cnt;
                }
                if (flags & WT_F_ADAPT) {
                    ga = ga * net.adapt_decay[n] + net.adapt[n] * s;
                    run.g_a[o] = ga;
                }
                const size_t out = ((size_t)b * run.T_total + t_abs) * N + n;
                run.spikes[out] = s;
                if (flags & WT_F_PROB) {
                    const float p = sigmoid(ksur * (v - theta));
                    run.prob[out] = (flags & WT_F_REFRACTORY) ? p * (1.0f - held) : p;
                }
                if ((flags & WT_F_TRACK) && (run.track_b < 0 || run.track_b == b)) {
                    const int bt = run.track_b < 0 ? b : 0;
                    const size_t to = ((size_t)bt * run.T_total + t_abs) * N + n;
                    run.track_v[to] = v_next;
                    float *tI = run.track_I + to * (S + 1);
#pragma unroll
                    for (int c = 0; c < S; c++) tI[c] = Gt[c] * (v - tab.E[c]);
                    tI[S] = I_leak;
                    if (flags & WT_F_ADAPT) run.track_a[to] = ga;
                }
                run.v[o] = v_next;
#pragma unroll
                for (int c = 0; c < S; c++) {
                    g_b[(size_t)c * N] = gr[c];
                    g_b[(size_t)(S + c) * N] = gd[c];
                }
                if (emit_next) {
                    float h2;
                    const float u2 = (flags & WT_F_SAMPLE) ? run.noise[((size_t)b * run.T_total + t_abs + 1) * N + n] : 0.0f;
                    s_next = spike_of(v_next, theta, cnt, u2, flags, ksur, h2);
                }
            }
            if (flags & WT_F_SAVE) {
                const unsigned sb = __ballot_sync(kFull, s > 0.0f);
                const unsigned hb = __ballot_sync(kFull, held > 0.0f);
                if (lane == 0) {
                    const size_t w = ((size_t)b * run.T_total + t_abs) * words + (n >> 5);
                    run.spike_bits[w] = sb;
                    if (flags & WT_F_REFRACTORY) run.held_bits[w] = hb;
                }
            }
            if (emit_next) emit(net, run, ws, t + 1, valid, b, n, s_next, gated, lane);
        }
        // ---------------- phase A: the input columns of the next step ----------------
        if (emit_next) {
            for (long long base = warp0; base < itemsI; base += nthreads) {
                const long long i = base + lane;
                const int b = (int)(i / Ip), c = (int)(i % Ip);
                const bool valid = c < n_in;
                const float xv = valid ? run.x[((size_t)b * run.T_total + t_abs + 1) * n_in + c] : 0.0f;
                emit(net, run, ws, t + 1, valid, b, N + c, xv, gated, lane);
            }
        }
        // ---------------- phase B: scatter the events of step t into X_t ----------------
        {
            const unsigned count = *reinterpret_cast<volatile unsigned *>(&ws.ev_count[t]);
            const uint32_t *items = ws.ev_item + (size_t)(t & 1) * ws.ev_cap;
            const float *amps = ws.ev_amp + (size_t)(t & 1) * ws.ev_cap;
            unsigned long long *X = ws.X + (size_t)(t & 1) * C * BN;
            const uint32_t nch = (uint32_t)net.n_chunks;
            for (long long it = gwarp; it < (long long)count; it += nwarps) {
                const uint32_t item = __ldcg(items + it);  // written by other blocks: L2, not L1
                const float amp = __ldcg(amps + it);
                const uint32_t b = item / nch, chunk = item - b * nch;
                const long long e0 = net.chunk_begin[chunk];
                const int len = net.chunk_len[chunk];
                unsigned long long *Xb = X + (size_t)b * N;
                if (ws.edges && lane == 0) atomicAdd(ws.edges + (chunk >= (uint32_t)net.n_rec_chunks), (unsigned long long)len);
                for (int q = lane; q < len; q += 32) {
                    const uint32_t pc = net.edge_col[e0 + q];
                    const float prod = net.edge_w[e0 + q] * amp;
                    if (fabsf(prod) >= 0x1p62f) {
                        set_error(ws.err, WT_ERR_FIXED_POINT);
                        continue;
                    }
                    const long long fx = __float2ll_rn(prod);
                    atomicAdd(Xb + (size_t)(pc >> 27) * BN + (pc & 0x7ffffffu), (unsigned long long)fx);
                }
            }
        }
        if (!bar.sync(ws.err)) return;
    }

    // The input of the last step completes the conductances the run leaves.
    if (T > 0) {
        const int t_last = run.t0 + T - 1;
        for (long long i = gtid; i < itemsN; i += nthreads) {
            const int b = (int)(i / Np), n = (int)(i % Np);
            if (n >= N) continue;
            const size_t o = (size_t)b * N + n;
            float *g_b = run.g + (size_t)b * 2 * S * N + n;
            const unsigned long long *Xp = ws.X + (size_t)((T - 1) & 1) * C * BN + o;
            float gr[S], gd[S];
#pragma unroll
            for (int c = 0; c < S; c++) {
                gr[c] = g_b[(size_t)c * N] * tab.dr[c];
                gd[c] = g_b[(size_t)(S + c) * N] * tab.dd[c];
                const int in = tab.in[c];
                if (in >= 0) {
                    const float xin = __ll2float_rn((long long)__ldcg(Xp + (size_t)in * BN)) * tab.fx_inv[in];
                    gr[c] = gr[c] + tab.jr[c] * xin;
                    gd[c] = gd[c] + tab.jd[c] * xin;
                }
                g_b[(size_t)c * N] = gr[c];
                g_b[(size_t)(S + c) * N] = gd[c];
            }
            if (flags & WT_F_SAVE_INPUT)
                for (int c = 0; c < C; c++)
                    run.X_saved[(((size_t)b * run.T_total + t_last) * C + c) * N + n] =
                        __ll2float_rn((long long)__ldcg(Xp + (size_t)c * BN)) * tab.fx_inv[c];
            if ((flags & WT_F_TRACK) && (run.track_b < 0 || run.track_b == b)) {
                const int bt = run.track_b < 0 ? b : 0;
                float *tg = run.track_g + (((size_t)bt * run.T_total + t_last) * N + n) * 2 * S;
#pragma unroll
                for (int c = 0; c < S; c++) {
                    tg[c] = gr[c];
                    tg[S + c] = gd[c];
                }
            }
        }
    }
}

}  // namespace

template <int S>
static cudaError_t launch_s(const WtNet &net, const WtForward &run, const WtWorkspace &ws, cudaStream_t st,
                            int grid_cap) {
    static int max_blocks[16] = {0};  // per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && max_blocks[dev] == 0) {
        int per_sm = 0, sms = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, forward_kernel<S>, kBlock, 0);
        if (e != cudaSuccess) return e;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        max_blocks[dev] = per_sm * sms;
    }
    int grid = dev < 16 ? max_blocks[dev] : 148;
    if (grid_cap > 0 && grid_cap < grid) grid = grid_cap;
    if (grid < 1) grid = 1;
    WtNet n = net;
    WtForward r = run;
    WtWorkspace w = ws;
    void *args[] = {&n, &r, &w};
    return cudaLaunchCooperativeKernel((const void *)forward_kernel<S>, dim3(grid), dim3(kBlock), args, 0, st);
}

cudaError_t launch_forward_s(const WtNet &net, const WtForward &run, const WtWorkspace &ws, cudaStream_t st,
                             int grid_cap) {
    switch (net.S) {
        case 1: return launch_s<1>(net, run, ws, st, grid_cap);
        case 2: return launch_s<2>(net, run, ws, st, grid_cap);
        case 3: return launch_s<3>(net, run, ws, st, grid_cap);
        case 4: return launch_s<4>(net, run, ws, st, grid_cap);
        case 5: return launch_s<5>(net, run, ws, st, grid_cap);
        case 6: return launch_s<6>(net, run, ws, st, grid_cap);
        case 7: return launch_s<7>(net, run, ws, st, grid_cap);
        case 8: return launch_s<8>(net, run, ws, st, grid_cap);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace wt
