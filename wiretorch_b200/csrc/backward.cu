// The backward pass when gradients do not flow through the recurrent spikes (the
// reference's default for conductance-based networks): the recurrent input is then input
// like any other, every (trial, neuron) is independent, and the adjoint of the whole run
// is one reverse scan per (trial, neuron) — the adjoint of conductance/dynamics.py's
// time step, as the reference's scan_backward (conductance/kernels.py:382-568) computes
// it. Then wt_edge_grads carries each step's input adjoint Q back along the edges to
// the kernel scales, the weights and the input.
//
// Reverse step t, with lv = dL/dv after the step, l_r, l_d = dL/dg after it:
//   Q_c      = sum over channels fed by c of  jump_r l_r + jump_d l_d     (dL/dX_t)
//   membrane adjoint of v' = (v - phi J)(1 - r) + U r  (exponential Euler, r = reset)
//     gives dL/dv and dL/dG of each clipped, Mg-blocked conductance, and the
//     physiology terms; then the spike's surrogate term is added to dL/dv.
//   l_r = decay_r l_r + dL/dG ;  l_d = decay_d l_d + dL/dG
// The decays' gradient sum_t l_t g_t needs no saved conductances per component: with
// H_{t-1} = l_t + decay H_t it is sum_t jump X_t H_t + g_init H_{-1}.
#include <algorithm>

#include "common.cuh"

namespace wt {
namespace {

// The saved quantities of one step, loaded ahead of their use: they do not depend on the
// adjoint recursion, so the scan keeps kAhead steps of loads in flight.
template <int S>
struct StepIn {
    float v, gs, ga, gp;
    unsigned sb, hb;
    float G[S];
};
constexpr int kAhead = 3;

// PHYS: some physiology gradient is wanted (else the scan carries only dL/dv, dL/dg and
// Q); SYN: some synapse parameter's.
// CUR: current-based neurons (WT_F_CURRENT), compiled apart so that the conductance
// kernels carry none of its code.
template <int S, bool PHYS, bool SYN, bool CUR>
__global__ void __launch_bounds__(kBlock, (PHYS || S > 2) ? 1 : 3) backward_kernel(const WtNet net, const WtBackward bw) {
    const int N = net.N, C = net.C, T = bw.T;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)net.B * N) return;
    const int b = (int)(i / N), n = (int)(i % N);
    const int flags = bw.flags, wants = PHYS ? bw.wants : 0;
    const bool REF = flags & WT_F_REFRACTORY, MG = flags & WT_F_MG_BLOCK, ADAPT = flags & WT_F_ADAPT;
    const bool SAMPLE = flags & WT_F_SAMPLE, PROB = flags & WT_F_PROB;
    const int words = (N + 31) >> 5;
    const float dt = net.dt, k = net.surr_scale;

    const float theta = net.theta[n], E_L = net.E_L[n], Cm = net.C_m[n], beta = net.beta[n];
    const float rate = -log1pf(beta - 1.0f) / dt;
    const float g_L = Cm * rate, inv_C = 1.0f / Cm;
    const float a_decay = ADAPT ? net.adapt_decay[n] : 0.0f;
    const float E_a = (ADAPT && !CUR) ? net.E_adapt[n] : 0.0f;
    const float adapt_n = (ADAPT && CUR) ? net.adapt[n] : 0.0f;
    int in_c[S];
#pragma unroll
    for (int c = 0; c < S; c++) in_c[c] = net.input_of[c];

    float dv = 0.0f, la = 0.0f;
    float lr[S], ld[S];
    float acc_E[SYN ? S : 1], acc_dr[SYN ? S : 1], acc_dd[SYN ? S : 1], acc_jr[SYN ? S : 1],
        acc_jd[SYN ? S : 1], H_r[SYN ? S : 1], H_d[SYN ? S : 1];
#pragma unroll
    for (int c = 0; c < S; c++) lr[c] = ld[c] = 0.0f;
    if (SYN) {
#pragma unroll
        for (int c = 0; c < S; c++) acc_E[c] = acc_dr[c] = acc_dd[c] = acc_jr[c] = acc_jd[c] = H_r[c] = H_d[c] = 0.0f;
    }
    float acc_theta = 0.0f, acc_reset = 0.0f, acc_E_L = 0.0f, acc_C_m = 0.0f, acc_beta = 0.0f;
    float acc_adapt = 0.0f, acc_adapt_decay = 0.0f, acc_E_a = 0.0f;

    const size_t TN = (size_t)T * N;
    const float *v_b = bw.v_saved + (size_t)b * TN + n;
    const float *gs_b = bw.grad_spikes + (size_t)b * TN + n;
    const float *G_b = bw.G_saved + (size_t)b * TN * S + n;
    const uint32_t *sb_b = bw.spike_bits + (size_t)b * T * words + (n >> 5);
    const uint32_t *hb_b = REF ? bw.held_bits + (size_t)b * T * words + (n >> 5) : nullptr;
    auto load = [&](int t, StepIn<S> &in) {
        const size_t o = (size_t)t * N;
        in.v = __ldg(v_b + o);
        in.gs = __ldg(gs_b + o);
        in.sb = __ldg(sb_b + (size_t)t * words);
        in.hb = REF ? __ldg(hb_b + (size_t)t * words) : 0u;
        in.ga = ADAPT ? __ldg(bw.a_saved + (size_t)b * TN + o + n) : 0.0f;
        in.gp = (PROB && bw.grad_prob) ? __ldg(bw.grad_prob + (size_t)b * TN + o + n) : 0.0f;
#pragma unroll
        for (int c = 0; c < S; c++) in.G[c] = __ldg(G_b + ((size_t)t * S + c) * N);
    };
    const int t_hi = bw.t_hi > 0 ? bw.t_hi : T, t_lo = bw.t_lo;
    // a chunk of a scan taken in pieces: the adjoint state entering it
    const int NA = 2 + 4 * S;
    float *adj = bw.adj ? bw.adj + (size_t)b * NA * N + n : nullptr;
    if (adj) {
        dv = adj[0];
        la = adj[(size_t)N];
#pragma unroll
        for (int c = 0; c < S; c++) {
            lr[c] = adj[(size_t)(2 + c) * N];
            ld[c] = adj[(size_t)(2 + S + c) * N];
            if (SYN) {
                H_r[c] = adj[(size_t)(2 + 2 * S + c) * N];
                H_d[c] = adj[(size_t)(2 + 3 * S + c) * N];
            }
        }
    }
    const float R_b = bw.R ? bw.R[(size_t)b * N + n] : 0.0f;
    // target-major adjoints (a whole scan): eight steps of each channel kept in registers
    // and written together, one 32-byte sector per thread; slots past T stay zero
    const int Tp = (T + 7) & ~7;
    float *const QT_n = bw.QT ? bw.QT + ((size_t)n * net.B + b) * Tp : nullptr;
    const size_t qt_c = (size_t)N * net.B * Tp;
    float qb[S][8];
#pragma unroll
    for (int c = 0; c < S; c++)
#pragma unroll
        for (int u = 0; u < 8; u++) qb[c][u] = 0.0f;
    StepIn<S> q[kAhead];
#pragma unroll
    for (int d = 0; d < kAhead; d++)
        if (t_hi - 1 - d >= t_lo) load(t_hi - 1 - d, q[d]);

    for (int t = t_hi - 1; t >= t_lo; t--) {
        const StepIn<S> cur = q[0];
#pragma unroll
        for (int d = 0; d + 1 < kAhead; d++) q[d] = q[d + 1];
        if (t - kAhead >= t_lo) load(t - kAhead, q[kAhead - 1]);
        const float v = cur.v;
        const float s = (cur.sb >> (n & 31)) & 1u ? 1.0f : 0.0f;
        const float held = (REF && ((cur.hb >> (n & 31)) & 1u)) ? 1.0f : 0.0f;
        const float r = fmaxf(s, held);
        const float *G = cur.G;

        // The input of step t entered the state step t + 1 saw: its adjoint.
        float *Qt = bw.Q ? bw.Q + ((size_t)b * T + t) * C * N + n : nullptr;
#pragma unroll
        for (int c = 0; c < S; c++) {
            if (c >= C) break;
            float qc = 0.0f;
#pragma unroll
            for (int j = 0; j < S; j++)
                if (in_c[j] == c) qc = qc + (net.jump_r[j] * lr[j] + net.jump_d[j] * ld[j]);
            if (Qt) Qt[(size_t)c * N] = qc;
            if (QT_n) {
#pragma unroll
                for (int u = 0; u < 8; u++)
                    if ((t & 7) == u) qb[c][u] = qc;
                if ((t & 7) == 0) {  // the group t .. t + 7 is complete
                    float4 *dst = reinterpret_cast<float4 *>(QT_n + c * qt_c + t);
                    dst[0] = make_float4(qb[c][0], qb[c][1], qb[c][2], qb[c][3]);
                    dst[1] = make_float4(qb[c][4], qb[c][5], qb[c][6], qb[c][7]);
                }
            }
        }
        if (SYN && !CUR && (wants & (WT_W_DECAY | WT_W_JUMP))) {
            const float *Xt = bw.X_saved + ((size_t)b * T + t) * C * N + n;
#pragma unroll
            for (int c = 0; c < S; c++) {
                const float base = in_c[c] >= 0 ? Xt[(size_t)in_c[c] * N] : 0.0f;
                if (wants & WT_W_JUMP) {
                    acc_jr[c] += lr[c] * base;
                    acc_jd[c] += ld[c] * base;
                }
                if (wants & WT_W_DECAY) {
                    acc_dr[c] += net.jump_r[c] * base * H_r[c];
                    acc_dd[c] += net.jump_d[c] * base * H_d[c];
                    H_r[c] = lr[c] + net.decay_r[c] * H_r[c];
                    H_d[c] = ld[c] + net.decay_d[c] * H_d[c];
                }
            }
        }
        if constexpr (CUR) {
            // Current-based step (current/dynamics.py:116-125, 166-183): the adjoint state
            // entering step t is dL/dv_{t+1} and the adjoints of I_{t+1} and I_a{t+1}
            // with the membrane of step t already added (so that Q_t above is complete,
            // and the recurrent carry, which reads Q_t from the same state, sees it too).
            const float gx = dv * (1.0f - r);
            // physiology gradients of step t, from the adjoints entering it (saved: the
            // currents after the step's input, G, and the adaptation current entering it)
            if (PHYS) {
                float Isyn = 0.0f;
#pragma unroll
                for (int c = 0; c < S; c++) Isyn = Isyn + G[c] * net.E_syn[c];
                if (ADAPT) Isyn = Isyn - (cur.ga * a_decay + adapt_n * s);  // - I_a{t+1}
                const float drive = E_L + Cm * Isyn;  // U_rest + R (sum_j sign_j I_j - I_a)
                if (wants & WT_W_BETA) acc_beta += gx * (v - drive);
                if (wants & WT_W_E_L) acc_E_L += gx * (1.0f - beta);
                if (wants & WT_W_C_M) acc_C_m += gx * (1.0f - beta) * Isyn;
                if (wants & WT_W_RESET) acc_reset += dv * r;
                if (ADAPT && (wants & WT_W_ADAPT)) acc_adapt += la * s;
                if (ADAPT && (wants & WT_W_ADAPT_DECAY)) acc_adapt_decay += la * cur.ga;
            }
            if (SYN && (wants & WT_W_DECAY)) {  // I_{t+1} = decay I_t + X_t
#pragma unroll
                for (int c = 0; c < S; c++) {
                    float It;
                    if (t == 0)
                        It = bw.g_init[((size_t)b * 2 * S + S + c) * N + n];
                    else if (t - 1 >= t_lo)
                        It = q[0].G[c];
                    else
                        It = __ldg(G_b + ((size_t)(t - 1) * S + c) * N);
                    acc_dd[c] += ld[c] * It;
                }
            }
            if (ADAPT) la = la * a_decay;  // I_a{t+1} = a_decay I_a{t} + adapt s_t (s detached)
            const float xv = v - theta;
            const float gs = cur.gs + R_b;
            float g_x;
            if (SAMPLE) {
                const float p = sigmoid(k * xv);
                g_x = gs * k * p * (1.0f - p);
            } else {
                const float d = k * fabsf(xv) + 1.0f;
                g_x = __fdividef(gs, d * d);
            }
            if (PROB && bw.grad_prob) {
                const float p = sigmoid(k * xv);
                g_x += cur.gp * k * p * (1.0f - p);
            }
            if (REF) g_x *= 1.0f - held;
            acc_theta -= g_x;
            dv = gx * beta + g_x;
#pragma unroll
            for (int c = 0; c < S; c++) {
                ld[c] = ld[c] * net.decay_d[c];
                lr[c] = 0.0f;
            }
            // the membrane of step t - 1 read I_t and I_a{t}: its term, ahead
            if (t >= 1) {
                unsigned sb1, hb1;
                if (t - 1 >= t_lo) {
                    sb1 = q[0].sb;
                    hb1 = q[0].hb;
                } else {
                    sb1 = __ldg(sb_b + (size_t)(t - 1) * words);
                    hb1 = REF ? __ldg(hb_b + (size_t)(t - 1) * words) : 0u;
                }
                const float r1 = ((sb1 >> (n & 31)) & 1u) || (REF && ((hb1 >> (n & 31)) & 1u)) ? 1.0f : 0.0f;
                const float c1 = dv * (1.0f - r1) * (1.0f - beta) * Cm;
#pragma unroll
                for (int c = 0; c < S; c++) ld[c] = ld[c] + c1 * net.E_syn[c];
                if (ADAPT) la = la - c1;
            }
            continue;
        }
        float g_a = 0.0f;
        if (ADAPT) {
            g_a = cur.ga;
            if (wants & WT_W_ADAPT) acc_adapt += la * s;
            if (wants & WT_W_ADAPT_DECAY) acc_adapt_decay += la * g_a;
        }

        // Membrane adjoint.
        float Gc[S], Bm[S], clampg[S], Ge[S];
        float Ssum = 0.0f, EG = 0.0f;
#pragma unroll
        for (int c = 0; c < S; c++) {
            Gc[c] = fminf(fmaxf(G[c], 0.0f), net.g_clip[c]);
            float cg = G[c] < net.g_clip[c] ? 1.0f : (G[c] == net.g_clip[c] ? 0.5f : 0.0f);
            clampg[c] = G[c] >= 0.0f ? cg : 0.0f;
            Bm[c] = MG ? sigmoid(net.mg_a[c] * v - net.mg_lc[c]) : 1.0f;
            Ge[c] = MG ? Gc[c] * Bm[c] : Gc[c];
            Ssum = Ssum + Ge[c];
            EG = EG + Ge[c] * net.E_syn[c];
        }
        const float gx = dv * (1.0f - r);
        float J = g_L * (v - E_L) + v * Ssum - EG;
        if (ADAPT) {
            Ssum = Ssum + g_a;
            J = J + g_a * (v - E_a);
        }
        const float em = expm1f(-dt * (rate + Ssum * inv_C));
        const float inv_g = __fdividef(1.0f, g_L + Ssum);  // a gradient: 2-ulp division suffices
        const float a = 1.0f + em, phi = -em * inv_g;
        const float phi_S = (a * dt * inv_C - phi) * inv_g;
        const float k0 = -gx * (phi_S * J + phi * v), k1 = gx * phi;
        float dv_in = gx * a;
        float dG[S];
#pragma unroll
        for (int c = 0; c < S; c++) {
            const float dGe = k0 + k1 * net.E_syn[c];
            if (MG) {
                dv_in += dGe * Gc[c] * net.mg_a[c] * Bm[c] * (1.0f - Bm[c]);
                dG[c] = dGe * Bm[c] * clampg[c];
            } else {
                dG[c] = dGe * clampg[c];
            }
            if (SYN && (wants & WT_W_E_SYN)) acc_E[c] += gx * phi * Ge[c];
        }
        if (wants & WT_W_RESET) acc_reset += dv * r;
        if (wants & WT_W_E_L) acc_E_L += gx * phi * g_L;
        if (wants & WT_W_C_M) {
            const float dphi = -(a * dt * Ssum * inv_C * inv_C + phi * g_L * inv_C) * inv_g;
            acc_C_m -= gx * (dphi * J + phi * (v - E_L) * g_L * inv_C);
        }
        if (wants & WT_W_BETA) {
            const float dg_L = -Cm / (beta * dt);
            const float dphi = -(a / beta + phi * dg_L) * inv_g;
            acc_beta -= gx * (dphi * J + phi * (v - E_L) * dg_L);
        }
        if (ADAPT) {
            const float d_ga = k0 + k1 * E_a;
            if (wants & WT_W_E_ADAPT) acc_E_a += gx * phi * g_a;
            la = la * a_decay + d_ga;
        }
        // The spike (surrogate) and probability of step t, both of v - theta.
        const float xv = v - theta;
        const float gs = cur.gs + R_b;
        float g_x;
        if (SAMPLE) {
            const float p = sigmoid(k * xv);
            g_x = gs * k * p * (1.0f - p);
        } else {
            const float d = k * fabsf(xv) + 1.0f;
            g_x = __fdividef(gs, d * d);
        }
        if (PROB && bw.grad_prob) {
            const float p = sigmoid(k * xv);
            g_x += cur.gp * k * p * (1.0f - p);
        }
        if (REF) g_x *= 1.0f - held;
        dv = dv_in + g_x;
        acc_theta -= g_x;
#pragma unroll
        for (int c = 0; c < S; c++) {
            lr[c] = lr[c] * net.decay_r[c] + dG[c];
            ld[c] = ld[c] * net.decay_d[c] + dG[c];
        }
    }

    if (adj) {  // the state leaving the chunk
        adj[0] = dv;
        adj[(size_t)N] = la;
#pragma unroll
        for (int c = 0; c < S; c++) {
            adj[(size_t)(2 + c) * N] = lr[c];
            adj[(size_t)(2 + S + c) * N] = ld[c];
            if (SYN) {
                adj[(size_t)(2 + 2 * S + c) * N] = H_r[c];
                adj[(size_t)(2 + 3 * S + c) * N] = H_d[c];
            }
        }
    }
    // outputs: written, or added to when the scan is taken in chunks
    auto put = [&](float *dst, float val) { *dst = adj ? *dst + val : val; };
    const size_t bn = (size_t)b * N + n;
    if (wants & WT_W_THETA) put(bw.g_theta + bn, acc_theta);
    if (wants & WT_W_RESET) put(bw.g_reset + bn, acc_reset);
    if (wants & WT_W_E_L) put(bw.g_E_L + bn, acc_E_L);
    if (wants & WT_W_C_M) put(bw.g_C_m + bn, acc_C_m);
    if (wants & WT_W_BETA) put(bw.g_beta + bn, acc_beta);
    if (wants & WT_W_ADAPT) put(bw.g_adapt + bn, acc_adapt);
    if (wants & WT_W_ADAPT_DECAY) put(bw.g_adapt_decay + bn, acc_adapt_decay);
    if (wants & WT_W_E_ADAPT) put(bw.g_E_adapt + bn, acc_E_a);
    if (SYN) {
        const float *gi = bw.g_init + (size_t)b * 2 * S * N + n;
        const bool first = t_lo == 0;  // the conductances entering the run: once, at its start
#pragma unroll
        for (int c = 0; c < S; c++) {
            if (wants & WT_W_E_SYN) put(bw.g_E_syn + ((size_t)b * S + c) * N + n, acc_E[c]);
            if (wants & WT_W_JUMP) {
                put(bw.g_jump + ((size_t)b * 2 * S + c) * N + n, acc_jr[c]);
                put(bw.g_jump + ((size_t)b * 2 * S + S + c) * N + n, acc_jd[c]);
            }
            if (wants & WT_W_DECAY) {
                put(bw.g_decay + ((size_t)b * 2 * S + c) * N + n, acc_dr[c] + (first ? gi[(size_t)c * N] * H_r[c] : 0.0f));
                put(bw.g_decay + ((size_t)b * 2 * S + S + c) * N + n,
                    acc_dd[c] + (first ? gi[(size_t)(S + c) * N] * H_d[c] : 0.0f));
            }
        }
    }
}

// The edge gradients, source by source. First each source's firing over the whole run
// is transposed into a bit row over (trial, step) ("fired"); then one warp per source
// (taken from a work counter) lists the (trial, step) of its events in shared memory and
// walks every edge of its slots with them: each lane sums a * Q[b, t, c, n] for its
// edges in registers and adds the sum once per edge — one reduction per edge instead of
// one per (event, edge), and each edge's target and weight read once per source instead
// of once per event.

constexpr int kFiredGroup = 8;  // 32-step words written together per source (32 bytes)

// Recurrent sources: a warp per (word of 32 neurons, group of 8 x 32 (trial, step)).
__global__ void fired_rec_kernel(const WtEdgeGrads eg, int N, long long BT, int words, long long BTw8) {
    const int lane = threadIdx.x & 31;
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long groups = BTw8 / kFiredGroup;
    if (warp >= (long long)words * groups) return;
    const int w = (int)(warp / groups);
    const long long g = warp % groups;
    uint32_t out[kFiredGroup];
#pragma unroll
    for (int k = 0; k < kFiredGroup; k++) {
        const long long bt = (g * kFiredGroup + k) * 32 + lane;
        const uint32_t word = bt < BT ? __ldg(eg.spike_bits + bt * words + w) : 0u;
        uint32_t mine = 0;
        for (int l = 0; l < 32; l++) {
            const uint32_t r = __ballot_sync(kFull, (word >> l) & 1u);
            if (lane == l) mine = r;
        }
        out[k] = mine;
    }
    const int src = w * 32 + lane;
    if (src < N) {
        uint4 *dst = reinterpret_cast<uint4 *>(eg.fired + (size_t)src * BTw8 + g * kFiredGroup);
        dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
        dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
    }
}

// Input columns (x != 0): a warp per (32 columns, group of 8 x 32 (trial, step)).
__global__ void fired_in_kernel(const WtEdgeGrads eg, int N, int n_in, long long BT, long long BTw8) {
    const int lane = threadIdx.x & 31;
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long groups = BTw8 / kFiredGroup;
    const int cblocks = (n_in + 31) >> 5;
    if (warp >= (long long)cblocks * groups) return;
    const int c = (int)(warp / groups) * 32 + lane;
    const long long g = warp % groups;
    uint32_t out[kFiredGroup];
#pragma unroll
    for (int k = 0; k < kFiredGroup; k++) {
        uint32_t mine = 0;
        const long long bt0 = (g * kFiredGroup + k) * 32;
        for (int i = 0; i < 32; i++) {
            const long long bt = bt0 + i;
            if (bt < BT && c < n_in && __ldg(eg.x + bt * n_in + c) != 0.0f) mine |= 1u << i;
        }
        out[k] = mine;
    }
    if (c < n_in) {
        uint4 *dst = reinterpret_cast<uint4 *>(eg.fired + (size_t)(N + c) * BTw8 + g * kFiredGroup);
        dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
        dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
    }
}

constexpr int kEventCap = 512;      // events a warp lists before walking its edges
constexpr int kEdgeWarps = 8;

__global__ void __launch_bounds__(kEdgeWarps * 32) edge_grads_kernel(const WtNet net, const WtEdgeGrads eg,
                                                                     long long BT, long long BTw8) {
    __shared__ int s_bt[kEdgeWarps][kEventCap];
    __shared__ float s_a[kEdgeWarps][kEventCap];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    int *lbt = s_bt[wib];
    float *la = s_a[wib];
    const int N = net.N, C = net.C, n_in = net.n_in;
    const int n_src = N + n_in;
    const long long BTw = (BT + 31) >> 5;
    for (;;) {
        int j = 0;
        if (lane == 0) j = (int)atomicAdd(eg.work, 1u);
        j = __shfl_sync(kFull, j, 0);
        if (j >= n_src) break;
        const int slot0 = net.src_slot[j], slot1 = net.src_slot[j + 1];
        if (slot0 == slot1) continue;
        const uint32_t *fw = eg.fired + (size_t)j * BTw8;
        const bool is_in = j >= N;
        const int col = j - N;

        // Walk every edge of the source with the listed events.
        auto flush = [&](int len) {
            __syncwarp();
            for (int slot = slot0; slot < slot1; slot++) {
                int fcol = -1;
                if (net.slot_gate) {
                    const int gate = net.slot_gate[slot];
                    if (gate >= 0) fcol = net.gate_cols[4 * gate + 3] + net.slot_row[slot];
                }
                for (int ch = net.slot_chunk[slot]; ch < net.slot_chunk[slot + 1]; ch++) {
                    const long long d = net.chunk_desc[ch];
                    const long long e0 = d & ((1LL << 56) - 1);
                    const int elen = (int)((unsigned long long)d >> 56);
                    const int kp = eg.chunk_path[ch];
                    for (int q0 = 0; q0 < elen; q0 += 128) {
                        int nq[4], cq[4];
                        float acc[4];
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            const int q = q0 + lane + 32 * u;
                            nq[u] = -1;
                            cq[u] = 0;
                            acc[u] = 0.0f;
                            if (q < elen) {
                                const uint32_t pc = net.edge_col[e0 + q];
                                nq[u] = (int)(pc & 0x7ffffffu);
                                cq[u] = (int)(pc >> 27);
                            }
                        }
#pragma unroll 4
                        for (int i = 0; i < len; i++) {
                            const long long bt = lbt[i];
                            float a = la[i];
                            if (fcol >= 0) a *= eg.f_saved[bt * net.R_f + fcol];
                            const float *Qb = eg.Q + bt * C * N;
#pragma unroll
                            for (int u = 0; u < 4; u++)
                                if (nq[u] >= 0) acc[u] += a * __ldg(Qb + (size_t)cq[u] * N + nq[u]);
                        }
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            if (nq[u] < 0) continue;
                            const long long e = e0 + q0 + lane + 32 * u;
                            const double jfv = eg.jf[(size_t)kp * C + cq[u]];
                            if (eg.g_scale)
                                atomicAdd(eg.g_scale + (size_t)kp * N + nq[u], (double)acc[u] * (double)eg.w_raw[e] * jfv);
                            if (eg.g_w)
                                atomicAdd(eg.g_w + e, (double)acc[u] * (double)eg.scale[(size_t)kp * N + nq[u]] * jfv);
                        }
                    }
                }
            }
            __syncwarp();
        };

        // List the source's events, kEventCap/32 words (of 32 steps) at a time.
        int len = 0;
        constexpr int kWin = kEventCap / 32;
        for (long long wb = 0; wb < BTw; wb += kWin) {
            uint32_t word = (lane < kWin && wb + lane < BTw) ? fw[wb + lane] : 0u;
            const int cnt = __popc(word);
            const int incl = warp_inclusive_sum(cnt, lane);
            const int total = __shfl_sync(kFull, incl, 31);
            if (total == 0) continue;
            if (len + total > kEventCap) {
                flush(len);
                len = 0;
            }
            int off = len + incl - cnt;
            while (word) {
                const int bit = __ffs(word) - 1;
                word &= word - 1;
                const long long bt = (wb + lane) * 32 + bit;
                lbt[off] = (int)bt;
                la[off] = is_in ? eg.x[bt * n_in + col] : 1.0f;
                off++;
            }
            len += total;
        }
        if (len) flush(len);
    }
}


// ---------------------------------------------------------------------------------------
// The edge gradients target by target (WtEdgeGrads.QT). Each source's events are listed
// once (b Tp + t, in (trial, step) order, with where each slice of trials starts); then a
// block per target stages the target's adjoints QT[c, n, b, :] of one slice of trials in
// shared memory and every thread sums, for its in-edges, a * QT over the source's events
// of that slice from there. Each adjoint is read from HBM once, by one coalesced copy; the
// per-edge sums are plain writes (the block owns its target's in-edges).
// ---------------------------------------------------------------------------------------

constexpr int kTargetThreads = 256;
constexpr int kSliceBytes = 64 * 1024;  // shared memory a block's slice may take

// Events per source: a warp per source over its fired row.
__global__ void event_count_kernel(const WtEdgeGrads eg, int n_src, int slices, long long BTw, long long BTw8) {
    const int lane = threadIdx.x & 31;
    const long long j = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (j >= n_src) return;
    const uint32_t *fw = eg.fired + (size_t)j * BTw8;
    int cnt = 0;
    for (long long w = lane; w < BTw; w += 32) cnt += __popc(__ldg(fw + w));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(kFull, cnt, o);
    if (lane == 0) eg.ev_start[(size_t)j * (slices + 1)] = cnt;
}

// Exclusive sums of the counts over the sources (one block): the start of each source's
// list; WT_ERR_EVENTS when the total exceeds the capacity.
__global__ void event_scan_kernel(const WtEdgeGrads eg, int n_src, int slices) {
    __shared__ long long part[1024];
    const int tid = threadIdx.x, nt = blockDim.x;
    const long long per = ((long long)n_src + nt - 1) / nt;
    const long long lo = tid * per, hi = min((long long)n_src, lo + per);
    long long sum = 0;
    for (long long j = lo; j < hi; j++) sum += eg.ev_start[(size_t)j * (slices + 1)];
    part[tid] = sum;
    __syncthreads();
    for (int o = 1; o < nt; o <<= 1) {  // inclusive scan of the per-thread sums
        const long long y = tid >= o ? part[tid - o] : 0;
        __syncthreads();
        part[tid] += y;
        __syncthreads();
    }
    long long run = part[tid] - sum;
    for (long long j = lo; j < hi; j++) {
        const long long c = eg.ev_start[(size_t)j * (slices + 1)];
        eg.ev_start[(size_t)j * (slices + 1)] = (int32_t)min(run, eg.ev_cap);
        run += c;
    }
    if (tid == nt - 1 && part[tid] > eg.ev_cap) set_error(eg.err, WT_ERR_EVENTS);
}

// Each source's list: a warp per source walks its fired row 32 words at a time, writes
// every event as b Tp + t and records where each slice of trials (bq trials) begins.
__global__ void event_list_kernel(const WtEdgeGrads eg, int n_src, int slices, int bq, int T, int Tp, long long BT,
                                  long long BTw, long long BTw8) {
    const int lane = threadIdx.x & 31;
    const long long j = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (j >= n_src) return;
    if (read_error(eg.err)) return;  // over capacity: no list is written
    int32_t *starts = eg.ev_start + (size_t)j * (slices + 1);
    const uint32_t *fw = eg.fired + (size_t)j * BTw8;
    int base = starts[0];
    const long long span = (long long)bq * T;  // bits of one slice
    for (long long w0 = 0; w0 < BTw; w0 += 32) {
        const long long w = w0 + lane;
        const uint32_t word = w < BTw ? __ldg(fw + w) : 0u;
        const int cnt = __popc(word);
        const int incl = warp_inclusive_sum(cnt, lane);
        const int total = __shfl_sync(kFull, incl, 31);
        int off = base + incl - cnt;
        // slice boundaries that fall inside this lane's word
        if (w < BTw) {
            for (long long sl = (w * 32 + span - 1) / span; sl * span < w * 32 + 32 && sl < slices; sl++) {
                if (sl == 0) continue;
                const int bits = (int)(sl * span - w * 32);
                starts[sl] = off + __popc(bits >= 32 ? word : (word & ((1u << bits) - 1u)));
            }
        }
        uint32_t m = word;
        while (m) {
            const int bit = __ffs(m) - 1;
            m &= m - 1;
            const long long bt = w * 32 + bit;
            const int b = (int)(bt / T), t = (int)(bt - (long long)b * T);
            eg.ev[off++] = b * Tp + t;
        }
        base += total;
    }
    if (lane == 0) starts[slices] = base;
}

// The sum over source j's events of one slice of a * QT (the slice staged at qc).
__device__ __forceinline__ float slice_sum(const WtNet &net, const WtEdgeGrads &eg, const float *qc, int j, int fcol,
                                           int q0, int q1, int T, int Tp) {
    float acc = 0.0f;
    if (j < net.N && fcol < 0) {
        for (int q = q0; q < q1; q++) acc += qc[__ldg(eg.ev + q)];
    } else {  // input values and gating factors scale the events
        for (int q = q0; q < q1; q++) {
            const int ev = __ldg(eg.ev + q);
            const int b = ev / Tp, t = ev - b * Tp;
            const size_t bt = (size_t)b * T + t;
            float a = j >= net.N ? eg.x[bt * net.n_in + (j - net.N)] : 1.0f;
            if (fcol >= 0) a *= eg.f_saved[bt * net.R_f + fcol];
            acc += a * qc[ev];
        }
    }
    return acc;
}

__global__ void __launch_bounds__(kTargetThreads, 3) edge_grads_target_kernel(const WtNet net, const WtEdgeGrads eg,
                                                                          int slices, int bq, int T, int Tp) {
    extern __shared__ __align__(16) float qs[];  // [c][b - b0][Tp]
    const int N = net.N, C = net.C, B = net.B;
    const int tid = threadIdx.x;
    const size_t BTp = (size_t)B * Tp;
    __shared__ int s_n;
    if (read_error(eg.err)) return;
    // the slice sl of this target's adjoints, every channel, into shared memory
    auto stage = [&](int n, int sl) {
        const int b0 = sl * bq, nb = min(bq, B - b0);
        const int row = nb * Tp;  // floats, a multiple of 8
        __syncthreads();
        for (int c = 0; c < C; c++) {
            const float4 *src = reinterpret_cast<const float4 *>(eg.QT + ((size_t)c * N + n) * BTp + (size_t)b0 * Tp);
            float4 *dst = reinterpret_cast<float4 *>(qs + (size_t)c * bq * Tp);
            for (int k = tid; k < row / 4; k += kTargetThreads) dst[k] = __ldcs(src + k);
        }
        __syncthreads();
    };
    // in-edge i's gradients from its sum over every event (this block alone writes them)
    auto finish = [&](int n, int i, float sum) {
        const int e = eg.in_edge[i];
        const int k = eg.in_path[i] >> 3, c = eg.in_path[i] & 7;
        const double acc = (double)sum;
        const double jfv = eg.jf[(size_t)k * C + c];
        if (eg.g_w) eg.g_w[e] += acc * (double)eg.scale[(size_t)k * N + n] * jfv;
        if (eg.g_scale) atomicAdd(eg.g_scale + (size_t)k * N + n, acc * (double)eg.w_raw[e] * jfv);
    };
    for (;;) {
        __syncthreads();
        if (tid == 0) s_n = (int)atomicAdd(eg.work, 1u);
        __syncthreads();
        const int n = s_n;
        if (n >= N) return;
        const int i0 = eg.in_ptr[n], i1 = eg.in_ptr[n + 1];
        if (i0 == i1) continue;
        // each thread's in-edges, slice by slice, the sums kept in in_acc (keeping up to
        // four in-edges in registers across the slices and summing them side by side
        // measured twice as slow on C2)
        for (int sl = 0; sl < slices; sl++) {
            stage(n, sl);
            const int base = sl * bq * Tp;
            for (int i = i0 + tid; i < i1; i += kTargetThreads) {
                const int j = eg.in_src[i];
                const int c = eg.in_path[i] & 7;
                const int fcol = eg.in_fcol ? eg.in_fcol[i] : -1;
                const int32_t *st = eg.ev_start + (size_t)j * (slices + 1) + sl;
                const float acc = slice_sum(net, eg, qs + (size_t)c * bq * Tp - base, j, fcol, st[0], st[1], T, Tp);
                eg.in_acc[i] = sl ? eg.in_acc[i] + acc : acc;
            }
        }
        for (int i = i0 + tid; i < i1; i += kTargetThreads) finish(n, i, eg.in_acc[i]);
    }
}

// One warp per (trial, step, input column): the input's gradient, fired or not.
__global__ void input_grads_kernel(const WtNet net, const WtEdgeGrads eg) {
    const int lane = threadIdx.x & 31;
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    const int N = net.N, C = net.C, n_in = net.n_in;
    const long long total = (long long)net.B * eg.T * n_in;
    for (long long w = warp; w < total; w += nwarps) {
        const long long bt = w / n_in;
        const int c_in = (int)(w % n_in);
        const int src = N + c_in;
        const float *Qbt = eg.Q + (size_t)bt * C * N;
        float acc = 0.0f;
        for (int slot = net.src_slot[src]; slot < net.src_slot[src + 1]; slot++) {
            float f = 1.0f;
            if (net.slot_gate) {
                const int gate = net.slot_gate[slot];
                if (gate >= 0) f = eg.f_saved[(size_t)bt * net.R_f + net.gate_cols[4 * gate + 3] + net.slot_row[slot]];
            }
            float part = 0.0f;
            for (int ch = net.slot_chunk[slot]; ch < net.slot_chunk[slot + 1]; ch++) {
                const long long d = net.chunk_desc[ch];
                const long long e0 = d & ((1LL << 56) - 1);
                const int len = (int)((unsigned long long)d >> 56);
                const int kp = eg.chunk_path[ch];
                for (int q = lane; q < len; q += 32) {
                    const uint32_t pc = net.edge_col[e0 + q];
                    const int n = pc & 0x7ffffffu, c = pc >> 27;
                    part += eg.w_raw[e0 + q] * eg.scale[(size_t)kp * N + n] * eg.jf[(size_t)kp * C + c] *
                            Qbt[(size_t)c * N + n];
                }
            }
            acc += f * part;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
        if (lane == 0) eg.g_x[w] = acc;
    }
}

template <int S>
cudaError_t launch_bwd_s(const WtNet &net, const WtBackward &bw, cudaStream_t st) {
    const long long items = (long long)net.B * net.N;
    const int blocks = (int)((items + kBlock - 1) / kBlock);
    const bool syn = bw.wants & (WT_W_E_SYN | WT_W_DECAY | WT_W_JUMP);
    if (bw.flags & WT_F_CURRENT) {
        if (syn)
            backward_kernel<S, true, true, true><<<blocks, kBlock, 0, st>>>(net, bw);
        else if (bw.wants)
            backward_kernel<S, true, false, true><<<blocks, kBlock, 0, st>>>(net, bw);
        else
            backward_kernel<S, false, false, true><<<blocks, kBlock, 0, st>>>(net, bw);
    } else if (syn) {
        backward_kernel<S, true, true, false><<<blocks, kBlock, 0, st>>>(net, bw);
    } else if (bw.wants) {
        backward_kernel<S, true, false, false><<<blocks, kBlock, 0, st>>>(net, bw);
    } else {
        backward_kernel<S, false, false, false><<<blocks, kBlock, 0, st>>>(net, bw);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_backward(const WtNet &net, const WtBackward &bw, cudaStream_t st) {
    switch (net.S) {
        case 1: return launch_bwd_s<1>(net, bw, st);
        case 2: return launch_bwd_s<2>(net, bw, st);
        case 3: return launch_bwd_s<3>(net, bw, st);
        case 4: return launch_bwd_s<4>(net, bw, st);
        case 5: return launch_bwd_s<5>(net, bw, st);
        case 6: return launch_bwd_s<6>(net, bw, st);
        case 7: return launch_bwd_s<7>(net, bw, st);
        case 8: return launch_bwd_s<8>(net, bw, st);
        default: return cudaErrorInvalidValue;
    }
}

int edge_grads_slice_trials(const WtNet &net, int T) {
    const long long per_trial = (long long)net.C * ((T + 7) & ~7) * 4;  // bytes of one trial's adjoints
    if (per_trial > kSliceBytes) return 0;
    return (int)std::min<long long>(net.B, kSliceBytes / per_trial);
}

long long edge_grads_fired_words(const WtNet &net, int T) {
    const long long BT = (long long)net.B * T;
    const long long BTw8 = ((BT + 31) / 32 + kFiredGroup - 1) / kFiredGroup * kFiredGroup;
    return (long long)(net.N + net.n_in) * BTw8;
}

cudaError_t launch_edge_grads(const WtNet &net, const WtEdgeGrads &eg, cudaStream_t st) {
    const long long BT = (long long)net.B * eg.T;
    const long long BTw8 = ((BT + 31) / 32 + kFiredGroup - 1) / kFiredGroup * kFiredGroup;
    if (eg.g_scale || eg.g_w) {
        const int words = (net.N + 31) >> 5;
        const long long groups = BTw8 / kFiredGroup;
        long long warps = (long long)words * groups;
        if (warps > 0) fired_rec_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(eg, net.N, BT, words, BTw8);
        warps = (long long)((net.n_in + 31) >> 5) * groups;
        if (warps > 0) fired_in_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(eg, net.N, net.n_in, BT, BTw8);
        cudaError_t e = cudaMemsetAsync(eg.work, 0, sizeof(uint32_t), st);
        if (e != cudaSuccess) return e;
        int sms = 0, dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (eg.QT) {  // target by target
            const int n_src = net.N + net.n_in;
            const int T = eg.T, Tp = (T + 7) & ~7;
            const int bq = edge_grads_slice_trials(net, T);
            const int slices = (net.B + bq - 1) / bq;
            const long long BTw = (BT + 31) >> 5;
            const unsigned wblocks = (unsigned)(((long long)n_src + 7) / 8);
            event_count_kernel<<<wblocks, 256, 0, st>>>(eg, n_src, slices, BTw, BTw8);
            event_scan_kernel<<<1, 1024, 0, st>>>(eg, n_src, slices);
            event_list_kernel<<<wblocks, 256, 0, st>>>(eg, n_src, slices, bq, T, Tp, BT, BTw, BTw8);
            const size_t smem = (size_t)net.C * bq * Tp * 4;
            e = cudaFuncSetAttribute(edge_grads_target_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            int per_sm = 0;
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, edge_grads_target_kernel, kTargetThreads, smem);
            if (e != cudaSuccess) return e;
            edge_grads_target_kernel<<<sms * (per_sm > 0 ? per_sm : 1), kTargetThreads, smem, st>>>(net, eg, slices,
                                                                                                     bq, T, Tp);
            e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        } else {  // source by source
            int per_sm = 0;
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, edge_grads_kernel, kEdgeWarps * 32, 0);
            if (e != cudaSuccess) return e;
            edge_grads_kernel<<<sms * (per_sm > 0 ? per_sm : 1), kEdgeWarps * 32, 0, st>>>(net, eg, BT, BTw8);
            e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
    }
    if (eg.g_x && net.n_in > 0) {
        const long long warps = (long long)net.B * eg.T * net.n_in;
        long long blocks = (warps + 7) / 8;
        if (blocks > 148 * 64) blocks = 148 * 64;
        input_grads_kernel<<<(int)blocks, 256, 0, st>>>(net, eg);
    }
    return cudaGetLastError();
}

}  // namespace wt
