// Gradients through the recurrent spikes (Drive.recurrent_gradients; the reference's
// _recurrent_backward, conductance/engine.py:386-436, with carry_to_sources and
// presynaptic, network_simulators/engine.py:257-306). Taken one reverse step t at a
// time, between two chunks of the reverse scan (wt_backward with t_lo = t, t_hi = t + 1):
//
//   1. q_kernel: each (trial, neuron)'s input adjoint of step t,
//      Q[b, c, n] = sum over channels j fed by c of jump_r[j] l_r[j] + jump_d[j] l_d[j],
//      from the adjoint state entering the step, written transposed (C, N, B) through a
//      shared-memory tile so that the next kernel reads it trials-fastest;
//   2. carry_kernel: one warp per recurrent source j, lanes over trials: for every edge
//      e of j (pathway k, target n, channel c), with the edge's folded weight
//      w_e scale[k, n] jf[k, c] (its fixed-point word over 2^s_c),
//      R[b, j] = sum_e coef_e Q[b, c, n]  (a gated slot's sum times its factor at t),
//      each lane decoding one of 32 edges, the warp then reading each edge's 64 trials
//      as one coalesced 256-byte row of the L2-resident Q (two trials per lane).
#include "common.cuh"

namespace wt {
namespace {

constexpr int kTile = 32;

__global__ void __launch_bounds__(256) q_kernel(const WtNet net, const WtRecurrentCarry rc) {
    __shared__ float tile[WT_MAX_CHANNELS][kTile][kTile + 1];
    const int N = net.N, B = net.B, S = net.S, C = net.C;
    const int NA = 2 + 4 * S;
    const int n0 = blockIdx.x * kTile, b0 = blockIdx.y * kTile;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    for (int i = ty; i < kTile; i += 8) {
        const int b = b0 + i, n = n0 + tx;
        float q[WT_MAX_CHANNELS];
        for (int c = 0; c < C; c++) q[c] = 0.0f;
        if (b < B && n < N) {
            const float *a = rc.adj + (size_t)b * NA * N + n;
            for (int j = 0; j < S; j++) {
                const int c = net.input_of[j];
                if (c < 0) continue;
                q[c] = q[c] + (net.jump_r[j] * a[(size_t)(2 + j) * N] + net.jump_d[j] * a[(size_t)(2 + S + j) * N]);
            }
        }
        for (int c = 0; c < C; c++) tile[c][i][tx] = q[c];
    }
    __syncthreads();
    for (int i = ty; i < kTile; i += 8) {
        const int n = n0 + i, b = b0 + tx;
        if (n < N && b < B)
            for (int c = 0; c < C; c++) rc.Qt[((size_t)c * N + n) * B + b] = tile[c][tx][i];
    }
}

__global__ void __launch_bounds__(256) carry_kernel(const WtNet net, const WtRecurrentCarry rc) {
    const int lane = threadIdx.x & 31;
    const int j = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int N = net.N, B = net.B;
    if (j >= N) return;  // whole warps
    const int slot0 = net.src_slot[j], slot1 = net.src_slot[j + 1];
    const bool pairs = (B & 1) == 0;  // trials two at a time: one 8-byte load per edge
    for (int bb = 0; bb < B; bb += 64) {
        // this lane's trials: bb + 2 lane, + 1 (pairs), else bb + lane, bb + 32 + lane
        const int b_a = pairs ? bb + 2 * lane : bb + lane;
        const int b_b = pairs ? b_a + 1 : bb + 32 + lane;
        const bool ok_a = b_a < B, ok_b = b_b < B;
        float acc_a = 0.0f, acc_b = 0.0f;
        for (int slot = slot0; slot < slot1; slot++) {
            float sub_a = 0.0f, sub_b = 0.0f;
            for (int ch = net.slot_chunk[slot]; ch < net.slot_chunk[slot + 1]; ch++) {
                const long long d = net.chunk_desc[ch];
                const long long e0 = d & ((1LL << 56) - 1);
                const int len = (int)((unsigned long long)d >> 56);
                for (int q0 = 0; q0 < len; q0 += 32) {
                    // each lane decodes one edge: its Q row (c N + n) and coefficient
                    unsigned row = 0;
                    float coef = 0.0f;
                    if (q0 + lane < len) {
                        const unsigned long long cw = __ldg(net.edge_cw + e0 + q0 + lane);
                        const unsigned lo = (unsigned)cw;
                        const int c = (int)(lo >> 27);
                        row = (unsigned)c * (unsigned)N + (lo & 0x7ffffffu);
                        coef = __uint_as_float((unsigned)(cw >> 32)) * net.fx_inv[c];
                    }
                    const int m = min(32, len - q0);
                    for (int i0 = 0; i0 < m; i0 += 8) {
                        float cf[8], qa[8], qb[8];
#pragma unroll
                        for (int u = 0; u < 8; u++) {  // lanes past m hold row 0, coefficient 0
                            const int src = (i0 + u) & 31;
                            const unsigned r = __shfl_sync(kFull, row, src);
                            cf[u] = __shfl_sync(kFull, coef, src);
                            const float *qrow = rc.Qt + (size_t)r * B;
                            if (pairs) {
                                float2 q2 = make_float2(0.0f, 0.0f);
                                if (ok_a) q2 = __ldcg(reinterpret_cast<const float2 *>(qrow + b_a));
                                qa[u] = q2.x;
                                qb[u] = q2.y;
                            } else {
                                qa[u] = ok_a ? __ldcg(qrow + b_a) : 0.0f;
                                qb[u] = ok_b ? __ldcg(qrow + b_b) : 0.0f;
                            }
                        }
#pragma unroll
                        for (int u = 0; u < 8; u++) {
                            if (i0 + u < m) {
                                sub_a += cf[u] * qa[u];
                                sub_b += cf[u] * qb[u];
                            }
                        }
                    }
                }
            }
            if (net.slot_gate && rc.f_saved) {  // a gated slot: this step's factor per trial
                const int gate = net.slot_gate[slot];
                if (gate >= 0) {
                    const int col = net.gate_cols[4 * gate + 3] + net.slot_row[slot];
                    if (ok_a) sub_a *= rc.f_saved[((size_t)b_a * rc.T + rc.t) * net.R_f + col];
                    if (ok_b) sub_b *= rc.f_saved[((size_t)b_b * rc.T + rc.t) * net.R_f + col];
                }
            }
            acc_a += sub_a;
            acc_b += sub_b;
        }
        if (ok_a) rc.R[(size_t)b_a * N + j] = acc_a;
        if (ok_b) rc.R[(size_t)b_b * N + j] = acc_b;
    }
}

}  // namespace

cudaError_t launch_recurrent_carry(const WtNet &net, const WtRecurrentCarry &rc, cudaStream_t st) {
    const dim3 qgrid((net.N + kTile - 1) / kTile, (net.B + kTile - 1) / kTile);
    q_kernel<<<qgrid, 256, 0, st>>>(net, rc);
    carry_kernel<<<(net.N + 7) / 8, 256, 0, st>>>(net, rc);
    return cudaGetLastError();
}

}  // namespace wt
