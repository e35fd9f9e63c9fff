// The factorised (low-rank) recurrent drive on the tensor cores. A pathway k whose weights
// are W_k = U_k V^T (rank r <= 64; the benchmark's factorised configuration C3, a linear
// low-rank product, where wiretorch's LowRankProjection, projections.py:167-216, assembles
// a dense W every forward, network.py:731-752) drives neuron n of trial b with
//
//   a_k[b, n] = sum_j s_j(b) W_k[j, n] = sum_r V[n, r] P_k[b, r],   P_k = S_k U_k,
//
// so a step's recurrent input is one small GEMM: D = V P^T per pathway, K = the rank.
// A CTA computes a tile of 128 neurons (M, TMEM lanes) x 128 trials (N, TMEM columns) per
// pathway with tcgen05.mma: V's 128 rows and P's 128 rows staged in shared memory in the
// 128-byte-swizzled K-major layout, the fp32 P split into three bf16 parts (hi + mid + lo
// carry its 24-bit mantissa, so the products are fp32-accurate) accumulated into one fp32
// TMEM tile, read back with tcgen05.ld.
#include "common.cuh"
#include "tcgen05.cuh"

namespace wt {
namespace {

constexpr int kLrTile = 128;        // neurons (M) and trials (N) of a tile
constexpr int kLrK = 64;            // rank slots: K of the product (a lower rank is zero-padded)
constexpr int kTileBytes = kLrTile * kLrK * 2;  // one bf16 operand tile: 16 KB
constexpr unsigned long long kMmaWaitLimit = 1ull << 20;

__host__ __device__ constexpr uint32_t tmem_cols_for(int KP) { return KP <= 1 ? 128u : KP == 2 ? 256u : 512u; }

// Stage V's rows n0.. (a 128 x 64 bf16 tile) in shared memory.
__device__ void lr_stage_v(uint8_t *sV, const __nv_bfloat16 *V, int n0, int N) {
    for (int u = threadIdx.x; u < kLrTile * 8; u += blockDim.x) {
        const int r = u >> 3, c = u & 7;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (n0 + r < N) val = __ldg(reinterpret_cast<const uint4 *>(V + (size_t)(n0 + r) * kLrK) + c);
        *reinterpret_cast<uint4 *>(sV + sw128(r, c)) = val;
    }
}

// Stage each pathway's P rows b0.. (fp32, (B, KP, 64), read through L2) in shared memory
// as three bf16 tiles: hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid).
__device__ void lr_stage_p(uint8_t *sP, const float *P, int KP, int b0, int B) {
    for (int u = threadIdx.x; u < KP * kLrTile * 8; u += blockDim.x) {
        const int k = u / (kLrTile * 8), r = (u >> 3) & (kLrTile - 1), c = u & 7;
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; i++) f[i] = 0.0f;
        if (b0 + r < B) {
            const float4 *src = reinterpret_cast<const float4 *>(P + ((size_t)(b0 + r) * KP + k) * kLrK + c * 8);
            const float4 a = __ldcg(src), b = __ldcg(src + 1);
            f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
        }
        uint32_t part[3][4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            __nv_bfloat16 h[2], m[2], l[2];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const float x = f[i + e];
                h[e] = __float2bfloat16_rn(x);
                const float r1 = x - __bfloat162float(h[e]);
                m[e] = __float2bfloat16_rn(r1);
                l[e] = __float2bfloat16_rn(r1 - __bfloat162float(m[e]));
            }
            part[0][i / 2] = (uint32_t)__bfloat16_as_ushort(h[0]) | ((uint32_t)__bfloat16_as_ushort(h[1]) << 16);
            part[1][i / 2] = (uint32_t)__bfloat16_as_ushort(m[0]) | ((uint32_t)__bfloat16_as_ushort(m[1]) << 16);
            part[2][i / 2] = (uint32_t)__bfloat16_as_ushort(l[0]) | ((uint32_t)__bfloat16_as_ushort(l[1]) << 16);
        }
#pragma unroll
        for (int p = 0; p < 3; p++)
            *reinterpret_cast<uint4 *>(sP + (size_t)(k * 3 + p) * kTileBytes + sw128(r, c)) =
                make_uint4(part[p][0], part[p][1], part[p][2], part[p][3]);
    }
}

// One thread: D_k (TMEM columns k * 128..) = V_tile * (P_k,hi + P_k,mid + P_k,lo)^T.
__device__ void lr_issue(const uint8_t *sV, const uint8_t *sP, int KP, uint32_t tmem, uint64_t *mbar) {
    constexpr uint32_t idesc = umma_idesc_bf16_f32(kLrTile, kLrTile);
    const uint32_t va = smem_u32(sV);
    for (int k = 0; k < KP; k++)
        for (int p = 0; p < 3; p++) {
            const uint32_t pa = smem_u32(sP + (size_t)(k * 3 + p) * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < kLrK / 16; kk++)
                umma_bf16(tmem + k * kLrTile, umma_desc_sw128(va + kk * 32), umma_desc_sw128(pa + kk * 32), idesc,
                          (p | kk) != 0);
        }
    umma_commit(mbar);
}

__global__ void __launch_bounds__(256) lowrank_product_kernel(const WtLowRankProduct a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_base;
    uint8_t *base = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sV = base, *sP = base + kTileBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kLrTile, b0 = blockIdx.y * kLrTile;
    const uint32_t ncols = tmem_cols_for(a.KP);
    if (warp == 0) {
        tmem_alloc(&tmem_base, ncols);
        tmem_relinquish();
    }
    if (threadIdx.x == 32) mbar_init(&mbar, 1);
    lr_stage_v(sV, reinterpret_cast<const __nv_bfloat16 *>(a.V), n0, a.N);
    lr_stage_p(sP, a.P, a.KP, b0, a.B);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    if (threadIdx.x == 0) lr_issue(sV, sP, a.KP, tmem, &mbar);
    const bool ok = mbar_wait(&mbar, 0, kMmaWaitLimit);
    tc_fence_after();
    if (!ok) {
        if (threadIdx.x == 0) set_error(a.err, WT_ERR_BARRIER);
    } else {
        // warp w reads lanes 32 (w % 4).. (its neurons) and column half w / 4 (its trials)
        const int q = warp & 3, half = warp >> 2;
        const int n = n0 + q * 32 + lane;
        for (int k = 0; k < a.KP; k++)
            for (int ch = 0; ch < 2; ch++) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + k * kLrTile + half * 64 + ch * 32, v);
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int b = b0 + half * 64 + ch * 32 + i;
                    if (b < a.B && n < a.N) a.D[((size_t)k * a.B + b) * a.N + n] = v[i];
                }
            }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, ncols);
}

// ---------------------------------------------------------------------------------------
// The fused simulation of a factorised network (wt_lowrank_forward): one persistent
// cooperative kernel for all T steps, one CTA of 16 warps per SM, a bounded grid barrier
// per step. A CTA owns a run of 128-neuron tiles for every 128-trial block. Per step t and
// per (trial block, neuron tile): the block's P_{t-1} (the sources fired at t - 1, summed
// U rows, fp32) is staged as three bf16 tiles, V's tile next to it, and one thread issues
// the tcgen05.mma product into tensor memory; then every warp reads its 32 neurons x 32
// trials of the accumulator (tcgen05.ld) straight into the membrane update of step t —
// g_t = decay g_{t-1} + jump X_{t-1}, spike, exponential-Euler step, reset, refractory
// count (conductance/dynamics.py:116-143, 199-208), the state streamed through HBM — and
// the neurons that fire add their U row into P_t (fp32 reductions). A last pass after the
// T steps completes g_T with the last step's input.
constexpr int kLfWarps = 16;

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

template <int S, int KP>
__global__ void __launch_bounds__(kLfWarps * 32, 1) lowrank_forward_kernel(const WtLowRankNet net, const WtLowRankRun run,
                                                                           int n_tiles, int b_tiles) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_base;
    __shared__ int mma_ok;
    uint8_t *base = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sV = base, *sP = base + kTileBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int B = net.B, N = net.N, T = run.T;
    const bool REF = net.n_ref != nullptr;
    const int it0 = (int)((long long)n_tiles * blockIdx.x / gridDim.x);
    const int it1 = (int)((long long)n_tiles * (blockIdx.x + 1) / gridDim.x);
    constexpr uint32_t ncols = tmem_cols_for(KP);
    const long long nthreads = (long long)gridDim.x * blockDim.x;
    const long long gtid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t PB = (size_t)B * KP * kLrK;  // one P buffer
    const size_t TN = (size_t)run.T_total * N;
    const float dt = net.dt;
    GridBarrier bar(run.barrier, gridDim.x);

    if (warp == 0) {
        tmem_alloc(&tmem_base, ncols);
        tmem_relinquish();
    }
    if (threadIdx.x == 32) mbar_init(&mbar, 1);
    for (long long i = gtid; i < 3LL * (long long)PB; i += nthreads) run.P[i] = 0.0f;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    uint32_t phase = 0;
    bool alive = bar.sync(run.err);

    const int q = warp & 3, cb = warp >> 2;  // lane quarter (neurons), 32-trial column block
    for (int t = 0; t <= T && alive; t++) {
        const bool finish = t == T;  // the pass completing g_T
        const int t_abs = run.t0 + t;
        const bool has_x = t > 0;
        const float *Pprev = run.P + (size_t)((t + 2) % 3) * PB;
        float *Pcur = run.P + (size_t)(t % 3) * PB;
        if (!finish) {
            float *Pnext = run.P + (size_t)((t + 1) % 3) * PB;
            for (long long i = gtid; i < (long long)PB; i += nthreads) Pnext[i] = 0.0f;
        }
        for (int bt = 0; bt < b_tiles; bt++) {
            const int b0 = bt * kLrTile;
            for (int it = it0; it < it1; it++) {
                const int n0 = it * kLrTile;
                if (has_x) {
                    if (it == it0) lr_stage_p(sP, Pprev, KP, b0, B);
                    lr_stage_v(sV, reinterpret_cast<const __nv_bfloat16 *>(net.V), n0, N);
                    fence_proxy_async_smem();
                }
                tc_fence_before();
                __syncthreads();
                tc_fence_after();
                if (has_x) {
                    if (threadIdx.x == 0) lr_issue(sV, sP, KP, tmem, &mbar);
                    const bool ok = mbar_wait(&mbar, phase, kMmaWaitLimit);
                    phase ^= 1u;
                    if (threadIdx.x == 0) mma_ok = 1;
                    __syncthreads();
                    if (!ok) mma_ok = 0;
                    __syncthreads();
                    tc_fence_after();
                    if (!mma_ok) {
                        if (threadIdx.x == 0) set_error(run.err, WT_ERR_BARRIER);
                        continue;
                    }
                }
                // ---- epilogue: neuron n of this lane, trials b0 + 32 cb + j ----
                const int n = n0 + q * 32 + lane;
                const bool nvalid = n < N;
                float theta = 0.0f, U_reset = 0.0f, E_L = 0.0f, Cm = 1.0f, rate = 0.0f, g_L = 0.0f, w_in = 0.0f;
                float sc[KP + 1];
                int n_ref = 0, path = -1;
#pragma unroll
                for (int k = 0; k <= KP; k++) sc[k] = 0.0f;
                if (nvalid) {
                    theta = net.theta[n];
                    U_reset = net.U_reset[n];
                    E_L = net.E_L[n];
                    Cm = net.C_m[n];
                    rate = -log1pf(net.beta[n] - 1.0f) / dt;
                    g_L = Cm * rate;
                    w_in = net.w_in[n];
                    if (REF) n_ref = net.n_ref[n];
                    path = net.path_of[n];
#pragma unroll
                    for (int k = 0; k <= KP; k++) sc[k] = net.scale[(size_t)k * N + n];
                }
                for (int j0 = 0; j0 < 32; j0 += 8) {
                    float A[KP][8];
                    if (has_x) {
#pragma unroll
                        for (int k = 0; k < KP; k++)
                            tmem_ld8(tmem + ((uint32_t)(q * 32) << 16) + k * kLrTile + cb * 32 + j0, A[k]);
                    }
#pragma unroll
                    for (int jb = 0; jb < 8; jb += 4) {
                    // 4 items' state and input, loaded together (their loads overlap)
                    float v8[4], x8[4], gr8[4][S], gd8[4][S];
                    int cnt8[4];
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) {
                        const int j = jb + jj;
                        const int b = b0 + cb * 32 + j0 + j;
                        const bool valid = nvalid && b < B;
                        const size_t o = (size_t)b * N + n;
                        const float *g_b = run.g + (size_t)b * 2 * S * N + n;
                        v8[jj] = 0.0f;
                        x8[jj] = 0.0f;
                        cnt8[jj] = 0;
#pragma unroll
                        for (int c = 0; c < S; c++) gr8[jj][c] = gd8[jj][c] = 0.0f;
                        if (valid) {
#pragma unroll
                            for (int c = 0; c < S; c++) {
                                gd8[jj][c] = g_b[(size_t)(S + c) * N];
                                if (net.decay_r[c] != 0.0f || t == 0) gr8[jj][c] = g_b[(size_t)c * N];
                            }
                            if (has_x) x8[jj] = run.x[(size_t)b * TN + (size_t)(t_abs - 1) * N + n];
                            if (!finish) {
                                v8[jj] = run.v[o];
                                if (REF) cnt8[jj] = run.counter[o];
                            }
                        }
                    }
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) {
                        const int j = jb + jj;
                        const int b = b0 + cb * 32 + j0 + j;
                        const bool valid = nvalid && b < B;
                        float s = 0.0f;
                        if (valid) {
                            const size_t o = (size_t)b * N + n;
                            float *g_b = run.g + (size_t)b * 2 * S * N + n;
                            float gr[S], gd[S];
#pragma unroll
                            for (int c = 0; c < S; c++) {
                                gd[c] = gd8[jj][c];
                                gr[c] = gr8[jj][c];
                            }
                            if (has_x) {
                                const float xin = w_in * sc[KP] * x8[jj];
#pragma unroll
                                for (int c = 0; c < S; c++) {
                                    float X = 0.0f;
#pragma unroll
                                    for (int k = 0; k < KP; k++)
                                        if ((net.made >> (8 * k + c)) & 1u) X = X + sc[k] * A[k][j];
                                    if ((net.made >> (8 * KP + c)) & 1u) X = X + xin;
                                    gr[c] = gr[c] * net.decay_r[c] + net.jump_r[c] * X;
                                    gd[c] = gd[c] * net.decay_d[c] + net.jump_d[c] * X;
                                }
                            }
                            if (finish) {
#pragma unroll
                                for (int c = 0; c < S; c++) {
                                    g_b[(size_t)c * N] = gr[c];
                                    g_b[(size_t)(S + c) * N] = gd[c];
                                }
                            } else {
                                const float v = v8[jj];
                                int cnt = cnt8[jj];
                                const float held = (REF && cnt > 0) ? 1.0f : 0.0f;
                                s = (v - theta) > 0.0f ? 1.0f : 0.0f;
                                if (REF) s = s * (1.0f - held);
                                float G = 0.0f, Isum = 0.0f, Gt[S];
#pragma unroll
                                for (int c = 0; c < S; c++) {
                                    float gs = gr[c] + gd[c];
                                    gs = fminf(fmaxf(gs, 0.0f), net.g_clip[c]);
                                    Gt[c] = gs;
                                }
#pragma unroll
                                for (int c = 0; c < S; c++) G = G + Gt[c];
#pragma unroll
                                for (int c = 0; c < S; c++) Isum = Isum + Gt[c] * (v - net.E_syn[c]);
                                const float I_leak = g_L * (v - E_L);
                                const float J = Isum + I_leak;
                                const float xx = dt * rate + dt * G / Cm;
                                const float step = -expm1f(-xx) / (g_L + G);
                                const float rr = fmaxf(s, held);
                                run.v[o] = (v - step * J) * (1.0f - rr) + U_reset * rr;
                                if (REF) {
                                    const int c1 = cnt - 1;
                                    cnt = s > 0.0f ? n_ref : (c1 > 0 ? c1 : 0);
                                    run.counter[o] = cnt;
                                }
#pragma unroll
                                for (int c = 0; c < S; c++) {
                                    g_b[(size_t)(S + c) * N] = gd[c];
                                    if (net.decay_r[c] != 0.0f) g_b[(size_t)c * N] = gr[c];
                                }
                                run.spikes[(size_t)b * TN + (size_t)t_abs * N + n] = s;
                            }
                        }
                        // the fired sources' U rows into P_t: the whole warp adds each row
                        unsigned m = __ballot_sync(kFull, s > 0.0f && path >= 0);
                        while (m) {
                            const int l = __ffs(m) - 1;
                            m &= m - 1;
                            const int kl = __shfl_sync(kFull, path, l);
                            const int nl = n0 + q * 32 + l;
                            const __nv_bfloat162 u2 =
                                reinterpret_cast<const __nv_bfloat162 *>(net.U + (size_t)nl * kLrK)[lane];
                            const float2 f2 = __bfloat1622float2(u2);
                            atomicAdd(reinterpret_cast<float2 *>(Pcur + ((size_t)b * KP + kl) * kLrK) + lane, f2);
                        }
                    }
                    }
                }
            }
        }
        if (!finish) alive = bar.sync(run.err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, ncols);
}

}  // namespace

size_t lowrank_product_smem(int KP) { return (size_t)(1 + 3 * KP) * kTileBytes + 1024; }

cudaError_t launch_lowrank_product(const WtLowRankProduct &a, cudaStream_t st) {
    const size_t smem = lowrank_product_smem(a.KP);
    cudaError_t e = cudaFuncSetAttribute(lowrank_product_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const dim3 grid((a.N + kLrTile - 1) / kLrTile, (a.B + kLrTile - 1) / kLrTile);
    lowrank_product_kernel<<<grid, 256, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace wt

namespace wt {

size_t lowrank_forward_smem(int KP) { return (size_t)(1 + 3 * KP) * 16384 + 1024; }

template <int S, int KP>
static cudaError_t launch_lf(const WtLowRankNet &net, const WtLowRankRun &run, cudaStream_t st) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int n_tiles = (net.N + 127) / 128, b_tiles = (net.B + 127) / 128;
    const size_t smem = lowrank_forward_smem(KP);
    cudaError_t e = cudaFuncSetAttribute(lowrank_forward_kernel<S, KP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lowrank_forward_kernel<S, KP>, kLfWarps * 32, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    int grid = sms < n_tiles ? sms : n_tiles;
    WtLowRankNet n = net;
    WtLowRankRun r = run;
    void *args[] = {&n, &r, (void *)&n_tiles, (void *)&b_tiles};
    int nt = n_tiles, bt = b_tiles;
    args[2] = &nt;
    args[3] = &bt;
    return cudaLaunchCooperativeKernel((const void *)lowrank_forward_kernel<S, KP>, dim3(grid), dim3(kLfWarps * 32),
                                       args, smem, st);
}

cudaError_t launch_lowrank_forward(const WtLowRankNet &net, const WtLowRankRun &run, cudaStream_t st) {
    const int key = net.S * 8 + net.KP;
    switch (key) {
        case 1 * 8 + 1: return launch_lf<1, 1>(net, run, st);
        case 1 * 8 + 2: return launch_lf<1, 2>(net, run, st);
        case 2 * 8 + 1: return launch_lf<2, 1>(net, run, st);
        case 2 * 8 + 2: return launch_lf<2, 2>(net, run, st);
        case 3 * 8 + 1: return launch_lf<3, 1>(net, run, st);
        case 3 * 8 + 2: return launch_lf<3, 2>(net, run, st);
        case 4 * 8 + 1: return launch_lf<4, 1>(net, run, st);
        case 4 * 8 + 2: return launch_lf<4, 2>(net, run, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace wt
