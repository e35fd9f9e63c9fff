// The factorised (low-rank) recurrent drive on the tensor cores. A pathway k whose weights
// are W_k = U_k V^T (rank r <= 64; the BASELINE's factorised configuration, a linear
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

// Stage V's rows n0.. and each pathway's P rows b0.. (three bf16 parts) in shared memory.
__device__ void lr_stage(uint8_t *sV, uint8_t *sP, const __nv_bfloat16 *V, const float *P, int KP, int n0, int b0,
                         int B, int N) {
    for (int u = threadIdx.x; u < kLrTile * 8; u += blockDim.x) {
        const int r = u >> 3, c = u & 7;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (n0 + r < N) val = __ldg(reinterpret_cast<const uint4 *>(V + (size_t)(n0 + r) * kLrK) + c);
        *reinterpret_cast<uint4 *>(sV + sw128(r, c)) = val;
    }
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
    lr_stage(sV, sP, reinterpret_cast<const __nv_bfloat16 *>(a.V), a.P, a.KP, n0, b0, a.B, a.N);
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
