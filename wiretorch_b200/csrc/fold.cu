// Per-call weight folding: the weight of edge_cw = w * scale[k, col] * jf[k, c] * 2^s_c, next
// to the edge's packed target, for every edge of every chunk (one warp per chunk,
// coalesced over the chunk's edges). Run once per forward
// call, since a learnt kernel scale (the reference's scaling-factor projections,
// network.py:816-854) changes with every optimiser step.
#include "common.cuh"

namespace wt {
namespace {

__global__ void fold_kernel(const int64_t *chunk_desc, const int32_t *chunk_path, const uint32_t *edge_col,
                            const float *w_raw, const float *scale, const float *jf, const float *fx_scale,
                            unsigned long long *out, int n_chunks, int N, int C) {
    const int lane = threadIdx.x & 31;
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long chunk = warp; chunk < n_chunks; chunk += nwarps) {
        const long long d = chunk_desc[chunk];
        const long long e0 = d & ((1LL << 56) - 1);
        const int len = (int)((unsigned long long)d >> 56);
        const int k = chunk_path[chunk];
        for (int q = lane; q < len; q += 32) {
            const uint32_t pc = edge_col[e0 + q];
            const uint32_t col = pc & 0x7ffffffu, c = pc >> 27;
            const float w = w_raw[e0 + q] * scale[(size_t)k * N + col] * jf[(size_t)k * C + c] * fx_scale[c];
            out[e0 + q] = (unsigned long long)pc | ((unsigned long long)__float_as_uint(w) << 32);
        }
    }
}

}  // namespace

cudaError_t launch_fold(const WtNet &net, const float *w_raw, const int32_t *chunk_path, const float *scale,
                        const float *jf, const float *fx_scale, uint64_t *out, cudaStream_t st) {
    if (net.n_chunks == 0) return cudaSuccess;
    int blocks = (int)((net.n_chunks + 7) / 8);  // 8 warps per block
    if (blocks > 148 * 32) blocks = 148 * 32;
    fold_kernel<<<blocks, 256, 0, st>>>(net.chunk_desc, chunk_path, net.edge_col, w_raw, scale, jf, fx_scale,
                                        (unsigned long long *)out, net.n_chunks, net.N, net.C);
    return cudaGetLastError();
}

}  // namespace wt
