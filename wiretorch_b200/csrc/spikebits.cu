// Spikes as bits on the device: rows of n spikes, each row packed into ceil(n / 8) bytes,
// spike i of a row in bit i % 8 (least significant first) of byte i / 8. The runners'
// data path moves spikes between host and device in this form (an eighth of a bool
// tensor's bytes, a thirty-second of a float's) and these kernels convert on the device:
// one thread per packed byte (per half byte when unpacking to float), its spikes read or
// written with vector accesses when the rows keep them aligned. Both are bound by the HBM
// bytes of the unpacked side.
#include "common.cuh"

namespace wt {
namespace {

__device__ __forceinline__ long long grid_index() { return (long long)blockIdx.x * blockDim.x + threadIdx.x; }
__device__ __forceinline__ long long grid_threads() { return (long long)gridDim.x * blockDim.x; }

// bits -> spikes (`T` float or uint8: 0 or 1)
template <typename T>
__global__ void unpack_kernel(const uint8_t *__restrict__ bits, T *__restrict__ out, long long rows, int n,
                              bool vec) {
    const int nb = (n + 7) >> 3;
    const long long total = rows * nb;
    for (long long i = grid_index(); i < total; i += grid_threads()) {
        const long long row = i / nb;
        const int jb = (int)(i - row * nb);
        const unsigned byte = bits[i];
        T *o = out + row * n + (long long)jb * 8;
        const int m = min(8, n - jb * 8);
        if (vec && m == 8) {
            if constexpr (sizeof(T) == 4) {
                float4 a, b;
                a.x = (float)(byte & 1u), a.y = (float)((byte >> 1) & 1u);
                a.z = (float)((byte >> 2) & 1u), a.w = (float)((byte >> 3) & 1u);
                b.x = (float)((byte >> 4) & 1u), b.y = (float)((byte >> 5) & 1u);
                b.z = (float)((byte >> 6) & 1u), b.w = (float)((byte >> 7) & 1u);
                reinterpret_cast<float4 *>(o)[0] = a;
                reinterpret_cast<float4 *>(o)[1] = b;
            } else {
                // spread the eight bits to the low bit of eight bytes
                unsigned long long v = 0;
#pragma unroll
                for (int k = 0; k < 8; k++) v |= (unsigned long long)((byte >> k) & 1u) << (8 * k);
                *reinterpret_cast<unsigned long long *>(o) = v;
            }
        } else {
            for (int k = 0; k < m; k++) o[k] = (T)((byte >> k) & 1u);
        }
    }
}

// bits -> float spikes, a thread per half byte: its four spikes one 16-byte store when the
// rows keep them aligned, so that a warp's stores cover 512 contiguous bytes
__global__ void unpack_f32_kernel(const uint8_t *__restrict__ bits, float *__restrict__ out, long long rows, int n,
                                  bool vec) {
    const int nb = (n + 7) >> 3, nq = (n + 3) >> 2;  // bytes and half bytes of a row
    const long long total = rows * nq;
    for (long long i = grid_index(); i < total; i += grid_threads()) {
        const long long row = i / nq;
        const int jq = (int)(i - row * nq);
        const unsigned q = (bits[row * nb + (jq >> 1)] >> ((jq & 1) * 4)) & 15u;
        float *o = out + row * n + (long long)jq * 4;
        const int m = min(4, n - jq * 4);
        if (vec && m == 4) {
            *reinterpret_cast<float4 *>(o) =
                make_float4((float)(q & 1u), (float)((q >> 1) & 1u), (float)((q >> 2) & 1u), (float)((q >> 3) & 1u));
        } else {
            for (int k = 0; k < m; k++) o[k] = (float)((q >> k) & 1u);
        }
    }
}

// spikes -> bits; a value other than 0 or 1 records WT_ERR_ARGS (its bit is set all the same)
template <typename T>
__global__ void pack_kernel(const T *__restrict__ in, uint8_t *__restrict__ bits, long long rows, int n, bool vec,
                            int32_t *err) {
    const int nb = (n + 7) >> 3;
    const long long total = rows * nb;
    bool bad = false;
    for (long long i = grid_index(); i < total; i += grid_threads()) {
        const long long row = i / nb;
        const int jb = (int)(i - row * nb);
        const T *p = in + row * n + (long long)jb * 8;
        const int m = min(8, n - jb * 8);
        unsigned byte = 0;
        if (vec && m == 8) {
            if constexpr (sizeof(T) == 4) {
                const float4 a = __ldcs(reinterpret_cast<const float4 *>(p));
                const float4 b = __ldcs(reinterpret_cast<const float4 *>(p) + 1);
                const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    byte |= (unsigned)(v[k] != 0.0f) << k;
                    bad |= v[k] != 0.0f && v[k] != 1.0f;
                }
            } else {
                const unsigned long long w = __ldcs(reinterpret_cast<const unsigned long long *>(p));
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const unsigned v = (unsigned)(w >> (8 * k)) & 255u;
                    byte |= (unsigned)(v != 0u) << k;
                    bad |= v > 1u;
                }
            }
        } else {
            for (int k = 0; k < m; k++) {
                const T v = p[k];
                byte |= (unsigned)(v != (T)0) << k;
                bad |= v != (T)0 && v != (T)1;
            }
        }
        bits[i] = (uint8_t)byte;
    }
    if (bad && err) set_error(err, WT_ERR_ARGS);
}

int grid_for(long long total) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long want = (total + 255) / 256, cap = (long long)sms * 8;
    return (int)(want < 1 ? 1 : want > cap ? cap : want);
}

// Whether the spikes sit at aligned vectors: a float row of a multiple of 4 spikes from a
// 16-byte-aligned base (16-byte accesses), a uint8 row of a multiple of 8 from an
// 8-byte-aligned base (one 8-byte access per byte of bits).
bool vector_rows(const WtSpikeBits &a) {
    const uintptr_t base = (uintptr_t)a.spikes;
    return a.kind == WT_SPIKES_F32 ? (a.n % 4 == 0 && base % 16 == 0) : (a.n % 8 == 0 && base % 8 == 0);
}

}  // namespace

cudaError_t launch_unpack_spikes(const WtSpikeBits &a, cudaStream_t st) {
    const long long total = a.rows * (long long)((a.n + 7) / 8);
    if (total == 0) return cudaSuccess;
    const bool vec = vector_rows(a);
    if (a.kind == WT_SPIKES_F32)
        unpack_f32_kernel<<<grid_for(a.rows * (long long)((a.n + 3) / 4)), 256, 0, st>>>(a.bits, (float *)a.spikes,
                                                                                        a.rows, a.n, vec);
    else
        unpack_kernel<uint8_t><<<grid_for(total), 256, 0, st>>>(a.bits, (uint8_t *)a.spikes, a.rows, a.n, vec);
    return cudaGetLastError();
}

cudaError_t launch_pack_spikes(const WtSpikeBits &a, cudaStream_t st) {
    const long long total = a.rows * (long long)((a.n + 7) / 8);
    if (total == 0) return cudaSuccess;
    const int grid = grid_for(total);
    const bool vec = vector_rows(a);
    if (a.kind == WT_SPIKES_F32)
        pack_kernel<float><<<grid, 256, 0, st>>>((const float *)a.spikes, a.bits, a.rows, a.n, vec, a.err);
    else
        pack_kernel<uint8_t><<<grid, 256, 0, st>>>((const uint8_t *)a.spikes, a.bits, a.rows, a.n, vec, a.err);
    return cudaGetLastError();
}

}  // namespace wt
