// Device helpers shared by the engine's kernels: the bounded grid barrier of the
// persistent kernels, the device error word, and small math helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "wiretorch_b200.h"

namespace wt {

constexpr int kBlock = 256;          // threads per block of the persistent kernels
constexpr unsigned kFull = 0xffffffffu;
// A grid barrier waits at most this many polls (each with a short sleep, well under a
// second in all) before it records WT_ERR_BARRIER and lets the kernel return.
constexpr unsigned long long kSpinLimit = 1ull << 22;

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void set_error(int32_t *err, int code) { atomicCAS(err, 0, code); }

__device__ __forceinline__ int read_error(const int32_t *err) {
    return *reinterpret_cast<const volatile int32_t *>(err);
}

// A sense-counting barrier over all blocks of a cooperative launch. `words` points to
// two counters on separate 128-byte lines: arrivals, and the generation. Returns false
// (all threads of the block) once any block has recorded an error, so that every block
// leaves its loop at the same barrier.
struct GridBarrier {
    unsigned *count;
    unsigned *gen;
    unsigned nblocks;
    unsigned local;

    __device__ GridBarrier(uint32_t *words, unsigned n)
        : count(words), gen(words + 32), nblocks(n), local(0) {}

    __device__ bool sync(int32_t *err) {
        __shared__ int ok;
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned g = local;
            __threadfence();
            const unsigned arrived = atomicAdd(count, 1u);
            if (arrived == nblocks - 1) {
                atomicExch(count, 0u);
                __threadfence();
                atomicExch(gen, g + 1);
            } else {
                unsigned long long spins = 0;
                while (ld_acquire(gen) == g) {
                    if (++spins > kSpinLimit) {
                        set_error(err, WT_ERR_BARRIER);
                        break;
                    }
                    __nanosleep(64);
                }
            }
            __threadfence();
            local = g + 1;
            ok = read_error(err) == 0;  // one reading for the whole block
        }
        __syncthreads();
        return ok;
    }
};

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// Warp-wide inclusive prefix sum.
__device__ __forceinline__ int warp_inclusive_sum(int v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += y;
    }
    return v;
}

}  // namespace wt
