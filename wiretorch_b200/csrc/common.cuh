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

    // The barrier of a neuron-partitioned run's step, fused with its exchange of progress:
    // the last block to arrive writes `mine` into every rank's progress slot of this rank
    // (`peer_progress[r] + rank`), waits (bounded) until every rank's slot here (`slots[r]`) holds at
    // least `mine`, and only then releases the blocks. One grid barrier instead of a barrier,
    // a progress exchange by one block and a second barrier. With `reserve` (a run that
    // pushes its events: this rank's event counts per step parity and destination rank,
    // [2][8]), the last block first writes parity `par`'s counts into every rank's inbound
    // counts (`push_count[r][par * 8 + rank]`) and clears them for the step after next.
    //
    // Ordering: the blocks' stores to the ranks (spike words, events) are ordered before
    // their arrival by the block barrier and a fence at GPU scope; the last block's one
    // fence at system scope then orders all of them (causality order is transitive across
    // the GPU-scope synchronisation with the other blocks) and its own counts before the
    // relaxed system-scope progress stores: one system fence per step on the path (each
    // costs microseconds), not one per thread, per block or per rank.
    __device__ bool sync_progress(int32_t *err, unsigned long long *const *peer_progress, int rank,
                                  const unsigned long long *slots, int n_ranks, unsigned long long mine,
                                  uint32_t *reserve = nullptr, uint32_t *const *push_count = nullptr, int par = 0) {
        __shared__ int ok;
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned g = local;
            __threadfence();  // this block's stores (here and to the ranks), before its arrival
            const unsigned arrived = atomicAdd(count, 1u);
            if (arrived == nblocks - 1) {
                atomicExch(count, 0u);
                __threadfence();
                if (reserve) {
                    for (int r = 0; r < n_ranks; r++) {
                        const unsigned v = atomicExch(reserve + par * 8 + r, 0u);
                        push_count[r][par * 8 + rank] = v;
                    }
                }
                __threadfence_system();  // every block's stores to the ranks and the counts, first
                for (int r = 0; r < n_ranks; r++)
                    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(peer_progress[r] + rank), "l"(mine)
                                 : "memory");
                for (int r = 0; r < n_ranks; r++) {
                    unsigned long long spins = 0, seen = 0;
                    for (;;) {
                        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(seen) : "l"(slots + r) : "memory");
                        if (seen >= mine) break;
                        if (++spins > kSpinLimit) {
                            set_error(err, WT_ERR_BARRIER);
                            break;
                        }
                        __nanosleep(64);
                    }
                }
                __threadfence();
                atomicExch(gen, g + 1);
            } else {
                unsigned long long spins = 0;
                while (ld_acquire(gen) == g) {
                    if (++spins > 4 * kSpinLimit) {  // the last block may wait its own limit for the ranks
                        set_error(err, WT_ERR_BARRIER);
                        break;
                    }
                    __nanosleep(64);
                }
            }
            __threadfence();
            local = g + 1;
            ok = read_error(err) == 0;
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
