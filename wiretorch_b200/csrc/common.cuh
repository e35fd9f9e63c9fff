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

// A counting barrier over all blocks of a cooperative launch. `words` points to two
// counters on separate 128-byte lines, zero at the launch: the arrivals, counted up over
// the whole launch (the last arrival of generation g is number (g + 1) * nblocks - 1, so
// nothing resets them), and the generation released, its top bit set when an error had
// been recorded. Each block reads the error word as it arrives, beside its arrival, and
// the last block puts what it read into the release, so that every block leaves its loop
// at the same barrier; an error recorded by a block that arrived at the same time as the
// last one ends the run at the next barrier. Returns false (all threads of the block) once
// the run is to end. A launch holds at most 2^32 / nblocks barriers (the host bounds T).
struct GridBarrier {
    static constexpr unsigned kBad = 0x80000000u;
    unsigned *count;
    unsigned *gen;
    unsigned nblocks;
    unsigned local;

    __device__ GridBarrier(uint32_t *words, unsigned n)
        : count(words), gen(words + 32), nblocks(n), local(0) {}

    // Releases generation g + 1 (the last block).
    __device__ void release(unsigned g, bool good) {
        const unsigned v = (g + 1) | (good ? 0u : kBad);
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(gen), "r"(v) : "memory");
    }

    // Waits, bounded, for generation g + 1; false when it came with an error or never came.
    __device__ bool wait(int32_t *err, unsigned g, unsigned long long limit) {
        unsigned long long spins = 0;
        unsigned v;
        while (((v = ld_acquire(gen)) & ~kBad) == g) {
            if (++spins > limit) {
                set_error(err, WT_ERR_BARRIER);
                return false;
            }
            __nanosleep(64);
        }
        return !(v & kBad);
    }

    __device__ bool sync(int32_t *err) {
        __shared__ int ok;
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned g = local;
            __threadfence();  // this block's stores, before its arrival
            const int seen = read_error(err);
            const unsigned arrived = atomicAdd(count, 1u);
            bool good;
            if (arrived == (g + 1) * nblocks - 1) {
                good = seen == 0;
                release(g, good);  // a release at GPU scope: every block's stores, first
            } else {
                good = wait(err, g, kSpinLimit);
            }
            local = g + 1;
            ok = good;
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
    // Warp 0 of the last block does the work of rank r on lane r.
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
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            const unsigned g = __shfl_sync(kFull, local, 0);
            unsigned arrived = 0;
            int seen = 0;
            if (lane == 0) {
                __threadfence();  // this block's stores (here and to the ranks), before its arrival
                seen = read_error(err);
                arrived = atomicAdd(count, 1u);
            }
            arrived = __shfl_sync(kFull, arrived, 0);
            bool good;
            if (arrived == (g + 1) * nblocks - 1) {
                __threadfence();
                const bool mine_lane = lane < n_ranks;
                if (reserve && mine_lane) {
                    const unsigned v = atomicExch(reserve + par * 8 + lane, 0u);
                    push_count[lane][par * 8 + rank] = v;
                }
                __threadfence_system();  // every block's stores to the ranks and the counts, first
                if (mine_lane)
                    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(peer_progress[lane] + rank), "l"(mine)
                                 : "memory");
                bool done = !mine_lane, gave_up = false;
                unsigned long long spins = 0;
                while (!__all_sync(kFull, done)) {
                    if (!done) {
                        unsigned long long v;
                        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(slots + lane) : "memory");
                        if (v >= mine) {
                            done = true;
                        } else if (++spins > kSpinLimit) {
                            gave_up = done = true;
                        } else {
                            __nanosleep(64);
                        }
                    }
                }
                gave_up = __any_sync(kFull, gave_up);
                __syncwarp();  // every lane's acquisition, before lane 0's release
                good = __shfl_sync(kFull, seen, 0) == 0 && !gave_up;
                if (lane == 0) {
                    if (gave_up) set_error(err, WT_ERR_BARRIER);
                    release(g, good);
                }
            } else {
                good = false;
                if (lane == 0) good = wait(err, g, 4 * kSpinLimit);  // the last block may wait its own limit
                good = __shfl_sync(kFull, good, 0);
            }
            local = g + 1;
            if (lane == 0) ok = good;
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
