// The double-exponential filter of the spike-train losses (wiretorch's
// training_utils/filtering.py:28-135, the van Rossum losses of training_utils/losses.py):
//
//   rise_t   = a_r rise_{t-1}   + x_t          (the carried state enters undecayed at t = 0)
//   smooth_t = a_d smooth_{t-1} + rise_t
//
// and its adjoint, the reverse recursion g_s,t = dL/dsmooth_t + a_d g_s,t+1,
// g_x,t = g_s,t + a_r g_x,t+1. The state (rise, smooth) evolves linearly,
// state_t = M state_{t-1} + (x_t, x_t) with M = [[a_r, 0], [a_r, a_d]], so a chunk of L
// steps is the affine map (M^L, v). Two kernels:
//
// * many columns (trial, neuron): one thread per column scans its T steps in order,
//   coalesced over neurons — every element read and written once;
// * few columns: the T steps of a column are cut into 32 chunks, one per lane of a warp;
//   each lane summarises its chunk as (M^L, v), a warp-shuffle inclusive scan composes
//   the summaries into each chunk's entering state, and each lane rescans its chunk from
//   there — a parallel scan over T, for when the columns alone cannot fill the GPU.
#include "common.cuh"

namespace wt {
namespace {

constexpr int kVrAhead = 8;  // steps of a column the sequential scans load at once

__global__ void filter_seq(const WtFilterArgs f) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)f.B * f.N) return;
    const int b = (int)(i / f.N), n = (int)(i % f.N);
    float r = f.carry_rise ? f.carry_rise[i] : 0.0f;
    float s = f.carry_smooth ? f.carry_smooth[i] : 0.0f;
    const float *__restrict__ x = f.x + b * f.x_bstride + n;
    float *__restrict__ rise = f.rise, *__restrict__ smooth = f.smooth;
    auto step = [&](int t, float xt) {
        r = (t == 0 ? r : f.a_rise * r) + xt;
        s = (t == 0 ? s : f.a_decay * s) + r;
        const size_t o = ((size_t)b * f.T + t) * f.N + n;
        if (rise) rise[o] = r;
        if (smooth) smooth[o] = s;
    };
    int t = 0;
    for (; t + kVrAhead <= f.T; t += kVrAhead) {  // kVrAhead steps' loads issued together
        float xs[kVrAhead];
#pragma unroll
        for (int k = 0; k < kVrAhead; k++) xs[k] = x[(t + k) * f.x_tstride];
#pragma unroll
        for (int k = 0; k < kVrAhead; k++) step(t + k, xs[k]);
    }
    for (; t < f.T; t++) step(t, x[t * f.x_tstride]);
    if (f.last_rise) f.last_rise[i] = r;
    if (f.last_smooth) f.last_smooth[i] = s;
}

// Lower-triangular 2x2 [[m00, 0], [m10, m11]] and a vector: an affine map of the state.
struct Aff {
    float m00, m10, m11, v0, v1;
};

// hi after lo
__device__ __forceinline__ Aff compose(const Aff &hi, const Aff &lo) {
    Aff o;
    o.m00 = hi.m00 * lo.m00;
    o.m10 = hi.m10 * lo.m00 + hi.m11 * lo.m10;
    o.m11 = hi.m11 * lo.m11;
    o.v0 = hi.m00 * lo.v0 + hi.v0;
    o.v1 = hi.m10 * lo.v0 + hi.m11 * lo.v1 + hi.v1;
    return o;
}

// One warp per column; lane p scans steps [p L, (p + 1) L).
__global__ void filter_chunked(const WtFilterArgs f) {
    const int lane = threadIdx.x & 31;
    const long long col = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (col >= (long long)f.B * f.N) return;  // whole warps leave together
    const int b = (int)(col / f.N), n = (int)(col % f.N);
    const int L = (f.T + 31) / 32;
    const int t0 = lane * L, t1 = min(f.T, t0 + L);
    const float *x = f.x + b * f.x_bstride + n;
    // Summary of the chunk: its map from the entering state, from zero (and, for the
    // first chunk, from the carried state, which enters undecayed).
    Aff a{1.0f, 0.0f, 1.0f, 0.0f, 0.0f};
    for (int t = t0; t < t1; t++) {
        const float xt = x[t * f.x_tstride];
        Aff step;
        if (t == 0) step = Aff{1.0f, 1.0f, 1.0f, xt, xt};
        else step = Aff{f.a_rise, f.a_rise, f.a_decay, xt, xt};
        a = compose(step, a);
    }
    // Inclusive scan over the lanes: lane p gets the map from the run's start to the end
    // of its chunk.
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        Aff lo;
        lo.m00 = __shfl_up_sync(kFull, a.m00, o);
        lo.m10 = __shfl_up_sync(kFull, a.m10, o);
        lo.m11 = __shfl_up_sync(kFull, a.m11, o);
        lo.v0 = __shfl_up_sync(kFull, a.v0, o);
        lo.v1 = __shfl_up_sync(kFull, a.v1, o);
        if (lane >= o) a = compose(a, lo);
    }
    // The state entering this chunk: the previous lane's map applied to the carried state.
    const float c0 = f.carry_rise ? f.carry_rise[col] : 0.0f;
    const float c1 = f.carry_smooth ? f.carry_smooth[col] : 0.0f;
    Aff prev;
    prev.m00 = __shfl_up_sync(kFull, a.m00, 1);
    prev.m10 = __shfl_up_sync(kFull, a.m10, 1);
    prev.m11 = __shfl_up_sync(kFull, a.m11, 1);
    prev.v0 = __shfl_up_sync(kFull, a.v0, 1);
    prev.v1 = __shfl_up_sync(kFull, a.v1, 1);
    float r, s;
    if (lane == 0) {
        r = c0;
        s = c1;
    } else {
        r = prev.m00 * c0 + prev.v0;
        s = prev.m10 * c0 + prev.m11 * c1 + prev.v1;
    }
    for (int t = t0; t < t1; t++) {
        const float xt = x[t * f.x_tstride];
        r = (t == 0 ? r : f.a_rise * r) + xt;
        s = (t == 0 ? s : f.a_decay * s) + r;
        const size_t o = ((size_t)b * f.T + t) * f.N + n;
        if (f.rise) f.rise[o] = r;
        if (f.smooth) f.smooth[o] = s;
    }
    if (lane == 31 || t1 == f.T) {
        if (t1 == f.T && t0 < f.T) {
            if (f.last_rise) f.last_rise[col] = r;
            if (f.last_smooth) f.last_smooth[col] = s;
        }
    }
}

__global__ void filter_grad_seq(const WtFilterGradArgs f) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)f.B * f.N) return;
    const int b = (int)(i / f.N), n = (int)(i % f.N);
    const size_t base = (size_t)b * f.T * f.N + n;
    const float *__restrict__ gsm = f.grad_smooth + base;
    float *__restrict__ gx = f.grad_x + base;
    float gs = 0.0f, gr = 0.0f;
    auto step = [&](int t, float g) {
        gs = g * f.grad_scale + f.a_decay * gs;
        gr = gs + f.a_rise * gr;
        gx[(size_t)t * f.N] = gr;
    };
    int t = f.T - 1;
    for (; t + 1 >= kVrAhead; t -= kVrAhead) {  // kVrAhead steps' loads issued together
        float g8[kVrAhead];
#pragma unroll
        for (int k = 0; k < kVrAhead; k++) g8[k] = gsm[(size_t)(t - k) * f.N];
#pragma unroll
        for (int k = 0; k < kVrAhead; k++) step(t - k, g8[k]);
    }
    for (; t >= 0; t--) step(t, gsm[(size_t)t * f.N]);
}

// The reverse recursion as a chunked parallel scan (state (g_s, g_x), map M^T).
__global__ void filter_grad_chunked(const WtFilterGradArgs f) {
    const int lane = threadIdx.x & 31;
    const long long col = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (col >= (long long)f.B * f.N) return;
    const int b = (int)(col / f.N), n = (int)(col % f.N);
    const int L = (f.T + 31) / 32;
    // lane p takes reverse chunk p: steps counted from the end.
    const int r0 = lane * L, r1 = min(f.T, r0 + L);
    // state (gs, gx): gs' = a_d gs + y, gx' = a_r gx + gs' = a_r gx + a_d gs + y
    Aff a{1.0f, 0.0f, 1.0f, 0.0f, 0.0f};  // component 0: gs, component 1: gx
    for (int q = r0; q < r1; q++) {
        const int t = f.T - 1 - q;
        const float y = f.grad_smooth[((size_t)b * f.T + t) * f.N + n] * f.grad_scale;
        const Aff step{f.a_decay, f.a_decay, f.a_rise, y, y};
        a = compose(step, a);
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        Aff lo;
        lo.m00 = __shfl_up_sync(kFull, a.m00, o);
        lo.m10 = __shfl_up_sync(kFull, a.m10, o);
        lo.m11 = __shfl_up_sync(kFull, a.m11, o);
        lo.v0 = __shfl_up_sync(kFull, a.v0, o);
        lo.v1 = __shfl_up_sync(kFull, a.v1, o);
        if (lane >= o) a = compose(a, lo);
    }
    float gs = __shfl_up_sync(kFull, a.v0, 1), gx = __shfl_up_sync(kFull, a.v1, 1);
    if (lane == 0) gs = gx = 0.0f;
    for (int q = r0; q < r1; q++) {
        const int t = f.T - 1 - q;
        const size_t o = ((size_t)b * f.T + t) * f.N + n;
        gs = f.grad_smooth[o] * f.grad_scale + f.a_decay * gs;
        gx = gs + f.a_rise * gx;
        f.grad_x[o] = gx;
    }
}

// The van Rossum rate loss (training_utils/losses.py:140-194) in one pass per column:
// both filters, the difference saved, its square summed in double (per thread, then
// over the block: one partial per block, summed by the caller in a fixed order).
__global__ void __launch_bounds__(256) van_rossum_fwd(const WtVanRossumArgs a) {
    __shared__ double part[8];
    const long long cols = (long long)a.B * a.N;
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    double sq = 0.0;
    if (i < cols) {
        const int b = (int)(i / a.N), n = (int)(i % a.N);
        float ro = 0.0f, so = 0.0f, rt = 0.0f, st = 0.0f;
        if (a.carry) {
            ro = a.carry[i];
            so = a.carry[cols + i];
            rt = a.carry[2 * cols + i];
            st = a.carry[3 * cols + i];
        }
        const float *__restrict__ x = a.x + b * a.x_bstride + n;
        const float *__restrict__ y = a.y + b * a.y_bstride + n;
        float *__restrict__ e = a.err + (size_t)b * a.T * a.N + n;
        // one step (the carried state enters undecayed at t = 0: filtering.py:112-117)
        auto step = [&](int t, float xt, float yt) {
            ro = (t == 0 ? ro : a.a_rise * ro) + xt;
            so = (t == 0 ? so : a.a_decay * so) + ro;
            rt = (t == 0 ? rt : a.a_rise * rt) + yt;
            st = (t == 0 ? st : a.a_decay * st) + rt;
            const float d = so - st;
            e[(size_t)t * a.N] = d;
            sq += (double)d * (double)d;
        };
        int t = 0;
        for (; t + kVrAhead <= a.T; t += kVrAhead) {  // kVrAhead steps' loads issued together
            float xs[kVrAhead], ys[kVrAhead];
#pragma unroll
            for (int k = 0; k < kVrAhead; k++) {
                xs[k] = x[(t + k) * a.x_tstride];
                ys[k] = y[(t + k) * a.y_tstride];
            }
#pragma unroll
            for (int k = 0; k < kVrAhead; k++) step(t + k, xs[k], ys[k]);
        }
        for (; t < a.T; t++) step(t, x[t * a.x_tstride], y[t * a.y_tstride]);
        if (a.T > 0) {
            a.last[i] = ro;
            a.last[cols + i] = so;
            a.last[2 * cols + i] = rt;
            a.last[3 * cols + i] = st;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_down_sync(kFull, sq, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int w = 0; w < 8; w++) tot += part[w];
        a.partial[blockIdx.x] = tot;
    }
}

__global__ void van_rossum_bwd(const WtVanRossumGradArgs a) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)a.B * a.N) return;
    const int b = (int)(i / a.N), n = (int)(i % a.N);
    const float c = a.scale * *a.grad_loss;
    const size_t base = (size_t)b * a.T * a.N + n;
    const float *__restrict__ err = a.err + base;
    float *__restrict__ grad_x = a.grad_x + base;
    float gs = 0.0f, gx = 0.0f;
    auto step = [&](int t, float et) {
        gs = et * c + a.a_decay * gs;
        gx = gs + a.a_rise * gx;
        grad_x[(size_t)t * a.N] = gx;
    };
    int t = a.T - 1;
    for (; t + 1 >= kVrAhead; t -= kVrAhead) {  // kVrAhead steps' loads issued together
        float es[kVrAhead];
#pragma unroll
        for (int k = 0; k < kVrAhead; k++) es[k] = err[(size_t)(t - k) * a.N];
#pragma unroll
        for (int k = 0; k < kVrAhead; k++) step(t - k, es[k]);
    }
    for (; t >= 0; t--) step(t, err[(size_t)t * a.N]);
}

// Columns below which the parallel-over-T kernels run (148 SMs x 2048 threads would
// want ~300k sequential columns to fill the GPU).
constexpr long long kParallelBelow = 1 << 16;

}  // namespace

cudaError_t launch_van_rossum(const WtVanRossumArgs &a, cudaStream_t st) {
    const long long cols = (long long)a.B * a.N;
    if (cols == 0) return cudaSuccess;
    van_rossum_fwd<<<(unsigned)((cols + 255) / 256), 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_van_rossum_grad(const WtVanRossumGradArgs &a, cudaStream_t st) {
    const long long cols = (long long)a.B * a.N;
    if (cols == 0 || a.T == 0) return cudaSuccess;
    van_rossum_bwd<<<(unsigned)((cols + 255) / 256), 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_filter(const WtFilterArgs &f, cudaStream_t st) {
    const long long cols = (long long)f.B * f.N;
    if (cols == 0 || f.T == 0) return cudaSuccess;
    if (cols < kParallelBelow && f.T >= 64) {
        const long long threads = cols * 32;
        filter_chunked<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(f);
    } else {
        filter_seq<<<(unsigned)((cols + 255) / 256), 256, 0, st>>>(f);
    }
    return cudaGetLastError();
}

cudaError_t launch_filter_grad(const WtFilterGradArgs &f, cudaStream_t st) {
    const long long cols = (long long)f.B * f.N;
    if (cols == 0 || f.T == 0) return cudaSuccess;
    if (cols < kParallelBelow && f.T >= 64) {
        const long long threads = cols * 32;
        filter_grad_chunked<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(f);
    } else {
        filter_grad_seq<<<(unsigned)((cols + 255) / 256), 256, 0, st>>>(f);
    }
    return cudaGetLastError();
}

}  // namespace wt
