// wt_forward_noalloc: the forward run of wt_forward with its workspace in a static
// device array instead of buffers the caller allocates.
//
// Some callers cannot allocate device memory on the path that runs the network: a host
// that drives the library through its C ABI without a device allocator of its own (a
// C, Go or Java service holding only the network's tables), or one that must not call
// cudaMalloc/cudaFree there because those calls synchronise the device and stall the
// work of every other stream. This entry point needs nothing from them beyond the
// network and run buffers: its scratch is a file-scope __device__ array of
// kNoAllocScratchBytes, allocated with the module.
//
// Set-up: the first call on a device (with that device current) looks up the array's
// address with cudaGetSymbolAddress and keeps it; later calls on that device reuse it,
// so the first call should come before any stream capture. The kept address belongs to
// the device's current context: after cudaDeviceReset (or anything else that destroys
// that context) it is stale, and this entry point must not be called again in the
// process. A call that fails its argument checks launches nothing and leaves the
// previous run's device error code in place; wt_noalloc_error waits on the stream it is
// given, which must be the stream of the run whose code is wanted. Runs whose workspace
// (wt_workspace_bytes) does not fit are rejected with WT_ERR_ARGS before any device
// work. Calls share the one array per device: two calls that overlap in time, on any
// streams, race on it and corrupt each other's results, so a caller serialises them.
#include <atomic>
#include <cstdio>

#include "common.cuh"

namespace wt {
int set_last_error(int code, const char *message);
int check_forward(const WtNet *net, const WtForward *run, const WtWorkspace *ws);
}

namespace {

constexpr long long kNoAllocScratchBytes = 32LL << 20;  // 32 MiB per device
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::atomic<void *> g_scratch_of[kMaxDevices];

long long align256(long long x) { return (x + 255) & ~255LL; }

}  // namespace

extern "C" {

int wt_forward_noalloc(const WtNet *net, const WtForward *run, void *stream) {
    if (!run) return wt::set_last_error(WT_ERR_ARGS, "run is null");
    int64_t bytes[6];
    const int rc = wt_workspace_bytes(net, run->T, bytes);
    if (rc) return rc;
    // the error word and the barrier at fixed offsets, then X, events and event counts
    // (no edge counter)
    long long off[5], total = 512;
    off[4] = 0;
    off[3] = 256;
    for (int i = 0; i < 3; i++) {
        off[i] = total;
        total = align256(total + bytes[i]);
    }
    if (total > kNoAllocScratchBytes) {
        char msg[200];
        std::snprintf(msg, sizeof msg,
                      "wt_forward_noalloc: this run needs %lld bytes of scratch, above its static limit of %lld "
                      "(use wt_forward with a caller-allocated workspace)",
                      total, kNoAllocScratchBytes);
        return wt::set_last_error(WT_ERR_ARGS, msg);
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return wt::set_last_error(WT_ERR_LAUNCH, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return wt::set_last_error(WT_ERR_UNSUPPORTED, "device ordinal above 63");
    unsigned char *base = static_cast<unsigned char *>(g_scratch_of[dev].load());
    if (!base) {  // set-up, once per device
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return wt::set_last_error(WT_ERR_LAUNCH, cudaGetErrorString(e));
        g_scratch_of[dev].store(p);
        base = static_cast<unsigned char *>(p);
    }
    WtWorkspace ws{};
    ws.X = reinterpret_cast<unsigned long long *>(base + off[0]);
    ws.ev = reinterpret_cast<WtEvent *>(base + off[1]);
    ws.ev_count = reinterpret_cast<uint32_t *>(base + off[2]);
    ws.barrier = reinterpret_cast<uint32_t *>(base + off[3]);
    ws.err = reinterpret_cast<int32_t *>(base + off[4]);
    ws.ev_cap = (long long)net->B * (net->n_chunks > 0 ? net->n_chunks : 1);
    ws.edges = nullptr;
    // Every check of wt_forward first: a call it rejects leaves the device error code of
    // the previous run in place. Then the error word must start at zero (wt_forward
    // clears the barrier; the kernel clears the accumulators and event counts itself).
    const int checked = wt::check_forward(net, run, &ws);
    if (checked) return checked;
    if (run->T == 0) return WT_OK;
    e = cudaMemsetAsync(ws.err, 0, sizeof(int32_t), (cudaStream_t)stream);
    if (e != cudaSuccess) return wt::set_last_error(WT_ERR_LAUNCH, cudaGetErrorString(e));
    return wt_forward(net, run, &ws, stream);
}

int wt_noalloc_error(void *stream, int32_t *code) {
    if (!code) return wt::set_last_error(WT_ERR_ARGS, "code is null");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return wt::set_last_error(WT_ERR_LAUNCH, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices || !g_scratch_of[dev].load()) {
        *code = 0;  // nothing has run on this device
        return WT_OK;
    }
    const int32_t *err = static_cast<const int32_t *>(g_scratch_of[dev].load());  // offset 0
    e = cudaMemcpyAsync(code, err, sizeof(int32_t), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return wt::set_last_error(WT_ERR_LAUNCH, cudaGetErrorString(e));
    return WT_OK;
}

}  // extern "C"
