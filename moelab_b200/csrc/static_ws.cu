// moeb_experts_q4_static: the expert forward with its scratch in a fixed device array instead of a
// caller-provided workspace.
//
// Some callers of this library cannot allocate device memory: a host runtime that owns the whole device heap
// and hands kernels nothing but their operands, or code that must run without touching an allocator (for
// example on a path whose memory plan is fixed up front). For them this entry point takes only the inputs and
// the output; its scratch (routing tables, h, per-slot partial rows, counters) lives in g_static_scratch below,
// a file-scope __device__ array of MOEB_STATIC_SCRATCH_BYTES that every GPU loading the library keeps until the
// process exits. Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>
#include <unordered_map>

#include "../../include/moelab_b200.h"
#include "kernels.h"

namespace {

__device__ __align__(256) unsigned char g_static_scratch[MOEB_STATIC_SCRATCH_BYTES];

// Device address of g_static_scratch for the current device. The host-side symbol is only a stand-in for the
// array: passing it to a kernel would fault or silently touch the wrong memory. So the first call on a device
// looks the address up with cudaGetSymbolAddress (with that device current) and caches it; that first call
// should therefore come before any stream capture. The cache is keyed by the current device, so the caller's
// stream must belong to the current device (as for every entry point of this library).
void *scratch_address(int *rc) {
    static std::mutex mu;
    static std::unordered_map<int, void *> addr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        *rc = MOEB_ELAUNCH;
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(mu);
    auto it = addr.find(dev);
    if (it != addr.end()) return it->second;
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
        char msg[256];
        snprintf(msg, sizeof msg, "cudaGetSymbolAddress(g_static_scratch): %s", cudaGetErrorString(e));
        moeb::set_error(msg);
        *rc = MOEB_ELAUNCH;
        return nullptr;
    }
    addr[dev] = p;
    return p;
}

}  // namespace

extern "C" int moeb_experts_q4_static(const void *x, const void *qg, const void *sbg, const void *qu,
                                      const void *sbu, const void *qd, const void *sbd, const float *bg,
                                      const float *bu, const float *bd, const int *idx, const float *wts, int T,
                                      int d, int f, int E, int k, int act, int policy, const void *residual,
                                      void *y, cudaStream_t stream) {
    if (T < 0 || d <= 0 || f <= 0 || E <= 0 || k <= 0 || d % 64 || f % 64) {
        moeb::set_error("bad shape: dimensions must be positive, d and f multiples of 64");
        return MOEB_EINVAL;
    }
    const size_t need = moeb_workspace_bytes(T, d, f, E, k);
    if (need > (size_t)MOEB_STATIC_SCRATCH_BYTES) {
        char msg[256];
        snprintf(msg, sizeof msg,
                 "T=%d needs %zu bytes of scratch but the static scratch holds %zu; use moeb_experts_q4 with a "
                 "workspace for this size",
                 T, need, (size_t)MOEB_STATIC_SCRATCH_BYTES);
        moeb::set_error(msg);
        return MOEB_EINVAL;
    }
    int rc = MOEB_OK;
    void *ws = scratch_address(&rc);
    if (!ws) return rc;
    // The array keeps the previous call's contents: clear the counters and the error word this call relies on.
    // The call sees only the first `need` bytes, so its layout (and the cleared region) scales with T; every other
    // region is written by this call before it is read.
    // The decode kernel's tagged records are cleared with it: their tags count calls from the cleared counters.
    const size_t z = moeb::zero_region_bytes(need, d, f, E, k);
    size_t roff = 0, rlen = 0;
    moeb::decode_record_span(need, d, f, E, k, &roff, &rlen);
    if ((z && cudaMemsetAsync(ws, 0, z, stream) != cudaSuccess) ||
        (rlen && cudaMemsetAsync(static_cast<char *>(ws) + roff, 0, rlen, stream) != cudaSuccess)) {
        moeb::set_error("clearing the static scratch failed");
        return MOEB_ELAUNCH;
    }
    return moeb_experts_q4(x, qg, sbg, qu, sbu, qd, sbd, bg, bu, bd, idx, wts, T, d, f, E, k, act, policy, residual,
                           y, ws, need, stream);
}

// The device error bits (MOEB_DEVERR_*) of the last moeb_experts_q4_static call on the current device: read from the
// static array's error word and cleared, with the stream synchronised. Allocates nothing.
extern "C" int moeb_experts_q4_static_read_error(unsigned *out, cudaStream_t stream) {
    if (!out) {
        moeb::set_error("out must not be null");
        return MOEB_EINVAL;
    }
    int rc = MOEB_OK;
    void *ws = scratch_address(&rc);
    if (!ws) return rc;
    return moeb_read_error(ws, out, stream);
}
