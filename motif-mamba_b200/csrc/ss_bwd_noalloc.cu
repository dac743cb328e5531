// ss_bwd_noalloc: the selective-scan backward without any caller-provided or runtime-
// allocated workspace.  Its scratch (the fp32 dB / dC accumulators ss_bwd otherwise takes
// from `workspace`: the fp32 dB / dC accumulators, plus the per-step scratch of dstate > 16
// and the P/Q checkpoints) is a fixed array of MSS_BWD_NOALLOC_SCRATCH_BYTES in this
// library's device image; it is placed on a GPU when the module loads there and held until
// the process exits.  A call is accepted when ss_bwd_workspace_size() <= that size.
//
// Host code cannot use the array's name as a device address (on the host it names a
// stand-in object), so the device address is looked up with cudaGetSymbolAddress once per
// device, on the first call made with that device current, and cached per device index.
// That first call should therefore happen before any stream capture, and a device reset
// after it (which would move the array) is not supported.  Every call reuses the same array:
// ss_bwd clears the accumulators at the start of each call, and two calls that overlap on
// the GPU (different streams, or different host threads) race on it.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

static __device__ __align__(256) unsigned char g_bwd_noalloc_scratch[MSS_BWD_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;
}  // namespace

extern "C" int ss_bwd_noalloc(const ss_bwd_args *a, void *stream) {
    if (!a) return ss_bwd(a, stream);  // reports the null struct the same way
    int64_t need = 0;
    int rc = ss_bwd_workspace_size(a, &need);
    if (rc) return rc;
    if (need > (int64_t)MSS_BWD_NOALLOC_SCRATCH_BYTES) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "ss_bwd_noalloc: these sizes need %lld bytes of scratch (ss_bwd_workspace_size: the fp32 "
                 "dB/dC accumulators, plus per-step sums for dstate > 16 and checkpoints for P/Q), "
                 "more than the %lld-byte static array; use ss_bwd",
                 (long long)need, (long long)MSS_BWD_NOALLOC_SCRATCH_BYTES);
        return mss::set_last_error(MSS_ERR_WORKSPACE, msg);
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return mss::set_last_error(MSS_ERR_CUDA, "ss_bwd_noalloc: no usable current CUDA device");
    void *ptr = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        ptr = g_scratch_ptr[dev];
        if (!ptr) {
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_bwd_noalloc_scratch);
            if (e != cudaSuccess || !ptr) {
                char msg[256];
                snprintf(msg, sizeof(msg), "ss_bwd_noalloc: cudaGetSymbolAddress failed: %s",
                         cudaGetErrorString(e));
                return mss::set_last_error(MSS_ERR_CUDA, msg);
            }
            g_scratch_ptr[dev] = ptr;
        }
    }
    ss_bwd_args t = *a;
    t.workspace = ptr;
    t.workspace_bytes = MSS_BWD_NOALLOC_SCRATCH_BYTES;
    return ss_bwd(&t, stream);
}
