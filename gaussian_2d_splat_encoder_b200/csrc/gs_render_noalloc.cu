// gs_render_noalloc.cu -- a forward render that allocates nothing.
//
// gs_render_fwd needs a caller-provided workspace (splat records, the (tile, splat) pair buffers and the
// group fields).  Some callers cannot obtain one: a host application whose device memory is owned by
// another allocator it cannot call into, or code on a latency-critical path where cudaMalloc and its
// implicit device synchronisation are not acceptable.  gs_render_fwd_noalloc serves them with a fixed
// scratch array that lives in the library itself (a file-scope __device__ array), so the only memory
// the caller provides is its inputs and its output.
//
// Limits and sharing:
//   * the array holds GS_NOALLOC_SCRATCH_BYTES (32 MiB); a render whose forward workspace
//     (gs_render_workspace_size(d, 0)) is larger is refused with GS_ERR_WORKSPACE, before any launch;
//   * every GPU that loads the library holds the array until the process exits;
//   * all calls on a device share the one array and it keeps the previous call's contents (the forward
//     clears the parts it needs zeroed), so calls whose work overlaps on the GPU -- different streams,
//     or other host threads -- race and must be serialised by the caller;
//   * the first call on each device looks up the array's device address (cudaGetSymbolAddress) with
//     that device current; make that first call before any stream capture.  The address is kept for the
//     life of the process: after a cudaDeviceReset the library has to be reloaded;
//   * the render's own checks apply as in gs_render_fwd: a pair_capacity below gs_render_pair_bound, or a
//     max_pairs the host bound cannot rule out, makes the call count the pairs first (one stream
//     synchronisation) and refuse with GS_ERR_WORKSPACE / GS_ERR_PAIR_BUDGET instead of truncating.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/gsplat_b200.h"
#include "gs_render_internal.cuh"

static __device__ __align__(256) unsigned char g_noalloc_scratch[GS_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device.  In host code the array's name is only a
// host-side stand-in, so the address has to come from cudaGetSymbolAddress, once per device.
int scratch_address(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        gs_set_last_error(cudaGetErrorString(e));
        return GS_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        gs_set_last_error("gs_render_fwd_noalloc: device index beyond the 64 this library tracks");
        return GS_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            gs_set_last_error(e != cudaSuccess ? cudaGetErrorString(e) : "cudaGetSymbolAddress returned NULL");
            return GS_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return GS_OK;
}
}  // namespace

extern "C" int gs_render_fwd_noalloc(const gs_render_desc *d, const float *mu, const float *log_scale,
                                     const float *color, const float *opacity, const float *bg, const float *theta,
                                     float *out, void *stream) {
    if (!d) return GS_ERR_BAD_ARGUMENT;
    const size_t need = gs_render_workspace_size(d, 0);
    if (need == 0) return GS_ERR_BAD_ARGUMENT;
    if (need > (size_t)GS_NOALLOC_SCRATCH_BYTES) return GS_ERR_WORKSPACE;
    void *ws = nullptr;
    int st = scratch_address(&ws);
    if (st != GS_OK) return st;
    return gs_render_fwd(d, mu, log_scale, color, opacity, bg, theta, out, ws, (size_t)GS_NOALLOC_SCRATCH_BYTES,
                         stream);
}
