// latent_expert_ffn_forward_noalloc: the fused expert FFN for callers that
// cannot allocate device memory at call time.
//
// Who needs it: a host framework that plans every device buffer before it
// runs a model graph and forbids allocation while the graph executes (the
// ggml graph allocator assigns all tensors up front; an op that allocated
// mid-compute would break that plan), real-time or embedded hosts that
// reserve all GPU memory at start-up, and processes sharing a GPU under a
// hard memory cap, where a late cudaMalloc can fail or stall the device.
// Such a caller still owns x, ids, weights, out and the factors, but cannot
// provide the workspace.  This entry point uses a fixed scratch array that
// the library itself carries in device memory instead.
//
// Limits and rules:
// * The scratch is kStaticScratchBytes (16 MiB) per GPU, reserved by every
//   GPU that loads this library until the process exits.  A call whose
//   workspace need (latent_expert_ffn_workspace_size) exceeds it returns
//   LATENT_ERR_WORKSPACE before any work is queued.
// * desc->workspace and desc->workspace_bytes are ignored.
// * All calls on a device share the one array, which keeps the last call's
//   contents.  Everything that must start at zero (arrival counters, error
//   word) is cleared by the routing kernel at the start of every call, so
//   calls queued one after another on a stream are independent.  Calls
//   that overlap on the GPU (two streams, two host threads without ordering)
//   race on the array and give undefined results.
// * The array's device address is looked up (cudaGetSymbolAddress) on every
//   call made outside stream capture, so a device reset or a new context is
//   picked up; a call made while `stream` is capturing reuses the address of
//   the last uncaptured call on that device, so make one call on each device
//   before capturing (a capture cannot span a device reset).
// * Device-side errors (a routed id >= n_expert, an expired wait) are
//   recorded in the array's error word; read them with
//   latent_expert_ffn_check_noalloc().
// Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <mutex>

#include "internal.h"

namespace latent {
namespace {

constexpr size_t kStaticScratchBytes = 16u << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_mu;
void *g_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device: looked up afresh
// unless `stream` is capturing, when the last looked-up address is used.
int static_scratch(cudaStream_t stream, void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LATENT_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return LATENT_ERR_UNSUPPORTED;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) return LATENT_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (cap == cudaStreamCaptureStatusNone) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return LATENT_ERR_CUDA;
        g_ptr[dev] = p;
    } else if (!g_ptr[dev]) {
        return LATENT_ERR_UNSUPPORTED;  // first call on this device is inside a capture
    }
    *out = g_ptr[dev];
    return LATENT_OK;
}

}  // namespace
}  // namespace latent

extern "C" LATENT_API int latent_expert_ffn_forward_noalloc(const latent_ffn_desc *desc, CUstream_st *stream) {
    if (!desc) return LATENT_ERR_INVALID;
    size_t need = 0;
    int st = latent_expert_ffn_workspace_size(desc, &need);
    if (st) return st;
    if (need > latent::kStaticScratchBytes) return LATENT_ERR_WORKSPACE;
    if (desc->n_tokens == 0) return latent_expert_ffn_forward(desc, stream);
    void *scratch = nullptr;
    if ((st = latent::static_scratch(reinterpret_cast<cudaStream_t>(stream), &scratch))) return st;
    latent_ffn_desc local = *desc;
    local.workspace = scratch;
    local.workspace_bytes = latent::kStaticScratchBytes;
    return latent_expert_ffn_forward(&local, stream);
}

extern "C" LATENT_API int latent_expert_ffn_check_noalloc(const latent_ffn_desc *desc, CUstream_st *stream) {
    if (!desc) return LATENT_ERR_INVALID;
    void *scratch = nullptr;
    int st = latent::static_scratch(reinterpret_cast<cudaStream_t>(stream), &scratch);
    if (st) return st;
    latent_ffn_desc local = *desc;
    local.workspace = scratch;
    local.workspace_bytes = latent::kStaticScratchBytes;
    return latent_expert_ffn_check(&local, stream);
}
