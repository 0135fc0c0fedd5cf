// Expert-parallel dispatch and combine (no counterpart in the reference,
// which has no multi-GPU code).  The rows a rank sends travel through NCCL
// all-to-all in the caller; these kernels only pack them in expert order
// (which is destination-rank order, experts being contiguous per rank) and
// fold the returned expert outputs into the top-k combine.
#include "internal.h"

namespace latent {

namespace {

// Row p of the routed order: send_x[p] = x[token], send_expert[p] = id,
// send_weight[p] = router weight.  One block per routed row.
template <int XT>
__global__ void __launch_bounds__(128) k_ep_gather(EpArgs a) {
    const int p = blockIdx.x;
    if (p >= a.offsets[a.E]) return;
    const int slot = a.order[p];
    const int t = slot / a.k;
    const size_t es = XT == LATENT_TYPE_F32 ? 4 : 2;
    const char *src = static_cast<const char *>(a.x) + (size_t)t * a.d * es;
    char *dst = static_cast<char *>(a.send_x) + (size_t)p * a.d * es;
    const int n16 = (int)(a.d * es / 16);
    for (int i = threadIdx.x; i < n16; i += blockDim.x)
        reinterpret_cast<uint4 *>(dst)[i] = __ldg(reinterpret_cast<const uint4 *>(src) + i);
    if (threadIdx.x == 0) {
        a.send_expert[p] = __ldg(a.ids + slot);
        a.send_weight[p] = load_weight(a.weights, a.w_type, slot);
    }
}

}  // namespace

cudaError_t launch_ep_gather(const EpArgs &a, cudaStream_t s) {
    const int rows = a.T * a.k;
    if (rows == 0) return cudaSuccess;
    switch (a.x_type) {
        case LATENT_TYPE_F32: k_ep_gather<LATENT_TYPE_F32><<<rows, 128, 0, s>>>(a); break;
        case LATENT_TYPE_F16: k_ep_gather<LATENT_TYPE_F16><<<rows, 128, 0, s>>>(a); break;
        default: k_ep_gather<LATENT_TYPE_BF16><<<rows, 128, 0, s>>>(a); break;
    }
    return cudaGetLastError();
}

}  // namespace latent
