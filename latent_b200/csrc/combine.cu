// Top-k combine of per-routed-row outputs (expert-parallel return path and
// the prefill path): out[t] = sum_j w[t,j] * y[pos[t*k+j]] in slot order.
#include "internal.h"

namespace latent {

namespace {

// Top-k combine of per-routed-row outputs in slot order (used by the
// expert-parallel return path), or zero rows of skipped slots in per-slot mode.
__global__ void __launch_bounds__(256) k_combine(DecodeArgs a) {
    const int t = blockIdx.y;
    const int c = (blockIdx.x * 256 + threadIdx.x) * 4;
    if (c >= a.d) return;
    const bool per_slot = a.flags & LATENT_FLAG_OUT_PER_SLOT;
    const bool wbd = a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < a.k; ++j) {
        const int slot = t * a.k + j;
        const int p = a.rt.pos[slot];
        if (per_slot) {
            if (p < 0) *reinterpret_cast<float4 *>(a.out + (int64_t)slot * a.d + c) = acc;
            continue;
        }
        if (p < 0) continue;
        const float w = wbd ? 1.f : load_weight(a.weights, a.w_type, slot);
        const float4 v = *reinterpret_cast<const float4 *>(a.y + (int64_t)p * a.d + c);
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
    }
    if (!per_slot) *reinterpret_cast<float4 *>(a.out + (int64_t)t * a.d + c) = acc;
}

}  // namespace

cudaError_t launch_combine(const DecodeArgs &a, cudaStream_t s) {
    if (a.T == 0) return cudaSuccess;
    dim3 grid((a.d / 4 + 255) / 256, a.T);
    k_combine<<<grid, 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace latent
