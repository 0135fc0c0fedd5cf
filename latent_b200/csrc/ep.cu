// Expert-parallel dispatch and combine (no counterpart in the reference,
// which has no multi-GPU code).  The rows a rank sends travel through NCCL
// all-to-all in the caller; these kernels only pack them in expert order
// (which is destination-rank order, experts being contiguous per rank),
// optionally into fixed-capacity blocks per destination rank, and fold the
// returned expert outputs into the top-k combine.
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

// One exchange block per destination in a single buffer, so that rows and
// their metadata travel in one all-to-all: block g = [cap rows of x][cap
// {id, weight bits} pairs, padded to 16 bytes].
__host__ __device__ inline size_t merged_block_bytes(int cap, int d, int es) {
    return (size_t)cap * d * es + (((size_t)cap * 8 + 15) & ~(size_t)15);
}

// Fixed-capacity block q of the send buffer: block g = q / cap holds the
// rows routed to rank g's experts [g*el, (g+1)*el) in routed order, rows past
// their count get expert id -1.  One block per padded row.  A destination
// with more rows than cap (only possible when a token routes one expert
// twice) keeps its first cap rows and sets kErrCapacity.  With `merged` the
// rows and the metadata of block g share its region of `rows`
// (merged_block_bytes); otherwise they go to rows[q] and meta[q].
template <int XT>
__global__ void __launch_bounds__(128) k_ep_pack_fixed(EpArgs a, int el, int cap, void *rows, int32_t *meta,
                                                       bool merged) {
    const int q = blockIdx.x;
    const int g = q / cap, i = q - g * cap;
    const size_t es = XT == LATENT_TYPE_F32 ? 4 : 2;
    char *row_dst;
    int32_t *meta_dst;
    if (merged) {
        char *blk = static_cast<char *>(rows) + (size_t)g * merged_block_bytes(cap, a.d, (int)es);
        row_dst = blk + (size_t)i * a.d * es;
        meta_dst = reinterpret_cast<int32_t *>(blk + (size_t)cap * a.d * es) + 2 * (size_t)i;
    } else {
        row_dst = static_cast<char *>(rows) + (size_t)q * a.d * es;
        meta_dst = meta + 2 * (size_t)q;
    }
    const int p = a.offsets[g * el] + i;
    const int end = a.offsets[(g + 1) * el];
    const bool valid = p < end;
    if (threadIdx.x == 0 && i == 0 && end - p > cap) atomicOr(a.err, kErrCapacity);
    if (threadIdx.x == 0) {
        meta_dst[0] = valid ? a.send_expert[p] : -1;
        meta_dst[1] = valid ? __float_as_int(a.send_weight[p]) : 0;
    }
    if (!valid) return;
    const char *src = static_cast<const char *>(a.send_x) + (size_t)p * a.d * es;
    const int n16 = (int)(a.d * es / 16);
    for (int j = threadIdx.x; j < n16; j += blockDim.x)
        reinterpret_cast<uint4 *>(row_dst)[j] = __ldg(reinterpret_cast<const uint4 *>(src) + j);
}

// Receive side of the merged exchange: block q = g*cap + i copies row i of
// source block g to x_out[q] and turns its metadata into the local op's
// inputs: ids_out[q] = id - base for a local expert, else -1; w_out[q] = the
// router weight with weight-before-down, else 1.
__global__ void __launch_bounds__(128) k_ep_unpack_fixed(const char *buf, int cap, int d, int es, int base,
                                                         int n_local, bool wbd, char *x_out, int32_t *ids_out,
                                                         float *w_out, uint32_t *err) {
    const int q = blockIdx.x;
    const int g = q / cap, i = q - g * cap;
    const char *blk = buf + (size_t)g * merged_block_bytes(cap, d, es);
    const int32_t *meta = reinterpret_cast<const int32_t *>(blk + (size_t)cap * d * es) + 2 * (size_t)i;
    const int n16 = (int)((size_t)d * es / 16);
    const uint4 *src = reinterpret_cast<const uint4 *>(blk + (size_t)i * d * es);
    uint4 *dst = reinterpret_cast<uint4 *>(x_out + (size_t)q * d * es);
    const int id = meta[0];
    if (id >= 0)
        for (int j = threadIdx.x; j < n16; j += blockDim.x) dst[j] = src[j];
    if (threadIdx.x == 0) {
        const int local = id - base;
        const bool ok = id >= 0 && local < n_local && local >= 0;
        if (id >= 0 && !ok && err) atomicOr(err, kErrExpertId);
        ids_out[q] = ok ? local : -1;
        w_out[q] = wbd ? __int_as_float(meta[1]) : 1.f;
    }
}

// out[t] = sum_j w[t,j] * y_rows[block row of slot (t,j)], the inverse of
// k_ep_pack_fixed's placement (row = g*cap + routed position - first
// position of rank g).  Skipped slots (id < 0), out-of-range ids and rows
// that did not fit their block contribute nothing.
__global__ void __launch_bounds__(256) k_ep_combine_fixed(EpArgs a, const int32_t *pos, int el, int cap,
                                                          const float *y, float *out, bool wbd) {
    const int t = blockIdx.y;
    const int c = (blockIdx.x * 256 + threadIdx.x) * 4;
    if (c >= a.d) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < a.k; ++j) {
        const int slot = t * a.k + j;
        const int e = __ldg(a.ids + slot);
        if (e < 0 || e >= a.E) continue;
        const int p = pos[slot];
        if (p < 0) continue;
        const int g = e / el;
        const int i = p - a.offsets[g * el];
        if (i < 0 || i >= cap) continue;   // beyond the block: never sent (cap too small)
        const int q = g * cap + i;
        const float w = wbd ? 1.f : load_weight(a.weights, a.w_type, slot);
        const float4 v = *reinterpret_cast<const float4 *>(y + (int64_t)q * a.d + c);
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
    }
    *reinterpret_cast<float4 *>(out + (int64_t)t * a.d + c) = acc;
}

}  // namespace

cudaError_t launch_ep_pack_fixed(const EpArgs &a, int world, int cap, void *rows, int32_t *meta, bool merged,
                                 cudaStream_t s) {
    const int n = world * cap;
    const int el = a.E / world;
    switch (a.x_type) {
        case LATENT_TYPE_F32: k_ep_pack_fixed<LATENT_TYPE_F32><<<n, 128, 0, s>>>(a, el, cap, rows, meta, merged); break;
        case LATENT_TYPE_F16: k_ep_pack_fixed<LATENT_TYPE_F16><<<n, 128, 0, s>>>(a, el, cap, rows, meta, merged); break;
        default: k_ep_pack_fixed<LATENT_TYPE_BF16><<<n, 128, 0, s>>>(a, el, cap, rows, meta, merged); break;
    }
    return cudaGetLastError();
}

size_t ep_merged_block_bytes(int cap, int d, int es) { return merged_block_bytes(cap, d, es); }

cudaError_t launch_ep_unpack_fixed(const void *buf, int world, int cap, int d, int es, int base, int n_local, bool wbd,
                                   void *x_out, int32_t *ids_out, float *w_out, uint32_t *err, cudaStream_t s) {
    const int n = world * cap;
    if (n == 0) return cudaSuccess;
    k_ep_unpack_fixed<<<n, 128, 0, s>>>(static_cast<const char *>(buf), cap, d, es, base, n_local, wbd,
                                        static_cast<char *>(x_out), ids_out, w_out, err);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine_fixed(const EpArgs &a, const int32_t *pos, int world, int cap, const float *y, float *out,
                                    bool wbd, cudaStream_t s) {
    if (a.T == 0) return cudaSuccess;
    dim3 grid((a.d / 4 + 255) / 256, a.T);
    k_ep_combine_fixed<<<grid, 256, 0, s>>>(a, pos, a.E / world, cap, y, out, wbd);
    return cudaGetLastError();
}

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
