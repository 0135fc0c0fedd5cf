// Adaptive top-k router: router scores -> (expert ids, combine weights) for
// the fused op.  Reference: loader/adaptive_topk.py:29-90
// (adaptive_topk_inclusive / adaptive_topk_batch), which keeps, of a token's
// top-k scores in descending order, the leading ones whose running sum stays
// within threshold x their total.  Dropped slots get id -1, which the fused op
// skips (kernels/latent_fused_expert_ffn.cu:33-40 treats id < 0 as a zero row).
//
// One warp per token.  Lane l holds scores l, l+32, ... of the row in
// registers (coalesced 128-byte loads) and tracks its best unselected one;
// k rounds of a warp arg-max (two warp reductions: the largest order-
// preserving key, then the lowest expert id holding it; only the winning
// lane rescans) produce the descending top-k, which lane 0 then scans with
// the reference's arithmetic (a NaN among the top k makes the total NaN, and
// every slot is kept, as in the reference): the total is numpy's
// float32 pairwise sum, the target threshold x total is formed in double and
// compared in float32, the running sum is float32.  Lane i writes slot i.
// Traffic: one read of the scores, k ids + k weights written per token.
#include "internal.h"

namespace latent {

namespace {

constexpr int kRouterWarps = 8;
constexpr int kMaxRouterTopK = 32;       // one arg-max round per slot
constexpr int kMaxRouterExperts = 1024;  // 32 scores per lane in registers

bool router_aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

// np.sum of n <= 32 float32 values: sequential from zero below 8 values, else
// eight strided accumulators combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))
// and then the tail (numpy's pairwise summation for short vectors).
__device__ float f32_sum(const float *a, int n) {
    if (n < 8) {
        float r = 0.f;
        for (int i = 0; i < n; ++i) r = __fadd_rn(r, a[i]);
        return r;
    }
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = a[j];
    int i = 8;
    for (; i < n - n % 8; i += 8)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], a[i + j]);
    float r = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])),
                        __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7])));
    for (; i < n; ++i) r = __fadd_rn(r, a[i]);
    return r;
}

// Order-preserving 32-bit key of a finite or infinite score: a larger score
// has a larger key, -0 and +0 share one key, and no score maps to 0 (the
// mark for "nothing left to select") or 1 (the key of NaN, below -inf: numpy's
// sort places NaN after every number, so the reference picks NaN scores only
// when fewer than k others remain, lowest expert id first).
__device__ __forceinline__ unsigned score_key(float v) {
    const unsigned b = v == 0.f ? 0u : __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// With SOFTMAX the row holds logits: p = exp(l - max) / sum in fp32 (the
// maximum and the sum by warp reductions), then the same selection.  With
// counts != NULL the kept slots are counted per expert (a shared-memory
// histogram per block, added to counts with one atomic per expert).
template <int NPL, bool SOFTMAX>
__global__ void __launch_bounds__(kRouterWarps * 32) k_router_topk(const float *__restrict__ scores, int T, int E,
                                                                    int k, double threshold, bool renorm,
                                                                    int *__restrict__ ids, float *__restrict__ weights,
                                                                    int *__restrict__ n_kept, int *__restrict__ counts) {
    __shared__ float s_val[kRouterWarps][kMaxRouterTopK];
    __shared__ int s_idx[kRouterWarps][kMaxRouterTopK];
    __shared__ int s_hist[kMaxRouterExperts];
    const unsigned full = 0xffffffffu;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (counts) {
        for (int i = threadIdx.x; i < E; i += blockDim.x) s_hist[i] = 0;
        __syncthreads();
    }
    const int t = blockIdx.x * kRouterWarps + warp;
    if (t < T) {
        const float *row = scores + (size_t)t * E;
        float v[NPL];
        unsigned key[NPL];    // 0: padding or already selected; 1: NaN
#pragma unroll
        for (int j = 0; j < NPL; ++j) {
            const int e = j * 32 + lane;
            v[j] = e < E ? __ldg(row + e) : 0.f;
        }
        if constexpr (SOFTMAX) {
            float m = -INFINITY;
#pragma unroll
            for (int j = 0; j < NPL; ++j)
                if (j * 32 + lane < E) m = fmaxf(m, v[j]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(full, m, o));
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < NPL; ++j) {
                v[j] = j * 32 + lane < E ? expf(__fsub_rn(v[j], m)) : 0.f;
                sum = __fadd_rn(sum, v[j]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(full, sum, o));
#pragma unroll
            for (int j = 0; j < NPL; ++j) v[j] = __fdiv_rn(v[j], sum);
        }
#pragma unroll
        for (int j = 0; j < NPL; ++j) {
            const int e = j * 32 + lane;
            key[j] = e >= E ? 0u : v[j] != v[j] ? 1u : score_key(v[j]);
        }
        // each lane's best remaining element (lowest index among equal scores)
        unsigned lkey = 0;
        int lj = 0;
        auto rescan = [&]() {
            lkey = 0;
            lj = 0;
#pragma unroll
            for (int j = 0; j < NPL; ++j) {
                if (key[j] > lkey) {
                    lkey = key[j];
                    lj = j;
                }
            }
        };
        auto value_at = [&](int jj) {
            float x = v[0];
#pragma unroll
            for (int j = 1; j < NPL; ++j) x = jj == j ? v[j] : x;
            return x;
        };
        rescan();
        for (int r = 0; r < k; ++r) {
            const unsigned m = __reduce_max_sync(full, lkey);
            const unsigned win = __reduce_min_sync(full, lkey == m ? (unsigned)(lj * 32 + lane) : 0xffffffffu);
            const bool none = m == 0u;
            // the score back from its key; a zero or NaN score takes the winner's own bits (the sign of -0, the payload)
            float val = __uint_as_float((m & 0x80000000u) ? (m & 0x7fffffffu) : ~m);
            if (m == 0x80000000u || m == 1u) val = __shfl_sync(full, value_at(lj), (int)(win & 31u));
            if (!none && lane == (int)(win & 31u)) {
#pragma unroll
                for (int j = 0; j < NPL; ++j) key[j] = j == lj ? 0u : key[j];
                rescan();
            }
            if (lane == 0) {
                s_val[warp][r] = none ? 0.f : val;
                s_idx[warp][r] = none ? -1 : (int)win;
            }
        }
        __syncwarp();
        const float my_val = lane < k ? s_val[warp][lane] : 0.f;   // lane i writes slot i
        const int my_idx = lane < k ? s_idx[warp][lane] : -1;
        // adaptive_topk_inclusive (loader/adaptive_topk.py:46-56), by lane 0 in slot order
        int n = k;
        float cum = 0.f;
        if (lane == 0) {
            const float *sv = s_val[warp];
            const float total = f32_sum(sv, k);
            if (total <= 0.f) {
                n = 0;
            } else {
                const float target = __double2float_rn(threshold * (double)total);
                for (int i = 0; i < k; ++i) {
                    const float next = __fadd_rn(cum, sv[i]);
                    if (next > target) {
                        n = i;
                        break;
                    }
                    cum = next;
                }
            }
        }
        n = __shfl_sync(full, n, 0);
        cum = __shfl_sync(full, cum, 0);
        if (lane < k) {
            const bool keep = lane < n && my_idx >= 0;
            ids[(size_t)t * k + lane] = keep ? my_idx : -1;
            weights[(size_t)t * k + lane] = keep ? (renorm ? __fdiv_rn(my_val, cum) : my_val) : 0.f;
            if (counts && keep) atomicAdd(&s_hist[my_idx], 1);
        }
        if (lane == 0 && n_kept) n_kept[t] = n;
    }
    if (counts) {
        __syncthreads();
        for (int i = threadIdx.x; i < E; i += blockDim.x)
            if (s_hist[i]) atomicAdd(counts + i, s_hist[i]);
    }
}

template <int NPL>
void launch(const float *scores, int T, int E, int k, double threshold, bool renorm, int *ids, float *w, int *nk,
            bool softmax, int *counts, cudaStream_t s) {
    const int blocks = (T + kRouterWarps - 1) / kRouterWarps;
    if (softmax)
        k_router_topk<NPL, true><<<blocks, kRouterWarps * 32, 0, s>>>(scores, T, E, k, threshold, renorm, ids, w, nk,
                                                                      counts);
    else
        k_router_topk<NPL, false><<<blocks, kRouterWarps * 32, 0, s>>>(scores, T, E, k, threshold, renorm, ids, w, nk,
                                                                       counts);
}

}  // namespace

cudaError_t launch_router_topk(const float *scores, int T, int E, int k, double threshold, bool renorm, int *ids,
                               float *weights, int *n_kept, bool softmax, int *counts, cudaStream_t s) {
    if (counts) {
        const cudaError_t e = cudaMemsetAsync(counts, 0, (size_t)E * sizeof(int), s);
        if (e != cudaSuccess) return e;
    }
    if (T == 0) return cudaSuccess;
    if (E <= 32) launch<1>(scores, T, E, k, threshold, renorm, ids, weights, n_kept, softmax, counts, s);
    else if (E <= 64) launch<2>(scores, T, E, k, threshold, renorm, ids, weights, n_kept, softmax, counts, s);
    else if (E <= 128) launch<4>(scores, T, E, k, threshold, renorm, ids, weights, n_kept, softmax, counts, s);
    else if (E <= 256) launch<8>(scores, T, E, k, threshold, renorm, ids, weights, n_kept, softmax, counts, s);
    else if (E <= 512) launch<16>(scores, T, E, k, threshold, renorm, ids, weights, n_kept, softmax, counts, s);
    else launch<32>(scores, T, E, k, threshold, renorm, ids, weights, n_kept, softmax, counts, s);
    return cudaGetLastError();
}

}  // namespace latent

namespace {

int router_entry(const float *scores, int32_t n_tokens, int32_t n_expert, int32_t top_k, double threshold,
                 uint32_t flags, int32_t *ids, float *weights, int32_t *n_kept, int32_t *counts, CUstream_st *stream) {
    using namespace latent;
    if (n_tokens < 0 || n_expert < 1 || top_k < 1 || top_k > n_expert) return LATENT_ERR_SHAPE;
    if (!(threshold > 0.0 && threshold <= 1.0)) return LATENT_ERR_INVALID;
    if (flags & ~(uint32_t)(LATENT_ROUTER_RENORMALIZE | LATENT_ROUTER_SOFTMAX)) return LATENT_ERR_INVALID;
    if (n_expert > kMaxRouterExperts || top_k > kMaxRouterTopK) return LATENT_ERR_UNSUPPORTED;
    if (n_tokens > 0 && (!scores || !ids || !weights)) return LATENT_ERR_INVALID;
    if (!router_aligned(scores, 4) || !router_aligned(ids, 4) || !router_aligned(weights, 4) ||
        (n_kept && !router_aligned(n_kept, 4)) || (counts && !router_aligned(counts, 4)))
        return LATENT_ERR_ALIGN;
    if (n_tokens == 0 && !counts) return LATENT_OK;
    const cudaError_t e = launch_router_topk(scores, n_tokens, n_expert, top_k, threshold,
                                             (flags & LATENT_ROUTER_RENORMALIZE) != 0, ids, weights, n_kept,
                                             (flags & LATENT_ROUTER_SOFTMAX) != 0, counts,
                                             reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? LATENT_OK : LATENT_ERR_CUDA;
}

}  // namespace

extern "C" LATENT_API int latent_router_topk(const float *scores, int32_t n_tokens, int32_t n_expert, int32_t top_k,
                                             double threshold, uint32_t flags, int32_t *ids, float *weights,
                                             int32_t *n_kept, CUstream_st *stream) {
    if (flags & LATENT_ROUTER_SOFTMAX) return LATENT_ERR_INVALID;  // scores are probabilities here
    return router_entry(scores, n_tokens, n_expert, top_k, threshold, flags, ids, weights, n_kept, nullptr, stream);
}

extern "C" LATENT_API int latent_router_route(const float *scores, int32_t n_tokens, int32_t n_expert, int32_t top_k,
                                              double threshold, uint32_t flags, int32_t *ids, float *weights,
                                              int32_t *n_kept, int32_t *expert_counts, CUstream_st *stream) {
    return router_entry(scores, n_tokens, n_expert, top_k, threshold, flags, ids, weights, n_kept, expert_counts,
                        stream);
}
