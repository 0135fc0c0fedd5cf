// Routing: group routed (token, slot) pairs by expert, stably.
//
// Output (all in the caller's workspace):
//   counts[E], offsets[E+1]   routed pairs per expert and their prefix
//   active[E], n_active       experts with >= 1 pair, ascending
//   order[R]                  flat slot index t*k+j per routed position,
//                             sorted by expert, then by slot index
//   pos[T*k]                  routed position of each slot, -1 when skipped
//   virt[], n_virt, vslot[R]  (decode path) each active expert split into
//                             virtual experts of <= kVirtTokens consecutive
//                             routed positions, in active order, and the
//                             virtual expert of every routed position
// Slots with id < 0 are skipped (the reference op writes a zero row for
// them, kernels/latent_fused_expert_ffn.cu:33-40); ids >= E are skipped and
// flag kErrExpertId.  The same stable order is what the CPU oracle's
// route() returns.
#include "internal.h"

namespace latent {

namespace {

constexpr int kRouteThreads = 1024;
constexpr int kRouteWarps = kRouteThreads / 32;

__device__ __forceinline__ int valid_expert(int e, int E, uint32_t *err) {
    if (e >= E) {
        atomicOr(err, kErrExpertId);
        return -1;
    }
    return e;
}

// Exclusive scan of v[0..n) in shared memory by one block; returns the total.
// scratch needs 33 ints.
__device__ int block_exclusive_scan(int *v, int n, int *scratch) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (n + kRouteThreads - 1) / kRouteThreads;
    const int lo = min(n, tid * per), hi = min(n, lo + per);
    int local = 0;
    for (int i = lo; i < hi; ++i) local += v[i];
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) scratch[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int w = scratch[lane];
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        scratch[lane] = wi - w;
        if (lane == 31) scratch[32] = wi;
    }
    __syncthreads();
    int run = scratch[warp] + incl - local;
    for (int i = lo; i < hi; ++i) {
        const int x = v[i];
        v[i] = run;
        run += x;
    }
    const int total = scratch[32];
    __syncthreads();
    return total;
}

// Stable placement of slots [lo, hi): base[e] holds the next free routed
// position of expert e and is advanced.  wcnt is [kRouteWarps][E] scratch.
__device__ void block_stable_scatter(const int32_t *ids, int lo, int hi, int E, int top_k, int *base,
                                     int *wcnt, int32_t *order, int32_t *pos, uint32_t *err) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int c0 = lo; c0 < hi; c0 += kRouteThreads) {
        for (int i = tid; i < kRouteWarps * E; i += kRouteThreads) wcnt[i] = 0;
        __syncthreads();
        const int slot = c0 + tid;
        int e = -1;
        if (slot < hi) {
            const int raw = __ldg(ids + slot);
            e = raw < 0 ? -1 : valid_expert(raw, E, err);
        }
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(same & ((1u << lane) - 1u));
        const int leader = __ffs(same) - 1;
        if (e >= 0 && lane == leader) wcnt[warp * E + e] = __popc(same);
        __syncthreads();
        for (int x = tid; x < E; x += kRouteThreads) {
            int run = base[x];
            for (int w = 0; w < kRouteWarps; ++w) {
                const int c = wcnt[w * E + x];
                wcnt[w * E + x] = run;
                run += c;
            }
            base[x] = run;
        }
        __syncthreads();
        if (slot < hi) {
            if (e >= 0) {
                const int p = wcnt[warp * E + e] + rank;
                order[p] = slot;
                pos[slot] = p;
            } else {
                pos[slot] = -1;
            }
        }
        __syncthreads();
    }
    (void)top_k;
}

// Virtual-expert table from counts/offsets/active (one block): per active
// expert ceil(count / kVirtTokens) virtual experts, each with the prefix of
// the token columns before it.  act/cnt/off are the active list, counts and
// offsets (shared or global memory); nv and wv hold at least E ints of
// shared scratch each; scratch as for block_exclusive_scan.
__device__ void block_build_virt(const RouteArgs &a, int n_act, const int *act, const int *cnt, const int *off,
                                 int *nv, int *wv, int *scratch) {
    const int tid = threadIdx.x;
    for (int i = tid; i < n_act; i += kRouteThreads) {
        const int ne = cnt[act[i]];
        const int full = ne / kVirtTokens, rest = ne - full * kVirtTokens;
        nv[i] = full + (rest > 0);
        wv[i] = full * virt_weight(kVirtTokens) + (rest > 0 ? virt_weight(rest) : 0);
    }
    __syncthreads();
    const int total = block_exclusive_scan(nv, n_act, scratch);
    const int wtotal = block_exclusive_scan(wv, n_act, scratch);
    for (int i = tid; i < n_act; i += kRouteThreads) {
        const int e = act[i], ne = cnt[e], p0 = off[e];
        int wsum = wv[i];
        for (int q = 0, v = nv[i]; q * kVirtTokens < ne; ++q, ++v) {
            const int first = p0 + q * kVirtTokens, n = min(kVirtTokens, ne - q * kVirtTokens);
            a.virt[v] = make_int4(e, first, n, wsum);
            wsum += virt_weight(n);
            for (int jj = 0; jj < n; ++jj) a.vslot[first + jj] = v;
        }
    }
    if (tid == 0) {
        a.n_virt[0] = total;
        a.n_virt[1] = wtotal;
    }
    __syncthreads();
}

// One block does everything (small R: decode).
__global__ void __launch_bounds__(kRouteThreads) k_route_single(RouteArgs a) {
    extern __shared__ int sm[];
    int *cnt = sm;                 // [E] counts, then running bases of the scatter
    int *scratch = cnt + a.E;      // [64]
    int *wcnt = scratch + 64;      // [32][E]
    int *cnt_k = wcnt + 32 * a.E;  // [E] counts (kept)
    int *off_k = cnt_k + a.E;      // [E] offsets (kept)
    int *act = off_k + a.E;        // [E] active list
    const int tid = threadIdx.x;
    for (int i = tid; i < a.n_sem; i += kRouteThreads) a.sem[i] = 0;
    if (tid < 4) a.err[tid] = 0;
    for (int i = tid; i < a.E; i += kRouteThreads) cnt[i] = 0;
    __syncthreads();
    for (int i = tid; i < a.R; i += kRouteThreads) {
        const int e = __ldg(a.ids + i);
        if (e >= 0 && e < a.E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    for (int i = tid; i < a.E; i += kRouteThreads) {
        const int c = cnt[i];
        cnt_k[i] = c;
        a.counts[i] = c;
        wcnt[i] = c > 0 ? 1 : 0;
    }
    __syncthreads();
    const int total = block_exclusive_scan(cnt, a.E, scratch);
    const int n_act = block_exclusive_scan(wcnt, a.E, scratch);
    for (int i = tid; i < a.E; i += kRouteThreads) {
        off_k[i] = cnt[i];
        a.offsets[i] = cnt[i];
        if (cnt_k[i] > 0) {
            act[wcnt[i]] = i;
            a.active[wcnt[i]] = i;
        }
    }
    if (tid == 0) {
        a.offsets[a.E] = total;
        *a.n_active = n_act;
    }
    __syncthreads();
    if (a.virt) block_build_virt(a, n_act, act, cnt_k, off_k, wcnt, wcnt + a.E, scratch);
    block_stable_scatter(a.ids, 0, a.R, a.E, a.top_k, cnt, wcnt, a.order, a.pos, a.err);
}

// Multi-block variant (large R: prefill).  Pass 1: per-block histograms.
__global__ void __launch_bounds__(kRouteThreads) k_route_hist(RouteArgs a) {
    extern __shared__ int sm[];
    int *cnt = sm;
    const int tid = threadIdx.x, b = blockIdx.x;
    if (b == 0) {
        for (int i = tid; i < a.n_sem; i += kRouteThreads) a.sem[i] = 0;
        if (tid < 4) a.err[tid] = 0;
    }
    for (int i = tid; i < a.E; i += kRouteThreads) cnt[i] = 0;
    __syncthreads();
    const int lo = b * a.chunk, hi = min(a.R, lo + a.chunk);
    for (int i = lo + tid; i < hi; i += kRouteThreads) {
        const int e = __ldg(a.ids + i);
        if (e >= 0 && e < a.E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    for (int i = tid; i < a.E; i += kRouteThreads) a.block_counts[(int64_t)b * a.E + i] = cnt[i];
}

// Pass 2: one block turns block histograms into offsets and block bases.
__global__ void __launch_bounds__(kRouteThreads) k_route_scan(RouteArgs a) {
    extern __shared__ int sm[];
    int *cnt = sm;
    int *scratch = cnt + a.E;
    int *flag = scratch + 64;
    const int tid = threadIdx.x;
    for (int e = tid; e < a.E; e += kRouteThreads) {
        int s = 0;
        for (int b = 0; b < a.n_blocks; ++b) s += a.block_counts[(int64_t)b * a.E + e];
        cnt[e] = s;
        a.counts[e] = s;
        flag[e] = s > 0 ? 1 : 0;
    }
    __syncthreads();
    const int total = block_exclusive_scan(cnt, a.E, scratch);
    const int n_act = block_exclusive_scan(flag, a.E, scratch);
    for (int e = tid; e < a.E; e += kRouteThreads) {
        a.offsets[e] = cnt[e];
        if (a.counts[e] > 0) a.active[flag[e]] = e;
        int run = cnt[e];
        for (int b = 0; b < a.n_blocks; ++b) {
            const int c = a.block_counts[(int64_t)b * a.E + e];
            a.block_counts[(int64_t)b * a.E + e] = run;
            run += c;
        }
    }
    if (tid == 0) {
        a.offsets[a.E] = total;
        *a.n_active = n_act;
    }
    __syncthreads();
    if (a.virt) block_build_virt(a, n_act, a.active, a.counts, a.offsets, flag, cnt, scratch);
}

// Pass 3: stable scatter within each block from its base offsets.
__global__ void __launch_bounds__(kRouteThreads) k_route_scatter(RouteArgs a) {
    extern __shared__ int sm[];
    int *base = sm;
    int *wcnt = base + a.E;
    const int tid = threadIdx.x, b = blockIdx.x;
    for (int e = tid; e < a.E; e += kRouteThreads) base[e] = a.block_counts[(int64_t)b * a.E + e];
    __syncthreads();
    const int lo = b * a.chunk, hi = min(a.R, lo + a.chunk);
    block_stable_scatter(a.ids, lo, hi, a.E, a.top_k, base, wcnt, a.order, a.pos, a.err);
}

}  // namespace

size_t route_block_counts_bytes(int E, int R) {
    const int nb = R <= kRouteSingleMax ? 1 : (R + kRouteChunk - 1) / kRouteChunk;
    return (size_t)nb * E * sizeof(int32_t);
}

cudaError_t launch_route(RouteArgs a, cudaStream_t s) {
    const size_t wsm = (size_t)(64 + (kRouteWarps + 1) * a.E) * sizeof(int);
    const size_t ssm = wsm + (size_t)3 * a.E * sizeof(int);
    cudaError_t err = ensure_smem((const void *)k_route_single, ssm);
    if (err == cudaSuccess) err = ensure_smem((const void *)k_route_scatter, wsm);
    if (err != cudaSuccess) return err;
    if (a.R <= kRouteSingleMax) {
        k_route_single<<<1, kRouteThreads, ssm, s>>>(a);
        return cudaGetLastError();
    }
    a.chunk = kRouteChunk;
    a.n_blocks = (a.R + kRouteChunk - 1) / kRouteChunk;
    k_route_hist<<<a.n_blocks, kRouteThreads, (size_t)a.E * sizeof(int), s>>>(a);
    k_route_scan<<<1, kRouteThreads, (size_t)(2 * a.E + 64) * sizeof(int), s>>>(a);
    k_route_scatter<<<a.n_blocks, kRouteThreads, wsm, s>>>(a);
    return cudaGetLastError();
}

}  // namespace latent
