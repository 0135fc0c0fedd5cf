// Dense-fallback experts and the dense projection utility.
//
// The reference compressor keeps a dense fp16 copy of a matrix whose
// quantised factors miss its error threshold (`<name>.dense_fallback`,
// loader/latent_loader.py:262-265); its dense expert forward is
// dense_swiglu_expert (loader/latent_runtime.py:62-73).  The reference
// runtime itself never reads the fallback.  Here a layer may flag experts
// as dense: the routed slots of those experts are taken out of the latent
// op (their ids set to -1 in the copy the latent op reads) and served by
// the kernels below, which add their contributions into the same output.
// A flagged expert may mix kinds: a kind with a dense matrix uses it, the
// others use their exact fp32 factor pair (dequantised once at load).
//
// Row space: the routed slots of the flagged experts, grouped by expert
// (expert di owns rows [offs[di], offs[di+1])).  Stages per batch of up to
// kJobs jobs (one launch each): x -> G|U (dense) or x -> T (pair), T -> G|U,
// SwiGLU in place, H -> combine (dense) or H -> S, S -> combine.
//
// k_rows_gemm: y[p][n] = sum_k src[row(p)][k] W[k][n] on the CUDA cores in
// fp32, 128 threads per block, a tile of RB rows x 256 columns (two adjacent
// columns per thread: one 4- or 8-byte weight load per k, coalesced), the
// source tile staged in shared memory as [k][row] so that a thread reads
// the RB values of one k with RB/4 broadcast 16-byte loads.  Each weight
// element is read once per RB rows: dense experts are the rare case, served
// at the bandwidth of a plain streamed GEMV for decode-sized batches.
#include <limits.h>
#include <string.h>

#include <algorithm>

#include "internal.h"

namespace latent {

namespace {

constexpr int kJobs = 16;
constexpr int kKTile = 64;
constexpr int kCols = 256;

struct DJob {
    const void *w;        // [K][N] row-major, element type wt
    const void *src;      // source rows (element type of the stage), row stride lds, first column scol
    float *dst;           // destination rows (fp32), row stride ldd, first column dcol (store epilogue)
    int64_t lds, ldd;
    int wt, K, N, scol, dcol;
    int di;               // dense expert whose rows the job covers; -1: rows [0, M)
    int combine;          // 1: the combine epilogue instead of a store
};

struct DStage {
    DJob job[kJobs];
    int n_jobs;
    int M;                // rows of di < 0 jobs
    int gather;           // source row of row p: token list[p] / k (1) or p (0)
    int k;
    const int *offs;      // [n_dense + 1] row offsets of the flagged experts
    const int *list;      // [rows] routed slot of each row
    // combine epilogue
    float *out;
    const void *weights;
    int w_type, d, wbd, per_slot;
};

__device__ __forceinline__ float2 load_w2(const void *w, int wt, int64_t i) {
    if (wt == LATENT_TYPE_F16) {
        const __half2 h = __ldg(reinterpret_cast<const __half2 *>(reinterpret_cast<const __half *>(w) + i));
        return __half22float2(h);
    }
    return __ldg(reinterpret_cast<const float2 *>(reinterpret_cast<const float *>(w) + i));
}

template <int XT, int RB>
__global__ void __launch_bounds__(128) k_rows_gemm(const __grid_constant__ DStage st) {
    const DJob &j = st.job[blockIdx.z];
    if ((int)blockIdx.x * kCols >= j.N) return;
    int r0 = 0, nr = st.M;
    if (j.di >= 0) {
        r0 = st.offs[j.di];
        nr = st.offs[j.di + 1] - r0;
    }
    __shared__ __align__(16) float xs[kKTile][RB];
    __shared__ int srow[RB];
    __shared__ int sslot[RB];
    const int c0 = blockIdx.x * kCols + threadIdx.x * 2;
    const bool live = c0 < j.N;
    for (int pb = blockIdx.y * RB; pb < nr; pb += gridDim.y * RB) {
        const int nrow = min(RB, nr - pb);
        __syncthreads();  // the previous chunk's readers of srow / xs
        if (threadIdx.x < RB) {
            const int p = r0 + pb + threadIdx.x;
            const bool in = threadIdx.x < nrow;
            const int slot = in && st.list ? st.list[p] : p;
            sslot[threadIdx.x] = in ? slot : -1;
            srow[threadIdx.x] = in ? (st.gather ? slot / st.k : p) : -1;
        }
        float acc[RB][2];
#pragma unroll
        for (int r = 0; r < RB; ++r) acc[r][0] = acc[r][1] = 0.f;
        for (int k0 = 0; k0 < j.K; k0 += kKTile) {
            __syncthreads();
            for (int i = threadIdx.x; i < kKTile * RB; i += 128) {
                const int rr = i / kKTile, kk = i % kKTile;
                const int row = srow[rr], kg = k0 + kk;
                float v = 0.f;
                if (row >= 0 && kg < j.K) v = load_act<XT>(j.src, (int64_t)row * j.lds + j.scol + kg);
                xs[kk][rr] = v;
            }
            __syncthreads();
            if (live) {
                const int kn = min(kKTile, j.K - k0);
                const int64_t wb = (int64_t)k0 * j.N + c0;
                float2 wv = load_w2(j.w, j.wt, wb);
                for (int kk = 0; kk < kn; ++kk) {
                    const float2 cur = wv;
                    if (kk + 1 < kn) wv = load_w2(j.w, j.wt, wb + (int64_t)(kk + 1) * j.N);
#pragma unroll
                    for (int r4 = 0; r4 < RB; r4 += 4) {
                        const float4 xv = *reinterpret_cast<const float4 *>(&xs[kk][r4]);
                        acc[r4 + 0][0] = fmaf(xv.x, cur.x, acc[r4 + 0][0]);
                        acc[r4 + 0][1] = fmaf(xv.x, cur.y, acc[r4 + 0][1]);
                        acc[r4 + 1][0] = fmaf(xv.y, cur.x, acc[r4 + 1][0]);
                        acc[r4 + 1][1] = fmaf(xv.y, cur.y, acc[r4 + 1][1]);
                        acc[r4 + 2][0] = fmaf(xv.z, cur.x, acc[r4 + 2][0]);
                        acc[r4 + 2][1] = fmaf(xv.z, cur.y, acc[r4 + 2][1]);
                        acc[r4 + 3][0] = fmaf(xv.w, cur.x, acc[r4 + 3][0]);
                        acc[r4 + 3][1] = fmaf(xv.w, cur.y, acc[r4 + 3][1]);
                    }
                }
            }
        }
        if (!live) continue;
#pragma unroll
        for (int r = 0; r < RB; ++r) {
            if (r >= nrow) break;
            const int p = r0 + pb + r;
            if (!j.combine) {
                *reinterpret_cast<float2 *>(j.dst + (int64_t)p * j.ldd + j.dcol + c0) =
                    make_float2(acc[r][0], acc[r][1]);
                continue;
            }
            const int slot = sslot[r];
            if (st.per_slot) {
                *reinterpret_cast<float2 *>(st.out + (int64_t)slot * st.d + c0) = make_float2(acc[r][0], acc[r][1]);
            } else {
                const float w = st.wbd ? 1.f : load_weight(st.weights, st.w_type, slot);
                float *o = st.out + (int64_t)(slot / st.k) * st.d + c0;
                atomicAdd(o, w * acc[r][0]);
                atomicAdd(o + 1, w * acc[r][1]);
            }
        }
    }
}

// Rows of the flagged experts: counts, offsets and the slot list (one block;
// the order within an expert is arrival order, which no result depends on
// beyond fp32 rounding of the combine), and the ids the latent op reads
// (flagged experts' slots set to -1).  dense_index[e] >= 0 flags expert e.
__global__ void __launch_bounds__(1024) k_dense_route(const int32_t *ids, int R, int E, const int32_t *dense_index,
                                                      int n_dense, int32_t *ids_latent, int *offs, int *list) {
    extern __shared__ int sh[];
    int *cnt = sh, *cur = sh + n_dense;
    for (int i = threadIdx.x; i < n_dense; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < R; i += blockDim.x) {
        const int e = ids[i];
        const int di = (e >= 0 && e < E) ? dense_index[e] : -1;
        if (di >= 0 && di < n_dense) atomicAdd(&cnt[di], 1);
        if (ids_latent) ids_latent[i] = (di >= 0 && di < n_dense) ? -1 : e;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0;
        for (int i = 0; i < n_dense; ++i) {
            offs[i] = s;
            cur[i] = s;
            s += cnt[i];
        }
        offs[n_dense] = s;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < R; i += blockDim.x) {
        const int e = ids[i];
        const int di = (e >= 0 && e < E) ? dense_index[e] : -1;
        if (di >= 0 && di < n_dense) list[atomicAdd(&cur[di], 1)] = i;
    }
}

// h = silu(g) * u (x the slot's router weight with weight_before_down), in
// place over g; rows [0, offs[n_dense]) of the row space, f columns.
__global__ void __launch_bounds__(256) k_dense_swiglu(float *g, const float *u, int64_t ld, int f, const int *offs,
                                                      int n_dense, const int *list, const void *weights, int w_type,
                                                      int wbd) {
    const int rows = offs[n_dense];
    const int64_t n = (int64_t)rows * f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = i / f, c = i - p * f;
        const float gv = g[p * ld + c];
        float h = gv / (1.f + expf(-gv)) * u[p * ld + c];
        if (wbd) h *= load_weight(weights, w_type, list[p]);
        g[p * ld + c] = h;
    }
}

template <int XT, int RB>
cudaError_t launch_gemm_t(const DStage &st, int max_n, int max_rows, cudaStream_t s) {
    const int gy = max(1, min(64, (max_rows + RB - 1) / RB));
    dim3 grid((max_n + kCols - 1) / kCols, gy, st.n_jobs);
    k_rows_gemm<XT, RB><<<grid, 128, 0, s>>>(st);
    return cudaGetLastError();
}

cudaError_t launch_gemm(const DStage &st, int xt, int max_n, int max_rows, cudaStream_t s) {
    if (st.n_jobs == 0 || max_rows == 0) return cudaSuccess;
    const bool small = max_rows <= 8;
    switch (xt) {
        case LATENT_TYPE_F32:
            return small ? launch_gemm_t<LATENT_TYPE_F32, 4>(st, max_n, max_rows, s)
                         : launch_gemm_t<LATENT_TYPE_F32, 16>(st, max_n, max_rows, s);
        case LATENT_TYPE_F16:
            return small ? launch_gemm_t<LATENT_TYPE_F16, 4>(st, max_n, max_rows, s)
                         : launch_gemm_t<LATENT_TYPE_F16, 16>(st, max_n, max_rows, s);
        default:
            return small ? launch_gemm_t<LATENT_TYPE_BF16, 4>(st, max_n, max_rows, s)
                         : launch_gemm_t<LATENT_TYPE_BF16, 16>(st, max_n, max_rows, s);
    }
}

}  // namespace

// Workspace of the dense-expert op: [offs (n_dense+1) | list (R) | T (R x 2r) | G (R x f) | U (R x f) | S (R x r)].
struct DenseLayout {
    size_t offs, list, t, g, u, s, total;
    int rmax;
};

static size_t align_up256(size_t v) { return (v + 255) & ~(size_t)255; }

static DenseLayout dense_layout(const latent_dense_desc *d) {
    DenseLayout L{};
    int rmax = 0;
    for (int i = 0; i < d->n_dense; ++i) rmax = d->experts[i].rank > rmax ? d->experts[i].rank : rmax;
    L.rmax = rmax;
    const size_t R = (size_t)d->n_tokens * d->top_k;
    size_t o = 0;
    L.offs = o;  o = align_up256(o + (size_t)(d->n_dense + 1) * 4);
    L.list = o;  o = align_up256(o + R * 4);
    L.t = o;     o = align_up256(o + R * 2 * rmax * 4);
    L.g = o;     o = align_up256(o + R * (size_t)d->n_ff * 4);
    L.u = o;     o = align_up256(o + R * (size_t)d->n_ff * 4);
    L.s = o;     o = align_up256(o + R * rmax * 4);
    L.total = o;
    return L;
}

int dense_validate(const latent_dense_desc *d, bool need_ptrs) {
    if (!d) return LATENT_ERR_INVALID;
    if (d->n_expert < 1 || d->n_expert > kMaxExperts) return LATENT_ERR_SHAPE;
    if (d->n_embd < 32 || d->n_embd % 32 || d->n_ff < 32 || d->n_ff % 32) return LATENT_ERR_SHAPE;
    if (d->n_tokens < 0 || d->top_k < 1 || (int64_t)d->n_tokens * d->top_k > ((int64_t)1 << 30)) return LATENT_ERR_SHAPE;
    if (d->n_dense < 0 || d->n_dense > d->n_expert) return LATENT_ERR_SHAPE;
    if (d->n_dense > 0 && !d->experts) return LATENT_ERR_INVALID;
    if (d->x_type != LATENT_TYPE_F32 && d->x_type != LATENT_TYPE_F16 && d->x_type != LATENT_TYPE_BF16)
        return LATENT_ERR_DTYPE;
    if (d->w_type != LATENT_TYPE_F32 && d->w_type != LATENT_TYPE_F16) return LATENT_ERR_DTYPE;
    if (d->dense_type != LATENT_TYPE_F32 && d->dense_type != LATENT_TYPE_F16) return LATENT_ERR_DTYPE;
    if (d->flags & ~(uint32_t)(LATENT_FLAG_WEIGHT_BEFORE_DOWN | LATENT_FLAG_OUT_PER_SLOT)) return LATENT_ERR_INVALID;
    for (int i = 0; i < d->n_dense; ++i) {
        const latent_dense_expert &x = d->experts[i];
        if (x.expert < 0 || x.expert >= d->n_expert) return LATENT_ERR_SHAPE;
        bool pair = false;
        for (int m = 0; m < 3; ++m) {
            if (x.dense[m]) continue;
            pair = true;
            if (need_ptrs && (!x.a[m] || !x.b[m])) return LATENT_ERR_INVALID;
        }
        if (pair && (x.rank < 2 || x.rank % 2 || x.rank > 4096)) return LATENT_ERR_SHAPE;
        if (need_ptrs)
            for (int m = 0; m < 3; ++m) {
                const void *p[3] = {x.dense[m], x.a[m], x.b[m]};
                for (const void *q : p)
                    if (q && (uintptr_t)q % 8) return LATENT_ERR_ALIGN;
            }
    }
    if (need_ptrs && d->n_tokens > 0) {
        if (!d->x || !d->ids || !d->weights || !d->out || !d->dense_index) return LATENT_ERR_INVALID;
        if ((uintptr_t)d->out % 8) return LATENT_ERR_ALIGN;
    }
    return LATENT_OK;
}

}  // namespace latent

using namespace latent;

namespace {

int dense_status(cudaError_t e) { return e == cudaSuccess ? LATENT_OK : LATENT_ERR_CUDA; }

template <class T>
T *ws_at(void *base, size_t off) {
    return reinterpret_cast<T *>(static_cast<char *>(base) + off);
}

int check_ws(const latent_dense_desc *d, const DenseLayout &L) {
    if (!d->workspace || d->workspace_bytes < L.total) return LATENT_ERR_WORKSPACE;
    if ((uintptr_t)d->workspace % 256) return LATENT_ERR_ALIGN;
    return LATENT_OK;
}

DStage stage_base(const latent_dense_desc *d, const DenseLayout &L, int gather) {
    DStage st;
    memset(&st, 0, sizeof(st));
    st.gather = gather;
    st.k = d->top_k;
    st.offs = ws_at<int>(d->workspace, L.offs);
    st.list = ws_at<int>(d->workspace, L.list);
    st.out = d->out;
    st.weights = d->weights;
    st.w_type = d->w_type;
    st.d = d->n_embd;
    st.wbd = (d->flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN) != 0;
    st.per_slot = (d->flags & LATENT_FLAG_OUT_PER_SLOT) != 0;
    return st;
}

DJob job(const void *w, int wt, int K, int N, const void *src, int64_t lds, int scol, float *dst, int64_t ldd,
         int dcol, int di, int combine) {
    DJob j;
    j.w = w;
    j.wt = wt;
    j.K = K;
    j.N = N;
    j.src = src;
    j.lds = lds;
    j.scol = scol;
    j.dst = dst;
    j.ldd = ldd;
    j.dcol = dcol;
    j.di = di;
    j.combine = combine;
    return j;
}

// Adds job j to the stage, launching the stage first when it is full.
int push(DStage &st, const DJob &j, int &max_n, int xt, int rows, cudaStream_t s) {
    if (st.n_jobs == kJobs) {
        const int e = dense_status(launch_gemm(st, xt, max_n, rows, s));
        if (e) return e;
        st.n_jobs = 0;
        max_n = 0;
    }
    st.job[st.n_jobs++] = j;
    max_n = j.N > max_n ? j.N : max_n;
    return LATENT_OK;
}

int flush(DStage &st, int &max_n, int xt, int rows, cudaStream_t s) {
    const int e = dense_status(launch_gemm(st, xt, max_n, rows, s));
    st.n_jobs = 0;
    max_n = 0;
    return e;
}

}  // namespace

extern "C" LATENT_API int latent_dense_workspace_size(const latent_dense_desc *desc, size_t *bytes) {
    if (!bytes) return LATENT_ERR_INVALID;
    const int st = dense_validate(desc, false);
    if (st) return st;
    *bytes = (desc->n_tokens == 0 || desc->n_dense == 0) ? 256 : dense_layout(desc).total;
    return LATENT_OK;
}

extern "C" LATENT_API int latent_dense_experts_prepare(const latent_dense_desc *d, int32_t *ids_latent,
                                                       CUstream_st *stream) {
    int st = dense_validate(d, true);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int R = d->n_tokens * d->top_k;
    if (R == 0) return LATENT_OK;
    if (!ids_latent) return LATENT_ERR_INVALID;
    if (d->n_dense == 0)
        return dense_status(cudaMemcpyAsync(ids_latent, d->ids, (size_t)R * 4, cudaMemcpyDeviceToDevice, s));
    const DenseLayout L = dense_layout(d);
    if ((st = check_ws(d, L))) return st;
    k_dense_route<<<1, 1024, (size_t)2 * d->n_dense * sizeof(int), s>>>(
        d->ids, R, d->n_expert, d->dense_index, d->n_dense, ids_latent, ws_at<int>(d->workspace, L.offs),
        ws_at<int>(d->workspace, L.list));
    return dense_status(cudaGetLastError());
}

extern "C" LATENT_API int latent_dense_experts_forward(const latent_dense_desc *d, CUstream_st *stream) {
    int st = dense_validate(d, true);
    if (st) return st;
    const int R = d->n_tokens * d->top_k;
    if (R == 0 || d->n_dense == 0) return LATENT_OK;
    const DenseLayout L = dense_layout(d);
    if ((st = check_ws(d, L))) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int dd = d->n_embd, f = d->n_ff, rm = L.rmax, dt = d->dense_type;
    float *T = ws_at<float>(d->workspace, L.t), *G = ws_at<float>(d->workspace, L.g);
    float *U = ws_at<float>(d->workspace, L.u), *S = ws_at<float>(d->workspace, L.s);
    int max_n = 0;
    // x -> G | U (dense kinds) or x -> T (pairs); then T -> G | U
    DStage st1 = stage_base(d, L, 1);
    for (int i = 0; i < d->n_dense; ++i) {
        const latent_dense_expert &e = d->experts[i];
        for (int m = 0; m < 2; ++m) {
            float *gu = m == 0 ? G : U;
            const DJob j = e.dense[m] ? job(e.dense[m], dt, dd, f, d->x, dd, 0, gu, f, 0, i, 0)
                                      : job(e.a[m], LATENT_TYPE_F32, dd, e.rank, d->x, dd, 0, T, 2 * rm, m * e.rank, i, 0);
            if ((st = push(st1, j, max_n, d->x_type, R, s))) return st;
        }
    }
    if ((st = flush(st1, max_n, d->x_type, R, s))) return st;
    DStage st2 = stage_base(d, L, 0);
    for (int i = 0; i < d->n_dense; ++i) {
        const latent_dense_expert &e = d->experts[i];
        for (int m = 0; m < 2; ++m) {
            if (e.dense[m]) continue;
            const DJob j = job(e.b[m], LATENT_TYPE_F32, e.rank, f, T, 2 * rm, m * e.rank, m == 0 ? G : U, f, 0, i, 0);
            if ((st = push(st2, j, max_n, LATENT_TYPE_F32, R, s))) return st;
        }
    }
    if ((st = flush(st2, max_n, LATENT_TYPE_F32, R, s))) return st;
    {
        const int64_t n = (int64_t)R * f;
        const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
        k_dense_swiglu<<<blocks, 256, 0, s>>>(G, U, f, f, st2.offs, d->n_dense, st2.list, d->weights, d->w_type,
                                              st2.wbd);
        if ((st = dense_status(cudaGetLastError()))) return st;
    }
    // H -> combine (dense down) or H -> S; then S -> combine
    DStage st4 = stage_base(d, L, 0);
    for (int i = 0; i < d->n_dense; ++i) {
        const latent_dense_expert &e = d->experts[i];
        const DJob j = e.dense[2] ? job(e.dense[2], dt, f, dd, G, f, 0, nullptr, 0, 0, i, 1)
                                  : job(e.a[2], LATENT_TYPE_F32, f, e.rank, G, f, 0, S, rm, 0, i, 0);
        if ((st = push(st4, j, max_n, LATENT_TYPE_F32, R, s))) return st;
    }
    if ((st = flush(st4, max_n, LATENT_TYPE_F32, R, s))) return st;
    DStage st5 = stage_base(d, L, 0);
    for (int i = 0; i < d->n_dense; ++i) {
        const latent_dense_expert &e = d->experts[i];
        if (e.dense[2]) continue;
        const DJob j = job(e.b[2], LATENT_TYPE_F32, e.rank, dd, S, rm, 0, nullptr, 0, 0, i, 1);
        if ((st = push(st5, j, max_n, LATENT_TYPE_F32, R, s))) return st;
    }
    return flush(st5, max_n, LATENT_TYPE_F32, R, s);
}

extern "C" LATENT_API int latent_dense_matmul(const void *x, int32_t x_type, const void *w, int32_t w_type, float *y,
                                              int64_t M, int64_t K, int64_t N, CUstream_st *stream) {
    if (M < 0 || K < 0 || N < 0) return LATENT_ERR_INVALID;
    if (M > INT32_MAX || K > INT32_MAX || N > INT32_MAX || K % 2 || N % 2) return LATENT_ERR_SHAPE;
    if (x_type != LATENT_TYPE_F32 && x_type != LATENT_TYPE_F16 && x_type != LATENT_TYPE_BF16) return LATENT_ERR_DTYPE;
    if (w_type != LATENT_TYPE_F32 && w_type != LATENT_TYPE_F16) return LATENT_ERR_DTYPE;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (M == 0 || N == 0) return LATENT_OK;
    if (!x || !w || !y) return LATENT_ERR_INVALID;
    if ((uintptr_t)w % 8 || (uintptr_t)y % 8) return LATENT_ERR_ALIGN;
    if (K == 0) return dense_status(cudaMemsetAsync(y, 0, (size_t)M * N * 4, s));
    DStage st;
    memset(&st, 0, sizeof(st));
    st.M = (int)M;
    st.job[0] = job(w, w_type, (int)K, (int)N, x, K, 0, y, N, 0, -1, 0);
    st.n_jobs = 1;
    return dense_status(launch_gemm(st, x_type, (int)N, (int)M, s));
}
