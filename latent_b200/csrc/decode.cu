// Decode path: the latent expert FFN as a chain of quantized vector-matrix
// products on CUDA cores with fp32 accumulation (rel-L2 <= 1e-5 vs the
// fp32 reference runtime, loader/latent_runtime.py:35-59).
//
// Per active expert e with n_e routed tokens (contiguous routed positions):
//   phase 1  t = x . [A_g | A_u]        K = d split in ks1 row chunks (split-K)
//   phase 2  h = silu(t_g . B_g) * (t_u . B_u) [* w]   column tiles of f
//   phase 3  s = h . A_d                K = f split in ks2 row chunks
//   phase 4  y = s . B_d                column tiles of d
//   combine  out[t] = sum_j w_tj * y_(t,j)  in slot order
// Split-K partials are summed in chunk order by the last CTA that finishes
// an expert (arrival counter, no waiting), so results are deterministic.
//
// Every factor element is read from HBM exactly once per call (per token
// chunk of up to 4 tokens).  A lane owns 16 consecutive columns of a row
// (8 code bytes, half of one 32-element scale group): it decodes each 4-bit
// code through a 16-entry shared-memory table (the 16 entries sit in 16
// distinct banks, so a warp's lookup is one wavefront) and accumulates
// x*scale*level with packed fp32x2 FMAs.
#include "internal.h"

namespace latent {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileN = 256;  // output columns per tile on the output side

__device__ __forceinline__ void fma2(float &a0, float &a1, float x, float v0, float v1) {
    unsigned long long acc, xx, vv;
    asm("mov.b64 %0, {%1,%2};" : "=l"(acc) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1,%1};" : "=l"(xx) : "f"(x));
    asm("mov.b64 %0, {%1,%2};" : "=l"(vv) : "f"(v0), "f"(v1));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(xx), "l"(vv));
    asm("mov.b64 {%0,%1}, %2;" : "=f"(a0), "=f"(a1) : "l"(acc));
}

__device__ __forceinline__ uint2 ldg_stream_v2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// One row of a lane's 16 columns: acc[t][j] += in[t] * scale * value(j).
template <int NT>
__device__ __forceinline__ void row_fma(const QView &M, int64_t group, int half, uint2 q, uint16_t sbits,
                                        const float *xin, int xstride, const float *lut, float (&acc)[NT][16]) {
    const float sc = half_bits_to_float(sbits);
    float xs[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) xs[t] = xin[t * xstride] * sc;
    uint32_t idx;
    if (M.i8.present() && M.i8.is_int8(group, &idx)) {
        const uint2 hi = *reinterpret_cast<const uint2 *>(M.i8.hi + (int64_t)idx * 16 + half * 8);
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint32_t lo_w = w ? q.y : q.x, hi_w = w ? hi.y : hi.x;
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const float v0 = int8_elem(lo_w, hi_w, i), v1 = int8_elem(lo_w, hi_w, i + 1);
#pragma unroll
                for (int t = 0; t < NT; ++t) fma2(acc[t][8 * w + i], acc[t][8 * w + i + 1], xs[t], v0, v1);
            }
        }
        return;
    }
#pragma unroll
    for (int w = 0; w < 2; ++w) {
        const uint32_t word = w ? q.y : q.x;
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            const float v0 = lut[(word >> (4 * i)) & 15u];
            const float v1 = lut[(word >> (4 * i + 4)) & 15u];
#pragma unroll
            for (int t = 0; t < NT; ++t) fma2(acc[t][8 * w + i], acc[t][8 * w + i + 1], xs[t], v0, v1);
        }
    }
}

// Accumulates rows [row0, row_end) x columns [col0, col0+ncols) of M against
// in_s[t * in_ld + (row - row0)] into the calling lane's 16-column slice.
// Lanes: LPR lanes span a row (16 columns each), 32/LPR rows per warp step.
template <int LPR, int NT>
__device__ __forceinline__ void vecmat_accum(const QView &M, int row0, int row_end, int col0, int ncols,
                                             const float *in_s, int in_ld, const float *lut,
                                             float (&acc)[NT][16]) {
    constexpr int RPW = 32 / LPR;
    constexpr int STEP = kWarps * RPW;
    constexpr int U = 4;
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[t][j] = 0.f;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cl = (lane % LPR) * 16;
    if (cl >= ncols) return;
    const int c = col0 + cl;
    const int64_t rb = M.cols >> 1, gpr = M.cols >> 5;
    const uint8_t *cp = M.codes + (c >> 1);
    const uint16_t *sp = M.scales + (c >> 5);
    const int half = (c >> 4) & 1;
    int row = row0 + warp * RPW + lane / LPR;
    for (; row + (U - 1) * STEP < row_end; row += U * STEP) {
        uint2 q[U];
        uint16_t sb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            q[u] = ldg_stream_v2(cp + (int64_t)(row + u * STEP) * rb);
            sb[u] = __ldg(sp + (int64_t)(row + u * STEP) * gpr);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int rr = row + u * STEP;
            row_fma<NT>(M, (int64_t)rr * gpr + (c >> 5), half, q[u], sb[u], in_s + (rr - row0), in_ld, lut, acc);
        }
    }
    for (; row < row_end; row += STEP) {
        const uint2 q = ldg_stream_v2(cp + (int64_t)row * rb);
        const uint16_t sb = __ldg(sp + (int64_t)row * gpr);
        row_fma<NT>(M, (int64_t)row * gpr + (c >> 5), half, q, sb, in_s + (row - row0), in_ld, lut, acc);
    }
}

// Sums the lanes that share columns (across the 32/LPR row lanes of a warp,
// then across warps through red_s[kWarps][NT][LPR*16]).  After the call,
// red_s[0..NT*ncols) -- indexed t * (LPR*16) + col -- holds the CTA's sums.
template <int LPR, int NT>
__device__ __forceinline__ void cta_reduce(float (&acc)[NT][16], int ncols, float *red_s) {
    constexpr int W = LPR * 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[t][j] += __shfl_xor_sync(0xffffffffu, acc[t][j], o);
    const int cl = lane * 16;
    if (lane < LPR && cl < ncols) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float4 *dst = reinterpret_cast<float4 *>(red_s + (warp * NT + t) * W + cl);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                dst[j] = make_float4(acc[t][4 * j], acc[t][4 * j + 1], acc[t][4 * j + 2], acc[t][4 * j + 3]);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NT * W; i += kThreads) {
        const int col = i % W;
        float v = 0.f;
        if (col < ncols) {
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += red_s[w * NT * W + i];
        }
        red_s[kWarps * NT * W + i] = v;
    }
    __syncthreads();
}

__device__ __forceinline__ void init_lut(float *lut) {
    if (threadIdx.x < 16) lut[threadIdx.x] = kNF4Levels[threadIdx.x];
}

}  // namespace

namespace {

// Runs one token chunk of the input side (split-K) and stores the chunk's
// partial sums; NT is picked at run time from the chunk size.
template <int LPR, int NT>
__device__ __forceinline__ void in_chunk(const QView &M, int row0, int row_end, int r, const float *in_s, int kc,
                                         const float *lut, float *red_s, float *part_rows, int ldo) {
    float acc[NT][16];
    vecmat_accum<LPR, NT>(M, row0, row_end, 0, r, in_s, kc, lut, acc);
    cta_reduce<LPR, NT>(acc, r, red_s);
    const float *res = red_s + kWarps * NT * r;
    for (int i = threadIdx.x; i < NT * r; i += kThreads) {
        const int t = i / r, col = i - t * r;
        part_rows[(int64_t)t * ldo + col] = res[i];
    }
}

// Phases 1 and 3: t = x.[A_g|A_u] (PH=1) or s = h.A_d (PH=3), split-K.
template <int LPR, int XT, int PH>
__global__ void __launch_bounds__(kThreads) k_in_phase(DecodeArgs a) {
    extern __shared__ float sm[];
    __shared__ int s_last;
    constexpr int nmat = PH == 1 ? 2 : 1;
    const int kc = PH == 1 ? a.kc1 : a.kc2;
    const int ks = PH == 1 ? a.ks1 : a.ks2;
    const int r = a.r;
    float *lut = sm;
    float *in_s = sm + 32;
    float *red_s = in_s + 4 * kc;
    int w = blockIdx.x;
    const int ksel = w % ks;
    w /= ks;
    const int m = w % nmat;
    const int ai = w / nmat;
    init_lut(lut);
    if (ai >= *a.rt.n_active) return;
    const int e = a.rt.active[ai];
    const int p0 = a.rt.offsets[e], ne = a.rt.offsets[e + 1] - p0;
    const latent_qmatrix &qm = PH == 1 ? (m == 0 ? a.gate_a : a.up_a) : a.down_a;
    const QView M = expert_view(qm, e);
    const int row0 = ksel * kc, row_end = min(M.rows, row0 + kc);
    const int ldo = nmat * r;
    float *part = PH == 1 ? a.part1 : a.part2;
    for (int tc = 0; tc < ne; tc += 4) {
        const int nt = min(4, ne - tc);
        __syncthreads();
        for (int i = threadIdx.x; i < nt * kc; i += kThreads) {
            const int t = i / kc, rr = i - t * kc, row = row0 + rr;
            float v = 0.f;
            if (row < row_end) {
                const int p = p0 + tc + t;
                if constexpr (PH == 1) {
                    const int tok = a.rt.order[p] / a.k;
                    v = load_act<XT>(a.x, (int64_t)tok * a.d + row);
                } else {
                    v = a.h[(int64_t)p * a.f + row];
                }
            }
            in_s[i] = v;
        }
        __syncthreads();
        float *rows = part + ((int64_t)ksel * a.R + p0 + tc) * ldo + m * r;
        if (nt == 1)
            in_chunk<LPR, 1>(M, row0, row_end, r, in_s, kc, lut, red_s, rows, ldo);
        else if (nt == 2)
            in_chunk<LPR, 2>(M, row0, row_end, r, in_s, kc, lut, red_s, rows, ldo);
        else if (nt == 3)
            in_chunk<LPR, 3>(M, row0, row_end, r, in_s, kc, lut, red_s, rows, ldo);
        else
            in_chunk<LPR, 4>(M, row0, row_end, r, in_s, kc, lut, red_s, rows, ldo);
    }
    // Arrival: the last CTA of this expert sums the split-K partials in order.
    __threadfence();
    __syncthreads();
    uint32_t *sem = a.rt.sem + (PH == 1 ? 0 : a.E) + e;
    if (threadIdx.x == 0) s_last = atomicAdd(sem, 1u) == (uint32_t)(nmat * ks - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    float *outv = PH == 1 ? a.t : a.s;
    for (int i = threadIdx.x; i < ne * ldo; i += kThreads) {
        const int pp = p0 + i / ldo, col = i % ldo;
        float v = 0.f;
        for (int q = 0; q < ks; ++q) v += __ldcg(part + ((int64_t)q * a.R + pp) * ldo + col);
        outv[(int64_t)pp * ldo + col] = v;
    }
    if (threadIdx.x == 0) *sem = 0u;
}

template <int NT>
__device__ __forceinline__ void gateup_chunk(const DecodeArgs &a, const QView &Mg, const QView &Mu, int col0,
                                             int ncols, int p, const float *in_g, const float *in_u,
                                             const float *lut, float *red_s, float *g_s) {
    constexpr int W = kTileN;
    const int r = a.r;
    float acc[NT][16];
    vecmat_accum<16, NT>(Mg, 0, r, col0, ncols, in_g, r, lut, acc);
    cta_reduce<16, NT>(acc, ncols, red_s);
    const float *res = red_s + kWarps * NT * W;
    for (int i = threadIdx.x; i < NT * W; i += kThreads) g_s[i] = res[i];
    __syncthreads();
    vecmat_accum<16, NT>(Mu, 0, r, col0, ncols, in_u, r, lut, acc);
    cta_reduce<16, NT>(acc, ncols, red_s);
    const bool wbd = a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN;
    for (int i = threadIdx.x; i < NT * W; i += kThreads) {
        const int t = i / W, col = i - t * W;
        if (col >= ncols) continue;
        float hv = silu_f32(g_s[i]) * res[i];
        if (wbd) hv *= load_weight(a.weights, a.w_type, a.rt.order[p + t]);
        a.h[(int64_t)(p + t) * a.f + col0 + col] = hv;
    }
}

// Phase 2: h = silu(t_g.B_g) * (t_u.B_u) [* w], one 256-column tile of f.
__global__ void __launch_bounds__(kThreads) k_gateup_out(DecodeArgs a) {
    extern __shared__ float sm[];
    const int r = a.r;
    float *lut = sm;
    float *in_g = sm + 32;
    float *in_u = in_g + 4 * r;
    float *red_s = in_u + 4 * r;
    float *g_s = red_s + (kWarps + 1) * 4 * kTileN;
    const int nct = (a.f + kTileN - 1) / kTileN;
    const int ct = blockIdx.x % nct, ai = blockIdx.x / nct;
    init_lut(lut);
    if (ai >= *a.rt.n_active) return;
    const int e = a.rt.active[ai];
    const int p0 = a.rt.offsets[e], ne = a.rt.offsets[e + 1] - p0;
    const QView Mg = expert_view(a.gate_b, e), Mu = expert_view(a.up_b, e);
    const int col0 = ct * kTileN, ncols = min(kTileN, a.f - col0);
    for (int tc = 0; tc < ne; tc += 4) {
        const int nt = min(4, ne - tc);
        __syncthreads();
        for (int i = threadIdx.x; i < nt * r; i += kThreads) {
            const int t = i / r, kk = i - t * r;
            const float *src = a.t + (int64_t)(p0 + tc + t) * 2 * r;
            in_g[i] = src[kk];
            in_u[i] = src[r + kk];
        }
        __syncthreads();
        const int p = p0 + tc;
        if (nt == 1)
            gateup_chunk<1>(a, Mg, Mu, col0, ncols, p, in_g, in_u, lut, red_s, g_s);
        else if (nt == 2)
            gateup_chunk<2>(a, Mg, Mu, col0, ncols, p, in_g, in_u, lut, red_s, g_s);
        else if (nt == 3)
            gateup_chunk<3>(a, Mg, Mu, col0, ncols, p, in_g, in_u, lut, red_s, g_s);
        else
            gateup_chunk<4>(a, Mg, Mu, col0, ncols, p, in_g, in_u, lut, red_s, g_s);
    }
}

template <int NT>
__device__ __forceinline__ void down_chunk(const DecodeArgs &a, const QView &M, int col0, int ncols, int p,
                                           const float *in_s, const float *lut, float *red_s) {
    constexpr int W = kTileN;
    float acc[NT][16];
    vecmat_accum<16, NT>(M, 0, a.r, col0, ncols, in_s, a.r, lut, acc);
    cta_reduce<16, NT>(acc, ncols, red_s);
    const float *res = red_s + kWarps * NT * W;
    const bool per_slot = a.flags & LATENT_FLAG_OUT_PER_SLOT;
    for (int i = threadIdx.x; i < NT * W; i += kThreads) {
        const int t = i / W, col = i - t * W;
        if (col >= ncols) continue;
        if (per_slot)
            a.out[(int64_t)a.rt.order[p + t] * a.d + col0 + col] = res[i];
        else
            a.y[(int64_t)(p + t) * a.d + col0 + col] = res[i];
    }
}

// Phase 4: y = s.B_d, one 256-column tile of d.
__global__ void __launch_bounds__(kThreads) k_down_out(DecodeArgs a) {
    extern __shared__ float sm[];
    const int r = a.r;
    float *lut = sm;
    float *in_s = sm + 32;
    float *red_s = in_s + 4 * r;
    const int nct = (a.d + kTileN - 1) / kTileN;
    const int ct = blockIdx.x % nct, ai = blockIdx.x / nct;
    init_lut(lut);
    if (ai >= *a.rt.n_active) return;
    const int e = a.rt.active[ai];
    const int p0 = a.rt.offsets[e], ne = a.rt.offsets[e + 1] - p0;
    const QView M = expert_view(a.down_b, e);
    const int col0 = ct * kTileN, ncols = min(kTileN, a.d - col0);
    for (int tc = 0; tc < ne; tc += 4) {
        const int nt = min(4, ne - tc);
        __syncthreads();
        for (int i = threadIdx.x; i < nt * r; i += kThreads) {
            const int t = i / r, kk = i - t * r;
            in_s[i] = a.s[(int64_t)(p0 + tc + t) * r + kk];
        }
        __syncthreads();
        const int p = p0 + tc;
        if (nt == 1)
            down_chunk<1>(a, M, col0, ncols, p, in_s, lut, red_s);
        else if (nt == 2)
            down_chunk<2>(a, M, col0, ncols, p, in_s, lut, red_s);
        else if (nt == 3)
            down_chunk<3>(a, M, col0, ncols, p, in_s, lut, red_s);
        else
            down_chunk<4>(a, M, col0, ncols, p, in_s, lut, red_s);
    }
}

// Top-k combine in slot order (or zero rows of skipped slots in per-slot mode).
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

int round_up(int x, int m) { return (x + m - 1) / m * m; }

void plan_split(int K, int nmax, int nmat, int step, int &kc, int &ks) {
    const int target = 2 * 148;
    int want = (target + nmax * nmat - 1) / (nmax * nmat);
    want = want < 1 ? 1 : want;
    const int unit = step > 64 ? step : 64;
    kc = round_up((K + want - 1) / want, unit);
    if (kc > 1024) kc = 1024;
    if (kc < unit) kc = unit;
    ks = (K + kc - 1) / kc;
}

template <int LPR>
cudaError_t launch_in_phases(const DecodeArgs &a, int ph, cudaStream_t s) {
    const size_t smem = (32 + 4 * (ph == 1 ? a.kc1 : a.kc2) + (kWarps + 1) * 4 * a.r) * sizeof(float);
    const int grid = a.nmax * (ph == 1 ? 2 * a.ks1 : a.ks2);
    const void *fn;
    if (ph == 1) {
        switch (a.x_type) {
            case LATENT_TYPE_F32: fn = (const void *)k_in_phase<LPR, LATENT_TYPE_F32, 1>; break;
            case LATENT_TYPE_F16: fn = (const void *)k_in_phase<LPR, LATENT_TYPE_F16, 1>; break;
            default: fn = (const void *)k_in_phase<LPR, LATENT_TYPE_BF16, 1>; break;
        }
    } else {
        fn = (const void *)k_in_phase<LPR, LATENT_TYPE_F32, 3>;
    }
    cudaError_t err = ensure_smem(fn, smem);
    if (err != cudaSuccess) return err;
    void *args[] = {(void *)&a};
    return cudaLaunchKernel(fn, dim3(grid), dim3(kThreads), args, smem, s);
}

cudaError_t launch_in(const DecodeArgs &a, int ph, cudaStream_t s) {
    switch (a.r) {
        case 32: return launch_in_phases<2>(a, ph, s);
        case 64: return launch_in_phases<4>(a, ph, s);
        case 128: return launch_in_phases<8>(a, ph, s);
        case 256: return launch_in_phases<16>(a, ph, s);
        case 512: return launch_in_phases<32>(a, ph, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

void decode_plan(DecodeArgs &a) {
    a.R = a.T * a.k;
    a.nmax = a.E < a.R ? a.E : a.R;
    if (a.nmax < 1) {  // empty batch: nothing is launched
        a.kc1 = a.kc2 = 64;
        a.ks1 = a.ks2 = 1;
        return;
    }
    const int lpr = a.r / 16;
    const int step = kWarps * (32 / (lpr > 32 ? 32 : lpr));
    plan_split(a.d, a.nmax, 2, step, a.kc1, a.ks1);
    plan_split(a.f, a.nmax, 1, step, a.kc2, a.ks2);
}

size_t decode_scratch_floats(const DecodeArgs &a) {
    const size_t R = (size_t)a.R, r = (size_t)a.r;
    return (size_t)a.ks1 * R * 2 * r + R * 2 * r + R * (size_t)a.f + (size_t)a.ks2 * R * r + R * r +
           R * (size_t)a.d + 6 * 64;
}

cudaError_t launch_decode(const DecodeArgs &a, cudaStream_t s, Marks *marks) {
    Marks none;
    Marks &m = marks ? *marks : none;
    cudaError_t err;
    if ((err = launch_in(a, 1, s)) != cudaSuccess) return err;
    m.mark(s);
    {
        const size_t smem = (32 + 8 * a.r + (kWarps + 1) * 4 * kTileN + 4 * kTileN) * sizeof(float);
        if ((err = ensure_smem((const void *)k_gateup_out, smem)) != cudaSuccess) return err;
        const int grid = a.nmax * ((a.f + kTileN - 1) / kTileN);
        k_gateup_out<<<grid, kThreads, smem, s>>>(a);
        if ((err = cudaGetLastError()) != cudaSuccess) return err;
    }
    m.mark(s);
    if ((err = launch_in(a, 3, s)) != cudaSuccess) return err;
    m.mark(s);
    {
        const size_t smem = (32 + 4 * a.r + (kWarps + 1) * 4 * kTileN) * sizeof(float);
        if ((err = ensure_smem((const void *)k_down_out, smem)) != cudaSuccess) return err;
        const int grid = a.nmax * ((a.d + kTileN - 1) / kTileN);
        k_down_out<<<grid, kThreads, smem, s>>>(a);
        if ((err = cudaGetLastError()) != cudaSuccess) return err;
    }
    m.mark(s);
    dim3 grid((a.d / 4 + 255) / 256, a.T);
    k_combine<<<grid, 256, 0, s>>>(a);
    err = cudaGetLastError();
    m.mark(s);
    return err;
}

}  // namespace latent

namespace latent {

cudaError_t launch_combine(const DecodeArgs &a, cudaStream_t s) {
    if (a.T == 0) return cudaSuccess;
    dim3 grid((a.d / 4 + 255) / 256, a.T);
    k_combine<<<grid, 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace latent
