// Decode path: the latent expert FFN as a chain of quantized vector-matrix
// products on CUDA cores with fp32 accumulation (rel-L2 <= 1e-5 vs the fp32
// reference runtime, loader/latent_runtime.py:35-59).
//
// One persistent, cooperatively launched kernel runs the whole chain.  Work
// items are handed out in phase order by an atomic counter:
//   phase 1  t = x . [A_g | A_u]   item = (expert, matrix, row chunk of d)  split-K
//   phase 2  h = silu(t_g.B_g) * (t_u.B_u) [* w]   item = (expert, 256-column tile of f)
//   phase 3  s = h . A_d           item = (expert, row chunk of f)          split-K
//   phase 4  y = s . B_d           item = (expert, 256-column tile of d), fused top-k combine
// An item waits (bounded) only for its own expert's previous phase:
// phase-1/3 partial sums are reduced in chunk order by the last item to
// arrive (arrival counter), which then publishes a ready flag; phase 3 waits
// for all phase-2 tiles of its expert; the last phase-4 tile to finish a
// (token, column tile) sums that token's top-k rows in slot order.  Items are
// handed out in phase order and every CTA is resident (cooperative launch),
// so every wait ends; a wait that exceeds its bound sets kErrTimeout and the
// kernel runs to completion without waiting further.  Results are bitwise
// deterministic.
//
// Inner loop: codes and scales stream through a 4-deep cp.async ring in
// shared memory (memory parallelism independent of registers).  A lane owns
// 16 consecutive columns of a row (8 code bytes, half a 32-element scale
// group), turns codes into table byte offsets with one shift and one
// and-or per 8 codes, looks each value up in a shared table and accumulates
// x*scale*value with packed fp32x2 FMAs on 64-bit accumulators.  The table
// has the 16 NF4 levels in banks 0-15 and the identity 0..15 in banks 16-31;
// the sign bit of a group's scale (set for INT8 groups) selects the second,
// so a warp lookup is one wavefront and INT8 groups cost the hot loop nothing
// extra.  The INT8 high nibbles are added afterwards to the CTA's reduced
// tile (int8_fix), in a fixed order.
#include "internal.h"

namespace latent {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileN = 256;  // output columns per tile on the output side
constexpr unsigned long long kWaitNs = 2000000000ull;  // a dependency wait gives up after 2 s

typedef unsigned long long u64;

__device__ __forceinline__ u64 pack2(float a, float b) {
    u64 r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ void unpack2(u64 v, float &a, float &b) {
    asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}

__device__ __forceinline__ void ffma2(u64 &acc, u64 x, u64 v) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(x), "l"(v));
}

__device__ __forceinline__ float lut_at(const float *lut, uint32_t byte_off) {
    return *reinterpret_cast<const float *>(reinterpret_cast<const char *>(lut) + byte_off);
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int b) { return __byte_perm(w, 0u, 0x4440u | b); }

// Bounded wait until *flag >= target (thread 0 of the CTA only).  Returns
// false (and records kErrTimeout) when the bound is exceeded or another CTA
// already gave up.
__device__ bool wait_ge(const uint32_t *flag, uint32_t target, uint32_t *err) {
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    unsigned ns = 32;
    while (true) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v >= target) return true;
        uint32_t e;
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(e) : "l"(err) : "memory");
        if (e & kErrTimeout) return false;
        unsigned long long now;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
        if (now - t0 > kWaitNs) {
            atomicOr(err, kErrTimeout);
            return false;
        }
        __nanosleep(ns);
        if (ns < 1024) ns <<= 1;
    }
}

// cp.async (LDGSTS) helpers.
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void cp_async16(void *s, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(s)), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async4(void *s, const void *g) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(s)), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int kStages = 4;
constexpr int kWarpStageCode = 1024;  // code bytes per warp per stage
constexpr int kWarpStageScale = 256;  // scale bytes per warp per stage
constexpr int kWarpStageBytes = kWarpStageCode + kWarpStageScale;
constexpr int kWarpRing = kStages * kWarpStageBytes;
constexpr int kStageBytes = kWarps * kWarpRing / kStages;  // per-CTA bytes of one stage (all warps)

// One staged row of a lane's 16 columns: acc[t][p] (columns 2p, 2p+1) += in[t]*scale*table[code].
// `tsel` adds 64 bytes to every table offset: the identity table that decodes
// the low nibble of an INT8 group (its high nibble is added by int8_fix).
template <int NT>
__device__ __forceinline__ void row_fma(uint2 q, uint32_t tsel, float sc, const float *xin, int xstride,
                                        const float *lut, u64 (&acc)[NT][8]) {
    u64 xs[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const float v = xin[t * xstride] * sc;
        xs[t] = pack2(v, v);
    }
#pragma unroll
    for (int w2 = 0; w2 < 2; ++w2) {
        const uint32_t word = w2 ? q.y : q.x;
        const uint32_t e4 = ((word << 2) & 0x3C3C3C3Cu) | tsel;  // even columns: table byte offsets
        const uint32_t o4 = ((word >> 2) & 0x3C3C3C3Cu) | tsel;  // odd columns
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const u64 vv = pack2(lut_at(lut, byte_of(e4, j)), lut_at(lut, byte_of(o4, j)));
#pragma unroll
            for (int t = 0; t < NT; ++t) ffma2(acc[t][4 * w2 + j], xs[t], vv);
        }
    }
}

// Accumulates rows [row0, row_end) x columns [col0, col0+ncols) of M against
// in_s[t * in_ld + (row - row0)] into the calling lane's 16-column slice.
// Each warp streams its own contiguous share of the rows through a private
// kStages-deep cp.async ring in `stages` (kWarpRing bytes per warp), so the
// loop synchronises only within the warp.  LPR lanes span a row (16 columns
// each), 32/LPR rows per warp step.  All threads of the CTA must call it.
// phase: kFull (prologue + loop), kPrologue (issue the first kStages-1
// stages and return: lets an item start streaming weights before it waits for
// its inputs), kLoop (the rest; the same geometry's prologue was issued).
enum : int { kFull = 0, kPrologue = 1, kLoop = 2 };

template <int LPR, int NT, int PHASE = kFull>
__device__ __forceinline__ void vecmat_staged(const QView &M, int row0, int row_end, int col0, int ncols,
                                              const float *in_s, int in_ld, const float *lut, uint8_t *stages,
                                              u64 (&acc)[NT][8]) {
    constexpr int RPW = 32 / LPR;
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[t][j] = 0ull;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cb = ncols >> 1, ng = ncols >> 5;
    const int spitch = (ng * 2 + 3) & ~3;
    // this warp's rows: a multiple of RPW
    const int nrows = row_end - row0;
    const int per = (nrows + kWarps * RPW - 1) / (kWarps * RPW) * RPW;
    const int wr0 = row0 + warp * per, wr1 = min(row_end, wr0 + per);
    uint8_t *ring = stages + warp * kWarpRing;
    int SR = kWarpStageCode / cb;
    if (SR * spitch > kWarpStageScale) SR = kWarpStageScale / spitch;
    SR = SR / RPW * RPW;
    const int nst = wr1 > wr0 ? (wr1 - wr0 + SR - 1) / SR : 0;
    const int64_t rb = M.cols >> 1, gpr = M.cols >> 5;
    const bool sc4 = ((gpr | ng | (col0 >> 5)) & 1) == 0;
    const int chunks = cb >> 4;
    const int cshift = (chunks & (chunks - 1)) == 0 ? __ffs(chunks) - 1 : -1;
    const int n4 = ng >> 1;
    const int sshift = (n4 & (n4 - 1)) == 0 && n4 > 0 ? __ffs(n4) - 1 : -1;
    const uint8_t *gcodes = M.codes + (col0 >> 1);
    const uint16_t *gscales = M.scales + (col0 >> 5);

    auto issue = [&](int s) {
        if (s < nst) {
            uint8_t *buf = ring + (s % kStages) * kWarpStageBytes;
            const int rbase = wr0 + s * SR;
            const int nr = min(SR, wr1 - rbase);
            for (int i = lane; i < nr * chunks; i += 32) {
                const int rr = cshift >= 0 ? i >> cshift : i / chunks;
                const int ch = i - rr * chunks;
                cp_async16(buf + rr * cb + ch * 16, gcodes + (int64_t)(rbase + rr) * rb + ch * 16);
            }
            uint8_t *sbuf = buf + kWarpStageCode;
            if (sc4) {
                for (int i = lane; i < nr * n4; i += 32) {
                    const int rr = sshift >= 0 ? i >> sshift : i / n4;
                    const int ch = i - rr * n4;
                    cp_async4(sbuf + rr * spitch + ch * 4, gscales + (int64_t)(rbase + rr) * gpr + ch * 2);
                }
            } else {
                for (int i = lane; i < nr * ng; i += 32) {
                    const int rr = i / ng, gi = i - rr * ng;
                    *reinterpret_cast<uint16_t *>(sbuf + rr * spitch + gi * 2) =
                        __ldg(gscales + (int64_t)(rbase + rr) * gpr + gi);
                }
            }
        }
        cp_commit();
    };

    if (PHASE != kLoop)
        for (int s = 0; s < kStages - 1; ++s) issue(s);
    if (PHASE == kPrologue) return;
    const int cl = (lane % LPR) * 16;
    const int rs = lane / LPR;
    for (int s = 0; s < nst; ++s) {
        cp_wait<kStages - 2>();
        __syncwarp();
        issue(s + kStages - 1);
        if (cl < ncols) {
            const uint8_t *buf = ring + (s % kStages) * kWarpStageBytes;
            const uint8_t *sbuf = buf + kWarpStageCode;
            const int rbase = wr0 + s * SR;
            const int nr = min(SR, wr1 - rbase);
            const float *xin = in_s + (rbase - row0);
            for (int rr = rs; rr < nr; rr += RPW) {
                const uint2 q = *reinterpret_cast<const uint2 *>(buf + rr * cb + (cl >> 1));
                const uint16_t sb = *reinterpret_cast<const uint16_t *>(sbuf + rr * spitch + (cl >> 5) * 2);
                const uint32_t tsel = (sb & 0x8000u) ? 0x40404040u : 0u;
                row_fma<NT>(q, tsel, half_bits_to_float(sb & 0x7FFFu), xin + rr, in_ld, lut, acc);
            }
        }
        __syncwarp();
    }
    cp_wait<0>();
    __syncthreads();
}

// Sums lanes that share columns (the 32/LPR row lanes of a warp, then the
// warps through red_s[kWarps][NT][W], W = LPR*16).  The CTA's sums end up at
// red_s + kWarps*NT*W, indexed t*W + col.
template <int LPR, int NT>
__device__ __forceinline__ float *cta_reduce(u64 (&acc)[NT][8], int ncols, float *red_s) {
    constexpr int W = LPR * 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float a[NT][16];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int p = 0; p < 8; ++p) unpack2(acc[t][p], a[t][2 * p], a[t][2 * p + 1]);
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int j = 0; j < 16; ++j) a[t][j] += __shfl_xor_sync(0xffffffffu, a[t][j], o);
    const int cl = lane * 16;
    if (lane < LPR && cl < ncols) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float4 *dst = reinterpret_cast<float4 *>(red_s + (warp * NT + t) * W + cl);
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[j] = make_float4(a[t][4 * j], a[t][4 * j + 1], a[t][4 * j + 2], a[t][4 * j + 3]);
        }
    }
    __syncthreads();
    float *res = red_s + kWarps * NT * W;
    for (int i = threadIdx.x; i < NT * W; i += kThreads) {
        const int col = i % W;
        float v = 0.f;
        if (col < ncols) {
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += red_s[w * NT * W + i];
        }
        res[i] = v;
    }
    __syncthreads();
    return res;
}

// Does expert e's factor have any INT8 group?  (prefix counts of the stacked tensor)
__device__ __forceinline__ bool expert_has_int8(const latent_qmatrix &m, int e) {
    if (!m.i8_mask) return false;
    const int64_t words = ((m.rows * m.cols >> 5) + 31) >> 5;
    const uint32_t *mask = m.i8_mask + (int64_t)e * words;
    const uint32_t *base = m.i8_base + (int64_t)e * words;
    const uint32_t first = __ldg(base), last = __ldg(base + words - 1) + __popc(__ldg(mask + words - 1));
    return last > first;
}

// Adds the high-nibble part of every INT8 group of the tile to the CTA's
// reduced sums res[t * W + col] (the main loop decoded only the low nibble,
// through the identity table): value = (16*h + l) * |scale| with h the
// signed high nibble from the i8_hi side table.  Per chunk of 256 rows it
// makes two round trips to memory: (1) the mask and prefix words of every
// row, (2) the high-nibble records and scale words of every INT8 group.
// Deterministic: thread (column chunk of 8, row slice) accumulates its rows
// in order, then the slices are summed in order.  `part` needs 8*NT*W
// floats; `scratch` kI8Scratch bytes.
constexpr int kI8Rows = 256;
constexpr int kI8Cap = 512;
constexpr int kI8Scratch = kI8Rows * 16 + kI8Rows * 8 + 64 + kI8Cap * 20;
static_assert(kI8Rows == kThreads, "int8_fix scans one row per thread");

template <int NT>
__device__ void int8_fix(const QView &M, int row0, int row_end, int col0, int ncols, const float *in_s, int in_ld,
                         float *res, int W, float *part, uint8_t *scratch) {
    const int ng = ncols >> 5, g0 = col0 >> 5;
    const int64_t gpr = M.cols >> 5;
    const int64_t words = (((int64_t)M.rows * gpr) + 31) >> 5;
    const int ccount = ncols >> 3;
    const int slices = min(8, kThreads / ccount);
    const int cc = threadIdx.x % ccount, sl = threadIdx.x / ccount;
    const bool active = sl < slices;
    const int col8 = cc * 8, gi = col8 >> 5, wsel = (col8 & 31) >> 3;
    uint32_t *msk = reinterpret_cast<uint32_t *>(scratch);                    // [kI8Rows][2]
    uint32_t *bas = msk + 2 * kI8Rows;                                         // [kI8Rows][2]
    uint32_t *rowbits = bas + 2 * kI8Rows;                                     // [kI8Rows]
    int *rowstart = reinterpret_cast<int *>(rowbits + kI8Rows);                // [kI8Rows + 1 + kWarps]
    uint4 *ent_hi = reinterpret_cast<uint4 *>(scratch + kI8Rows * 16 + kI8Rows * 8 + 64);  // [kI8Cap]
    float *ent_sc = reinterpret_cast<float *>(ent_hi + kI8Cap);               // [kI8Cap] 16*|scale|
    float acc[NT][8];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[t][j] = 0.f;
    for (int rc = row0; rc < row_end;) {
        int nr = min(kI8Rows, row_end - rc);
        __syncthreads();
        // round trip 1: mask and prefix words of each row's tile groups
        for (int i = threadIdx.x; i < nr; i += kThreads) {
            const int64_t pos = (int64_t)(rc + i) * gpr + g0;
            const int64_t w = pos >> 5;
            cp_async4(msk + 2 * i, M.i8.mask + w);
            cp_async4(bas + 2 * i, M.i8.base + w);
            if ((int)(pos & 31) + ng > 32 && w + 1 < words) {
                cp_async4(msk + 2 * i + 1, M.i8.mask + w + 1);
                cp_async4(bas + 2 * i + 1, M.i8.base + w + 1);
            } else {
                msk[2 * i + 1] = 0u;
            }
        }
        cp_commit();
        cp_wait<0>();
        __syncthreads();
        {   // one row per thread (kI8Rows == kThreads): bits, then a block scan of their counts
            const int i = threadIdx.x, lane = i & 31, wid = i >> 5;
            uint32_t bits = 0u;
            if (i < nr) {
                const int64_t pos = (int64_t)(rc + i) * gpr + g0;
                const int b = (int)(pos & 31);
                const uint64_t two = (uint64_t)msk[2 * i] | ((uint64_t)msk[2 * i + 1] << 32);
                bits = (uint32_t)(two >> b) & ((1u << ng) - 1u);
                rowbits[i] = bits;
            }
            const int c = __popc(bits);
            int v = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += y;
            }
            if (lane == 31) rowstart[kI8Rows + 1 + wid] = v;  // warp totals (scratch slots)
            __syncthreads();
            int base = 0;
            for (int w2 = 0; w2 < wid; ++w2) base += rowstart[kI8Rows + 1 + w2];
            const int start = base + v - c;
            const bool ok = i < nr && start + c <= kI8Cap;
            __syncthreads();
            if (ok) rowstart[i] = start;
            nr = __syncthreads_count(ok);  // rows handled this pass (a prefix of the chunk)
        }
        // round trip 2: high-nibble records and scale words of the INT8 groups
        for (int i = threadIdx.x; i < nr; i += kThreads) {
            const int64_t pos = (int64_t)(rc + i) * gpr + g0;
            const int b = (int)(pos & 31);
            int k = rowstart[i];
            for (uint32_t rest = rowbits[i]; rest; rest &= rest - 1, ++k) {
                const int q = __ffs(rest) - 1;
                const int bb = b + q;                       // bit position relative to word w
                const int wi = bb >> 5;                     // 0 or 1
                const uint32_t mw = msk[2 * i + wi];
                const uint32_t idx = bas[2 * i + wi] + __popc(mw & ((1u << (bb & 31)) - 1u));
                cp_async16(ent_hi + k, M.i8.hi + (int64_t)idx * 16);
                ent_sc[k] = 16.f * half_bits_to_float(__ldg(M.scales + pos + q) & 0x7FFFu);
            }
        }
        cp_commit();
        cp_wait<0>();
        __syncthreads();
        if (active) {
            for (int rr = sl; rr < nr; rr += slices) {
                const uint32_t bits = rowbits[rr];
                if (!((bits >> gi) & 1u)) continue;
                const int k = rowstart[rr] + __popc(bits & ((1u << gi) - 1u));
                const uint32_t hw = reinterpret_cast<const uint32_t *>(ent_hi + k)[wsel];
                const float s16 = ent_sc[k];
                float xv[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) xv[t] = in_s[t * in_ld + (rc - row0 + rr)] * s16;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float h = (float)((int)(((hw >> (4 * j)) & 15u) ^ 8u) - 8);
#pragma unroll
                    for (int t = 0; t < NT; ++t) acc[t][j] = fmaf(xv[t], h, acc[t][j]);
                }
            }
        }
        rc += nr;
    }
    __syncthreads();
    if (active) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int j = 0; j < 8; ++j) part[(sl * NT + t) * W + col8 + j] = acc[t][j];
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < NT; ++t)
        for (int col = threadIdx.x; col < ncols; col += kThreads) {
            float s = 0.f;
            for (int q = 0; q < slices; ++q) s += part[(q * NT + t) * W + col];
            res[t * W + col] += s;
        }
    __syncthreads();
}

struct Smem {
    float *lut;    // 32: NF4 levels, then the identity table 0..15
    uint8_t *stages;  // kStages * kStageBytes
    uint8_t *i8s;     // kI8Scratch
    float *in_s;   // staged input vectors
    float *red_s;  // (kWarps+1) * 4 * max(r, kTileN)
    float *g_s;    // 4 * kTileN
    int *list;     // kThreads token ids
    int *flag;     // 2 ints
};

__device__ __forceinline__ void cta_wait(const uint32_t *flag, uint32_t target, const DecodeArgs &a, const Smem &S) {
    if (threadIdx.x == 0) wait_ge(flag, target, a.rt.err);
    __syncthreads();
}

// Publishes this CTA's global writes, then adds 1 to *ctr; returns the old value (all threads).
__device__ __forceinline__ uint32_t cta_arrive(uint32_t *ctr, const Smem &S) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) S.flag[0] = (int)atomicAdd(ctr, 1u);
    __syncthreads();
    return (uint32_t)S.flag[0];
}

template <int LPR, int NT>
__device__ __forceinline__ void in_chunk(const QView &M, bool has_i8, int row0, int row_end, int r, const float *in_s,
                                         int kc, const Smem &S, float *part_rows, int ldo, bool pre) {
    u64 acc[NT][8];
    if (pre)
        vecmat_staged<LPR, NT, kLoop>(M, row0, row_end, 0, r, in_s, kc, S.lut, S.stages, acc);
    else
        vecmat_staged<LPR, NT>(M, row0, row_end, 0, r, in_s, kc, S.lut, S.stages, acc);
    float *res = cta_reduce<LPR, NT>(acc, r, S.red_s);
    if (has_i8) int8_fix<NT>(M, row0, row_end, 0, r, in_s, kc, res, LPR * 16, S.red_s, S.i8s);
#pragma unroll
    for (int t = 0; t < NT; ++t)
        for (int col = threadIdx.x; col < r; col += kThreads) part_rows[(int64_t)t * ldo + col] = res[t * r + col];
}

// Phase 1 (PH=1: t = x.A_{g|u}) and phase 3 (PH=3: s = h.A_d): one split-K row chunk.
template <int LPR, int XT, int PH>
__device__ void item_in(const DecodeArgs &a, const Smem &S, int ai, int m, int ksel) {
    constexpr int nmat = PH == 1 ? 2 : 1;
    const int kc = PH == 1 ? a.kc1 : a.kc2, ks = PH == 1 ? a.ks1 : a.ks2, r = a.r;
    const int e = a.rt.active[ai];
    const int p0 = a.rt.offsets[e], ne = a.rt.offsets[e + 1] - p0;
    const latent_qmatrix &qm = PH == 1 ? (m == 0 ? a.gate_a : a.up_a) : a.down_a;
    const QView M = expert_view(qm, e);
    const bool has_i8 = expert_has_int8(qm, e);
    const int row0 = ksel * kc, row_end = min(M.rows, row0 + kc);
    {   // start streaming the weights before waiting for inputs
        u64 none[1][8];
        vecmat_staged<LPR, 1, kPrologue>(M, row0, row_end, 0, r, nullptr, 0, S.lut, S.stages, none);
    }
    if (PH == 3) cta_wait(a.cnt2 + e, (uint32_t)a.nct_f, a, S);
    const int ldo = nmat * r;
    float *part = PH == 1 ? a.part1 : a.part2;
    for (int tc = 0; tc < ne; tc += 4) {
        const int nt = min(4, ne - tc);
        __syncthreads();
        for (int t = 0; t < nt; ++t) {
            const int p = p0 + tc + t;
            const int64_t src = PH == 1 ? (int64_t)(a.rt.order[p] / a.k) * a.d : (int64_t)p * a.f;
            for (int rr = threadIdx.x; rr < kc; rr += kThreads) {
                const int row = row0 + rr;
                float v = 0.f;
                if (row < row_end) {
                    if constexpr (PH == 1)
                        v = load_act<XT>(a.x, src + row);
                    else
                        v = __ldcg(a.h + src + row);
                }
                S.in_s[t * kc + rr] = v;
            }
        }
        __syncthreads();
        float *rows = part + ((int64_t)ksel * a.R + p0 + tc) * ldo + m * r;
        if (nt == 1)
            in_chunk<LPR, 1>(M, has_i8, row0, row_end, r, S.in_s, kc, S, rows, ldo, tc == 0);
        else if (nt == 2)
            in_chunk<LPR, 2>(M, has_i8, row0, row_end, r, S.in_s, kc, S, rows, ldo, tc == 0);
        else if (nt == 3)
            in_chunk<LPR, 3>(M, has_i8, row0, row_end, r, S.in_s, kc, S, rows, ldo, tc == 0);
        else
            in_chunk<LPR, 4>(M, has_i8, row0, row_end, r, S.in_s, kc, S, rows, ldo, tc == 0);
    }
    uint32_t *arr = (PH == 1 ? a.arr1 : a.arr3) + e;
    if (cta_arrive(arr, S) != (uint32_t)(nmat * ks - 1)) return;
    // Last chunk of this expert: sum the partials in chunk order, publish.
    __threadfence();
    float *outv = PH == 1 ? a.t : a.s;
    for (int pp = p0; pp < p0 + ne; ++pp) {
        for (int col = threadIdx.x; col < ldo; col += kThreads) {
            float v = 0.f;
            for (int q = 0; q < ks; ++q) v += __ldcg(part + ((int64_t)q * a.R + pp) * ldo + col);
            outv[(int64_t)pp * ldo + col] = v;
        }
    }
    cta_arrive(PH == 1 ? a.flag1 + e : a.flag3 + e, S);
}

template <int NT>
__device__ __forceinline__ void gateup_chunk(const DecodeArgs &a, const Smem &S, const QView &Mg, bool gi8,
                                             const QView &Mu, bool ui8, int col0, int ncols, int p,
                                             const float *in_g, const float *in_u, bool pre) {
    constexpr int W = kTileN;
    const int r = a.r;
    u64 acc[NT][8];
    if (pre)
        vecmat_staged<16, NT, kLoop>(Mg, 0, r, col0, ncols, in_g, r, S.lut, S.stages, acc);
    else
        vecmat_staged<16, NT>(Mg, 0, r, col0, ncols, in_g, r, S.lut, S.stages, acc);
    {   // the up matrix starts streaming while the gate sums are reduced
        u64 none[1][8];
        vecmat_staged<16, 1, kPrologue>(Mu, 0, r, col0, ncols, nullptr, 0, S.lut, S.stages, none);
    }
    float *res = cta_reduce<16, NT>(acc, ncols, S.red_s);
    if (gi8) int8_fix<NT>(Mg, 0, r, col0, ncols, in_g, r, res, W, S.red_s, S.i8s);
    for (int i = threadIdx.x; i < NT * W; i += kThreads) S.g_s[i] = res[i];
    __syncthreads();
    vecmat_staged<16, NT, kLoop>(Mu, 0, r, col0, ncols, in_u, r, S.lut, S.stages, acc);
    res = cta_reduce<16, NT>(acc, ncols, S.red_s);
    if (ui8) int8_fix<NT>(Mu, 0, r, col0, ncols, in_u, r, res, W, S.red_s, S.i8s);
    const bool wbd = a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN;
    for (int i = threadIdx.x; i < NT * W; i += kThreads) {
        const int t = i / W, col = i - t * W;
        if (col >= ncols) continue;
        float hv = silu_f32(S.g_s[i]) * res[i];
        if (wbd) hv *= load_weight(a.weights, a.w_type, a.rt.order[p + t]);
        a.h[(int64_t)(p + t) * a.f + col0 + col] = hv;
    }
}

// Phase 2: h = silu(t_g.B_g) * (t_u.B_u) [* w] for one 256-column tile of f.
__device__ void item_gateup(const DecodeArgs &a, const Smem &S, int ai, int ct) {
    const int r = a.r;
    const int e = a.rt.active[ai];
    const int p0 = a.rt.offsets[e], ne = a.rt.offsets[e + 1] - p0;
    const QView Mg = expert_view(a.gate_b, e), Mu = expert_view(a.up_b, e);
    const bool gi8 = expert_has_int8(a.gate_b, e), ui8 = expert_has_int8(a.up_b, e);
    const int col0 = ct * kTileN, ncols = min(kTileN, a.f - col0);
    {
        u64 none[1][8];
        vecmat_staged<16, 1, kPrologue>(Mg, 0, r, col0, ncols, nullptr, 0, S.lut, S.stages, none);
    }
    cta_wait(a.flag1 + e, 1u, a, S);
    float *in_g = S.in_s, *in_u = S.in_s + 4 * r;
    for (int tc = 0; tc < ne; tc += 4) {
        const int nt = min(4, ne - tc);
        __syncthreads();
        for (int t = 0; t < nt; ++t) {
            const float *src = a.t + (int64_t)(p0 + tc + t) * 2 * r;
            for (int kk = threadIdx.x; kk < r; kk += kThreads) {
                in_g[t * r + kk] = __ldcg(src + kk);
                in_u[t * r + kk] = __ldcg(src + r + kk);
            }
        }
        __syncthreads();
        const int p = p0 + tc;
        if (nt == 1)
            gateup_chunk<1>(a, S, Mg, gi8, Mu, ui8, col0, ncols, p, in_g, in_u, tc == 0);
        else if (nt == 2)
            gateup_chunk<2>(a, S, Mg, gi8, Mu, ui8, col0, ncols, p, in_g, in_u, tc == 0);
        else if (nt == 3)
            gateup_chunk<3>(a, S, Mg, gi8, Mu, ui8, col0, ncols, p, in_g, in_u, tc == 0);
        else
            gateup_chunk<4>(a, S, Mg, gi8, Mu, ui8, col0, ncols, p, in_g, in_u, tc == 0);
    }
    cta_arrive(a.cnt2 + e, S);
}

template <int NT>
__device__ __forceinline__ void down_chunk(const DecodeArgs &a, const Smem &S, const QView &M, bool i8, int col0,
                                           int ncols, int p, bool pre) {
    constexpr int W = kTileN;
    u64 acc[NT][8];
    if (pre)
        vecmat_staged<16, NT, kLoop>(M, 0, a.r, col0, ncols, S.in_s, a.r, S.lut, S.stages, acc);
    else
        vecmat_staged<16, NT>(M, 0, a.r, col0, ncols, S.in_s, a.r, S.lut, S.stages, acc);
    float *res = cta_reduce<16, NT>(acc, ncols, S.red_s);
    if (i8) int8_fix<NT>(M, 0, a.r, col0, ncols, S.in_s, a.r, res, W, S.red_s, S.i8s);
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

__device__ __forceinline__ int live_slots(const DecodeArgs &a, int t) {
    int n = 0;
    for (int j = 0; j < a.k; ++j) n += a.rt.pos[t * a.k + j] >= 0;
    return n;
}

// Phase 4: y = s.B_d for one 256-column tile of d, then the top-k combine of
// every token whose last routed slot for this tile just finished.
__device__ void item_down(const DecodeArgs &a, const Smem &S, int ai, int ct) {
    const int r = a.r;
    const int e = a.rt.active[ai];
    const int p0 = a.rt.offsets[e], ne = a.rt.offsets[e + 1] - p0;
    const QView M = expert_view(a.down_b, e);
    const bool i8 = expert_has_int8(a.down_b, e);
    const int col0 = ct * kTileN, ncols = min(kTileN, a.d - col0);
    {
        u64 none[1][8];
        vecmat_staged<16, 1, kPrologue>(M, 0, r, col0, ncols, nullptr, 0, S.lut, S.stages, none);
    }
    cta_wait(a.flag3 + e, 1u, a, S);
    for (int tc = 0; tc < ne; tc += 4) {
        const int nt = min(4, ne - tc);
        __syncthreads();
        for (int t = 0; t < nt; ++t)
            for (int kk = threadIdx.x; kk < r; kk += kThreads)
                S.in_s[t * r + kk] = __ldcg(a.s + (int64_t)(p0 + tc + t) * r + kk);
        __syncthreads();
        const int p = p0 + tc;
        if (nt == 1)
            down_chunk<1>(a, S, M, i8, col0, ncols, p, tc == 0);
        else if (nt == 2)
            down_chunk<2>(a, S, M, i8, col0, ncols, p, tc == 0);
        else if (nt == 3)
            down_chunk<3>(a, S, M, i8, col0, ncols, p, tc == 0);
        else
            down_chunk<4>(a, S, M, i8, col0, ncols, p, tc == 0);
    }
    if (a.flags & LATENT_FLAG_OUT_PER_SLOT) return;
    __threadfence();
    const bool wbd = a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN;
    for (int base = 0; base < ne; base += kThreads) {
        __syncthreads();
        if (threadIdx.x == 0) S.flag[1] = 0;
        __syncthreads();
        const int i = base + threadIdx.x;
        if (i < ne) {
            const int t = a.rt.order[p0 + i] / a.k;
            const uint32_t old = atomicAdd(a.tokcnt + (int64_t)t * a.nct_d + ct, 1u);
            if ((int)old + 1 == live_slots(a, t)) S.list[atomicAdd(&S.flag[1], 1)] = t;
        }
        __syncthreads();
        const int n_done = S.flag[1];
        if (n_done == 0) continue;
        __threadfence();
        for (int q = 0; q < n_done; ++q) {
            const int t = S.list[q];
            for (int col = threadIdx.x; col < ncols; col += kThreads) {
                float acc = 0.f;
                for (int j = 0; j < a.k; ++j) {
                    const int slot = t * a.k + j;
                    const int pp = a.rt.pos[slot];
                    if (pp < 0) continue;
                    const float w = wbd ? 1.f : load_weight(a.weights, a.w_type, slot);
                    acc = fmaf(w, __ldcg(a.y + (int64_t)pp * a.d + col0 + col), acc);
                }
                a.out[(int64_t)t * a.d + col0 + col] = acc;
            }
        }
    }
}

template <int LPR, int XT>
__global__ void __launch_bounds__(kThreads, 2) k_decode(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t sm_raw[];
    __shared__ __align__(128) float s_lut[32];
    __shared__ int s_list[kThreads];
    __shared__ int s_flag[2];
    __shared__ int s_item;
    Smem S;
    S.lut = s_lut;
    S.stages = sm_raw;
    S.i8s = sm_raw + kStages * kStageBytes;
    float *sm = reinterpret_cast<float *>(sm_raw + kStages * kStageBytes + kI8Scratch);
    S.in_s = sm;
    S.red_s = sm + a.in_floats;
    S.g_s = S.red_s + a.red_floats;
    S.list = s_list;
    S.flag = s_flag;
    if (threadIdx.x < 16) s_lut[threadIdx.x] = kNF4Levels[threadIdx.x];
    else if (threadIdx.x < 32) s_lut[threadIdx.x] = (float)(threadIdx.x - 16);
    const int n_active = *a.rt.n_active;
    const int n1 = n_active * 2 * a.ks1, n2 = n_active * a.nct_f, n3 = n_active * a.ks2, n4 = n_active * a.nct_d;
    // Rows no expert writes: skipped slots (per-slot output) or tokens with no live slot.
    const bool per_slot = a.flags & LATENT_FLAG_OUT_PER_SLOT;
    const int n_rows = per_slot ? a.T * a.k : a.T;
    for (int i = blockIdx.x; i < n_rows; i += gridDim.x) {
        const bool empty = per_slot ? a.rt.pos[i] < 0 : live_slots(a, i) == 0;
        if (empty)
            for (int c = threadIdx.x * 4; c < a.d; c += kThreads * 4)
                *reinterpret_cast<float4 *>(a.out + (int64_t)i * a.d + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    while (true) {
        __syncthreads();
        if (threadIdx.x == 0) s_item = (int)atomicAdd(a.work, 1u);
        __syncthreads();
        int it = s_item;
        if (it < n1) {
            item_in<LPR, XT, 1>(a, S, it / (2 * a.ks1), (it / a.ks1) % 2, it % a.ks1);
            continue;
        }
        it -= n1;
        if (it < n2) {
            item_gateup(a, S, it / a.nct_f, it % a.nct_f);
            continue;
        }
        it -= n2;
        if (it < n3) {
            item_in<LPR, LATENT_TYPE_F32, 3>(a, S, it / a.ks2, 0, it % a.ks2);
            continue;
        }
        it -= n3;
        if (it < n4) {
            item_down(a, S, it / a.nct_d, it % a.nct_d);
            continue;
        }
        break;
    }
}

int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Rows per split-K item: about 32 KB of codes, whole warp steps, at most 1024.
void plan_split(int K, int r, int &kc, int &ks) {
    const int lpr = r / 16;
    const int step = kWarps * (32 / lpr);
    int rows = 32768 / (r / 2);
    rows = rows < step ? step : rows;
    rows = rows > 512 ? 512 : rows;
    kc = round_up(rows, 64);
    if (kc > round_up(K, 64)) kc = round_up(K, 64);
    ks = (K + kc - 1) / kc;
}

template <int LPR>
const void *decode_fn(int x_type) {
    switch (x_type) {
        case LATENT_TYPE_F32: return (const void *)k_decode<LPR, LATENT_TYPE_F32>;
        case LATENT_TYPE_F16: return (const void *)k_decode<LPR, LATENT_TYPE_F16>;
        default: return (const void *)k_decode<LPR, LATENT_TYPE_BF16>;
    }
}

const void *pick_decode_fn(int r, int x_type) {
    switch (r) {
        case 32: return decode_fn<2>(x_type);
        case 64: return decode_fn<4>(x_type);
        case 128: return decode_fn<8>(x_type);
        case 256: return decode_fn<16>(x_type);
        case 512: return decode_fn<32>(x_type);
        default: return nullptr;
    }
}

}  // namespace

void decode_plan(DecodeArgs &a) {
    a.R = a.T * a.k;
    a.nmax = a.E < a.R ? a.E : a.R;
    a.nct_f = (a.f + kTileN - 1) / kTileN;
    a.nct_d = (a.d + kTileN - 1) / kTileN;
    plan_split(a.d, a.r, a.kc1, a.ks1);
    plan_split(a.f, a.r, a.kc2, a.ks2);
    int in_f = 4 * (a.kc1 > a.kc2 ? a.kc1 : a.kc2);
    if (in_f < 8 * a.r) in_f = 8 * a.r;
    a.in_floats = round_up(in_f, 32);
    const int w = a.r > kTileN ? a.r : kTileN;
    a.red_floats = (kWarps + 1) * 4 * w;
}

int decode_sem_count(const DecodeArgs &a) { return 1 + 5 * a.E + a.T * a.nct_d; }

size_t decode_scratch_floats(const DecodeArgs &a) {
    const size_t R = (size_t)a.R, r = (size_t)a.r;
    return (size_t)a.ks1 * R * 2 * r + R * 2 * r + R * (size_t)a.f + (size_t)a.ks2 * R * r + R * r +
           R * (size_t)a.d + 6 * 64;
}

cudaError_t launch_decode(const DecodeArgs &a, cudaStream_t s, Marks *marks) {
    const void *fn = pick_decode_fn(a.r, a.x_type);
    if (!fn) return cudaErrorInvalidValue;
    const size_t smem = (size_t)kStages * kStageBytes + kI8Scratch +
                        (size_t)(a.in_floats + a.red_floats + 4 * kTileN) * sizeof(float);
    cudaError_t err = ensure_smem(fn, smem);
    if (err != cudaSuccess) return err;
    int dev = 0, sms = 0, per_sm = 0;
    if ((err = cudaGetDevice(&dev)) != cudaSuccess) return err;
    if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return err;
    if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem)) != cudaSuccess) return err;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int grid = sms * per_sm;
    void *args[] = {(void *)&a};
    err = cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kThreads), args, smem, s);
    if (marks) marks->mark(s);
    return err;
}

}  // namespace latent

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
