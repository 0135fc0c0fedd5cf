// Prefill path: many tokens per expert.  The latent chain runs as four
// grouped GEMMs on the 5th-generation tensor cores (tcgen05, kind::f16 with
// f16 operands, fp32 accumulation in TMEM):
//   G1  T  = Xp . [A_g|A_u]           Xp: routed rows of x in expert order
//   G2  H  = silu(T_g.B_g) * (T_u.B_u) [* w]   dual accumulator, SwiGLU epilogue
//   G3  S  = H . A_d
//   G4  Y  = S . B_d                   the epilogue adds w * Y into the
//                                      token's output row (red.add on an output
//                                      zeroed before G1), or stores Y per slot
// Factors are first dequantized (NF4 / INT8, bit-exact fp32 values rounded
// once to f16) into K-major f16 copies in the workspace; activations between
// GEMMs are f16.  f16 rather than bf16 operands: a numpy emulation of this
// chain at a Mixtral-like shape gives rel-L2 9e-4 with f16 and 4.8e-3 with
// bf16 against the fp32 reference (tolerance 2e-3).
//
// GEMM kernel: persistent, one CTA per SM, warp-specialised: warp 0 issues
// TMA tile loads (128B swizzle) into a 3-4 stage shared-memory ring, warp 1
// issues tcgen05.mma from a single thread into one of two 256-column TMEM
// accumulators, warps 4-7 drain the other accumulator (tcgen05.ld) and run
// the epilogue, so the epilogue of tile i overlaps the MMAs of tile i+1.
// Every mbarrier wait is bounded; on a timeout the kernel records
// kErrTimeout, drains its TMA loads, frees TMEM and exits.  Every TMA load
// is a plain per-CTA load into the issuing CTA's own shared memory.
#include <cuda.h>

#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace latent {

namespace {

using namespace sm100;

constexpr int kBM = 128;  // rows per tile (TMEM lanes)
constexpr int kBK = 64;   // K per stage (128 bytes of f16: one swizzle atom)

// ---------------------------------------------------------------------------
// Dequantize-transpose: NF4/INT8 factor [K rows][N cols] of every expert into
// f16 [N][K] rows at dst + e*dst_expert_stride + (row_off + n)*K.  One block
// per (expert, 256-column tile, 64-row block).  Decode: thread t takes row
// k0 + t % 64 of group column t / 64 (and +4), so that a warp writes 32
// consecutive k of one n into the [n][k] shared tile (conflict-free); the
// group loads are L1-cached 16-byte loads.  Store: 8 lanes per output row,
// each a 16-byte run: every warp store writes four whole 128-byte lines.
constexpr int kDqK = 64;             // K rows per block
constexpr int kDqLd = kDqK + 8;      // tile row pitch in halves (144 B)

__global__ void __launch_bounds__(256) k_pf_dequant_t(latent_qmatrix m, __half *dst, int64_t dst_expert_stride,
                                                       int row_off) {
    __shared__ __align__(16) __half tile[256][kDqLd];
    __shared__ float lut[16];  // per-thread table indices: shared memory, not the constant cache
    if (threadIdx.x < 16) lut[threadIdx.x] = kNF4Levels[threadIdx.x];
    const int e = blockIdx.z;
    const QView M = expert_view(m, e);
    const int K = M.rows, N = M.cols;
    const int c = blockIdx.x;
    const int ng = min(8, (N >> 5) - 8 * c);
    const int k0 = blockIdx.y * kDqK;
    const int nk = min(kDqK, K - k0);
    const int64_t q0 = (int64_t)c * K * 8 + (int64_t)k0 * ng;  // tile_group(K, N, k0, 256 c)
    __syncthreads();
    const int kk = threadIdx.x % kDqK;
    for (int gi = threadIdx.x / kDqK; gi < ng; gi += 256 / kDqK) {
        if (kk >= nk) continue;
        const int64_t g = q0 + (int64_t)kk * ng + gi;
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(M.codes) + g);
        const uint16_t sb = __ldg(M.scales + g);
        const float sc = half_bits_to_float(sb & 0x7FFFu);
        uint4 h = make_uint4(0u, 0u, 0u, 0u);
        uint32_t idx;
        const bool i8 = (sb & 0x8000u) && M.i8.present() && M.i8.is_int8(g, &idx);
        if (i8) h = __ldg(reinterpret_cast<const uint4 *>(M.i8.hi + (int64_t)idx * 16));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w}, hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
        for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float v = i8 ? int8_elem(w[s], hw[s], j) : lut[(w[s] >> (4 * j)) & 15u];
                tile[gi * 32 + s * 8 + j][kk] = __float2half_rn(__fmul_rn(v, sc));
            }
        }
    }
    __syncthreads();
    const int nn = ng * 32;
    for (int i = threadIdx.x; i < nn * (kDqK / 8); i += blockDim.x) {
        const int n = i >> 3, ch = i & 7;
        const int kc = ch * 8;
        if (kc >= nk) continue;
        __half *out = dst + (int64_t)e * dst_expert_stride + (int64_t)(row_off + 256 * c + n) * K + k0 + kc;
        const uint4 v = *reinterpret_cast<const uint4 *>(&tile[n][kc]);
        if (kc + 8 <= nk) {
            *reinterpret_cast<uint4 *>(out) = v;
        } else {
            const __half *hv = reinterpret_cast<const __half *>(&v);
            for (int j = 0; kc + j < nk; ++j) out[j] = hv[j];
        }
    }
}

// Routed rows of x in expert order, converted to f16: xp[p] = f16(x[order[p] / k]); 8 elements per thread.
template <int XT>
__global__ void __launch_bounds__(256) k_pf_gather(const void *x, const int32_t *order, const int32_t *offsets, int E,
                                                   int k, int d, __half *xp) {
    const int p = blockIdx.x;
    if (p >= __ldg(offsets + E)) return;
    const int64_t src = (int64_t)(__ldg(order + p) / k) * d;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0) {  // x only element-aligned: scalar loads
        for (int c = threadIdx.x * 2; c < d; c += blockDim.x * 2) {
            const float v0 = load_act<XT>(x, src + c), v1 = load_act<XT>(x, src + c + 1);
            reinterpret_cast<__half2 *>(xp + (int64_t)p * d)[c >> 1] = __floats2half2_rn(v0, v1);
        }
        return;
    }
    for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
        __align__(16) __half hv[8];
        if constexpr (XT == LATENT_TYPE_F16) {
            *reinterpret_cast<uint4 *>(hv) = __ldg(reinterpret_cast<const uint4 *>(static_cast<const __half *>(x) + src + c));
        } else if constexpr (XT == LATENT_TYPE_BF16) {
            __align__(16) __nv_bfloat16 bv[8];
            *reinterpret_cast<uint4 *>(bv) =
                __ldg(reinterpret_cast<const uint4 *>(static_cast<const __nv_bfloat16 *>(x) + src + c));
#pragma unroll
            for (int j = 0; j < 8; ++j) hv[j] = __float2half_rn(__bfloat162float(bv[j]));
        } else {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(x) + src + c));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(x) + src + c) + 1);
            const float f8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) hv[j] = __float2half_rn(f8[j]);
        }
        *reinterpret_cast<uint4 *>(xp + (int64_t)p * d + c) = *reinterpret_cast<const uint4 *>(hv);
    }
}

// mtile_off[e] = sum over e' < e of ceil(count[e'] / 128); mtile_off[E] = total.
__global__ void __launch_bounds__(1024) k_pf_mtiles(const int32_t *counts, int E, int32_t *mtile_off) {
    __shared__ int warp_sum[32];
    const int per = (E + 1023) / 1024;
    const int lo = min(E, (int)threadIdx.x * per), hi = min(E, lo + per);
    int s = 0;
    for (int e = lo; e < hi; ++e) s += (counts[e] + kBM - 1) / kBM;
    // inclusive scan over 1024 partials (warp shuffles, then warp totals)
    int v = s;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    if (lane == 31) warp_sum[w] = v;
    __syncthreads();
    if (w == 0) {
        int t = warp_sum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        warp_sum[lane] = t;
    }
    __syncthreads();
    int run = v - s + (w > 0 ? warp_sum[w - 1] : 0);
    for (int e = lo; e < hi; ++e) {
        mtile_off[e] = run;
        run += (counts[e] + kBM - 1) / kBM;
    }
    if (threadIdx.x == 1023) mtile_off[E] = run;
}

// Epilogue / operand modes of the grouped GEMM.
enum : int { kModeF16 = 0, kModeSwiGLU = 1, kModeF32 = 2 };

struct GemmArgs {
    int E;
    int K;          // contraction length
    int N;          // output columns per expert (rows of the B operand per expert)
    int a_koff2;    // SwiGLU: column offset of the up half inside the A operand
    int ldo;        // output row stride (elements)
    void *out;      // row-major [R][ldo] (f16 for kModeF16/SwiGLU, f32 for kModeF32)
    const int32_t *offsets;    // [E+1] routed-row offsets
    const int32_t *mtile_off;  // [E+1] m-tile offsets
    const int32_t *order;      // routed row -> slot
    const void *weights;
    int w_type;
    uint32_t flags;
    int per_slot_d;            // kModeF32: row length d of out_slot
    float *out_slot;           // kModeF32: the op's output; [slot][d] with OUT_PER_SLOT, else [token][d] += w * y
    int top_k;
    uint32_t *err;
};

template <int MODE>
struct GemmCfg {
    static constexpr int BN = MODE == kModeSwiGLU ? 128 : 256;           // output columns per tile
    static constexpr int A_BYTES = kBM * kBK * 2;                        // 16 KB
    static constexpr int B_BYTES = BN * kBK * 2;                         // 16 / 32 KB
    static constexpr int STAGE = MODE == kModeSwiGLU ? 2 * (A_BYTES + B_BYTES) : A_BYTES + B_BYTES;
    static constexpr int STAGES = MODE == kModeSwiGLU ? 3 : 4;
    static constexpr int SMEM = STAGES * STAGE + 1024 /*barriers*/ + 1024 /*alignment*/;
    static constexpr uint32_t IDESC = idesc_f16_f32(BN);
};

__device__ __forceinline__ void decode_tile(const GemmArgs &g, int ntn, int tile, int &row0, int &nrows, int &brow,
                                            int &n0) {
    const int mt = tile / ntn, nt = tile - mt * ntn;
    int lo = 0, hi = g.E;  // largest e with mtile_off[e] <= mt
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(g.mtile_off + mid) <= mt) lo = mid; else hi = mid;
    }
    const int e = lo;
    const int m = mt - __ldg(g.mtile_off + e);
    const int start = __ldg(g.offsets + e), cnt = __ldg(g.offsets + e + 1) - start;
    row0 = start + m * kBM;
    nrows = min(kBM, cnt - m * kBM);
    n0 = nt * GemmCfg<0>::BN;  // overwritten by caller for other modes
    brow = e * g.N;
    (void)n0;
}

template <int MODE>
__global__ void __launch_bounds__(256, 1) k_pf_gemm(const __grid_constant__ CUtensorMap mA,
                                                    const __grid_constant__ CUtensorMap mB,
                                                    const __grid_constant__ CUtensorMap mB2, GemmArgs g) {
    using C = GemmCfg<MODE>;
    constexpr int BN = C::BN, S = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * C::STAGE);
    uint64_t *empty = full + S;
    uint64_t *acc_full = empty + S;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntn = (g.N + BN - 1) / BN;
    const int total = __ldg(g.mtile_off + g.E) * ntn;
    const int nk = (g.K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 128);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        prefetch_tensormap(&mA);
        prefetch_tensormap(&mB);
        if (MODE == kModeSwiGLU) prefetch_tensormap(&mB2);
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
            int row0, nrows, brow, n0;
            decode_tile(g, ntn, tile, row0, nrows, brow, n0);
            n0 = (tile % ntn) * BN;
            for (int ks = 0; ks < nk; ++ks, ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (it >= S && !mbar_wait(empty + s, ph ^ 1u)) { ok = false; break; }
                if (*abort_flag) { ok = false; break; }
                uint8_t *st = smem + s * C::STAGE;
                mbar_arrive_expect_tx(full + s, C::STAGE);
                tma_load_2d(st, &mA, ks * kBK, row0, full + s);
                tma_load_2d(st + C::A_BYTES, &mB, ks * kBK, brow + n0, full + s);
                if (MODE == kModeSwiGLU) {
                    tma_load_2d(st + C::A_BYTES + C::B_BYTES, &mA, g.a_koff2 + ks * kBK, row0, full + s);
                    tma_load_2d(st + 2 * C::A_BYTES + C::B_BYTES, &mB2, ks * kBK, brow + n0, full + s);
                }
            }
        }
        if (!ok) {
            atomicOr(g.err, kErrTimeout);
            *abort_flag = 1;
            // drain: the last load issued into each slot must land before the CTA exits
            for (int j = 0; j < S && j < it; ++j) {
                const int i2 = it - 1 - j;
                mbar_wait(full + (i2 % S), (uint32_t)(i2 / S) & 1u);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        int it = 0, tl = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++tl) {
            const int b = tl & 1;
            const uint32_t use = (uint32_t)(tl >> 1);
            if (tl >= 2 && !mbar_wait(acc_empty + b, (use - 1u) & 1u)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d = tmem_base + (uint32_t)b * 256u;
            for (int ks = 0; ks < nk; ++ks, ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (!mbar_wait(full + s, ph) || *abort_flag) { ok = false; break; }
                tc_fence_after();
                const uint8_t *st = smem + s * C::STAGE;
                const uint32_t a_addr = smem_addr(st), b_addr = smem_addr(st + C::A_BYTES);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint32_t acc = (ks | kk) != 0;
                    mma_f16(d, desc_kmajor_sw128(a_addr + kk * 32), desc_kmajor_sw128(b_addr + kk * 32), C::IDESC, acc);
                    if (MODE == kModeSwiGLU) {
                        const uint32_t a2 = smem_addr(st + C::A_BYTES + C::B_BYTES);
                        const uint32_t b2 = smem_addr(st + 2 * C::A_BYTES + C::B_BYTES);
                        mma_f16(d + 128u, desc_kmajor_sw128(a2 + kk * 32), desc_kmajor_sw128(b2 + kk * 32), C::IDESC,
                                acc);
                    }
                }
                mma_commit(empty + s);
            }
            if (!ok) break;
            mma_commit(acc_full + b);
        }
        if (!ok) {
            atomicOr(g.err, kErrTimeout);
            *abort_flag = 1;
            mma_commit(acc_full + 0);  // releases a waiting epilogue; MMAs already issued complete first
            mma_commit(acc_full + 1);
        }
    } else if (warp >= 4) {
        // ---------------- epilogue (128 threads = 128 TMEM lanes) ----------------
        const int q = warp - 4;
        const int row = q * 32 + lane;
        int tl = 0;
        const bool wbd = g.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++tl) {
            const int b = tl & 1;
            const uint32_t use = (uint32_t)(tl >> 1);
            if (!mbar_wait(acc_full + b, use & 1u) || *abort_flag) {
                atomicOr(g.err, kErrTimeout);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            int row0, nrows, brow, n0;
            decode_tile(g, ntn, tile, row0, nrows, brow, n0);
            n0 = (tile % ntn) * BN;
            const uint32_t taddr = tmem_base + (uint32_t)b * 256u + ((uint32_t)(q * 32) << 16);
            const bool live = row < nrows;
            const int64_t grow = (int64_t)row0 + row;
            float wrow = 1.f;
            if (MODE == kModeSwiGLU && wbd && live) wrow = load_weight(g.weights, g.w_type, g.order[grow]);
            for (int c = 0; c < BN; c += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + (uint32_t)c, v);
                if (MODE == kModeSwiGLU) {
                    uint32_t u[32];
                    tmem_ld32(taddr + 128u + (uint32_t)c, u);
                    tmem_ld_wait();
                    if (live) {
                        __half *o = reinterpret_cast<__half *>(g.out) + grow * g.ldo + n0 + c;
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            __align__(16) __half hv[8];
#pragma unroll
                            for (int t = 0; t < 8; ++t) {
                                const float gg = __uint_as_float(v[j + t]), uu = __uint_as_float(u[j + t]);
                                hv[t] = __float2half_rn(silu_fast(gg) * uu * wrow);
                            }
                            if (n0 + c + j + 8 <= g.N) *reinterpret_cast<uint4 *>(o + j) = *reinterpret_cast<uint4 *>(hv);
                        }
                    }
                } else {
                    tmem_ld_wait();
                    if (live) {
                        if (MODE == kModeF16) {
                            __half *o = reinterpret_cast<__half *>(g.out) + grow * g.ldo + n0 + c;
#pragma unroll
                            for (int j = 0; j < 32; j += 8) {
                                __align__(16) __half hv[8];
#pragma unroll
                                for (int t = 0; t < 8; ++t) hv[t] = __float2half_rn(__uint_as_float(v[j + t]));
                                if (n0 + c + j + 8 <= g.N) *reinterpret_cast<uint4 *>(o + j) = *reinterpret_cast<uint4 *>(hv);
                            }
                        } else if (g.flags & LATENT_FLAG_OUT_PER_SLOT) {
                            float *o = g.out_slot + (int64_t)g.order[grow] * g.per_slot_d + n0 + c;
#pragma unroll
                            for (int j = 0; j < 32; j += 4) {
                                if (n0 + c + j + 4 <= g.N)
                                    *reinterpret_cast<float4 *>(o + j) =
                                        make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                    __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
                            }
                        } else {  // the top-k combine: out[token] += w * y (out zeroed before G1)
                            const int slot = g.order[grow];
                            const float w = (g.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN)
                                                ? 1.f : load_weight(g.weights, g.w_type, slot);
                            float *o = g.out_slot + (int64_t)(slot / g.top_k) * g.per_slot_d + n0 + c;
#pragma unroll
                            for (int j = 0; j < 32; j += 4) {
                                if (n0 + c + j + 4 <= g.N)
                                    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(o + j),
                                                 "f"(w * __uint_as_float(v[j])), "f"(w * __uint_as_float(v[j + 1])),
                                                 "f"(w * __uint_as_float(v[j + 2])), "f"(w * __uint_as_float(v[j + 3]))
                                                 : "memory");
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(acc_empty + b);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem_base, 512);
}

}  // namespace

}  // namespace latent

namespace latent {

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Row-major f16 matrix [rows][cols] as a 2-D TMA map with a {64, box_rows} box, 128B swizzle.
bool make_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_dequant_t(const latent_qmatrix &m, int E, __half *dst, int64_t stride, int row_off, cudaStream_t s) {
    dim3 grid((unsigned)((m.cols + 255) / 256), (unsigned)((m.rows + kDqK - 1) / kDqK), (unsigned)E);
    k_pf_dequant_t<<<grid, 256, 0, s>>>(m, dst, stride, row_off);
    return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_gemm(const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &b2, const GemmArgs &g,
                        cudaStream_t s) {
    const void *fn = (const void *)k_pf_gemm<MODE>;
    cudaError_t err = ensure_smem(fn, GemmCfg<MODE>::SMEM);
    if (err != cudaSuccess) return err;
    int dev = 0, sms = 0;
    if ((err = cudaGetDevice(&dev)) != cudaSuccess) return err;
    if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return err;
    k_pf_gemm<MODE><<<sms, 256, GemmCfg<MODE>::SMEM, s>>>(a, b, b2, g);
    return cudaGetLastError();
}

size_t al(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

size_t prefill_scratch_bytes(const DecodeArgs &a) {
    const size_t E = a.E, R = a.R, d = a.d, f = a.f, r = a.r;
    return al((E + 1) * 4) + al(R * d * 2) + al(E * 2 * r * d * 2) + 2 * al(E * f * r * 2) + al(E * r * f * 2) +
           al(E * d * r * 2) + al(R * 2 * r * 2) + al(R * f * 2) + al(R * r * 2);
}

cudaError_t launch_prefill(const DecodeArgs &a, void *scratch, cudaStream_t s, Marks *marks) {
    const size_t E = a.E, R = a.R, d = a.d, f = a.f, r = a.r;
    char *p = static_cast<char *>(scratch);
    auto take = [&](size_t bytes) { char *q = p; p += al(bytes); return q; };
    int32_t *mtile_off = reinterpret_cast<int32_t *>(take((E + 1) * 4));
    __half *xp = reinterpret_cast<__half *>(take(R * d * 2));
    __half *w1t = reinterpret_cast<__half *>(take(E * 2 * r * d * 2));
    __half *bgt = reinterpret_cast<__half *>(take(E * f * r * 2));
    __half *but = reinterpret_cast<__half *>(take(E * f * r * 2));
    __half *adt = reinterpret_cast<__half *>(take(E * r * f * 2));
    __half *bdt = reinterpret_cast<__half *>(take(E * d * r * 2));
    __half *tb = reinterpret_cast<__half *>(take(R * 2 * r * 2));
    __half *hb = reinterpret_cast<__half *>(take(R * f * 2));
    __half *sb = reinterpret_cast<__half *>(take(R * r * 2));
    cudaError_t err;
    Marks none;
    Marks &mk = marks ? *marks : none;

    const bool per_slot = a.flags & LATENT_FLAG_OUT_PER_SLOT;
    if (!per_slot && (err = cudaMemsetAsync(a.out, 0, (size_t)a.T * d * sizeof(float), s)) != cudaSuccess) return err;
    k_pf_mtiles<<<1, 1024, 0, s>>>(a.rt.counts, a.E, mtile_off);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    if ((err = launch_dequant_t(a.gate_a, a.E, w1t, (int64_t)2 * r * d, 0, s)) != cudaSuccess) return err;
    if ((err = launch_dequant_t(a.up_a, a.E, w1t, (int64_t)2 * r * d, (int)r, s)) != cudaSuccess) return err;
    if ((err = launch_dequant_t(a.gate_b, a.E, bgt, (int64_t)f * r, 0, s)) != cudaSuccess) return err;
    if ((err = launch_dequant_t(a.up_b, a.E, but, (int64_t)f * r, 0, s)) != cudaSuccess) return err;
    if ((err = launch_dequant_t(a.down_a, a.E, adt, (int64_t)r * f, 0, s)) != cudaSuccess) return err;
    if ((err = launch_dequant_t(a.down_b, a.E, bdt, (int64_t)d * r, 0, s)) != cudaSuccess) return err;
    switch (a.x_type) {
        case LATENT_TYPE_F32: k_pf_gather<LATENT_TYPE_F32><<<a.R, 256, 0, s>>>(a.x, a.rt.order, a.rt.offsets, a.E, a.k, a.d, xp); break;
        case LATENT_TYPE_F16: k_pf_gather<LATENT_TYPE_F16><<<a.R, 256, 0, s>>>(a.x, a.rt.order, a.rt.offsets, a.E, a.k, a.d, xp); break;
        default: k_pf_gather<LATENT_TYPE_BF16><<<a.R, 256, 0, s>>>(a.x, a.rt.order, a.rt.offsets, a.E, a.k, a.d, xp); break;
    }
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    mk.mark(s);

    CUtensorMap mX, mW1, mT, mBg, mBu, mH, mAd, mS, mBd;
    if (!make_map(&mX, xp, R, d, kBM) || !make_map(&mW1, w1t, E * 2 * r, d, 256) || !make_map(&mT, tb, R, 2 * r, kBM) ||
        !make_map(&mBg, bgt, E * f, r, 128) || !make_map(&mBu, but, E * f, r, 128) || !make_map(&mH, hb, R, f, kBM) ||
        !make_map(&mAd, adt, E * r, f, 256) || !make_map(&mS, sb, R, r, kBM) || !make_map(&mBd, bdt, E * d, r, 256))
        return cudaErrorInvalidValue;

    GemmArgs g{};
    g.E = a.E;
    g.offsets = a.rt.offsets;
    g.mtile_off = mtile_off;
    g.order = a.rt.order;
    g.weights = a.weights;
    g.w_type = a.w_type;
    g.flags = a.flags;
    g.err = a.rt.err;

    g.K = a.d; g.N = 2 * a.r; g.ldo = 2 * a.r; g.out = tb;
    if ((err = launch_gemm<kModeF16>(mX, mW1, mW1, g, s)) != cudaSuccess) return err;
    mk.mark(s);
    g.K = a.r; g.N = a.f; g.ldo = a.f; g.out = hb; g.a_koff2 = a.r;
    if ((err = launch_gemm<kModeSwiGLU>(mT, mBg, mBu, g, s)) != cudaSuccess) return err;
    mk.mark(s);
    g.K = a.f; g.N = a.r; g.ldo = a.r; g.out = sb; g.a_koff2 = 0;
    if ((err = launch_gemm<kModeF16>(mH, mAd, mAd, g, s)) != cudaSuccess) return err;
    mk.mark(s);
    g.K = a.r; g.N = a.d; g.ldo = a.d; g.out = nullptr;
    g.out_slot = a.out;
    g.per_slot_d = a.d;
    g.top_k = a.k;
    if ((err = launch_gemm<kModeF32>(mS, mBd, mBd, g, s)) != cudaSuccess) return err;
    mk.mark(s);
    // per-slot output: the rows of skipped slots are zeroed here; the combined
    // output was summed by G4's epilogue
    if (per_slot) err = launch_combine(a, s);
    mk.mark(s);
    return err;
}

}  // namespace latent
