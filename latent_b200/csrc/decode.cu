// Decode path: the latent expert FFN as a chain of quantized vector-matrix
// products on CUDA cores with fp32 accumulation (rel-L2 <= 1e-5 vs the fp32
// reference runtime, loader/latent_runtime.py:35-59).
//
// One persistent, cooperatively launched kernel (one CTA per SM) streams the
// whole chain.  Routed positions are grouped into virtual experts (an expert
// and up to 4 of its consecutive routed positions).  For every virtual expert
// the chain is four phases of "segments", a segment being one 256-column tile
// of one factor matrix over all of its rows:
//   phase 1  t = x . [A_g | A_u]        segments (matrix, tile of r), rows d
//   phase 2  g|u = t . B_{g|u}          segments (tile of f, matrix), rows r
//   phase 3  s = h . A_d, h = silu(g)u  segments (tile of r),         rows f
//   phase 4  y = s . B_d                segments (tile of d),         rows r
// followed by the top-k combine of y into out (phase 5).
//
// Work partition: the segments of a phase, in order, form one stream of
// 8-row blocks weighted by their width; each warp of the grid takes one
// contiguous, equally weighted range of it (no work queue, no CTA-wide
// synchronisation).  A warp's range covers parts ("pieces") of one or a few
// segments.  A piece accumulates its rows in registers and adds the sums of
// its columns into the phase output with vector atomic adds (the outputs are
// zeroed at kernel start, before any piece adds), then adds its row count to
// the segment's arrival counter.  A piece of the next phase waits (bounded)
// until all rows of the segments it reads have arrived; the SwiGLU (and
// the optional router weight) is applied where phase 3 loads its inputs.
// Every CTA is resident (cooperative launch) and every warp takes its ranges
// in phase order, so every wait ends; a wait that exceeds its bound sets
// kErrTimeout and the kernel runs to completion without waiting further.
// The split-K sums are added in arrival order, so results agree between
// calls to fp32 rounding, not bitwise.
//
// Memory path: each warp streams its codes and scales through a private
// 3-deep cp.async ring of 16-row stages (2 KB of codes + 256 B of scales at
// full width), issued from per-piece pointers two stages ahead across piece
// and phase boundaries, so the weight stream never waits for a dependency.
// Inputs and INT8 records of the next stage are prefetched into registers.
//
// Inner loop: one code path for every virtual expert (fewer than 4 tokens are
// zero-padded: one instantiation keeps the hot code in the instruction
// cache); a lane owns 8 consecutive columns (4 code bytes) of a row, which
// keeps the accumulators at 32 registers and lets 16 warps share an SM (the
// kernel is latency-bound: more warps beat fewer instructions per element).
// One PRMT builds
// the shared-memory address of a code byte's entry in a 64 KB table of float
// pairs (16 replicas x 256 byte values x 2 tables, replica = lane % 16, so a
// warp lookup touches every bank exactly twice) and one 64-bit load returns
// the two decoded values, which feed packed fp32x2 FMAs directly.  Table 0
// holds NF4 level pairs; table 1 holds (lo - 8, hi - 8) pairs and is selected
// by the sign bit of the group's scale, which flags INT8 groups.
//
// INT8 groups: int8(hi:lo) = (lo - 8) + 16 * (hi' - 8) + 8 with hi' = hi ^ 8.
// The main loop adds (lo - 8) through table 1.  After each stage the warp
// walks the stage's INT8 records (one contiguous run in the tile-major order;
// a lane takes its share of the rows of its own group) and adds
// 16 * (hi' - 8) + 8 through the same table.
#include <map>
#include <mutex>

#include "internal.h"

namespace latent {

namespace {

typedef unsigned long long u64;

#ifndef LATENT_DECODE_WARPS
#define LATENT_DECODE_WARPS 16
#endif
constexpr int kSW = LATENT_DECODE_WARPS;                 // warps per CTA
constexpr int kSThreads = kSW * 32;
constexpr int kMaxCtas = 160;           // grid cap the workspace is sized for
constexpr int kRing = 3;                // stages per warp ring (two issued ahead)
constexpr int kStRows = 16;             // rows per stage
constexpr int kStCode = kStRows * 128;  // code bytes per stage (at most)
constexpr int kStScale = kStRows * 16;  // scale bytes per stage (at most)
constexpr int kStBytes = kStCode + kStScale;
constexpr int kRecStage = 32;           // INT8 records per stage staged in shared memory
constexpr int kNT = kVirtTokens;        // tokens per virtual expert (4)
constexpr int kMinUnits = 64;           // least work per warp, in (8 rows x 32 columns) units
constexpr unsigned long long kWaitNs = 2000000000ull;  // a dependency wait gives up after 2 s

// Per-warp shared memory (byte offsets); "x2" areas alternate by stage parity
// because a stage's INT8 pass runs after the next stage's main loop.
constexpr int kWRing = 0;
constexpr int kWIn = kWRing + kRing * kStBytes;   // x2 float [kStRows][kNT] inputs of the stage
constexpr int kWStash = kWIn + 2 * kStRows * kNT * 4;  // x2 uint16 [kStRows][8] scales of INT8 groups
constexpr int kWRow = kWStash + 2 * kStRows * 8 * 2;   // x2 uint16 [kStRows] INT8 prefix | flags << 8
constexpr int kWRec = kWRow + 2 * kStRows * 2;    // x2 uint8 [kRecStage][16] INT8 records of the stage
constexpr int kWMeta = kWRec + 2 * kRecStage * 16;  // 4 x uint32 [4] INT8 table words of upcoming pieces
constexpr int kWIter = kWMeta + 4 * 16;           // Iter of the consumer
constexpr int kWIssue = kWIter + 48;              // Iter of the stage issuer
constexpr int kWarpBytes = kWIssue + 48;
static_assert(kWarpBytes % 16 == 0, "warp area alignment");
// CTA area at the start of dynamic shared memory, then the areas of the low
// warps, the pair table at shared address 64 K, the remaining warps after it.
constexpr int kCumCap = 1024;          // virtual experts whose cost prefix is kept in shared memory
constexpr int kCtaRange = 512 + (kCumCap + 4) * 4;     // Pos [4][kSW + 1] phase ranges of the CTA's warps
constexpr int kCtaBytes = kCtaRange + ((4 * (kSW + 1) * 12 + 15) / 16) * 16;
constexpr uint32_t kTableAddr = 65536;
constexpr int kTableBytes = 65536;
constexpr int kMaxSmemBase = 4096;      // dynamic shared memory must start below this address
constexpr int kLowWarpsFit = (int)((kTableAddr - kMaxSmemBase - kCtaBytes) / kWarpBytes);
constexpr int kLowWarps = kLowWarpsFit < kSW ? kLowWarpsFit : kSW;
constexpr int kDynSmem = (int)kTableAddr + kTableBytes + (kSW - kLowWarps) * kWarpBytes;
static_assert(kDynSmem <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ u64 pack2(float a, float b) {
    u64 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void unpack2(u64 v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ void ffma2(u64 &acc, u64 x, u64 v) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(x), "l"(v));
}
__device__ __forceinline__ u64 fadd2(u64 a, u64 b) {
    u64 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ u64 lds64(uint32_t addr) {
    u64 v;
    asm("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void cp_async16(uint32_t s, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait until *flag >= target (one lane).  Returns false (and records
// kErrTimeout) when the bound is exceeded or another warp already gave up.
__device__ bool wait_ge(const uint32_t *flag, uint32_t target, uint32_t *err) {
    const unsigned long long t0 = gtime();
    unsigned ns = 256;
    while (true) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v >= target) return true;
        uint32_t e;
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(e) : "l"(err) : "memory");
        if (e & kErrTimeout) return false;
        if (gtime() - t0 > kWaitNs) {
            atomicOr(err, kErrTimeout);
            return false;
        }
        // long sleeps: a polling warp takes issue slots from the warps still computing
        __nanosleep(ns);
        if (ns < 512) ns <<= 1;
    }
}

// ---------------------------------------------------------------------------
// Phase geometry.  A phase has M matrices (1 or 2) of C column tiles of L
// rows; segment j is (m = j / C, c = j % C), except in phase 2 where it is
// (c = j / 2, m = j % 2) so that the gate and up tiles of a column range are
// neighbours.  Work units: an 8-row block of a tile of width w weighs w / 32.
struct Geo {
    int P;        // 1..4
    int M, C, L;  // matrices, tiles, rows
    int N;        // matrix columns
    int S;        // segments per virtual expert
    int wl;       // width of the last tile
    int Gp;       // warps the phase is spread over
    int pad[2];
    int64_t Uf, Ul, Wm, Wv;  // units of a full tile, the last tile, a matrix, a virtual expert
    int64_t total;           // cost-weighted units of the phase: Wv * (sum of the virtual experts' weights)
};

// Cost-weight prefix of virtual expert v (cum(n_virt) = total weight), from
// shared memory when it fits there, else from the virtual-expert table.
struct Pos;
struct CumView {
    const int *s;      // [n + 1] or nullptr
    const int4 *virt;
    const Pos *rng;    // phase ranges of the CTA's warps (see iter_next)
    int n, total;
    __device__ __forceinline__ int operator()(int v) const {
        if (s) return s[v];
        return v >= n ? total : __ldg(&virt[v].w);
    }
};

__device__ __forceinline__ int tile_w(const Geo &g, int c) { return c == g.C - 1 ? g.wl : 256; }
__device__ __forceinline__ int seg_m(const Geo &g, int j) { return g.P == 2 ? (j & 1) : j / g.C; }
__device__ __forceinline__ int seg_c(const Geo &g, int j) { return g.P == 2 ? (j >> 1) : j % g.C; }

__device__ Geo make_geo(const DecodeArgs &a, int P, int n_virt, int wtot, int G) {
    Geo g;
    g.P = P;
    g.L = P == 1 ? a.d : P == 2 ? a.r : P == 3 ? a.f : a.r;
    g.N = P == 1 ? a.r : P == 2 ? a.f : P == 3 ? a.r : a.d;
    g.M = P <= 2 ? 2 : 1;
    g.C = (g.N + 255) / 256;
    g.S = g.M * g.C;
    g.wl = g.N - 256 * (g.C - 1);
    g.Uf = (int64_t)(g.L / 8) * 8;
    g.Ul = (int64_t)(g.L / 8) * (g.wl / 32);
    g.Wm = (int64_t)(g.C - 1) * g.Uf + g.Ul;
    g.Wv = g.Wm * g.M;
    g.total = g.Wv * wtot;
    const int64_t gp = (g.Wv * n_virt + kMinUnits - 1) / kMinUnits;  // warps used: by bytes, not weights
    g.Gp = (int)(gp < G ? gp : G);
    if (g.Gp < 1) g.Gp = 1;
    g.pad[0] = g.pad[1] = 0;
    return g;
}

struct Pos {
    int v, j, blk;
};

// The block containing weighted unit u (0 <= u < total).  Offsets inside one
// virtual expert (< Wv * weight, far below 2^31) use 32-bit arithmetic.
__device__ Pos pos_of(const Geo &g, int64_t u, const CumView &cum) {
    Pos p;
    int lo = 0, hi = cum.n - 1;  // largest v with cum(v) * Wv <= u
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if ((int64_t)cum(mid) * g.Wv <= u) lo = mid; else hi = mid - 1;
    }
    p.v = lo;
    const int wt = cum(lo + 1) - cum(lo);
    const int rem0 = (int)(u - (int64_t)cum(lo) * g.Wv);
    const int rem = wt == 1 ? rem0 : rem0 / wt;
    const int Uf = (int)g.Uf, Ul = (int)g.Ul;
    int c, r3;
    if (g.P == 2) {
        c = rem / (2 * Uf);
        if (c > g.C - 1) c = g.C - 1;
        const int r2 = rem - c * 2 * Uf;
        const int U = c == g.C - 1 ? Ul : Uf;
        const int m = r2 / U;
        r3 = r2 - m * U;
        p.j = 2 * c + m;
    } else {
        const int Wm = (int)g.Wm;
        const int m = rem / Wm;
        const int r2 = rem - m * Wm;
        c = r2 / Uf;
        if (c > g.C - 1) c = g.C - 1;
        r3 = r2 - c * Uf;
        p.j = m * g.C + c;
    }
    p.blk = r3 / (tile_w(g, c) / 32);
    return p;
}

// First block of warp w's range (w in [0, Gp]); warp w owns [start(w), start(w+1)).
__device__ Pos range_start(const Geo &g, int w, const CumView &cum) {
    const int64_t u = g.total * w / g.Gp;
    if (u >= g.total) return Pos{cum.n, 0, 0};
    return pos_of(g, u, cum);
}

__device__ __forceinline__ bool pos_less(const Pos &a, const Pos &b) {
    return a.v != b.v ? a.v < b.v : a.j != b.j ? a.j < b.j : a.blk < b.blk;
}

// ---------------------------------------------------------------------------
// Piece iteration: the pieces of a warp's ranges in phase order.  The
// consumer and the stage issuer each run one iterator over the same sequence
// (kept in the warp's shared area between pieces).
struct Iter {
    int P;         // phase of the current piece (5 once all ranges are done)
    Pos cur, end;  // start of the next piece, end of the warp's range in phase P
    int v, j;      // current piece: virtual expert, segment
    int row, row1; // first row, end row of the piece
};
static_assert(sizeof(Iter) <= 48, "iterator area");

// Moves to the next non-empty piece; false when all phases are done.  rng
// holds range_start of phase P for the CTA's warps 0..kSW at rng[(P-1)*(kSW+1) + w].
__device__ bool iter_next(Iter &it, const Geo *geo, int gw, const Pos *rng) {
    while (true) {
        if (it.P >= 1 && it.P <= 4 && pos_less(it.cur, it.end)) {
            const Geo &g = geo[it.P - 1];
            it.v = it.cur.v;
            it.j = it.cur.j;
            it.row = it.cur.blk * 8;
            it.row1 = (it.cur.v == it.end.v && it.cur.j == it.end.j) ? it.end.blk * 8 : g.L;
            if (++it.cur.j == g.S) {
                it.cur.j = 0;
                ++it.cur.v;
            }
            it.cur.blk = 0;
            if (it.row1 > it.row) return true;
            continue;
        }
        if (it.P >= 4) {
            it.P = 5;
            return false;
        }
        ++it.P;
        const Geo &g = geo[it.P - 1];
        if (gw < g.Gp) {
            const Pos *r = rng + (it.P - 1) * (kSW + 1) + (gw % kSW);
            it.cur = r[0];
            it.end = r[1];
        } else {
            it.cur = it.end = Pos{0, 0, 0};
        }
    }
}

__device__ __forceinline__ const latent_qmatrix &phase_matrix(const DecodeArgs &a, int P, int m) {
    return P == 1 ? (m ? a.up_a : a.gate_a) : P == 2 ? (m ? a.up_b : a.gate_b) : P == 3 ? a.down_a : a.down_b;
}

// Iterator step shared by all lanes: load from the warp area, advance, store back.
__device__ __forceinline__ bool shared_iter_next(Iter *itp, Iter &it, const Geo *geo, int gw, const CumView &cum,
                                                 int lane) {
    it = *itp;
    const bool more = iter_next(it, geo, gw, cum.rng);
    __syncwarp();
    if (lane == 0) *itp = it;
    __syncwarp();
    return more;
}

// Stage issuer: source pointers of the next stage of its current piece.
struct Issuer {
    const uint8_t *codes;
    const uint8_t *scales;
    int row, row1;  // next row, end row of the piece
    int cstride;    // code bytes per row (tile width / 2)
    int P;          // 0 before the first piece, 5 when all are issued
    int pc;         // pieces entered
};

// Mask/base words of the INT8 table around expert-local group q: word
// index, and whether q is past the last group (then all bits count).
__device__ __forceinline__ int64_t int8_word(const latent_qmatrix &m, int64_t q, bool &past) {
    const int64_t groups = m.rows * m.cols / 32, words = (groups + 31) / 32;
    past = q >= groups;
    return past ? words - 1 : (q >> 5);
}

// INT8 records before group q from the copied (base, mask) words.
__device__ __forceinline__ uint32_t int8_count(uint32_t base, uint32_t mask, int64_t q, bool past) {
    return base + __popc(past ? mask : (mask & ((1u << (q & 31)) - 1u)));
}

__device__ void issuer_next_piece(const DecodeArgs &a, Issuer &is, uint8_t *warea, const Geo *geo, int gw,
                                  const CumView &cum, int lane) {
    Iter it;
    if (!shared_iter_next(reinterpret_cast<Iter *>(warea + kWIssue), it, geo, gw, cum, lane)) {
        is.P = 5;
        return;
    }
    const Geo &g = geo[it.P - 1];
    const int m = seg_m(g, it.j), c = seg_c(g, it.j), w = tile_w(g, c), ng = w >> 5;
    const int e = __ldg(&a.rt.virt[it.v].x);
    const latent_qmatrix &qm = phase_matrix(a, it.P, m);
    const int64_t q0 = (int64_t)c * g.L * 8 + (int64_t)it.row * ng;  // expert-local flat group
    is.codes = qm.codes + (int64_t)e * (qm.rows * qm.cols / 2) + q0 * 16;
    is.scales = reinterpret_cast<const uint8_t *>(qm.scales + (int64_t)e * (qm.rows * qm.cols / 32) + q0);
    is.row = it.row;
    is.row1 = it.row1;
    is.cstride = w >> 1;
    is.P = it.P;
    // INT8 table words at the piece's first and end row; they land with the
    // piece's first stage, before the consumer needs them.
    if (qm.i8_mask && lane < 4) {
        const int64_t words = (qm.rows * qm.cols / 32 + 31) / 32;
        bool past;
        const int64_t q = (int64_t)c * g.L * 8 + (int64_t)(lane < 2 ? it.row : it.row1) * ng;
        const int64_t wi = (int64_t)e * words + int8_word(qm, q, past);
        const uint32_t *src = (lane & 1) ? qm.i8_mask + wi : qm.i8_base + wi;
        const uint32_t dst = smem_u32(warea + kWMeta + (is.pc & 3) * 16 + lane * 4);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
    }
    ++is.pc;
}

// Issues the next stage into ring slot `slot` (all lanes) and commits one
// cp.async group (empty once everything is issued).
__device__ __forceinline__ void issue_stage(const DecodeArgs &a, Issuer &is, uint8_t *warea, const Geo *geo, int gw,
                                            const CumView &cum, uint32_t slot, int lane) {
    if (is.P <= 4 && is.row >= is.row1) issuer_next_piece(a, is, warea, geo, gw, cum, lane);
    if (is.P <= 4) {
        const int n = min(kStRows, is.row1 - is.row);
        const int cb = n * is.cstride;  // code bytes, a multiple of 128
        for (int o = lane * 16; o < cb; o += 512) cp_async16(slot + o, is.codes + o);
        const int sbytes = cb >> 3;     // scale bytes, a multiple of 16
        if (lane * 16 < sbytes) cp_async16(slot + kStCode + lane * 16, is.scales + lane * 16);
        is.codes += cb;
        is.scales += sbytes;
        is.row += n;
    }
    cp_commit();
}

// ---------------------------------------------------------------------------
#ifndef LATENT_DECODE_COLS
#define LATENT_DECODE_COLS 8
#endif
template <int NT>
struct Mode {
    static constexpr int COLS = NT <= 4 ? LATENT_DECODE_COLS : 8;  // columns per lane
    static constexpr int NB = COLS / 2;            // code bytes per lane and row
};

// Inner loop over the n rows of one stage.  acc[t * NB + b] holds columns
// (2b, 2b+1) of the lane's COLS columns for token t.
template <int NT>
__device__ __forceinline__ void stage_rows(uint32_t slot, int n, int w, int ng, int rs, int ch, int rps,
                                           uint32_t in_s, uint32_t lb, u64 (&acc)[32]) {
    constexpr int NB = Mode<NT>::NB, COLS = Mode<NT>::COLS;
    const int wb = w >> 1;
    const int gofs = (ch * COLS) >> 5;
#pragma unroll 1
    for (int row = rs; row < n; row += rps) {
        const uint32_t cb = slot + row * wb + ch * NB;
        uint32_t q[2];
        if constexpr (NB == 8) {
            const uint2 v = lds_v2(cb);
            q[0] = v.x;
            q[1] = v.y;
        } else {
            q[0] = lds32(cb);
            q[1] = 0;
        }
        const uint32_t sb = lds16(slot + kStCode + (row * ng + gofs) * 2);
        const uint32_t lr = lb | ((sb >> 8) & 0x80u);
        const float sc = half_bits_to_float((uint16_t)(sb & 0x7FFFu));
        const uint32_t xa = in_s + (uint32_t)row * (kNT * 4);
        float xv[8];
        {
            const float4 x0 = lds_f4(xa);
            xv[0] = x0.x; xv[1] = x0.y; xv[2] = x0.z; xv[3] = x0.w;
            if constexpr (NT > 4) {
                const float4 x1 = lds_f4(xa + 16);
                xv[4] = x1.x; xv[5] = x1.y; xv[6] = x1.z; xv[7] = x1.w;
            }
        }
        u64 xs[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float v = xv[t] * sc;
            xs[t] = pack2(v, v);
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const uint32_t addr = __byte_perm(q[b >> 2], lr, 0x7604u | ((uint32_t)(b & 3) << 4));
            const u64 vv = lds64(addr);
#pragma unroll
            for (int t = 0; t < NT; ++t) ffma2(acc[t * NB + b], xs[t], vv);
        }
    }
}

// INT8 flags of one stage (from its scales, still in the ring): lanes
// 0..n-1 take row `lane`, store the row's record prefix and flags and the
// scales of its INT8 groups (buffer `par`), and every lane gets the row mask
// of its own group g.  Returns the stage's INT8 record count.
__device__ __forceinline__ int stage_flags(uint32_t slot, int n, int ng, int g, int lane, uint8_t *warea, int par,
                                           uint32_t &mask) {
    uint32_t flags = 0;
    if (lane < n) {
        uint8_t *stash = warea + kWStash + par * (kStRows * 16) + lane * 16;
        if (ng == 8) {  // full tile: the row's 8 scales are one 16-byte word; keep them all
            const float4 f = lds_f4(slot + kStCode + lane * 16);
            const uint32_t w0 = __float_as_uint(f.x), w1 = __float_as_uint(f.y);
            const uint32_t w2 = __float_as_uint(f.z), w3 = __float_as_uint(f.w);
            flags = ((w0 >> 15) & 1u) | ((w0 >> 30) & 2u) | ((w1 >> 13) & 4u) | ((w1 >> 28) & 8u) |
                    ((w2 >> 11) & 16u) | ((w2 >> 26) & 32u) | ((w3 >> 9) & 64u) | ((w3 >> 24) & 128u);
            *reinterpret_cast<float4 *>(stash) = f;
        } else {
            for (int gg = 0; gg < ng; ++gg) {
                const uint32_t sb = lds16(slot + kStCode + (lane * ng + gg) * 2);
                flags |= ((sb >> 15) & 1u) << gg;
                reinterpret_cast<uint16_t *>(stash)[gg] = (uint16_t)sb;
            }
        }
    }
    const int cnt = __popc(flags);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if ((lane & 15) >= o) incl += y;
    }
    if (lane < n)
        *reinterpret_cast<uint16_t *>(warea + kWRow + par * (kStRows * 2) + lane * 2) =
            (uint16_t)((incl - cnt) | (flags << 8));
    mask = 0;
    for (int gg = 0; gg < ng; ++gg) {
        const uint32_t b = __ballot_sync(0xffffffffu, (flags >> gg) & 1u);
        mask = gg == g ? (b & 0xFFFFu) : mask;
    }
    return __shfl_sync(0xffffffffu, incl, 15);
}

// INT8 high-nibble pass of a stage whose flags, scales, inputs and records
// sit in the buffers of parity `par`: the lane adds 16 * (hi' - 8) + 8 for
// its share of the rows of its own group (records past the first kRecStage
// are read from global memory at hi_stage).
template <int NT>
__device__ __forceinline__ void int8_pass(uint32_t wbase, int par, uint32_t mask, int g, int rs, int ch, int rps,
                                          const uint8_t *hi_stage, uint32_t lb, u64 (&acc)[32]) {
    constexpr int NB = Mode<NT>::NB, COLS = Mode<NT>::COLS;
    const int colb = ((ch * COLS) & 31) >> 1;  // byte offset of the lane's nibbles in a record
    const int cntg = __popc(mask);
    const int beg = rs * cntg / rps, end = (rs + 1) * cntg / rps;
    if (beg >= end) return;
    int row = (int)__fns(mask, 0, beg + 1);
    const uint32_t lr = lb | 0x80u;
    const uint32_t rowb = wbase + kWRow + par * (kStRows * 2);
    const uint32_t stb = wbase + kWStash + par * (kStRows * 16);
    const uint32_t recb = wbase + kWRec + par * (kRecStage * 16);
    const uint32_t inb = wbase + kWIn + par * (kStRows * kNT * 4);
    float cc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) cc[t] = 0.f;
    auto next_row = [&](int r) {
        const uint32_t rest = r >= 31 ? 0u : mask & (0xFFFFFFFEu << r);
        return __ffs(rest) - 1;
    };
    // the high nibbles (XOR 8), scale and inputs of the record of row r
    auto fetch = [&](int r, uint32_t (&hw)[2], float &sc, float (&xv)[NT]) {
        const uint32_t ri = lds16(rowb + r * 2);
        const int idx = (int)(ri & 0xFFu) + __popc((ri >> 8) & ((1u << g) - 1u));
        if (idx < kRecStage) {
            const uint32_t ra = recb + idx * 16 + colb;
            if constexpr (NB == 8) {
                const uint2 v = lds_v2(ra);
                hw[0] = v.x;
                hw[1] = v.y;
            } else {
                hw[0] = lds32(ra);
                hw[1] = 0;
            }
        } else {
            const uint8_t *q = hi_stage + (int64_t)idx * 16 + colb;
            if constexpr (NB == 8) {
                const uint2 v = __ldg(reinterpret_cast<const uint2 *>(q));
                hw[0] = v.x;
                hw[1] = v.y;
            } else {
                hw[0] = __ldg(reinterpret_cast<const uint32_t *>(q));
                hw[1] = 0;
            }
        }
        hw[0] ^= 0x88888888u;
        hw[1] ^= 0x88888888u;
        sc = half_bits_to_float((uint16_t)(lds16(stb + r * 16 + g * 2) & 0x7FFFu));
        const uint32_t xa = inb + (uint32_t)r * (kNT * 4);
        const float4 x0 = lds_f4(xa);
        float xt[8] = {x0.x, x0.y, x0.z, x0.w, 0.f, 0.f, 0.f, 0.f};
        if constexpr (NT > 4) {
            const float4 x1 = lds_f4(xa + 16);
            xt[4] = x1.x; xt[5] = x1.y; xt[6] = x1.z; xt[7] = x1.w;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) xv[t] = xt[t];
    };
    auto apply = [&](const uint32_t (&hw)[2], float sc, const float (&xv)[NT]) {
        u64 xs[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float v = xv[t] * sc;
            cc[t] = fmaf(8.f, v, cc[t]);
            const float v16 = 16.f * v;
            xs[t] = pack2(v16, v16);
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const uint32_t addr = __byte_perm(hw[b >> 2], lr, 0x7604u | ((uint32_t)(b & 3) << 4));
            const u64 vv = lds64(addr);
#pragma unroll
            for (int t = 0; t < NT; ++t) ffma2(acc[t * NB + b], xs[t], vv);
        }
    };    for (int it = beg; it < end; it += 2) {  // two records in flight
        const bool two = it + 1 < end;
        const int row2 = two ? next_row(row) : row;
        uint32_t hwa[2], hwb[2];
        float sca, scb, xa[NT], xb[NT];
        fetch(row, hwa, sca, xa);
        fetch(row2, hwb, scb, xb);
        apply(hwa, sca, xa);
        if (two) apply(hwb, scb, xb);
        row = next_row(row2);
    }
    // the "+ 8" of every INT8 group visited, on all of the lane's columns
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const u64 k = pack2(cc[t], cc[t]);
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[t * NB + b] = fadd2(acc[t * NB + b], k);
    }
}

// ---------------------------------------------------------------------------

// Where the inputs of a piece come from (kept in registers for the piece):
// token k of the lane's four reads element row of row tok[k] (-1: padded
// token) of the row-major [*, ld] matrix at base.  Phase 3 reads g at base
// and u half a row further and forms h = silu(g) * u [* w].
struct InSrc {
    const void *base;
    int tok[4];
    int ld;
    int kind;  // 0/1/2: x as f32/f16/bf16 (phase 1), 3: fp32 sums, 4: phase 3
};

__device__ __forceinline__ InSrc make_insrc(const DecodeArgs &a, int P, int m, int p0, int nt, int tq) {
    InSrc src;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int t = 4 * tq + k;
        src.tok[k] = t >= nt ? -1 : P == 1 ? __ldg(&a.rt.order[p0 + t]) / a.k : p0 + t;
    }
    if (P == 1) {
        src.base = a.x;
        src.ld = a.d;
        src.kind = a.x_type == LATENT_TYPE_F32 ? 0 : a.x_type == LATENT_TYPE_F16 ? 1 : 2;
    } else if (P == 2) {
        src.base = a.t + m * a.r;
        src.ld = 2 * a.r;
        src.kind = 3;
    } else if (P == 3) {
        src.base = a.gu;
        src.ld = 2 * a.f;
        src.kind = 4;
    } else {
        src.base = a.s;
        src.ld = a.r;
        src.kind = 3;
    }
    return src;
}

// Inputs of one stage row for the lane's four tokens (zero when not live),
// as raw bits (and phase 3's u): the loads complete while the stage before
// is processed, and in_value converts them when they are stored.
__device__ __forceinline__ void load_inputs(const InSrc &src, int row, bool live, uint32_t (&raw)[4],
                                            float (&rawu)[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t v = 0;
        float u = 0.f;
        if (live && src.tok[k] >= 0) {
            const int64_t i = (int64_t)src.tok[k] * src.ld + row;
            if (src.kind == 1 || src.kind == 2) {
                v = __ldg(reinterpret_cast<const unsigned short *>(src.base) + i);
            } else if (src.kind == 0) {
                v = __ldg(reinterpret_cast<const uint32_t *>(src.base) + i);
            } else {
                const uint32_t *g = reinterpret_cast<const uint32_t *>(src.base) + i;
                v = __ldcg(g);
                if (src.kind == 4) u = __uint_as_float(__ldcg(g + (src.ld >> 1)));
            }
        }
        raw[k] = v;
        rawu[k] = u;
    }
}

__device__ __forceinline__ float in_value(int kind, uint32_t v, float u, float w) {
    switch (kind) {
        case 1: return __half2float(__ushort_as_half((unsigned short)v));
        case 2: return __uint_as_float(v << 16);  // bf16 -> f32
        case 4: return silu_f32(__uint_as_float(v)) * u * w;
        default: return __uint_as_float(v);
    }
}

// Index of the arrival counter of segment (v, j) of phase P.
__device__ __forceinline__ int flag_index(const Geo &g, int v, int j) {
    return g.P == 2 ? v * g.C + (j >> 1) : v * g.S + j;
}

// Piece end: the lane-row reduction, the vector atomic adds into the phase
// output (after the kernel-start zeroing is complete), the arrival count.
template <int NT>
__device__ __forceinline__ void flush_piece(const DecodeArgs &a, const Geo &g, int v, int j, int p0, int nt, int rows,
                                            int lane, int rs, int ch, int lpr, bool active, bool &zeroed,
                                            u64 (&acc)[32]) {
    constexpr int NB = Mode<NT>::NB, COLS = Mode<NT>::COLS;
    for (int o = lpr; o < 32; o <<= 1) {
#pragma unroll
        for (int i = 0; i < NT * NB; ++i) acc[i] = fadd2(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], o));
    }
    if (!zeroed) {
        if (lane == 0) wait_ge(a.zero_done, gridDim.x, a.rt.err);
        __syncwarp();
        zeroed = true;
    }
    if (rs == 0 && active) {
        const int m = seg_m(g, j), col = 256 * seg_c(g, j) + ch * COLS;
        float *dst;
        int64_t ld;
        if (g.P == 1) {
            ld = 2 * a.r;
            dst = a.t + (int64_t)p0 * ld + m * a.r + col;
        } else if (g.P == 2) {
            ld = 2 * a.f;
            dst = a.gu + (int64_t)p0 * ld + m * a.f + col;
        } else if (g.P == 3) {
            ld = a.r;
            dst = a.s + (int64_t)p0 * ld + col;
        } else {
            ld = a.d;
            dst = a.y + (int64_t)p0 * ld + col;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < nt) {
#pragma unroll
                for (int b = 0; b < NB; b += 2) {
                    float x0, x1, x2, x3;
                    unpack2(acc[t * NB + b], x0, x1);
                    unpack2(acc[t * NB + b + 1], x2, x3);
                    atomicAdd(reinterpret_cast<float4 *>(dst + t * ld + 2 * b), make_float4(x0, x1, x2, x3));
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0ull;
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(a.arrive[g.P - 1] + flag_index(g, v, j), (uint32_t)rows);
}

// Bounded wait (lane 0) until every row of segment (v, j) of phase g.P
// (phase 2: of the gate/up pair) has arrived: pieces count their rows in.
__device__ __forceinline__ bool wait_segment(const DecodeArgs &a, const Geo &g, int v, int j) {
    return wait_ge(a.arrive[g.P - 1] + flag_index(g, v, j), (uint32_t)(g.P == 2 ? 2 * g.L : g.L), a.rt.err);
}

// Bounded wait (lane 0) for the previous-phase segments holding input rows
// [row0, row1) of a piece of phase P: phase 2 reads t_m (phase-1 segment
// (m, c)), phase 3 reads h (phase-2 pair c), phase 4 reads s (phase-3 segment c).
__device__ void wait_inputs(const DecodeArgs &a, const Geo *geo, int P, int v, int m, int row0, int row1, int lane) {
    if (P == 1 || lane != 0) return;
    const Geo &gp = geo[P - 2];
    for (int c = row0 / 256; c <= (row1 - 1) / 256; ++c) {
        const int j = P == 2 ? m * gp.C + c : P == 3 ? 2 * c : c;
        if (!wait_segment(a, gp, v, j)) return;
    }
}

struct WarpCtx {
    const Geo *geo;
    uint8_t *warea;
    uint32_t wbase, ring, lb;
    int gw, lane;
    CumView cum;
};

// Copies INT8 records [first, first + kRecStage) clamped to `end` into the
// record buffer of parity `par` and commits them as one cp.async group.
__device__ __forceinline__ void issue_records(const uint8_t *hi, uint32_t first, uint32_t end, uint32_t wbase,
                                              int par, int lane) {
    if (hi && first + (uint32_t)lane < end)
        cp_async16(wbase + kWRec + par * (kRecStage * 16) + lane * 16, hi + (int64_t)(first + lane) * 16);
    cp_commit();
}

// One piece: rows [it.row, it.row1) of segment (it.v, it.j) of phase it.P.
// Per stage k the warp commits the stage's INT8 records (R_k), then the
// codes of stage k+2 (S_{k+2}); the groups after S_k are always R_{k-1} and
// S_{k+1}, after R_{k-1} always S_{k+1}, R_k and S_{k+2}.
template <int NT>
__device__ __forceinline__ void run_piece(const DecodeArgs &a, const WarpCtx &wc, const Iter &it, Issuer &is,
                                          int &si, int &sc_, int cpc, bool &zeroed, u64 (&acc)[32]) {
    constexpr int COLS = Mode<NT>::COLS;
    const int lane = wc.lane;
    const Geo &g = wc.geo[it.P - 1];
    const int P = it.P, v = it.v, j = it.j, row1 = it.row1;
    const int m = seg_m(g, j), c = seg_c(g, j), w = tile_w(g, c), ng = w >> 5;
    const int4 ve = __ldg(&a.rt.virt[v]);
    const int p0 = ve.y, nt = ve.z;  // nt <= NT; tokens nt..NT-1 are zero inputs
    int lpr = 1;
    while (lpr * COLS < w) lpr <<= 1;
    const int rps = 32 / lpr, rs = lane / lpr, ch = lane % lpr;
    const bool active = ch * COLS < w;
    const int grp = (ch * COLS) >> 5;
    const latent_qmatrix &qm = phase_matrix(a, P, m);
    const int rl = lane & 15, tq = lane >> 4;
    const InSrc src = make_insrc(a, P, m, p0, nt, tq);
    float pw[4] = {1.f, 1.f, 1.f, 1.f};  // phase 3: router weights applied to h
    if (P == 3 && (a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN)) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (4 * tq + k < nt) pw[k] = load_weight(a.weights, a.w_type, a.rt.order[p0 + 4 * tq + k]);
    }
    wait_inputs(a, wc.geo, P, v, m, it.row, row1, lane);
    __syncwarp();
    uint32_t pre[4];
    float preu[4];
    load_inputs(src, it.row + rl, rl < row1 - it.row, pre, preu);
    const uint8_t *hi = nullptr;
    uint32_t rec_next = 0, rec_end = 0, prev_mask = 0;
    int prev_par = -1;
    const uint8_t *prev_hi = nullptr;
    // One pass of the loop per stage, plus one for the deferred INT8 pass of
    // the last stage (a single copy of the pass code).
    for (int row = it.row, k = 0;; ++k) {
        const bool main = row < row1;
        if (!main && prev_par < 0) break;
        const int n = main ? min(kStRows, row1 - row) : 0;
        const int par = k & 1;
        uint32_t mask = 0;
        int crec = 0;
        if (main) {
            if (tq * 4 < kNT)  // a row holds kNT tokens: lanes 16..31 carry tokens 4..7 when kNT == 8
                *reinterpret_cast<float4 *>(wc.warea + kWIn + par * (kStRows * kNT * 4) + rl * (kNT * 4) + tq * 16) =
                    make_float4(in_value(src.kind, pre[0], preu[0], pw[0]), in_value(src.kind, pre[1], preu[1], pw[1]),
                                in_value(src.kind, pre[2], preu[2], pw[2]), in_value(src.kind, pre[3], preu[3], pw[3]));
            if (row + n < row1) load_inputs(src, row + n + rl, rl < row1 - row - n, pre, preu);
            cp_wait<2>();  // S_k
            __syncwarp();
            if (k == 0 && qm.i8_mask) {  // the piece's INT8 range, from the words issued with S_0
                const uint32_t *meta = reinterpret_cast<const uint32_t *>(wc.warea + kWMeta + (cpc & 3) * 16);
                bool past;
                const int64_t q0 = (int64_t)c * g.L * 8;
                int8_word(qm, q0 + (int64_t)it.row * ng, past);
                rec_next = int8_count(meta[0], meta[1], q0 + (int64_t)it.row * ng, past);
                int8_word(qm, q0 + (int64_t)row1 * ng, past);
                rec_end = int8_count(meta[2], meta[3], q0 + (int64_t)row1 * ng, past);
                if (rec_end > rec_next) hi = qm.i8_hi;
            }
            issue_records(hi, rec_next, rec_end, wc.wbase, par, lane);  // R_k
            issue_stage(a, is, wc.warea, wc.geo, wc.gw, wc.cum, wc.ring + (si % kRing) * kStBytes, lane);  // S_{k+2}
            ++si;
            const uint32_t slot = wc.ring + (sc_ % kRing) * kStBytes;
            ++sc_;
            const uint32_t in_s = wc.wbase + kWIn + par * (kStRows * kNT * 4);
            if (active) stage_rows<NT>(slot, n, w, ng, rs, ch, rps, in_s, wc.lb, acc);
            if (hi) crec = stage_flags(slot, n, ng, grp, lane, wc.warea, par, mask);
        }
        if (prev_par >= 0) {  // deferred INT8 pass of stage k-1
            if (main)
                cp_wait<3>();  // R_{k-1}
            else
                cp_wait<1>();  // R_last
            __syncwarp();
            if (active && prev_mask) int8_pass<NT>(wc.wbase, prev_par, prev_mask, grp, rs, ch, rps, prev_hi, wc.lb, acc);
        }
        prev_par = main && hi ? par : -1;
        prev_mask = mask;
        prev_hi = hi ? hi + (int64_t)rec_next * 16 : nullptr;
        rec_next += crec;
        __syncwarp();
        row += n;
    }
    flush_piece<NT>(a, g, v, j, p0, nt, row1 - it.row, lane, rs, ch, lpr, active, zeroed, acc);
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSThreads, 1) k_decode(DecodeArgs args) {
    // Device functions take the arguments by reference; a reference to the
    // kernel parameter would give every thread a local-memory copy, so they
    // read this shared copy instead.
    __shared__ DecodeArgs sargs;
    if (threadIdx.x == 0) sargs = args;
    const DecodeArgs &a = sargs;
    extern __shared__ __align__(16) uint8_t dsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t a0 = smem_u32(dsm);
    Geo *geo = reinterpret_cast<Geo *>(dsm);
    int *cta_cum = reinterpret_cast<int *>(dsm + 512);                    // [kCumCap + 1]
    uint8_t *table = dsm + (kTableAddr - a0);
    uint8_t *warea = warp < kLowWarps ? dsm + kCtaBytes + warp * kWarpBytes
                                      : dsm + (kTableAddr + kTableBytes - a0) + (warp - kLowWarps) * kWarpBytes;
    static_assert(4 * sizeof(Geo) + 16 <= 512, "CTA area");
    if (a0 > (uint32_t)kMaxSmemBase) {  // layout assumption violated: fail loudly, touch nothing
        if (threadIdx.x == 0) atomicOr(args.rt.err, kErrLayout);
        return;
    }
    // pair table: entry (tbl, byte e, replica c) at e*256 + tbl*128 + c*8
    for (int i = threadIdx.x; i < 2 * 256 * 16; i += kSThreads) {
        const int tbl = i >> 12, e = (i >> 4) & 255, c = i & 15;
        float lo, hi;
        if (tbl == 0) {
            lo = kNF4Levels[e & 15];
            hi = kNF4Levels[e >> 4];
        } else {
            lo = (float)((e & 15) - 8);
            hi = (float)((e >> 4) - 8);
        }
        *reinterpret_cast<float2 *>(table + e * 256 + tbl * 128 + c * 8) = make_float2(lo, hi);
    }
    const int G = gridDim.x * kSW, gw = blockIdx.x * kSW + warp;
    __syncthreads();  // sargs
    const int nv = args.rt.n_virt[0], wtot = args.rt.n_virt[1];
    if (threadIdx.x < 4) geo[threadIdx.x] = make_geo(a, threadIdx.x + 1, nv, wtot, G);
    if (nv <= kCumCap)
        for (int v = threadIdx.x; v <= nv; v += kSThreads) cta_cum[v] = v < nv ? __ldg(&args.rt.virt[v].w) : wtot;
    {   // zero this CTA's share of the phase outputs t, gu, s, y (contiguous)
        const int64_t n4 = (int64_t)a.R * (3 * a.r + 2 * a.f + a.d) / 4;
        float4 *z = reinterpret_cast<float4 *>(a.t);
        for (int64_t i = (int64_t)blockIdx.x * kSThreads + threadIdx.x; i < n4; i += (int64_t)gridDim.x * kSThreads)
            __stcg(z + i, make_float4(0.f, 0.f, 0.f, 0.f));
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(args.zero_done, 1u);
    CumView cv;
    cv.s = nv <= kCumCap ? cta_cum : nullptr;
    cv.virt = args.rt.virt;
    cv.n = nv;
    cv.total = wtot;
    // the ranges of every phase for this CTA's warps, once (range_start of
    // warps blockIdx.x * kSW + 0 .. kSW, clamped to the phase's warp count)
    Pos *cta_rng = reinterpret_cast<Pos *>(dsm + kCtaRange);
    cv.rng = cta_rng;
    for (int t = threadIdx.x; t < 4 * (kSW + 1); t += kSThreads) {
        const int P = t / (kSW + 1), w = blockIdx.x * kSW + (t - P * (kSW + 1));
        cta_rng[t] = range_start(geo[P], w < geo[P].Gp ? w : geo[P].Gp, cv);
    }
    __syncthreads();
    WarpCtx wc;
    wc.geo = geo;
    wc.warea = warea;
    wc.wbase = smem_u32(warea);
    wc.ring = wc.wbase + kWRing;
    wc.lb = (kTableAddr & 0xFFFF0000u) | (uint32_t)((lane & 15) * 8);
    wc.gw = gw;
    wc.lane = lane;
    wc.cum = cv;
    Iter *cit = reinterpret_cast<Iter *>(warea + kWIter);
    if (lane == 0) {
        Iter z;
        z.P = 0;
        z.cur = z.end = Pos{0, 0, 0};
        z.v = z.j = z.row = z.row1 = 0;
        *cit = z;
        *reinterpret_cast<Iter *>(warea + kWIssue) = z;
    }
    __syncwarp();
    Issuer is;
    is.codes = is.scales = nullptr;
    is.row = is.row1 = is.cstride = 0;
    is.P = 0;
    is.pc = 0;
    int si = 0, sc_ = 0;  // stages issued / consumed
    // prologue: E, S_0, E, S_1 (E = empty group standing for R_-2, R_-1)
    for (int k = 0; k < kRing - 1; ++k, ++si) {
        cp_commit();
        issue_stage(a, is, warea, geo, gw, wc.cum, wc.ring + (si % kRing) * kStBytes, lane);
    }
    u64 acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0ull;
    Iter it;
    bool zeroed = false;  // the kernel-start zeroing is known complete
    for (int cpc = 0; shared_iter_next(cit, it, geo, gw, wc.cum, lane); ++cpc)
        run_piece<kNT>(a, wc, it, is, si, sc_, cpc, zeroed, acc);  // one code path: fewer tokens are zero-padded
    cp_wait<0>();

    // Phase 5: top-k combine per (token, 256-column tile of d), slot order;
    // zero rows of tokens without a live slot.  With OUT_PER_SLOT: y rows
    // copied to their slots, zero rows for skipped slots.
    const bool per_slot = a.flags & LATENT_FLAG_OUT_PER_SLOT;
    const bool wbd = a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN;
    const Geo &g4 = geo[3];
    const int n_units = (per_slot ? a.T * a.k : a.T) * g4.C;
    for (int u = gw; u < n_units; u += G) {
        const int row = u / g4.C, c = u - row * g4.C, w = tile_w(g4, c);
        const int col = 256 * c + lane * 8;
        const bool live_col = lane * 8 < w;
        if (per_slot) {
            const int p = a.rt.pos[row];
            float4 y0 = make_float4(0.f, 0.f, 0.f, 0.f), y1 = y0;
            if (p >= 0) {
                if (lane == 0) wait_segment(a, g4, a.rt.vslot[p], c);
                __syncwarp();
                if (live_col) {
                    const float4 *y = reinterpret_cast<const float4 *>(a.y + (int64_t)p * a.d + col);
                    y0 = __ldcg(y);
                    y1 = __ldcg(y + 1);
                }
            }
            if (live_col) {
                float4 *o = reinterpret_cast<float4 *>(a.out + (int64_t)row * a.d + col);
                o[0] = y0;
                o[1] = y1;
            }
            continue;
        }
        float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
        for (int jj = 0; jj < a.k; ++jj) {
            const int slot = row * a.k + jj;
            const int p = a.rt.pos[slot];
            if (p < 0) continue;
            if (lane == 0) wait_segment(a, g4, a.rt.vslot[p], c);
            __syncwarp();
            const float wt = wbd ? 1.f : load_weight(a.weights, a.w_type, slot);
            if (live_col) {
                const float4 *y = reinterpret_cast<const float4 *>(a.y + (int64_t)p * a.d + col);
                const float4 y0 = __ldcg(y), y1 = __ldcg(y + 1);
                s0.x = fmaf(wt, y0.x, s0.x); s0.y = fmaf(wt, y0.y, s0.y);
                s0.z = fmaf(wt, y0.z, s0.z); s0.w = fmaf(wt, y0.w, s0.w);
                s1.x = fmaf(wt, y1.x, s1.x); s1.y = fmaf(wt, y1.y, s1.y);
                s1.z = fmaf(wt, y1.z, s1.z); s1.w = fmaf(wt, y1.w, s1.w);
            }
        }
        if (live_col) {
            float4 *o = reinterpret_cast<float4 *>(a.out + (int64_t)row * a.d + col);
            o[0] = s0;
            o[1] = s1;
        }
    }
}


// Host-side mirror of make_geo for sizing (upper bounds over n_virt <= n_virt_max).
int host_flags(const DecodeArgs &a, int P) {
    const int N = P == 1 ? a.r : P == 2 ? a.f : P == 3 ? a.r : a.d;
    const int C = (N + 255) / 256, S = (P <= 2 ? 2 : 1) * C;
    return a.n_virt_max * (P == 2 ? C : S);
}

}  // namespace

void decode_plan(DecodeArgs &a) {
    a.R = a.T * a.k;
    a.nmax = a.E < a.R ? a.E : a.R;
    a.n_virt_max = a.nmax + a.R / kVirtTokens + 1;
}

int decode_sem_count(const DecodeArgs &a) {
    int n = 1;  // zero_done
    for (int P = 1; P <= 4; ++P) n += host_flags(a, P);
    return n;
}

size_t decode_scratch_floats(const DecodeArgs &a) {
    const size_t R = (size_t)a.R, r = (size_t)a.r;
    return R * 2 * r + R * 2 * (size_t)a.f + R * r + R * (size_t)a.d + 64;
}

void decode_bind_sem(DecodeArgs &a, uint32_t *sem) {
    for (int P = 1; P <= 4; ++P) {
        a.arrive[P - 1] = sem;
        sem += host_flags(a, P);
    }
    a.zero_done = sem;
}

void decode_bind_scratch(DecodeArgs &a, float *f) {
    const size_t R = (size_t)a.R, r = (size_t)a.r;
    a.t = f;  f += R * 2 * r;
    a.gu = f; f += R * 2 * (size_t)a.f;
    a.s = f;  f += R * r;
    a.y = f;
}

cudaError_t launch_decode(const DecodeArgs &a, cudaStream_t s, Marks *marks) {
    const void *fn = (const void *)k_decode;
    cudaError_t err = ensure_smem(fn, kDynSmem);
    if (err != cudaSuccess) return err;
    int dev = 0;
    if ((err = cudaGetDevice(&dev)) != cudaSuccess) return err;
    // SM count and residency per device, queried once
    static std::mutex mu;
    static std::map<int, int> grid_of;
    int grid = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto f = grid_of.find(dev);
        if (f != grid_of.end()) {
            grid = f->second;
        } else {
            int sms = 0, per_sm = 0;
            if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return err;
            if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kSThreads, kDynSmem)) != cudaSuccess)
                return err;
            if (per_sm < 1) return cudaErrorInvalidConfiguration;
            grid = sms < kMaxCtas ? sms : kMaxCtas;
            grid_of[dev] = grid;
        }
    }
    void *args[] = {(void *)&a};
    err = cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kSThreads), args, kDynSmem, s);
    if (marks) marks->mark(s);
    return err;
}

}  // namespace latent
