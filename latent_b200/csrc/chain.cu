// Decode path: the latent expert FFN as a chain of quantized vector-matrix
// products on CUDA cores with fp32 accumulation (rel-L2 <= 1e-5 against the
// fp32 reference runtime, loader/latent_runtime.py:35-59).
//
// Work.  Routing groups the routed (token, slot) positions of every active
// expert into virtual experts of at most 8 positions (NT = 4 or 8 token
// columns, zero-padded), so that each virtual expert streams its expert's
// factors once for all of its tokens.  Per virtual expert v the chain is
//   P1  T[v]  += x[v] . A_{g|u}       K-chunks of d, red.add (fp32)
//   P2  H[v]   = silu(T_g . B_g) * (T_u . B_u) [* w]     full K = r
//   P3  S[v]  += H[v] . A_d           K-chunks of f, red.add
//   P4  out   += w * (S[v] . B_d)     full K = r; or out[slot] = y
// Intermediates are [rows][NT] fp32 per virtual expert (token columns
// innermost), so the rows a stage needs are one contiguous run; T, S and out
// are zeroed by every CTA's share at kernel start.
//
// Items.  An item is (phase, v, matrix, 256-column tile, K-chunk); items are
// numbered phase-major, virtual-expert-major inside a phase, and handed out
// by one atomic counter, so an item's inputs come from items numbered before
// it and a CTA waits only on items taken earlier.  Each item of phase p
// counts its completion into done[p][v] (once per consumer warp); the inputs
// of a phase-p item are read only after done[p-1][v] reached its target.
//
// CTA.  One persistent CTA per SM (cooperative launch: every CTA is resident,
// which the zeroing at kernel start relies on), three roles:
//  - the producer warp takes items one at a time from the queue, loads their
//    virtual-expert entry and INT8 list blocks, and
//    fills a ring of kSlots stages (128 rows of one tile) with cp.async.bulk
//    copies completing on the slot's mbarrier: codes, scales, INT8 records
//    and the stage's INT8 list block.  Weight copies never wait for a
//    dependency.
//  - the input warp follows the stage headers: P1 stages get their x rows
//    gathered, converted and transposed into the slot; later phases wait for
//    their item's dependency and get their input rows by bulk copy.  Its
//    arrival on the slot's barrier orders those inputs before the consumers.
//  - consumer warp w owns quant group w % G of the tile (G = tile width / 32)
//    and rows part w / G of every stage: a lane holds CPL columns of one row
//    (CPL = 16 for NT = 4, 8 for NT = 8), so accumulators stay at 64 floats.
//    At the end of an item the lanes reduce-scatter their sums with shuffles
//    (each lane ends with one column), warps sharing a group add through
//    shared memory, and the epilogue writes the outputs; the completion count
//    is released one stage later (or before the warp would block), when the
//    writes have long been performed.
//
// Inner loop (per code byte: one PRMT + one 64-bit shared load).  A 64 KB
// table at shared address 64 K holds, per byte value, the pair of decoded
// values, replicated 16 times (replica = lane % 16: a warp's lookup touches
// every bank twice); table 0 holds NF4 level pairs, table 1 unsigned nibble
// pairs, selected by the sign bit of the group's scale (the INT8 flag).  An
// INT8 group adds the high nibbles afterwards: int8 = lo + 16 * sext(hi);
// the warp's INT8 rows are listed in shared memory and spread over its lanes,
// which look the high nibbles up in the unsigned table at byte ^ 0x88 and
// subtract 8 (sext(n) = (n ^ 8) - 8).
//
// Every wait is bounded (kWaitNs): a wait that gives up sets kErrTimeout,
// which every other wait sees, and the kernel unwinds (the producer lets its
// bulk copies land before the CTA exits).
#include <cuda.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>

#include "internal.h"

namespace latent {

namespace {

typedef unsigned long long u64;

constexpr int kNW = 8;                     // consumer warps
constexpr int kThreads = (kNW + 2) * 32;   // + the producer and the input warp
constexpr int kSlots = 4;
constexpr int kStageRows = 128;
constexpr int kListCap = 384;              // INT8 list entries staged per stage (more are read from global memory)
constexpr int kRecCap = 384;               // INT8 records staged per stage (more are read from global memory)
constexpr unsigned long long kWaitNs = 2000000000ull;

// Slot layout (bytes from the slot base, which is 1024-byte aligned: full
// tiles' codes arrive as one 128B-swizzled TMA box).
constexpr int kOffCodes = 0;
constexpr int kOffScales = kOffCodes + kStageRows * 128;
constexpr int kOffIn = kOffScales + kStageRows * 16;
constexpr int kOffLoff = kOffIn + kStageRows * 8 * 4;  // the stage's INT8 list block words (12 x int32)
constexpr int kOffList = kOffLoff + 64;                // its INT8 list entries (kListCap)
constexpr int kOffRec = kOffList + kListCap * 4;
constexpr int kOffHdr = kOffRec + kRecCap * 16;
constexpr int kOffPre = kOffHdr + 128;  // P4 (and weighted P2) first stage: the item's 8 output rows and router weights
constexpr int kSlotBytes = (kOffPre + 64 + 1023) / 1024 * 1024;
static_assert(kOffHdr % 16 == 0, "slot alignment");

// Dynamic shared memory: region A (barriers, per-warp item data, cross-warp
// buffer, slot 0) below shared address 64 K, the lookup table at
// [64 K, 128 K), slots 1.. above it.
constexpr int kBarBytes = 256;                        // mbarriers: full, empty, hdr per slot; consumers
static_assert(8 * (3 * kSlots + 1) <= kBarBytes, "mbarrier area");
constexpr int kPreBytes = kNW * 64;                   // per-warp slots and router weights of the current item
constexpr int kXbufBytes = 2 * kNW * 32 * 8 * 4;      // [matrix][warp][lane][8] cross-warp partial sums
constexpr uint32_t kTableAddr = 65536;
constexpr int kTableBytes = 65536;
constexpr int kRegionA = kBarBytes + kPreBytes + kXbufBytes + 1024 + kSlotBytes;  // + slot 0 alignment
constexpr int kMaxSmemBase = 65536 - kRegionA;  // dynamic shared memory must start below this
constexpr int kDynEnd = (int)kTableAddr + kTableBytes + (kSlots - 1) * kSlotBytes;
static_assert(kMaxSmemBase > 4096, "region A");
static_assert(kDynEnd <= 226 * 1024, "shared memory budget");

enum : int { kStop = -1 };
enum : int { kFirst = 1, kFlush = 2, kLast = 4, kSwz = 8 };  // kSwz: codes are 128B-swizzled

// Stage header, written by the producer before it arrives on the slot.
struct Hdr {
    int kind;     // phase 1..4, or kStop
    int v, e, m;  // virtual expert, expert, matrix (P1/P2: 0 gate, 1 up)
    int tc, tile_w, ng, nrows;
    int row0, nt, NT, off;
    int first_pos, flags, rec0, nrec_s;  // first INT8 record, records staged in the slot
    int list0, q0, nrec, in_row;         // first INT8 list entry of the stage's block, first group
                                         // (expert-local), INT8 records of the stage, first input row
};
static_assert(sizeof(Hdr) <= 128, "header");

struct Args {
    int E, d, f, r, T, k;
    int x_type, w_type;
    uint32_t flags;
    const void *x;
    const void *weights;
    float *out;
    latent_qmatrix mat[6];  // gate_a, up_a, gate_b, up_b, down_a, down_b
    const int32_t *order;
    const int4 *virt;       // {expert, first position, positions, token-column offset}
    const int32_t *n_virt;  // [0] virtual experts, [1] token columns
    uint32_t *err;
    uint32_t *queue;        // item counter
    uint32_t *zero_done;    // CTAs that zeroed their share of out, T and S
    uint32_t *done;         // [5][n_virt_max] completion counts (x kNW)
    int n_virt_max;
    float *tb, *hb, *sb;    // intermediates [token columns][rows] of 2r, f, r
    int chunk1, chunk3;     // K-chunk rows of P1 (over d) and P3 (over f)
    uint32_t tma_mask;      // bit i: maps.m[i] is valid (codes of mat[i] as [rows of 128 B])
    unsigned long long wait_ns;  // limit of every bounded wait (kWaitNs unless a test shortens it)
    uint32_t dep_extra;          // test hook: completions each dependency wait wants beyond the real count
};

// TMA maps of the factors' codes viewed as rows of 128 bytes (one full
// 256-column tile row each), 128B swizzle, {128 B, 128 rows} box.
struct CodeMaps {
    CUtensorMap m[6];
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Ring slots: slot 0 in region A, slots 1.. after the table.
struct Slots {
    uint8_t *s0, *s1;
    __device__ __forceinline__ uint8_t *operator[](int s) const { return s == 0 ? s0 : s1 + (s - 1) * kSlotBytes; }
};

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool aborted(const uint32_t *err) {
    uint32_t e;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(e) : "l"(err) : "memory");
    return (e & kErrTimeout) != 0;
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// --- mbarriers and bulk copies ------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}
// Bounded wait for phase `parity` of the barrier; false once the wait gave up
// (kErrTimeout recorded) or another wait already did.
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t *err, unsigned long long limit) {
    unsigned long long t0 = 0;
    for (unsigned i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 100000;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 15u) == 0) {
            if (aborted(err)) return false;
            const unsigned long long now = gtime();
            if (i == 0) {
                t0 = now;
            } else if (now - t0 > limit) {
                atomicOr(err, kErrTimeout);
                return false;
            }
        }
    }
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, u64 policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar,
                                            u64 policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void bulk_g2s_plain(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// --- shared-memory loads and packed fp32 ---------------------------------------
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
    asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
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
__device__ __forceinline__ void sts_v4(uint32_t addr, int x, int y, int z, int w) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ void sts_f4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// --- item geometry ---------------------------------------------------------------
__device__ __forceinline__ int tiles_of(int n) { return (n + 255) >> 8; }
__device__ __forceinline__ int tile_width(int n, int c) { return min(256, n - 256 * c); }
__device__ __forceinline__ int stages_of(int rows) { return (rows + kStageRows - 1) / kStageRows; }

struct Geo {
    int per_v[5];  // items per virtual expert of phases 1..4 (index 0 unused)
    int base[6];   // first item of phases 1..4 at base[1..4]; base[5] = total
    int kc1, kc3;  // K-chunks of P1 and P3
};

__device__ Geo make_geo(const Args &a, int nv) {
    Geo g;
    g.kc1 = (a.d + a.chunk1 - 1) / a.chunk1;
    g.kc3 = (a.f + a.chunk3 - 1) / a.chunk3;
    g.per_v[0] = 0;
    g.per_v[1] = 2 * tiles_of(a.r) * g.kc1;
    g.per_v[2] = tiles_of(a.f);
    g.per_v[3] = tiles_of(a.r) * g.kc3;
    g.per_v[4] = tiles_of(a.d);
    g.base[0] = g.base[1] = 0;
    for (int p = 1; p < 5; ++p) g.base[p + 1] = g.base[p] + nv * g.per_v[p];
    return g;
}

// One item.  Its shape follows from its index alone; its virtual-expert
// entry `ve` ({expert, first position, positions, token-column offset}) is
// loaded one item ahead of use.
struct Item {
    int phase, v, tc, kc;
    int m0;            // P1: the matrix (0 gate, 1 up); P2 covers both
    int row_b, row_e;  // K rows [row_b, row_e) of each matrix
    int tile_w, n_stages;
    int4 ve;
};

__device__ __forceinline__ const latent_qmatrix &phase_mat(const Args &a, int phase, int m) {
    // mat[]: 0 gate_a, 1 up_a, 2 gate_b, 3 up_b, 4 down_a, 5 down_b
    return phase == 1 ? a.mat[m] : phase == 2 ? a.mat[2 + m] : phase == 3 ? a.mat[4] : a.mat[5];
}

__device__ Item item_shape(const Args &a, const Geo &g, int i) {
    Item it;
    int p = 1;
    while (p < 4 && i >= g.base[p + 1]) ++p;
    const int j = i - g.base[p];
    it.phase = p;
    it.v = j / g.per_v[p];
    const int rest = j - it.v * g.per_v[p];
    it.kc = 0;
    it.tc = 0;
    it.m0 = 0;
    it.row_b = 0;
    it.row_e = 0;
    it.tile_w = 256;
    it.n_stages = 1;
    it.ve = make_int4(0, 0, 0, 0);
    if (p == 1) {
        const int C = tiles_of(a.r);
        it.m0 = rest / (C * g.kc1);
        it.tc = (rest / g.kc1) % C;
        it.kc = rest % g.kc1;
        it.row_b = it.kc * a.chunk1;
        it.row_e = min(a.d, it.row_b + a.chunk1);
        it.tile_w = tile_width(a.r, it.tc);
        it.n_stages = stages_of(it.row_e - it.row_b);
    } else if (p == 2) {
        it.tc = rest;
        it.row_e = a.r;
        it.tile_w = tile_width(a.f, it.tc);
        it.n_stages = 2 * stages_of(a.r);
    } else if (p == 3) {
        it.tc = rest / g.kc3;
        it.kc = rest % g.kc3;
        it.row_b = it.kc * a.chunk3;
        it.row_e = min(a.f, it.row_b + a.chunk3);
        it.tile_w = tile_width(a.r, it.tc);
        it.n_stages = stages_of(it.row_e - it.row_b);
    } else {
        it.tc = rest;
        it.row_e = a.r;
        it.tile_w = tile_width(a.d, it.tc);
        it.n_stages = stages_of(a.r);
    }
    return it;
}

// Stage s of an item: matrix, first row, rows.
__device__ __forceinline__ void stage_rows(const Item &it, int s, int &m, int &row0, int &n) {
    const int rows = it.row_e - it.row_b;
    int ss = s;
    m = it.m0;
    if (it.phase == 2) {
        const int per = stages_of(rows);
        m = s / per;
        ss = s - m * per;
    }
    row0 = it.row_b + ss * kStageRows;
    n = min(kStageRows, it.row_e - row0);
}

// Input of phase p >= 2 for the virtual expert at token column `off`: row 0
// of its [rows][NT] block (P2 reads rows m*r.. of the [2r][NT] block).
__device__ __forceinline__ const float *input_base(const Args &a, int p, int off) {
    if (p == 2) return a.tb + (int64_t)off * 2 * a.r;
    if (p == 3) return a.hb + (int64_t)off * a.f;
    return a.sb + (int64_t)off * a.r;
}

// INT8 list block of stage `lane` of an item (128-row block of one column
// tile of one expert, see latent_qmatrix.i8_blocks): its entry count, first
// list entry and first record, loaded one item before they are used.
struct MetaRaw {
    int n, list0, rec0, b;
};

__device__ MetaRaw meta_load(const Args &a, const Item &it, int lane) {
    MetaRaw r{0, 0, 0, -1};
    if (lane >= it.n_stages) return r;
    int m, row0, n;
    stage_rows(it, lane, m, row0, n);
    const latent_qmatrix &qm = phase_mat(a, it.phase, m);
    if (!qm.i8_blocks) return r;
    const int tiles = (int)((qm.cols + 255) >> 8), rblk = (int)((qm.rows + kStageRows - 1) / kStageRows);
    r.b = (it.ve.x * tiles + it.tc) * rblk + row0 / kStageRows;
    const int4 w2 = __ldg(reinterpret_cast<const int4 *>(qm.i8_blocks + (int64_t)r.b * 12 + 8));  // words 8..11
    r.n = w2.x;
    r.list0 = w2.y;
    r.rec0 = w2.z;
    return r;
}

// --- producer --------------------------------------------------------------------
// Items come from the counter one at a time: the next index is claimed once
// the current item's last stage has a slot, and its virtual-expert entry and
// INT8 block words are loaded after that stage is issued, while the ring
// (up to kSlots stages) keeps the consumers busy.  Claiming later keeps the
// end of the queue balanced: a CTA holds no item it cannot start soon (items
// claimed two ahead left CTAs idle at the end while others still held
// several: config 1 136 -> 126 us).  Every CTA handles its items in counter
// order and every dependency points to a lower item, so the lowest unfinished
// item is always at the head of some CTA: no deadlock.
__device__ __forceinline__ int mat_index(int phase, int m) { return phase == 1 ? m : phase == 2 ? 2 + m : phase == 3 ? 4 : 5; }

// One expert's view of a stacked factor, held in registers by the producer.
struct MatView {
    const uint8_t *codes;    // the expert's codes
    const uint16_t *scales;  // the expert's scales
    const int32_t *blocks;   // INT8 list blocks and entries (latent_qmatrix.i8_blocks / i8_list)
    const uint32_t *list;
    const uint8_t *hi;
    int64_t rows;
    int64_t cbyte;           // byte offset of the expert's codes in the stacked tensor
};

__device__ __forceinline__ MatView mat_view(const Args &a, int phase, int m, int e) {
    const latent_qmatrix &qm = phase_mat(a, phase, m);
    MatView v;
    const int64_t epe = qm.rows * qm.cols;
    v.cbyte = (int64_t)e * (epe >> 1);
    v.codes = qm.codes + v.cbyte;
    v.scales = qm.scales + (int64_t)e * (epe >> 5);
    v.blocks = qm.i8_blocks;
    v.list = qm.i8_list;
    v.hi = qm.i8_hi;
    v.rows = qm.rows;
    return v;
}

__device__ void producer_run(const Args &a, const CodeMaps &maps, const Geo &g, const Slots &slot_ptr, uint32_t bars,
                             int total) {
    const int lane = threadIdx.x & 31;
    const uint32_t full0 = bars, empty0 = bars + 8 * kSlots, hdr0 = bars + 16 * kSlots;
    u64 policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    int slot = 0;
    uint32_t empty_par = (1u << kSlots) - 1u;  // a fresh barrier passes a wait for parity 1
    uint32_t armed = 0, full_par = 0;
    bool ok = true;
    int q = 0;
    if (lane == 0) q = (int)atomicAdd(a.queue, 1u);
    const int i0 = __shfl_sync(0xffffffffu, q, 0);
    Item cur{};
    MetaRaw mc{0u, 0u, 0u, 0u};
    bool have_cur = i0 < total;
    if (have_cur) {
        cur = item_shape(a, g, i0);
        cur.ve = __ldg(&a.virt[cur.v]);
        mc = meta_load(a, cur, lane);
    }
    while (have_cur && ok) {
        const int ph = cur.phase;
        const int4 ve = cur.ve;
        const int NT = ve.z <= 4 ? 4 : 8;
        const int ng = cur.tile_w >> 5;
        // this lane's stage (s = lane): its INT8 list block
        // the item's matrices in registers (P2 covers gate and up)
        const MatView mv0 = mat_view(a, ph, cur.m0, ve.x);
        const MatView mv1 = ph == 2 ? mat_view(a, ph, 1, ve.x) : mv0;
        const uint32_t tma_bits = a.tma_mask;
        const int r_rows = a.r;
        for (int s = 0; s < cur.n_stages; ++s) {
            const uint32_t full = full0 + 8 * slot, empty = empty0 + 8 * slot, hdrb = hdr0 + 8 * slot;
            if (lane == 0) ok = mbar_wait(empty, (empty_par >> slot) & 1u, a.err, a.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            // the next item is claimed once the last stage of this one has a slot
            if (lane == 0 && s == cur.n_stages - 1) q = (int)atomicAdd(a.queue, 1u);
            const uint32_t sbase = smem_u32(slot_ptr[slot]);
            int m = 0, row0 = 0, n = 0;
            stage_rows(cur, s, m, row0, n);
            const bool second = ph == 2 && m == 1;
            MatView mv;
            mv.codes = second ? mv1.codes : mv0.codes;
            mv.scales = second ? mv1.scales : mv0.scales;
            mv.blocks = second ? mv1.blocks : mv0.blocks;
            mv.list = second ? mv1.list : mv0.list;
            mv.hi = second ? mv1.hi : mv0.hi;
            mv.rows = second ? mv1.rows : mv0.rows;
            mv.cbyte = second ? mv1.cbyte : mv0.cbyte;
            const uint32_t rec0 = (uint32_t)__shfl_sync(0xffffffffu, mc.rec0, s & 31);
            const uint32_t nrec = (uint32_t)__shfl_sync(0xffffffffu, mc.n, s & 31);
            const int list0 = __shfl_sync(0xffffffffu, mc.list0, s & 31);
            const int blk = __shfl_sync(0xffffffffu, mc.b, s & 31);
            const uint32_t nrec_s = min(nrec, (uint32_t)kRecCap);
            const int64_t q0 = (int64_t)cur.tc * mv.rows * 8 + (int64_t)row0 * ng;
            int fl = 0;
            if (s == 0) fl |= kFirst;
            if (s == cur.n_stages - 1) fl |= kFlush | kLast;
            if (ph == 2 && s == cur.n_stages / 2 - 1) fl |= kFlush;
            const int mi = mat_index(ph, m);
            const bool swz = ng == 8 && n == kStageRows && ((tma_bits >> mi) & 1u);
            if (swz) fl |= kSwz;
            if (lane == 0) {
                const uint32_t hp = sbase + kOffHdr;
                sts_v4(hp, ph, cur.v, ve.x, m);
                sts_v4(hp + 16, cur.tc, cur.tile_w, ng, n);
                sts_v4(hp + 32, row0, ve.z, NT, ve.w);
                sts_v4(hp + 48, ve.y, fl, (int)rec0, (int)nrec_s);
                sts_v4(hp + 64, list0, (int)q0, (int)nrec, (ph == 2 ? m * r_rows : 0) + row0);
                const uint32_t cbytes = (uint32_t)n * ng * 16, sbytes = (uint32_t)n * ng * 2;
                const uint32_t ibytes = ph >= 2 ? (uint32_t)n * NT * 4 : 0u;  // P1 inputs are stored by the input warp
                const uint32_t rbytes = nrec_s * 16;
                // the block's list words and its first entries (blocks pad their entries to 4: 16-byte copies)
                const uint32_t lbytes = nrec ? 48u + min((nrec + 3u) & ~3u, (uint32_t)kListCap) * 4u : 0u;
                // the input copy (issued by the input warp) completes on the same phase
                mbar_arrive_tx(full, cbytes + sbytes + ibytes + rbytes + lbytes);
                if (swz)  // rows of 128 bytes: row index of the stage's first code byte
                    tma_load_2d(sbase + kOffCodes, &maps.m[mi], 0, (int)((mv.cbyte + q0 * 16) >> 7), full, policy);
                else
                    bulk_g2s(sbase + kOffCodes, mv.codes + q0 * 16, cbytes, full, policy);
                bulk_g2s(sbase + kOffScales, mv.scales + q0, sbytes, full, policy);
                if (rbytes) bulk_g2s(sbase + kOffRec, mv.hi + (int64_t)rec0 * 16, rbytes, full, policy);
                if (lbytes) {
                    bulk_g2s(sbase + kOffLoff, mv.blocks + (int64_t)blk * 12, 48u, full, policy);
                    bulk_g2s(sbase + kOffList, mv.list + list0, lbytes - 48u, full, policy);
                }
                mbar_arrive(hdrb);
            }
            __syncwarp();
            if (armed & (1u << slot)) full_par ^= 1u << slot;
            armed |= 1u << slot;
            empty_par ^= 1u << slot;
            slot = slot + 1 == kSlots ? 0 : slot + 1;
        }
        if (!ok) break;
        const int i1 = __shfl_sync(0xffffffffu, q, 0);
        have_cur = i1 < total;
        if (have_cur) {
            cur = item_shape(a, g, i1);
            cur.ve = __ldg(&a.virt[cur.v]);
            mc = meta_load(a, cur, lane);
        }
    }
    if (lane == 0) {
        if (ok && mbar_wait(empty0 + 8 * slot, (empty_par >> slot) & 1u, a.err, a.wait_ns)) {
            reinterpret_cast<Hdr *>(slot_ptr[slot] + kOffHdr)->kind = kStop;
            mbar_arrive(full0 + 8 * slot);
            mbar_arrive(hdr0 + 8 * slot);
        } else {
            atomicOr(a.err, kErrTimeout);
            // unwinding: let every armed stage's copies land before the CTA exits (bounded)
            for (int s = 0; s < kSlots; ++s) {
                if (!(armed & (1u << s))) continue;
                const unsigned long long t1 = gtime();
                while (!mbar_test(full0 + 8 * s, (full_par >> s) & 1u)) {
                    if (gtime() - t1 > 200000000ull) break;
                    __nanosleep(1000);
                }
            }
        }
    }
    __syncwarp();
}

// First stage of an item whose epilogue needs its slots and router weights
// (P4; P2 when the weights scale the down projection's input).
__device__ __forceinline__ bool needs_pre(const Args &a, const Hdr &h) {
    return (h.flags & kFirst) && (h.kind == 4 || (h.kind == 2 && (a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN)));
}

// --- input warp ------------------------------------------------------------------
// Follows the stage headers in ring order.  P1 stages: the lanes gather the
// stage's rows of x for the item's tokens, convert them to fp32 and store
// them as [row][NT] in the slot.  Later phases: once the item's dependency is
// met (done[phase-1][v] reached its target), one bulk copy of the input rows.
// The first stage of a P4 item (and of a P2 item under weight-before-down)
// also gets the item's slots and router weights (global loads kept off the
// consumers).  Either way the warp then arrives on the slot's barrier
// (release: the inputs are ordered before the consumers' reads).  On an abort the copy is issued
// anyway, so that every byte the slot expects arrives.
template <int XT>
__device__ __forceinline__ void gather_rows(const Args &a, const Hdr &h, const int (&tok)[8], uint32_t in, int lane) {
    float xv[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int row = lane + 32 * j;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            float v = 0.f;
            if (row < h.nrows && tok[t] >= 0) v = load_act<XT>(a.x, (int64_t)tok[t] * a.d + h.row0 + row);
            xv[j][t] = v;
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int row = lane + 32 * j;
        if (row >= h.nrows) break;
        const uint32_t dst = in + row * h.NT * 4;
        sts_f4(dst, make_float4(xv[j][0], xv[j][1], xv[j][2], xv[j][3]));
        if (h.NT == 8) sts_f4(dst + 16, make_float4(xv[j][4], xv[j][5], xv[j][6], xv[j][7]));
    }
}

__device__ void input_run(const Args &a, const Geo &g, const Slots &slot_ptr, uint32_t bars) {
    const int lane = threadIdx.x & 31;
    const uint32_t full0 = bars, hdr0 = bars + 16 * kSlots;
    int slot = 0;
    uint32_t par = 0;
    const uint32_t *ok_ptr = nullptr;
    uint32_t ok_target = 0;
    int tok_v = -1;
    int tok[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) tok[t] = -1;
    while (true) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(hdr0 + 8 * slot, (par >> slot) & 1u, a.err, a.wait_ns);
        if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) return;
        par ^= 1u << slot;
        const uint8_t *sp = slot_ptr[slot];
        const Hdr h = *reinterpret_cast<const Hdr *>(sp + kOffHdr);
        const uint32_t full = full0 + 8 * slot;
        if (h.kind == kStop) {
            if (lane == 0) mbar_arrive(full);
            return;
        }
        if (needs_pre(a, h)) {  // the item's slots and router weights, staged for the consumers' epilogue
            if (lane < 8) {
                const int sl = lane < h.nt ? __ldg(&a.order[h.first_pos + lane]) : 0;
                int *pre = reinterpret_cast<int *>(const_cast<uint8_t *>(sp) + kOffPre);
                // the output row: the slot's own row, or its token's for the combined output
                pre[lane] = (a.flags & LATENT_FLAG_OUT_PER_SLOT) ? sl : sl / a.k;
                pre[8 + lane] = __float_as_int(lane < h.nt ? load_weight(a.weights, a.w_type, sl) : 0.f);
            }
            __syncwarp();  // before lane 0's arrival on the slot
        }
        if (h.kind == 1) {
            if (h.v != tok_v) {
                tok_v = h.v;
                const int mine = lane < h.nt ? __ldg(&a.order[h.first_pos + lane]) / a.k : -1;
#pragma unroll
                for (int t = 0; t < 8; ++t) tok[t] = __shfl_sync(0xffffffffu, mine, t);
            }
            const uint32_t in = smem_u32(sp) + kOffIn;
            if (a.x_type == LATENT_TYPE_F32)
                gather_rows<LATENT_TYPE_F32>(a, h, tok, in, lane);
            else if (a.x_type == LATENT_TYPE_F16)
                gather_rows<LATENT_TYPE_F16>(a, h, tok, in, lane);
            else
                gather_rows<LATENT_TYPE_BF16>(a, h, tok, in, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(full);
        } else if (lane == 0) {
            const uint32_t *dep = a.done + (int64_t)(h.kind - 1) * a.n_virt_max + h.v;
            const uint32_t target = (uint32_t)(kNW * g.per_v[h.kind - 1]) + a.dep_extra;
            if (!(dep == ok_ptr && target <= ok_target)) {
                const unsigned long long t0 = gtime();
                unsigned ns = 32;
                while (ld_acquire(dep) < target) {
                    if (aborted(a.err)) break;
                    if (gtime() - t0 > a.wait_ns) {
                        atomicOr(a.err, kErrTimeout);
                        break;
                    }
                    __nanosleep(ns);
                    if (ns < 512) ns <<= 1;
                }
                ok_ptr = dep;
                ok_target = target;
            }
            // the inputs were written through the generic proxy by other CTAs
            asm volatile("fence.proxy.async.global;" ::: "memory");
            const float *src = input_base(a, h.kind, h.off) + (int64_t)h.in_row * h.NT;
            bulk_g2s_plain(smem_u32(sp) + kOffIn, src, (uint32_t)h.nrows * h.NT * 4, full);
            mbar_arrive(full);
        }
        __syncwarp();
        slot = slot + 1 == kSlots ? 0 : slot + 1;
    }
}

// --- consumers -----------------------------------------------------------------------
template <int NT>
struct Cfg {
    static constexpr int CPL = NT == 4 ? 16 : 8;  // columns per lane
    static_assert(NT == 4 || NT == 8, "token columns");
    static constexpr int LPR = 32 / CPL;           // lanes per 32-column group row
    static constexpr int S = 32 / LPR;             // row slots per warp
    static constexpr int NB = CPL / 2;             // code bytes per lane and row
};

struct Warp {
    int w, lane;
    uint32_t lb;      // replica bits of the lookup address
    uint8_t *xbuf;
    int *pre;         // [8] output rows, [8] router weights (float bits) of the current item's tokens
    bool zeroed;      // the kernel-start zeroing is known complete
    int pend_kind, pend_v;  // completion count not yet released
    uint32_t xbar, xpar;    // the consumer warps' barrier and the phase this warp waits for next
};

// Bounded barrier of the kNW consumer warps (an mbarrier taking one arrival
// per warp; arrive releases, try_wait acquires).  False once the wait gave
// up: the warp then unwinds.  A bar.sync would wait forever for a consumer
// warp that had already unwound after an expired wait.
__device__ __forceinline__ bool consumers_sync(const Args &a, Warp &wc) {
    __syncwarp();
    if (wc.lane == 0) mbar_arrive(wc.xbar);
    const bool ok = mbar_wait(wc.xbar, wc.xpar, a.err, a.wait_ns);
    wc.xpar ^= 1u;
    return __all_sync(0xffffffffu, ok);
}

// Main loop over the warp's rows of one stage, then the stage's INT8 rows.
template <int NT>
__device__ __forceinline__ void consume_stage(const Args &a, const Hdr &h, uint32_t sb, const Warp &wc, int g, int rr0,
                                              int rr1, u64 (&acc)[32]) {
    using C = Cfg<NT>;
    const int lane = wc.lane;
    const int rs = lane / C::LPR, ch = lane % C::LPR;
    const uint32_t codes = sb + kOffCodes + ch * C::NB;
    const uint32_t scales = sb + kOffScales + g * 2;
    const uint32_t in = sb + kOffIn;
    const int rowb = h.ng * 16, srow = h.ng * 2;
    // 128B-swizzled stage: the 16-byte chunk of group g in row r sits at chunk g ^ (r & 7)
    const int swz = (h.flags & kSwz) ? 7 : 0;
#pragma unroll 1
    for (int row = rr0 + rs; row < rr1; row += C::S) {
        uint32_t q[2];
        const uint32_t ca = codes + row * rowb + ((g ^ (row & swz)) << 4);
        if constexpr (C::NB == 8) {
            const uint2 v = lds_v2(ca);
            q[0] = v.x;
            q[1] = v.y;
        } else {
            q[0] = lds32(ca);
            q[1] = 0;
        }
        const uint32_t sbits = lds16(scales + row * srow);
        const uint32_t lr = wc.lb | ((sbits >> 8) & 0x80u);
        const float sc = __half2float(__ushort_as_half((unsigned short)(sbits & 0x7FFFu)));
        u64 xs[NT];
#pragma unroll
        for (int t4 = 0; t4 < NT; t4 += 4) {
            const float4 xv = lds_f4(in + (row * NT + t4) * 4);
            xs[t4 + 0] = pack2(xv.x * sc, xv.x * sc);
            xs[t4 + 1] = pack2(xv.y * sc, xv.y * sc);
            xs[t4 + 2] = pack2(xv.z * sc, xv.z * sc);
            xs[t4 + 3] = pack2(xv.w * sc, xv.w * sc);
        }
#pragma unroll
        for (int b = 0; b < C::NB; ++b) {
            const uint32_t addr = __byte_perm(q[b >> 2], lr, 0x7604u | ((uint32_t)(b & 3) << 4));
            const u64 vv = lds64(addr);
#pragma unroll
            for (int t = 0; t < NT; ++t) ffma2(acc[t * C::NB + b], xs[t], vv);
        }
    }
    // INT8 groups: add 16 * sext(hi) for the warp's INT8 rows of group g.  The
    // stage's list block holds column g's entries (row, record) in row order;
    // the row slots take them in turn.
    if (h.nrec == 0) return;
    const latent_qmatrix &qm = phase_mat(a, h.kind, h.m);
    const int o0 = (int)lds32(sb + kOffLoff + 4 * g);
    const int o1 = min((int)lds32(sb + kOffLoff + 4 * (g + 1)), h.nrec);  // tables are not trusted past nrec
#pragma unroll 1
    for (int k = o0 + rs; k < o1; k += C::S) {
        const uint32_t ent = k < kListCap ? lds32(sb + kOffList + 4 * k) : __ldg(qm.i8_list + h.list0 + k);
        const int r = (int)(ent >> 16);
        if (r < rr0 || r >= rr1) continue;  // another warp's rows
        const uint32_t ri = ent & 0xFFFFu;
        const uint32_t sbits = lds16(scales + r * srow);
        float4 xv[NT / 4];
#pragma unroll
        for (int t4 = 0; t4 < NT / 4; ++t4) xv[t4] = lds_f4(in + (r * NT + 4 * t4) * 4);
        const uint32_t rho = ri + (uint32_t)h.rec0;
        uint32_t hw[2];
        if (ri < (uint32_t)h.nrec_s) {
            const uint32_t ra = sb + kOffRec + ri * 16 + ch * C::NB;
            if constexpr (C::NB == 8) {
                const uint2 v = lds_v2(ra);
                hw[0] = v.x;
                hw[1] = v.y;
            } else {
                hw[0] = lds32(ra);
                hw[1] = 0;
            }
        } else {
            if (ri >= (uint32_t)h.nrec) {  // an entry past the block's records: bad tables
                if (ch == 0) atomicOr(a.err, kErrLayout);
                continue;
            }
            const uint8_t *gp = qm.i8_hi + (int64_t)rho * 16 + ch * C::NB;
            if constexpr (C::NB == 8) {
                const uint2 v = __ldg(reinterpret_cast<const uint2 *>(gp));
                hw[0] = v.x;
                hw[1] = v.y;
            } else {
                hw[0] = __ldg(reinterpret_cast<const uint32_t *>(gp));
                hw[1] = 0;
            }
        }
        const float sc16 = 16.f * __half2float(__ushort_as_half((unsigned short)(sbits & 0x7FFFu)));
        u64 xs[NT];
#pragma unroll
        for (int t4 = 0; t4 < NT / 4; ++t4) {
            xs[4 * t4 + 0] = pack2(xv[t4].x * sc16, xv[t4].x * sc16);
            xs[4 * t4 + 1] = pack2(xv[t4].y * sc16, xv[t4].y * sc16);
            xs[4 * t4 + 2] = pack2(xv[t4].z * sc16, xv[t4].z * sc16);
            xs[4 * t4 + 3] = pack2(xv[t4].w * sc16, xv[t4].w * sc16);
        }
        // sext(n) = (n ^ 8) - 8: table 1 (unsigned nibble pairs) at byte ^ 0x88, minus 8
        const u64 bias = pack2(-8.f, -8.f);
        const uint32_t lr1 = wc.lb | 0x80u;
        const uint32_t hx[2] = {hw[0] ^ 0x88888888u, hw[1] ^ 0x88888888u};
#pragma unroll
        for (int b = 0; b < C::NB; ++b) {
            const uint32_t addr = __byte_perm(hx[b >> 2], lr1, 0x7604u | ((uint32_t)(b & 3) << 4));
            const u64 vv = fadd2(lds64(addr), bias);
#pragma unroll
            for (int t = 0; t < NT; ++t) ffma2(acc[t * C::NB + b], xs[t], vv);
        }
    }
}

// Lane reduce-scatter over the row slots: afterwards lane (rs, ch) holds
// column ch*CPL + rs of its group for every token in v[0..NT).
template <int NT>
__device__ __forceinline__ void reduce_scatter(u64 (&acc)[32], float (&v)[8], int lane) {
    using C = Cfg<NT>;
    float f[NT][C::CPL];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int b = 0; b < C::NB; ++b) unpack2(acc[t * C::NB + b], f[t][2 * b], f[t][2 * b + 1]);
#pragma unroll
    for (int half = C::CPL / 2, xm = 16; half >= 1; half >>= 1, xm >>= 1) {
        const bool up = (lane & xm) != 0;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int c = 0; c < half; ++c) {
                const float lo = f[t][c], hi = f[t][c + half];
                const float send = up ? lo : hi;
                const float keep = up ? hi : lo;
                f[t][c] = keep + __shfl_xor_sync(0xffffffffu, send, xm);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = t < NT ? f[t < NT ? t : 0][0] : 0.f;
}

// Bounded wait (lane 0) for the zeroing of out, T and S by every CTA.
__device__ void wait_zeroed(const Args &a) {
    const unsigned long long t0 = gtime();
    while (ld_acquire(a.zero_done) < gridDim.x) {
        if (aborted(a.err)) return;
        if (gtime() - t0 > a.wait_ns) {
            atomicOr(a.err, kErrTimeout);
            return;
        }
        __nanosleep(256);
    }
}

// Writes the item's results for column `col` (tile-relative) of tokens 0..NT.
template <int NT>
__device__ __forceinline__ void epilogue(const Args &a, const Hdr &h, int col, const float (&g)[8], const float (&u)[8],
                                         const int *pre) {
    const int gc = 256 * h.tc + col;  // column within the factor
    if (h.kind == 1 || h.kind == 3) {
        float *dst = h.kind == 1 ? a.tb + (int64_t)h.off * 2 * a.r + ((int64_t)h.m * a.r + gc) * NT
                                 : a.sb + (int64_t)h.off * a.r + (int64_t)gc * NT;
#pragma unroll
        for (int t4 = 0; t4 < NT; t4 += 4)
            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + t4), "f"(g[t4]), "f"(g[t4 + 1]),
                         "f"(g[t4 + 2]), "f"(g[t4 + 3])
                         : "memory");
    } else if (h.kind == 2) {
        const bool wbd = a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN;
        float hv[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) hv[t] = t < h.nt ? silu_f32(g[t]) * u[t] * (wbd ? __int_as_float(pre[8 + t]) : 1.f) : 0.f;
        float *dst = a.hb + (int64_t)h.off * a.f + (int64_t)gc * NT;
#pragma unroll
        for (int t4 = 0; t4 < NT; t4 += 4)
            *reinterpret_cast<float4 *>(dst + t4) = make_float4(hv[t4], hv[t4 + 1], hv[t4 + 2], hv[t4 + 3]);
    } else {
        const bool per_slot = a.flags & LATENT_FLAG_OUT_PER_SLOT;
        const bool wbd = a.flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            if (t < h.nt) {
                const int orow = pre[t];  // output row (slot, or token of the combined output)
                if (per_slot) {
                    a.out[(int64_t)orow * a.d + gc] = g[t];
                } else {
                    float *o = a.out + (int64_t)orow * a.d + gc;
                    const float y = wbd ? g[t] : __int_as_float(pre[8 + t]) * g[t];
                    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(o), "f"(y) : "memory");
                }
            }
        }
    }
}

// Group and row part of warp w for a tile of ng groups; rows [rr0, rr1) of a
// stage of n rows.  Warps past G * P have no columns (ng not a power of two).
__device__ __forceinline__ void warp_part(int w, int ng, int n, int &g, int &rp, int &P, int &rr0, int &rr1) {
    if (ng == kNW) {  // full tiles: one warp per group, every row (no divisions)
        P = 1;
        g = w;
        rp = 0;
        rr0 = 0;
        rr1 = n;
        return;
    }
    if ((ng & (ng - 1)) == 0) {  // 1, 2 or 4 groups: shifts
        const int lg = __ffs(ng) - 1;
        P = kNW >> lg;
        g = w & (ng - 1);
        rp = w >> lg;
        const int lp = __ffs(P) - 1;
        const int per = (n + P - 1) >> lp;
        rr0 = min(n, rp * per);
        rr1 = min(n, rr0 + per);
        return;
    }
    P = kNW / ng;
    if (P < 1) P = 1;
    g = w % ng;
    rp = w / ng;
    if (rp >= P) {
        g = -1;
        rr0 = rr1 = 0;
        return;
    }
    const int per = (n + P - 1) / P;
    rr0 = min(n, rp * per);
    rr1 = min(n, rr0 + per);
}

// Releases the warp's pending completion count: the lanes' epilogue writes
// are ordered before lane 0's release reduction by the warp barrier.
__device__ __forceinline__ void release_pending(const Args &a, Warp &wc) {
    if (wc.pend_kind < 0) return;
    __syncwarp();
    if (wc.lane == 0) {
        uint32_t *p = a.done + (int64_t)wc.pend_kind * a.n_virt_max + wc.pend_v;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p) : "memory");
    }
    wc.pend_kind = -1;
}

// Consumer warp main loop.
__device__ void consumer_run(const Args &a, const Slots &slot_ptr, uint32_t bars, Warp &wc) {
    const int lane = wc.lane;
    const uint32_t full0 = bars, empty0 = bars + 8 * kSlots;
    int slot = 0;
    uint32_t par_bits = 0;
    u64 acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0ull;
    float gv[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) gv[t] = 0.f;
    while (true) {
        const uint32_t full = full0 + 8 * slot, empty = empty0 + 8 * slot;
        const uint32_t par = (par_bits >> slot) & 1u;
        // a pending completion must not wait behind a stage that may depend on it
        if (wc.pend_kind >= 0 && !mbar_test(full, par)) release_pending(a, wc);
        if (!__all_sync(0xffffffffu, mbar_wait(full, par, a.err, a.wait_ns))) return;
        par_bits ^= 1u << slot;
        const uint8_t *sp = slot_ptr[slot];
        const uint32_t sb = smem_u32(sp);
        const Hdr h = *reinterpret_cast<const Hdr *>(sp + kOffHdr);
        if (h.kind == kStop) {
            release_pending(a, wc);
            return;
        }
        if (needs_pre(a, h) && lane < 16)  // the item's slots and router weights, read by its epilogue
            wc.pre[lane] = reinterpret_cast<const int *>(sp + kOffPre)[lane];
        int g, rp, P, rr0, rr1;
        warp_part(wc.w, h.ng, h.nrows, g, rp, P, rr0, rr1);
        if (g >= 0) {
            if (h.NT == 4)
                consume_stage<4>(a, h, sb, wc, g, rr0, rr1, acc);
            else
                consume_stage<8>(a, h, sb, wc, g, rr0, rr1, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty);
        slot = slot + 1 == kSlots ? 0 : slot + 1;
        release_pending(a, wc);  // the previous item's writes are long performed by now
        if (!(h.flags & kFlush)) continue;
        // a matrix of the item is complete: reduce the warp's sums
        float v[8];
        if (g >= 0) {
            if (h.NT == 4)
                reduce_scatter<4>(acc, v, lane);
            else
                reduce_scatter<8>(acc, v, lane);
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0ull;
        if (h.kind == 2 && !(h.flags & kLast)) {  // P2: the gate half; keep it until the up half is done
#pragma unroll
            for (int t = 0; t < 8; ++t) gv[t] = v[t];
            continue;
        }
        float uv[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            uv[t] = h.kind == 2 ? v[t] : 0.f;
            if (h.kind != 2) gv[t] = v[t];
        }
        // warps sharing a group add through shared memory (tiles narrower than kNW groups)
        if (P > 1) {
            float *xb = reinterpret_cast<float *>(wc.xbuf);
            if (g >= 0 && rp > 0) {
                float *d0 = xb + ((size_t)(0 * kNW + wc.w) * 32 + lane) * 8;
                float *d1 = xb + ((size_t)(1 * kNW + wc.w) * 32 + lane) * 8;
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    d0[t] = gv[t];
                    d1[t] = uv[t];
                }
            }
            if (!consumers_sync(a, wc)) return;
            if (g >= 0 && rp == 0) {
                for (int q = 1; q < P; ++q) {
                    const int ow = q * h.ng + g;
                    const float *s0 = xb + ((size_t)(0 * kNW + ow) * 32 + lane) * 8;
                    const float *s1 = xb + ((size_t)(1 * kNW + ow) * 32 + lane) * 8;
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        gv[t] += s0[t];
                        uv[t] += s1[t];
                    }
                }
            }
            if (!consumers_sync(a, wc)) return;  // the buffer is rewritten by the next narrow item
        }
        if (h.kind != 2 && !wc.zeroed) {  // red.add targets are zeroed by every CTA at kernel start
            if (lane == 0) wait_zeroed(a);
            __syncwarp();
            wc.zeroed = true;
        }
        if (g >= 0 && rp == 0) {
            // lane (rs, ch) holds column ch * CPL + rs (LPR = 2 or 4: shifts, not divisions)
            const int llpr = h.NT == 4 ? 1 : 2;  // log2(Cfg<NT>::LPR)
            const int cpl = h.NT == 4 ? Cfg<4>::CPL : Cfg<8>::CPL;
            const int col = 32 * g + (lane & ((1 << llpr) - 1)) * cpl + (lane >> llpr);
            if (col < h.tile_w) {
                if (h.NT == 4)
                    epilogue<4>(a, h, col, gv, uv, wc.pre);
                else
                    epilogue<8>(a, h, col, gv, uv, wc.pre);
            }
        }
        if (h.kind < 4) {  // P4 has no dependents
            wc.pend_kind = h.kind;
            wc.pend_v = h.v;
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) k_chain(Args args, const __grid_constant__ CodeMaps maps) {
    __shared__ Args sargs;
    if (threadIdx.x == 0) sargs = args;
    static_assert(kNW == 8, "warp roles: consumers 0..7, producer 8, input 9");
    extern __shared__ __align__(16) uint8_t dsm[];
    const uint32_t a0 = smem_u32(dsm);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (a0 > (uint32_t)kMaxSmemBase) {  // layout assumption violated: fail loudly, touch nothing
        if (threadIdx.x == 0) atomicOr(args.err, kErrLayout);
        return;
    }
    uint8_t *ctl = dsm;
    uint8_t *xbuf = ctl + kBarBytes + kPreBytes;
    Slots slot_ptr;
    {
        const uint32_t s0 = (smem_u32(xbuf + kXbufBytes) + 1023u) & ~1023u;  // 1024-byte aligned
        slot_ptr.s0 = dsm + (s0 - a0);
    }
    slot_ptr.s1 = dsm + (kTableAddr + kTableBytes - a0);
    uint8_t *table = dsm + (kTableAddr - a0);
    const uint32_t bars = smem_u32(ctl);  // full[kSlots], empty[kSlots], hdr[kSlots], consumer barrier
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(bars + 8 * s, 2);                 // producer + input warp (+ transaction bytes)
            mbar_init(bars + 8 * (kSlots + s), kNW);    // consumer warps
            mbar_init(bars + 8 * (2 * kSlots + s), 1);  // producer
        }
        mbar_init(bars + 8 * 3 * kSlots, kNW);  // the consumer warps' barrier
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();  // sargs and the barriers
    const Args &a = sargs;
    if (warp == kNW) {  // the producer starts at once: it touches neither the table nor the zeroed buffers
        const Geo g = make_geo(a, __ldg(a.n_virt));
        producer_run(a, maps, g, slot_ptr, bars, g.base[5]);
        return;
    }
    // lookup table: entry (tbl, byte e, replica c) at e*256 + tbl*128 + c*8
    constexpr int kOthers = (kNW + 1) * 32;  // consumers and the input warp
    const int ot = warp < kNW ? (int)threadIdx.x : (int)threadIdx.x - 32;  // 0 .. kOthers-1 without the producer
    for (int i = ot; i < 2 * 256 * 16; i += kOthers) {
        const int tbl = i >> 12, e = (i >> 4) & 255, c = i & 15;
        float lo, hi;
        if (tbl == 0) {
            lo = kNF4Levels[e & 15];
            hi = kNF4Levels[e >> 4];
        } else {
            lo = (float)(e & 15);
            hi = (float)(e >> 4);
        }
        *reinterpret_cast<float2 *>(table + e * 256 + tbl * 128 + c * 8) = make_float2(lo, hi);
    }
    // zero this CTA's share of out, T and S (the red.add targets)
    {
        const bool per_slot = a.flags & LATENT_FLAG_OUT_PER_SLOT;
        const int64_t cols = __ldg(a.n_virt + 1);
        const int64_t n_out = (int64_t)(per_slot ? a.T * a.k : a.T) * a.d / 4;
        const int64_t n_t = cols * 2 * a.r / 4, n_s = cols * a.r / 4;
        const int64_t stride = (int64_t)gridDim.x * kOthers;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t i = (int64_t)blockIdx.x * kOthers + ot; i < n_out + n_t + n_s; i += stride) {
            float4 *p = i < n_out ? reinterpret_cast<float4 *>(a.out) + i
                        : i < n_out + n_t ? reinterpret_cast<float4 *>(a.tb) + (i - n_out)
                                          : reinterpret_cast<float4 *>(a.sb) + (i - n_out - n_t);
            *p = z;
        }
        __threadfence();
    }
    asm volatile("bar.sync 2, %0;" ::"n"(kOthers) : "memory");  // the table and this CTA's zeroing
    if (threadIdx.x == 0) atomicAdd(a.zero_done, 1u);
    const Geo g = make_geo(a, __ldg(a.n_virt));
    if (warp == kNW + 1) {
        input_run(a, g, slot_ptr, bars);
    } else {
        Warp wc;
        wc.w = warp;
        wc.lane = lane;
        wc.lb = kTableAddr | (uint32_t)((lane & 15) * 8);
        wc.pre = reinterpret_cast<int *>(ctl + kBarBytes + warp * 64);
        wc.xbuf = xbuf;
        wc.zeroed = false;
        wc.pend_kind = -1;
        wc.pend_v = 0;
        wc.xbar = bars + 8 * 3 * kSlots;
        wc.xpar = 0;
        consumer_run(a, slot_ptr, bars, wc);
    }
}

}  // namespace

// Decode-path workspace: virtual-expert token columns are bounded by 8 per
// virtual expert.
static size_t token_cols(const DecodeArgs &a) { return (size_t)a.n_virt_max * 8; }

void decode_plan(DecodeArgs &a) {
    a.R = a.T * a.k;
    a.nmax = a.E < a.R ? a.E : a.R;
    a.n_virt_max = a.nmax + a.R / kVirtTokens + 1;
}

int decode_sem_count(const DecodeArgs &a) { return 2 + 5 * a.n_virt_max; }

size_t decode_scratch_floats(const DecodeArgs &a) {
    return token_cols(a) * (2 * (size_t)a.r + (size_t)a.f + (size_t)a.r) + 64;
}

void decode_bind_sem(DecodeArgs &a, uint32_t *sem) {
    a.queue = sem;
    a.zero_done = sem + 1;
    a.done = sem + 2;
}

void decode_bind_scratch(DecodeArgs &a, float *f) {
    const size_t tc = token_cols(a);
    a.x0 = nullptr;
    a.tb = f;
    f += tc * 2 * (size_t)a.r;
    a.hb = f;
    f += tc * (size_t)a.f;
    a.sb = f;
}

// K-chunk rows of the split phases: chunks of about `stages` stages, even,
// multiples of the stage rows.
static int chunk_rows(int K, int stages) {
    if (stages < 1) stages = 1;
    if (stages > 32) stages = 32;  // the producer keeps one stage's metadata per lane
    int rows = stages * kStageRows;
    const int n = (K + rows - 1) / rows;  // even chunks, multiples of the stage rows
    rows = ((K + n - 1) / n + kStageRows - 1) / kStageRows * kStageRows;
    return rows < K ? rows : K;
}

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
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

// The codes of one stacked factor (E experts) as rows of 128 bytes for the
// 128B-swizzled stage loads; cached per buffer and shape (the factors outlive
// many calls; encoding costs host time).  False when the factor has no full
// 256-column tile or the driver entry point is missing.
bool codes_map(CUtensorMap *out, const latent_qmatrix &m, int E) {
    if (m.cols < 256) return false;
    const uint64_t bytes = (uint64_t)E * (uint64_t)(m.rows * m.cols / 2);
    const uint64_t rows = bytes / 128;
    if (rows < (uint64_t)kStageRows || rows > 0xFFFFFFFFull) return false;
    struct Key {
        const void *p;
        int64_t r, c;
        int e;
        bool operator<(const Key &o) const {
            return p != o.p ? p < o.p : r != o.r ? r < o.r : c != o.c ? c < o.c : e < o.e;
        }
    };
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key k{m.codes, m.rows, m.cols, E};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(k);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    cuuint64_t dims[2] = {128, rows};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {128, (cuuint32_t)kStageRows};
    cuuint32_t es[2] = {1, 1};
    CUtensorMap map;
    if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(m.codes), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache.size() > 4096) cache.clear();
    cache[k] = map;
    *out = map;
    return true;
}

}  // namespace

// Failure-path test hook (latent_debug_set_wait_limit).
std::atomic<unsigned long long> g_wait_ns{kWaitNs};
std::atomic<uint32_t> g_dep_extra{0};

cudaError_t launch_decode(const DecodeArgs &d, cudaStream_t s, Marks *marks) {
    const void *fn = (const void *)k_chain;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    static std::mutex mu;
    static std::map<int, int> grid_of;
    int grid = 0;
    const size_t smem = (size_t)kDynEnd;  // upper bound: the dynamic base is at least 0
    if ((err = ensure_smem(fn, smem)) != cudaSuccess) return err;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = grid_of.find(dev);
        if (it != grid_of.end()) {
            grid = it->second;
        } else {
            int sms = 0, per_sm = 0;
            if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return err;
            if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem)) != cudaSuccess)
                return err;
            if (per_sm < 1) return cudaErrorInvalidConfiguration;
            grid = sms;
            grid_of[dev] = grid;
        }
    }
    Args a{};
    a.E = d.E;
    a.d = d.d;
    a.f = d.f;
    a.r = d.r;
    a.T = d.T;
    a.k = d.k;
    a.x_type = d.x_type;
    a.w_type = d.w_type;
    a.flags = d.flags;
    a.x = d.x;
    a.weights = d.weights;
    a.out = d.out;
    a.mat[0] = d.gate_a;
    a.mat[1] = d.up_a;
    a.mat[2] = d.gate_b;
    a.mat[3] = d.up_b;
    a.mat[4] = d.down_a;
    a.mat[5] = d.down_b;
    a.order = d.rt.order;
    a.virt = d.rt.virt;
    a.n_virt = d.rt.n_virt;
    a.err = d.rt.err;
    a.queue = d.queue;
    a.zero_done = d.zero_done;
    a.done = d.done;
    a.n_virt_max = d.n_virt_max;
    a.tb = d.tb;
    a.hb = d.hb;
    a.sb = d.sb;
    // K-chunks: about four P1 items per CTA for the active experts the batch
    // can have.  Longer items cut the per-item epilogues and split-K adds,
    // shorter ones keep the CTAs busy to the end (config 1: 4 x 512 rows;
    // config 4 rank 256 at batch 1 / 64: 28 x 256 / 2 x 3584 rows).  P3
    // takes chunks of the same size.
    const int nact = d.nmax > 0 ? d.nmax : 1;
    const int kc1 = (4 * grid + 2 * nact - 1) / (2 * nact);
    const int st = ((d.d + kc1 - 1) / kc1 + kStageRows - 1) / kStageRows;
    a.chunk1 = chunk_rows(d.d, st);
    a.chunk3 = chunk_rows(d.f, st);
    a.wait_ns = g_wait_ns.load();
    a.dep_extra = g_dep_extra.load();
    CodeMaps maps;
    memset(&maps, 0, sizeof(maps));
    a.tma_mask = 0;
    for (int i = 0; i < 6; ++i)
        if (codes_map(&maps.m[i], a.mat[i], d.E)) a.tma_mask |= 1u << i;
    void *args[] = {(void *)&a, (void *)&maps};
    err = cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kThreads), args, smem, s);
    if (marks) marks->mark(s);
    return err;
}

}  // namespace latent

extern "C" LATENT_API int latent_debug_set_wait_limit(uint64_t wait_ns, int32_t unreachable_dependency) {
    if (wait_ns != 0 && (wait_ns < 1000000ull || wait_ns > latent::kWaitNs)) return LATENT_ERR_INVALID;
    latent::g_wait_ns.store(wait_ns ? wait_ns : latent::kWaitNs);
    latent::g_dep_extra.store(unreachable_dependency ? 1u : 0u);
    return LATENT_OK;
}
