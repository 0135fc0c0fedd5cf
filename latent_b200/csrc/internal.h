// Internal declarations shared by the CUDA translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace latent {

constexpr int kRouteSingleMax = 4096;  // routed slots served by one routing block
constexpr int kRouteChunk = 8192;      // slots per block in the multi-block routing
constexpr int kMaxExperts = 1024;
constexpr int kVirtTokens = 8;         // routed positions per virtual expert (decode path)

// Token columns of a virtual expert of nt routed positions: the decode
// kernel runs 4-column and 8-column code paths (fewer positions are
// zero-padded), and lays its intermediates out with this many columns.
__host__ __device__ constexpr int virt_weight(int nt) { return nt <= 0 ? 0 : nt <= 4 ? 4 : 8; }

struct RouteArgs {
    const int32_t *ids;
    int R;          // T * k slots
    int E;
    int top_k;
    uint32_t *err;  // [4]
    uint32_t *sem;  // [n_sem] zeroed here
    int n_sem;
    int32_t *counts;
    int32_t *offsets;
    int32_t *active;
    int32_t *n_active;
    int32_t *order;
    int32_t *pos;
    int32_t *block_counts;  // [n_blocks][E]
    int chunk;
    int n_blocks;
    // Virtual experts (decode path only; NULL otherwise): every active expert
    // split into groups of at most kVirtTokens routed positions, in active order.
    int4 *virt;       // [n_virt] {expert, first position, positions, token columns before it}
    int32_t *n_virt;  // [2] virtual experts, token columns
    int32_t *vslot;   // [R] virtual expert of each routed position
};

size_t route_block_counts_bytes(int E, int R);
cudaError_t launch_route(RouteArgs a, cudaStream_t s);

// Routing results as the FFN kernels read them.
struct Routing {
    const int32_t *counts;
    const int32_t *offsets;
    const int32_t *active;
    const int32_t *n_active;
    const int32_t *order;
    const int32_t *pos;
    uint32_t *sem;
    uint32_t *err;
    const int4 *virt;
    const int32_t *n_virt;
    const int32_t *vslot;
};

struct DecodeArgs {
    int E, d, f, r, T, k;
    int x_type, w_type;
    uint32_t flags;
    const void *x;
    const void *weights;
    float *out;
    latent_qmatrix gate_a, gate_b, up_a, up_b, down_a, down_b;
    Routing rt;
    int R;           // T * k
    int nmax;        // upper bound on active experts: min(E, R)
    int n_virt_max;  // upper bound on virtual experts
    // Per-routed-row outputs s.B_d (the combine input of the prefill and EP paths).
    float *y;   // [R][d]
    // Decode chain: intermediates per virtual expert, [rows][token columns]
    // fp32 (x0: gathered x, tb: x.[A_g | A_u], hb: silu(t_g.B_g) * (t_u.B_u)
    // [* w], sb: h.A_d), and its counters (zeroed by the routing kernel): the
    // item counter, the CTAs that zeroed their share of out, per phase and
    // virtual expert the completed items.
    float *x0, *tb, *hb, *sb;
    uint32_t *queue;
    uint32_t *zero_done;
    uint32_t *done;  // [5][n_virt_max]
};

int decode_sem_count(const DecodeArgs &a);

// Optional caller events recorded between kernel launches (profiling).
struct Marks {
    cudaEvent_t const *ev = nullptr;
    int n = 0;
    int i = 0;
    void mark(cudaStream_t s) {
        if (ev && i < n) cudaEventRecord(ev[i], s);
        ++i;
    }
};

void decode_plan(DecodeArgs &a);
size_t decode_scratch_floats(const DecodeArgs &a);
// Decode-path counters (zeroed by the routing kernel) and their carve-up.
void decode_bind_sem(DecodeArgs &a, uint32_t *sem);
// Carves the decode scratch (decode_scratch_floats floats) into a's buffers.
void decode_bind_scratch(DecodeArgs &a, float *scratch);
cudaError_t launch_decode(const DecodeArgs &a, cudaStream_t s, Marks *marks);

// Prefill path (tcgen05 grouped GEMMs); scratch is prefill_scratch_bytes(a) bytes.
size_t prefill_scratch_bytes(const DecodeArgs &a);
cudaError_t launch_prefill(const DecodeArgs &a, void *scratch, cudaStream_t s, Marks *marks);

// Top-k combine of per-routed-row outputs (a.y) into a.out, slot order.
cudaError_t launch_combine(const DecodeArgs &a, cudaStream_t s);

struct EpArgs {
    int E, d, T, k;
    int x_type, w_type;
    const void *x;
    const int32_t *ids;
    const void *weights;
    const int32_t *offsets;  // routing results (workspace)
    const int32_t *order;
    void *send_x;
    int32_t *send_expert;
    float *send_weight;
    uint32_t *err;           // workspace error word (kErrCapacity)
};

cudaError_t launch_ep_gather(const EpArgs &a, cudaStream_t s);
cudaError_t launch_ep_pack_fixed(const EpArgs &a, int world, int cap, void *rows, int32_t *meta, bool merged,
                                 cudaStream_t s);
size_t ep_merged_block_bytes(int cap, int d, int es);
cudaError_t launch_ep_unpack_fixed(const void *buf, int world, int cap, int d, int es, int base, int n_local, bool wbd,
                                   void *x_out, int32_t *ids_out, float *w_out, uint32_t *err, cudaStream_t s);
cudaError_t launch_ep_combine_fixed(const EpArgs &a, const int32_t *pos, int world, int cap, const float *y, float *out,
                                    bool wbd, cudaStream_t s);

cudaError_t launch_dequant(const latent_qmatrix &m, int expert, float *out, cudaStream_t s);
cudaError_t launch_silu(const float *x, float *y, int64_t n, cudaStream_t s);
cudaError_t launch_router_topk(const float *scores, int T, int E, int k, double threshold, bool renorm, int *ids,
                               float *weights, int *n_kept, bool softmax, int *counts, cudaStream_t s);
cudaError_t launch_pack_tiles(const uint8_t *codes, const uint16_t *scales, int n_expert, int64_t rows, int64_t cols,
                              uint8_t *dcodes, uint16_t *dscales, cudaStream_t s);

// Raises the dynamic shared memory limit of `func` on the current device once.
cudaError_t ensure_smem(const void *func, size_t bytes);

}  // namespace latent
