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
    float *part1;  // [ks1][R][2r]
    float *t;      // [R][2r]
    float *h;      // [R][f]
    float *part2;  // [ks2][R][r]
    float *s;      // [R][r]
    float *y;      // [R][d]
    int R;         // T * k
    int nmax;      // upper bound on active experts: min(E, R)
    int kc1, ks1;  // rows per split-K chunk / chunks, x -> t
    int kc2, ks2;  // rows per split-K chunk / chunks, h -> s
    int nct_f, nct_d;          // 256-column tiles of f and d
    int in_floats, red_floats;  // shared-memory carve-up of the fused kernel
    // Counters in the routing block's zeroed region (decode_sem_count of them):
    uint32_t *work;    // [1] next work item
    uint32_t *arr1;    // [E] phase-1 chunk arrivals
    uint32_t *flag1;   // [E] t of the expert is complete
    uint32_t *cnt2;    // [E] finished phase-2 tiles
    uint32_t *arr3;    // [E] phase-3 chunk arrivals
    uint32_t *flag3;   // [E] s of the expert is complete
    uint32_t *tokcnt;  // [T][nct_d] finished slots per (token, d tile)
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
};

cudaError_t launch_ep_gather(const EpArgs &a, cudaStream_t s);

cudaError_t launch_dequant(const latent_qmatrix &m, int expert, float *out, cudaStream_t s);
cudaError_t launch_silu(const float *x, float *y, int64_t n, cudaStream_t s);

// Raises the dynamic shared memory limit of `func` on the current device once.
cudaError_t ensure_smem(const void *func, size_t bytes);

}  // namespace latent
