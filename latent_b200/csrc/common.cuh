// Shared device helpers for the latent expert FFN kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/latent_ffn.h"

namespace latent {

// Device-side error bits, kept in the first word of the workspace.
enum : uint32_t {
    kErrExpertId = 1u << 0,
    kErrTimeout = 1u << 1,
    kErrLayout = 1u << 2,  // a kernel's shared-memory layout assumption did not hold
    kErrCapacity = 1u << 3,  // a fixed-capacity exchange block had more rows than it holds
};

// NF4 levels in code order.  Must equal the reference table
// (loader/latent_loader.py:28-48) bit for bit; tests compare the GPU decode
// with the reference decode byte by byte.
__constant__ float kNF4Levels[16] = {
    -1.0f, -0.6961928f, -0.52507305f, -0.3949175f,
    -0.28444138f, -0.18477343f, -0.09105004f, 0.0f,
    0.0795803f, 0.1609302f, 0.2461123f, 0.33791524f,
    0.44070983f, 0.562617f, 0.72295684f, 1.0f,
};

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

template <int XT>
__device__ __forceinline__ float load_act(const void *p, int64_t i) {
    if constexpr (XT == LATENT_TYPE_F32) {
        return __ldg(reinterpret_cast<const float *>(p) + i);
    } else if constexpr (XT == LATENT_TYPE_F16) {
        return __half2float(__ldg(reinterpret_cast<const __half *>(p) + i));
    } else {
        return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16 *>(p) + i));
    }
}

__device__ __forceinline__ float load_weight(const void *p, int wt, int64_t i) {
    return wt == LATENT_TYPE_F16 ? __half2float(__ldg(reinterpret_cast<const __half *>(p) + i))
                                 : __ldg(reinterpret_cast<const float *>(p) + i);
}

// 16-byte read-only streaming load (weights are touched once per call).
__device__ __forceinline__ uint4 ldg_stream_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_stream_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// SiLU in fp32: x / (1 + exp(-x)).  The reference evaluates it in float64
// and rounds to fp32 (loader/latent_runtime.py:39-45); the fp32 form differs
// by a few ulp, far inside the decode tolerance.
__device__ __forceinline__ float silu_f32(float x) {
    return x / (1.0f + expf(-x));
}

// SiLU with the fast exponential and division (about 2 ulp); used where the
// result is rounded to f16 anyway (the prefill epilogue).
__device__ __forceinline__ float silu_fast(float x) {
    return __fdividef(x, 1.0f + __expf(-x));
}

// Per-group INT8 lookup for a stacked factor: is group g (expert-local) INT8,
// and where are its high nibbles?
struct Int8Side {
    const uint32_t *mask;  // expert-local words
    const uint32_t *base;  // expert-local words, global group index
    const uint8_t *hi;
    __device__ __forceinline__ bool present() const { return mask != nullptr; }
    __device__ __forceinline__ bool is_int8(int64_t g, uint32_t *index) const {
        const uint32_t w = __ldg(mask + (g >> 5));
        const uint32_t bit = 1u << (g & 31);
        if (!(w & bit)) return false;
        *index = __ldg(base + (g >> 5)) + __popc(w & (bit - 1u));
        return true;
    }
};

// Flat group index of element (row, col) of a [rows][cols] factor in the
// 256-column tile-major device order: tile c = col/256 holds its rows in
// turn, each row its min(8, cols/32 - 8c) groups.  The index addresses the
// 16 code bytes (codes + 16*q), the fp16 scale (scales[q]) and the INT8 bit.
__device__ __forceinline__ int64_t tile_group(int rows, int cols, int row, int col) {
    const int c = col >> 8;
    const int ng = min(8, (cols >> 5) - 8 * c);
    return (int64_t)c * rows * 8 + (int64_t)row * ng + ((col & 255) >> 5);
}

// Expert-local view of one stacked factor.
struct QView {
    const uint8_t *codes;   // [rows][cols/2]
    const uint16_t *scales; // [rows][cols/32]
    Int8Side i8;
    int rows;
    int cols;
};

__device__ __forceinline__ QView expert_view(const latent_qmatrix &m, int e) {
    QView v;
    const int64_t n = m.rows * m.cols;
    v.codes = m.codes + (int64_t)e * (n >> 1);
    v.scales = m.scales + (int64_t)e * (n >> 5);
    const int64_t words = ((n >> 5) + 31) >> 5;
    v.i8.mask = m.i8_mask ? m.i8_mask + (int64_t)e * words : nullptr;
    v.i8.base = m.i8_base ? m.i8_base + (int64_t)e * words : nullptr;
    v.i8.hi = m.i8_hi;
    v.rows = (int)m.rows;
    v.cols = (int)m.cols;
    return v;
}

// Sign-extended int8 value of element j (0..7) of an INT8 group, given the
// 32-bit word of low nibbles and the matching word of high nibbles.
__device__ __forceinline__ float int8_elem(uint32_t lo, uint32_t hi, int j) {
    const uint32_t l = (lo >> (4 * j)) & 0xFu;
    const uint32_t h = (hi >> (4 * j)) & 0xFu;
    return (float)(int8_t)(uint8_t)((h << 4) | l);
}

}  // namespace latent
