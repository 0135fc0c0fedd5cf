// Load-time quantisation of float factors on the GPU: the encoders of the
// reference compressor (loader/latent_loader.py:111-158) applied per
// 32-element group, with the per-group NF4 -> INT8 fallback of the device
// format.  One warp per group, lane i holding element i:
//
//  * NF4 (latent_loader.py:111-130): absmax (0 -> 1.0), normalise by the
//    fp32 absmax (IEEE division), nearest of the 16 levels by fp32 distance
//    with the lowest code winning a tie (numpy's argmin), scale fp16(absmax).
//  * SNR (latent_loader.py:173-185): ||v|| / max(||v - nf4(v)||, 1e-12),
//    nf4(v) = level * fp32(fp16 scale), in fp32 as numpy evaluates the
//    reference (squares that underflow give 0, as there).  An all-zero
//    group (SNR 0) stays NF4.
//  * INT8 when the SNR is below 10^(snr_db/20) (latent_loader.py:148-158 on
//    the group): scale = absmax / 127 in fp32 (0 -> 1.0), q = clip(rint(v /
//    scale), -127, 127), fp16 scale; the low nibbles of q go to `lo`, the
//    high nibbles to `hi`.
//
// Outputs per group: lo[16] / hi[16] bytes (even element in the low nibble),
// the fp16 scale bits and an INT8 flag byte.
#include "internal.h"

namespace latent {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(256) k_quantize_groups(const float *__restrict__ values, int64_t n_groups,
                                                         int mixed, float threshold, uint8_t *lo, uint8_t *hi,
                                                         uint16_t *scales, uint8_t *is_int8, float *snr) {
    const int64_t grp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (grp >= n_groups) return;  // whole warps: n_groups is per warp
    const float v = values[grp * 32 + lane];
    const unsigned abits = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
    float amax = __uint_as_float(abits);
    if (amax == 0.f) amax = 1.f;
    const float norm = __fdiv_rn(v, amax);
    int code = 0;
    float best = fabsf(__fsub_rn(norm, kNF4Levels[0]));
#pragma unroll
    for (int c = 1; c < 16; ++c) {
        const float dd = fabsf(__fsub_rn(norm, kNF4Levels[c]));
        if (dd < best) {
            best = dd;
            code = c;
        }
    }
    const __half s16 = __float2half_rn(amax);
    uint16_t sbits = __half_as_ushort(s16);
    bool i8 = false;
    int q = 0;
    if (mixed || snr) {
        const float dq = __fmul_rn(kNF4Levels[code], __half2float(s16));
        const float e = __fsub_rn(v, dq);
        const float sig = __fsqrt_rn(warp_sum(__fmul_rn(v, v)));
        const float noise = fmaxf(__fsqrt_rn(warp_sum(__fmul_rn(e, e))), 1e-12f);
        const float ratio = __fdiv_rn(sig, noise);
        if (snr && lane == 0) snr[grp] = ratio;
        i8 = mixed && sig > 0.f && ratio < threshold;  // an all-zero group stays NF4
        if (i8) {
            float s = __fdiv_rn(__uint_as_float(abits), 127.f);  // the group's own absmax
            if (s == 0.f) s = 1.f;
            q = (int)rintf(__fdiv_rn(v, s));
            q = q < -127 ? -127 : q > 127 ? 127 : q;
            sbits = __half_as_ushort(__float2half_rn(s));
        }
    }
    const unsigned low = i8 ? (unsigned)(q & 15) : (unsigned)code;
    const unsigned high = i8 ? (unsigned)((q >> 4) & 15) : 0u;
    const unsigned low_n = __shfl_down_sync(0xffffffffu, low, 1);
    const unsigned high_n = __shfl_down_sync(0xffffffffu, high, 1);
    if ((lane & 1) == 0) {
        lo[grp * 16 + (lane >> 1)] = (uint8_t)(low | (low_n << 4));
        hi[grp * 16 + (lane >> 1)] = (uint8_t)(high | (high_n << 4));
    }
    if (lane == 0) {
        scales[grp] = sbits;
        is_int8[grp] = i8 ? 1 : 0;
    }
}

}  // namespace
}  // namespace latent

extern "C" LATENT_API int latent_quantize_groups(const float *values, int64_t n_groups, float snr_db, uint8_t *lo,
                                                 uint8_t *hi, uint16_t *scales, uint8_t *is_int8, float *snr,
                                                 CUstream_st *stream) {
    if (n_groups < 0) return LATENT_ERR_INVALID;
    if (n_groups == 0) return LATENT_OK;
    if (!values || !lo || !hi || !scales || !is_int8) return LATENT_ERR_INVALID;
    if ((uintptr_t)values % 4 || (uintptr_t)scales % 2) return LATENT_ERR_ALIGN;
    if (n_groups > (int64_t)8 * 0x7fffffff) return LATENT_ERR_SHAPE;  // grid limit: 8 groups per block
    const bool mixed = !(snr_db != snr_db);  // NaN: every group NF4
    const float thr = mixed ? (float)pow(10.0, (double)snr_db / 20.0) : 0.f;
    const int64_t threads = n_groups * 32;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    latent::k_quantize_groups<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        values, n_groups, mixed ? 1 : 0, thr, lo, hi, scales, is_int8, snr);
    return cudaGetLastError() == cudaSuccess ? LATENT_OK : LATENT_ERR_CUDA;
}
