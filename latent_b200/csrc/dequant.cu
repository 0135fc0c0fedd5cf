// Standalone dequantization (bit-exact with the reference decoders) and SiLU.
#include "internal.h"

namespace latent {

namespace {

// Eight elements per thread: one 32-bit word of codes.  value =
// level[code] * float(scale) (NF4, loader/latent_loader.py:144) or
// float(int8) * float(scale) (INT8, :169) -- a single fp32 rounding.
__global__ void __launch_bounds__(256) k_dequant(latent_qmatrix m, int expert, float *out) {
    __shared__ float lut[16];
    if (threadIdx.x < 16) lut[threadIdx.x] = kNF4Levels[threadIdx.x];
    __syncthreads();
    const QView M = expert_view(m, expert);
    const int64_t n = (int64_t)M.rows * M.cols;
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (i >= n) return;
    const int row = (int)(i / M.cols), col = (int)(i - (int64_t)row * M.cols);
    const int64_t g = tile_group(M.rows, M.cols, row, col);
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(M.codes + g * 16 + ((col & 31) >> 1)));
    const uint16_t sb = __ldg(M.scales + g);
    const float sc = half_bits_to_float(sb & 0x7FFFu);
    float v[8];
    uint32_t idx;
    if ((sb & 0x8000u) && M.i8.present() && M.i8.is_int8(g, &idx)) {
        const uint32_t hw = __ldg(reinterpret_cast<const uint32_t *>(M.i8.hi + (int64_t)idx * 16 + ((col & 31) >> 1)));
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(int8_elem(w, hw, j), sc);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(lut[(w >> (4 * j)) & 15u], sc);
    }
    float4 *dst = reinterpret_cast<float4 *>(out + i);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// One thread per group: the 16 code bytes and the scale of row-major group
// (row, g) go to its tile-major position.
__global__ void __launch_bounds__(256) k_pack_tiles(const uint8_t *codes, const uint16_t *scales, int64_t rows,
                                                    int64_t cols, int64_t n_groups, uint8_t *dcodes,
                                                    uint16_t *dscales) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // global row-major group index
    if (i >= n_groups) return;
    const int64_t per = rows * (cols >> 5);
    const int64_t e = i / per, r = i - e * per;
    const int row = (int)(r / (cols >> 5)), col = (int)(r - (int64_t)row * (cols >> 5)) * 32;
    const int64_t q = e * per + tile_group((int)rows, (int)cols, row, col);
    reinterpret_cast<uint4 *>(dcodes)[q] = __ldg(reinterpret_cast<const uint4 *>(codes) + i);
    dscales[q] = __ldg(scales + i);
}

__global__ void __launch_bounds__(256) k_silu(const float *x, float *y, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = silu_f32(x[i]);
}

}  // namespace

cudaError_t launch_dequant(const latent_qmatrix &m, int expert, float *out, cudaStream_t s) {
    const int64_t n8 = m.rows * m.cols / 8;
    if (n8 == 0) return cudaSuccess;
    k_dequant<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(m, expert, out);
    return cudaGetLastError();
}

cudaError_t launch_pack_tiles(const uint8_t *codes, const uint16_t *scales, int n_expert, int64_t rows, int64_t cols,
                              uint8_t *dcodes, uint16_t *dscales, cudaStream_t s) {
    const int64_t n = (int64_t)n_expert * rows * (cols / 32);
    if (n == 0) return cudaSuccess;
    k_pack_tiles<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(codes, scales, rows, cols, n, dcodes, dscales);
    return cudaGetLastError();
}

cudaError_t launch_silu(const float *x, float *y, int64_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    k_silu<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, y, n);
    return cudaGetLastError();
}

}  // namespace latent
