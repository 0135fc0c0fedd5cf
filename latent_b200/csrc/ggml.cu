// The ggml op adapter: the body of the reference's ggml_cuda_latent_expert_ffn
// (kernels/latent_fused_expert_ffn.cu:134-292) as two library calls.
//
// Load time, latent_ggml_pack_layer: the op's twelve factor sources (src[3..14]:
// codes and fp16 scales of gate_a, gate_b, up_a, up_b, down_a, down_b, as the
// reference GGUF writer stores them, loader/write_latent_gguf.py:101-123 and
// :412-436) are copied into one caller-owned device buffer in the library's
// layout: 256-column tile-major group order, every factor padded to one
// power-of-two rank with zero groups (code 7 = 0.0, scale 1.0), which changes
// no result.  The writer records each tensor's dims as (n_expert, rows,
// cols/2) for codes and (n_expert, rows, cols/32) for scales, with the bytes
// in C order of those dims; the reference op reads the same ne[] order
// (kernels/latent_fused_expert_ffn.cu:152-160), and so does this adapter.
// A factors are [n_in, max_rank] (columns zero-padded by the writer), B
// factors [largest actual rank, n_out].
//
// Per call, latent_ggml_expert_ffn: src[0] x [n_embd, T] (F16, BF16 or F32),
// src[1] ids [k, T] I32, src[2] weights [k, T] (F16 or F32) and dst
// [n_embd, k, T] F32 (the op's per-slot output) or [n_embd, T] F32 (combined
// by the library) -> latent_expert_ffn_forward with a caller workspace.
#include <algorithm>

#include "internal.h"

namespace latent {
namespace {

// Row-major source group (e, row, g) of [rows][cols] -> padded destination
// [prow][pcol] in tile order; padding groups are zero (code 7, scale 1.0).
__global__ void __launch_bounds__(256) k_pack_pad(const uint8_t *codes, const uint16_t *scales, int64_t rows,
                                                  int64_t cols, int64_t prow, int64_t pcol, int64_t n_groups,
                                                  uint8_t *dcodes, uint16_t *dscales) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // destination row-major group index
    if (i >= n_groups) return;
    const int64_t per = prow * (pcol >> 5);
    const int64_t e = i / per, r = i - e * per;
    const int row = (int)(r / (pcol >> 5)), col = (int)(r - (int64_t)row * (pcol >> 5)) * 32;
    uint4 c = make_uint4(0x77777777u, 0x77777777u, 0x77777777u, 0x77777777u);
    uint16_t sc = 0x3C00u;
    if (row < rows && col < cols) {
        const int64_t src = (e * rows + row) * (cols >> 5) + (col >> 5);
        c = __ldg(reinterpret_cast<const uint4 *>(codes) + src);
        sc = __ldg(scales + src);
    }
    const int64_t q = e * per + tile_group((int)prow, (int)pcol, row, col);
    reinterpret_cast<uint4 *>(dcodes)[q] = c;
    dscales[q] = sc;
}

int rank_pad(int64_t r) {
    int p = 32;
    while (p < r) p *= 2;
    return p;
}

size_t up256(size_t v) { return (v + 255) & ~(size_t)255; }

struct Shapes {
    int64_t E, rows[6], cols[6], prow[6], pcol[6];
    int d, f, R;
};

int read_shapes(const latent_ggml_tensor *fac, Shapes &s) {
    if (!fac) return LATENT_ERR_INVALID;
    for (int m = 0; m < 6; ++m) {
        const latent_ggml_tensor &c = fac[2 * m], &sc = fac[2 * m + 1];
        if (c.type != LATENT_GGML_I8 || sc.type != LATENT_GGML_F16) return LATENT_ERR_DTYPE;
        if (c.ne[3] > 1 || sc.ne[3] > 1) return LATENT_ERR_SHAPE;
        if (c.ne[0] != sc.ne[0] || c.ne[1] != sc.ne[1] || c.ne[2] * 2 != sc.ne[2] * 32) return LATENT_ERR_SHAPE;
        if (m == 0) s.E = c.ne[0];
        if (c.ne[0] != s.E || s.E < 1 || s.E > kMaxExperts) return LATENT_ERR_SHAPE;
        s.rows[m] = c.ne[1];
        s.cols[m] = c.ne[2] * 2;
        if (s.rows[m] < 1 || s.cols[m] < 32) return LATENT_ERR_SHAPE;
    }
    // gate_a [d][ra], gate_b [rb][f], up_a [d][ra], up_b [rb][f], down_a [f][ra], down_b [rb][d]
    s.d = (int)s.rows[0];
    s.f = (int)s.cols[1];
    if (s.rows[2] != s.d || s.cols[3] != s.f || s.rows[4] != s.f || s.cols[5] != s.d) return LATENT_ERR_SHAPE;
    if (s.d % 32 || s.f % 32) return LATENT_ERR_SHAPE;
    int64_t rmax = 0;
    for (int m = 0; m < 6; ++m) rmax = std::max(rmax, (m % 2 == 0) ? s.cols[m] : s.rows[m]);
    s.R = rank_pad(rmax);
    if (s.R > 512) return LATENT_ERR_UNSUPPORTED;
    for (int m = 0; m < 6; ++m) {
        const bool a_side = m % 2 == 0;
        s.prow[m] = a_side ? s.rows[m] : s.R;
        s.pcol[m] = a_side ? s.R : s.cols[m];
    }
    return LATENT_OK;
}

}  // namespace
}  // namespace latent

using namespace latent;

extern "C" LATENT_API int latent_ggml_pack_layer(const latent_ggml_tensor *factors, void *dst, size_t dst_bytes,
                                                 size_t *bytes_needed, latent_ffn_desc *desc, CUstream_st *stream) {
    Shapes s{};
    int st = read_shapes(factors, s);
    if (st) return st;
    size_t off[6][2], total = 0;
    for (int m = 0; m < 6; ++m) {
        const size_t groups = (size_t)s.E * s.prow[m] * (s.pcol[m] / 32);
        off[m][0] = total;
        total = up256(total + groups * 16);
        off[m][1] = total;
        total = up256(total + groups * 2);
    }
    if (bytes_needed) *bytes_needed = total;
    if (!dst) return LATENT_OK;
    if (!desc) return LATENT_ERR_INVALID;
    if (dst_bytes < total) return LATENT_ERR_WORKSPACE;
    if ((uintptr_t)dst % 256) return LATENT_ERR_ALIGN;
    for (int m = 0; m < 12; ++m)
        if (!factors[m].data) return LATENT_ERR_INVALID;
    for (int m = 0; m < 6; ++m)
        if ((uintptr_t)factors[2 * m].data % 16 || (uintptr_t)factors[2 * m + 1].data % 2) return LATENT_ERR_ALIGN;
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    uint8_t *base = static_cast<uint8_t *>(dst);
    latent_qmatrix q[6];
    for (int m = 0; m < 6; ++m) {
        const int64_t n = s.E * s.prow[m] * (s.pcol[m] / 32);
        uint8_t *dc = base + off[m][0];
        uint16_t *ds = reinterpret_cast<uint16_t *>(base + off[m][1]);
        k_pack_pad<<<(unsigned)((n + 255) / 256), 256, 0, cs>>>(
            static_cast<const uint8_t *>(factors[2 * m].data), static_cast<const uint16_t *>(factors[2 * m + 1].data),
            s.rows[m], s.cols[m], s.prow[m], s.pcol[m], n, dc, ds);
        if (cudaGetLastError() != cudaSuccess) return LATENT_ERR_CUDA;
        q[m] = latent_qmatrix{};
        q[m].codes = dc;
        q[m].scales = ds;
        q[m].rows = s.prow[m];
        q[m].cols = s.pcol[m];
    }
    *desc = latent_ffn_desc{};
    desc->n_expert = (int32_t)s.E;
    desc->n_embd = s.d;
    desc->n_ff = s.f;
    desc->rank = s.R;
    desc->gate_a = q[0];
    desc->gate_b = q[1];
    desc->up_a = q[2];
    desc->up_b = q[3];
    desc->down_a = q[4];
    desc->down_b = q[5];
    return LATENT_OK;
}

namespace {

int act_type(int32_t ggml_type, bool allow_bf16) {
    switch (ggml_type) {
        case LATENT_GGML_F32: return LATENT_TYPE_F32;
        case LATENT_GGML_F16: return LATENT_TYPE_F16;
        case LATENT_GGML_BF16: return allow_bf16 ? LATENT_TYPE_BF16 : -1;
        default: return -1;
    }
}

}  // namespace

extern "C" LATENT_API int latent_ggml_expert_ffn(const latent_ffn_desc *layer, const latent_ggml_tensor *src,
                                                 const latent_ggml_tensor *dst, void *workspace,
                                                 size_t workspace_bytes, size_t *workspace_needed,
                                                 CUstream_st *stream) {
    if (!layer || !src || !dst) return LATENT_ERR_INVALID;
    const latent_ggml_tensor &x = src[0], &ids = src[1], &w = src[2];
    latent_ffn_desc d = *layer;
    d.n_tokens = (int32_t)x.ne[1];
    d.top_k = (int32_t)ids.ne[0];
    if (x.ne[0] != d.n_embd || ids.ne[1] != x.ne[1] || w.ne[0] != ids.ne[0] || w.ne[1] != ids.ne[1])
        return LATENT_ERR_SHAPE;
    if (x.ne[2] > 1 || ids.ne[2] > 1 || w.ne[2] > 1) return LATENT_ERR_SHAPE;
    if (ids.type != LATENT_GGML_I32 || dst->type != LATENT_GGML_F32) return LATENT_ERR_DTYPE;
    d.x_type = act_type(x.type, true);
    d.w_type = act_type(w.type, false);
    if (d.x_type < 0 || d.w_type < 0) return LATENT_ERR_DTYPE;
    if (dst->ne[0] != d.n_embd) return LATENT_ERR_SHAPE;
    if (dst->ne[1] == ids.ne[0] && dst->ne[2] == x.ne[1])
        d.flags = LATENT_FLAG_OUT_PER_SLOT;            // [n_embd, k, T]: the op's per-slot dst
    else if (dst->ne[1] == x.ne[1] && dst->ne[2] <= 1)
        d.flags = 0;                                   // [n_embd, T]: combined by the library
    else
        return LATENT_ERR_SHAPE;
    d.path = LATENT_PATH_AUTO;
    d.x = x.data;
    d.ids = static_cast<const int32_t *>(ids.data);
    d.weights = w.data;
    d.out = static_cast<float *>(const_cast<void *>(dst->data));
    size_t need = 0;
    int st = latent_expert_ffn_workspace_size(&d, &need);
    if (st) return st;
    if (workspace_needed) *workspace_needed = need;
    if (!workspace) return LATENT_OK;
    d.workspace = workspace;
    d.workspace_bytes = workspace_bytes;
    return latent_expert_ffn_forward(&d, stream);
}
