// C-ABI entry points (include/latent_ffn.h): validation, workspace layout,
// launch sequencing.  Nothing here allocates device memory.
#include <map>
#include <mutex>
#include <utility>

#include "internal.h"

namespace latent {

cudaError_t ensure_smem(const void *func, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, size_t> done;
    std::lock_guard<std::mutex> lock(mu);
    size_t &have = done[{func, dev}];
    if (have >= bytes) return cudaSuccess;
    err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err == cudaSuccess) have = bytes;
    return err;
}

namespace {

constexpr size_t kAlign = 256;

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct Layout {
    size_t err, counts, offsets, active, n_active, sem, order, pos, block_counts, virt, n_virt, vslot, scratch, total;
    int n_sem;
};

bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

int check_qmatrix(const latent_qmatrix &m, int64_t rows, int64_t cols, bool need_ptrs) {
    if (m.rows != rows || m.cols != cols) return LATENT_ERR_SHAPE;
    if (!need_ptrs) return LATENT_OK;
    if (!m.codes || !m.scales) return LATENT_ERR_INVALID;
    if (!aligned(m.codes, 16) || !aligned(m.scales, 16)) return LATENT_ERR_ALIGN;
    const bool any = m.i8_mask || m.i8_base || m.i8_hi || m.i8_blocks || m.i8_list;
    if (any && !(m.i8_mask && m.i8_base && m.i8_hi && m.i8_blocks && m.i8_list)) return LATENT_ERR_INVALID;
    if (m.i8_hi && (!aligned(m.i8_hi, 16) || !aligned(m.i8_mask, 16) || !aligned(m.i8_base, 16) ||
                    !aligned(m.i8_blocks, 16) || !aligned(m.i8_list, 16)))
        return LATENT_ERR_ALIGN;
    return LATENT_OK;
}

bool rank_supported(int r) { return r == 32 || r == 64 || r == 128 || r == 256 || r == 512; }

// Shape/type validation; `need_ptrs` also checks pointers and alignment.
int validate(const latent_ffn_desc *d, bool need_ptrs) {
    if (!d) return LATENT_ERR_INVALID;
    if (d->n_expert < 1 || d->n_expert > kMaxExperts) return LATENT_ERR_SHAPE;
    if (d->n_embd < 32 || d->n_embd % 32 || d->n_ff < 32 || d->n_ff % 32) return LATENT_ERR_SHAPE;
    if (d->n_tokens < 0 || d->top_k < 1) return LATENT_ERR_SHAPE;
    if ((int64_t)d->n_tokens * d->top_k > (int64_t)1 << 30) return LATENT_ERR_SHAPE;
    if (!rank_supported(d->rank)) return LATENT_ERR_UNSUPPORTED;
    if (d->x_type != LATENT_TYPE_F32 && d->x_type != LATENT_TYPE_F16 && d->x_type != LATENT_TYPE_BF16)
        return LATENT_ERR_DTYPE;
    if (d->w_type != LATENT_TYPE_F32 && d->w_type != LATENT_TYPE_F16) return LATENT_ERR_DTYPE;
    if (d->flags & ~(uint32_t)(LATENT_FLAG_WEIGHT_BEFORE_DOWN | LATENT_FLAG_OUT_PER_SLOT)) return LATENT_ERR_INVALID;
    if (d->path != LATENT_PATH_AUTO && d->path != LATENT_PATH_DECODE && d->path != LATENT_PATH_PREFILL)
        return LATENT_ERR_INVALID;
    const int64_t D = d->n_embd, F = d->n_ff, R = d->rank;
    const bool ptrs = need_ptrs && d->n_tokens > 0;
    int st;
    if ((st = check_qmatrix(d->gate_a, D, R, ptrs))) return st;
    if ((st = check_qmatrix(d->up_a, D, R, ptrs))) return st;
    if ((st = check_qmatrix(d->gate_b, R, F, ptrs))) return st;
    if ((st = check_qmatrix(d->up_b, R, F, ptrs))) return st;
    if ((st = check_qmatrix(d->down_a, F, R, ptrs))) return st;
    if ((st = check_qmatrix(d->down_b, R, D, ptrs))) return st;
    if (ptrs) {
        if (!d->x || !d->ids || !d->weights || !d->out) return LATENT_ERR_INVALID;
        const size_t xs = d->x_type == LATENT_TYPE_F32 ? 4 : 2;
        if (!aligned(d->x, xs) || !aligned(d->ids, 4) || !aligned(d->weights, d->w_type == LATENT_TYPE_F32 ? 4 : 2))
            return LATENT_ERR_ALIGN;
        if (!aligned(d->out, 16)) return LATENT_ERR_ALIGN;
    }
    return LATENT_OK;
}

// AUTO: the tensor-core path once an expert sees ~64 rows on average (a
// 128-row MMA tile is then at least half full); the CUDA-core chain below.
int pick_path(const latent_ffn_desc *d) {
    if (d->path != LATENT_PATH_AUTO) return d->path;
    const int64_t R = (int64_t)d->n_tokens * d->top_k;
    return (R >= 4096 && R >= 64 * (int64_t)d->n_expert) ? LATENT_PATH_PREFILL : LATENT_PATH_DECODE;
}

DecodeArgs decode_args(const latent_ffn_desc *d) {
    DecodeArgs a{};
    a.E = d->n_expert;
    a.d = d->n_embd;
    a.f = d->n_ff;
    a.r = d->rank;
    a.T = d->n_tokens;
    a.k = d->top_k;
    a.x_type = d->x_type;
    a.w_type = d->w_type;
    a.flags = d->flags;
    a.x = d->x;
    a.weights = d->weights;
    a.out = d->out;
    a.gate_a = d->gate_a;
    a.gate_b = d->gate_b;
    a.up_a = d->up_a;
    a.up_b = d->up_b;
    a.down_a = d->down_a;
    a.down_b = d->down_b;
    decode_plan(a);
    return a;
}

Layout layout(const latent_ffn_desc *d, const DecodeArgs &a, int path) {
    Layout L{};
    const size_t E = (size_t)d->n_expert, R = (size_t)d->n_tokens * (size_t)d->top_k;
    size_t o = 0;
    L.err = o;           o = align_up(o + 16);
    L.counts = o;        o = align_up(o + E * 4);
    L.offsets = o;       o = align_up(o + (E + 1) * 4);
    L.active = o;        o = align_up(o + E * 4);
    L.n_active = o;      o = align_up(o + 4);
    L.n_sem = path == LATENT_PATH_PREFILL ? 0 : decode_sem_count(a);
    L.sem = o;           o = align_up(o + (size_t)L.n_sem * 4);
    L.order = o;         o = align_up(o + R * 4);
    L.pos = o;           o = align_up(o + R * 4);
    L.block_counts = o;  o = align_up(o + route_block_counts_bytes((int)E, (int)R));
    const bool dec = path != LATENT_PATH_PREFILL;
    L.virt = o;          o = align_up(o + (dec ? (size_t)a.n_virt_max * 16 : 0));
    L.n_virt = o;        o = align_up(o + (dec ? 8 : 0));
    L.vslot = o;         o = align_up(o + (dec ? R * 4 : 0));
    L.scratch = o;
    o = align_up(o + (path == LATENT_PATH_PREFILL ? prefill_scratch_bytes(a) : decode_scratch_floats(a) * sizeof(float)));
    L.total = o;
    return L;
}

template <class T>
T *at(void *base, size_t off) {
    return reinterpret_cast<T *>(static_cast<char *>(base) + off);
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? LATENT_OK : LATENT_ERR_CUDA; }

}  // namespace

}  // namespace latent

using namespace latent;

extern "C" LATENT_API int latent_abi_version(void) { return LATENT_ABI_VERSION; }

extern "C" LATENT_API const char *latent_status_string(int status) {
    switch (status) {
        case LATENT_OK: return "ok";
        case LATENT_ERR_INVALID: return "invalid argument (NULL pointer, bad flag or negative size)";
        case LATENT_ERR_SHAPE: return "inconsistent or unsupported shape";
        case LATENT_ERR_DTYPE: return "unsupported data type";
        case LATENT_ERR_ALIGN: return "buffer not aligned as required";
        case LATENT_ERR_EXPERT_ID: return "routed expert id >= n_expert";
        case LATENT_ERR_WORKSPACE: return "workspace missing or too small";
        case LATENT_ERR_TIMEOUT: return "bounded device wait timed out";
        case LATENT_ERR_CUDA: return "CUDA runtime error";
        case LATENT_ERR_UNSUPPORTED: return "request not supported by this build";
        case LATENT_ERR_CAPACITY: return "a fixed-capacity exchange block overflowed";
        default: return "unknown status";
    }
}

extern "C" LATENT_API int latent_expert_ffn_workspace_size(const latent_ffn_desc *desc, size_t *bytes) {
    if (!bytes) return LATENT_ERR_INVALID;
    const int st = validate(desc, false);
    if (st) return st;
    const DecodeArgs a = decode_args(desc);
    *bytes = layout(desc, a, pick_path(desc)).total;
    return LATENT_OK;
}

namespace {

int forward_impl(const latent_ffn_desc *desc, CUstream_st *stream, Marks *marks) {
    int st = validate(desc, true);
    if (st) return st;
    if (desc->n_tokens == 0) return LATENT_OK;
    const int path = pick_path(desc);
    DecodeArgs a = decode_args(desc);
    const Layout L = layout(desc, a, path);
    if (!desc->workspace || desc->workspace_bytes < L.total) return LATENT_ERR_WORKSPACE;
    if (!aligned(desc->workspace, kAlign)) return LATENT_ERR_ALIGN;
    void *ws = desc->workspace;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

    RouteArgs ra{};
    ra.ids = desc->ids;
    ra.R = a.R;
    ra.E = a.E;
    ra.top_k = a.k;
    ra.err = at<uint32_t>(ws, L.err);
    ra.sem = at<uint32_t>(ws, L.sem);
    ra.n_sem = L.n_sem;
    ra.counts = at<int32_t>(ws, L.counts);
    ra.offsets = at<int32_t>(ws, L.offsets);
    ra.active = at<int32_t>(ws, L.active);
    ra.n_active = at<int32_t>(ws, L.n_active);
    ra.order = at<int32_t>(ws, L.order);
    ra.pos = at<int32_t>(ws, L.pos);
    ra.block_counts = at<int32_t>(ws, L.block_counts);
    if (path != LATENT_PATH_PREFILL) {
        ra.virt = at<int4>(ws, L.virt);
        ra.n_virt = at<int32_t>(ws, L.n_virt);
        ra.vslot = at<int32_t>(ws, L.vslot);
    }
    if (marks) marks->mark(s);
    if ((st = cuda_status(launch_route(ra, s)))) return st;
    if (marks) marks->mark(s);

    a.rt.counts = ra.counts;
    a.rt.offsets = ra.offsets;
    a.rt.active = ra.active;
    a.rt.n_active = ra.n_active;
    a.rt.order = ra.order;
    a.rt.pos = ra.pos;
    a.rt.sem = ra.sem;
    a.rt.err = ra.err;
    if (path == LATENT_PATH_PREFILL) return cuda_status(launch_prefill(a, at<void>(ws, L.scratch), s, marks));
    a.rt.virt = ra.virt;
    a.rt.n_virt = ra.n_virt;
    a.rt.vslot = ra.vslot;
    decode_bind_scratch(a, at<float>(ws, L.scratch));
    decode_bind_sem(a, ra.sem);
    return cuda_status(launch_decode(a, s, marks));
}

}  // namespace

extern "C" LATENT_API int latent_expert_ffn_forward(const latent_ffn_desc *desc, CUstream_st *stream) {
    return forward_impl(desc, stream, nullptr);
}

extern "C" LATENT_API int latent_expert_ffn_forward_timed(const latent_ffn_desc *desc, CUstream_st *stream,
                                                          CUevent_st *const *events, int n_events) {
    if (n_events < 0 || (n_events > 0 && !events)) return LATENT_ERR_INVALID;
    Marks m;
    m.ev = reinterpret_cast<cudaEvent_t const *>(events);
    m.n = n_events;
    return forward_impl(desc, stream, &m);
}

extern "C" LATENT_API int latent_expert_ffn_check(const latent_ffn_desc *desc, CUstream_st *stream) {
    if (!desc || !desc->workspace) return LATENT_ERR_INVALID;
    uint32_t err = 0;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (cudaStreamSynchronize(s) != cudaSuccess) return LATENT_ERR_CUDA;
    if (desc->n_tokens == 0) return LATENT_OK;
    if (cudaMemcpy(&err, desc->workspace, sizeof(err), cudaMemcpyDeviceToHost) != cudaSuccess)
        return LATENT_ERR_CUDA;
    if (err & kErrExpertId) return LATENT_ERR_EXPERT_ID;
    if (err & kErrTimeout) return LATENT_ERR_TIMEOUT;
    if (err & kErrLayout) return LATENT_ERR_UNSUPPORTED;
    return LATENT_OK;
}

namespace {

int ep_validate(const latent_ep_desc *d) {
    if (!d) return LATENT_ERR_INVALID;
    if (d->n_expert < 1 || d->n_expert > kMaxExperts) return LATENT_ERR_SHAPE;
    if (d->n_embd < 32 || d->n_embd % 32 || d->n_tokens < 0 || d->top_k < 1) return LATENT_ERR_SHAPE;
    if ((int64_t)d->n_tokens * d->top_k > (int64_t)1 << 30) return LATENT_ERR_SHAPE;
    if (d->x_type != LATENT_TYPE_F32 && d->x_type != LATENT_TYPE_F16 && d->x_type != LATENT_TYPE_BF16)
        return LATENT_ERR_DTYPE;
    if (d->w_type != LATENT_TYPE_F32 && d->w_type != LATENT_TYPE_F16) return LATENT_ERR_DTYPE;
    if (d->flags & ~(uint32_t)LATENT_FLAG_WEIGHT_BEFORE_DOWN) return LATENT_ERR_INVALID;
    return LATENT_OK;
}

// Routing-only layout (the prefix of the forward layout, no FFN scratch).
Layout ep_layout(const latent_ep_desc *d) {
    latent_ffn_desc f{};
    f.n_expert = d->n_expert;
    f.n_embd = d->n_embd;
    f.n_ff = 32;
    f.rank = 32;
    f.n_tokens = d->n_tokens;
    f.top_k = d->top_k;
    DecodeArgs a = decode_args(&f);
    Layout L = layout(&f, a, LATENT_PATH_PREFILL);
    L.total = L.scratch;
    return L;
}

}  // namespace

extern "C" LATENT_API int latent_ep_workspace_size(const latent_ep_desc *desc, size_t *bytes) {
    if (!bytes) return LATENT_ERR_INVALID;
    const int st = ep_validate(desc);
    if (st) return st;
    *bytes = ep_layout(desc).total;
    return LATENT_OK;
}

extern "C" LATENT_API int latent_ep_dispatch(const latent_ep_desc *desc, CUstream_st *stream) {
    int st = ep_validate(desc);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (!desc->expert_counts) return LATENT_ERR_INVALID;
    if (desc->n_tokens == 0)
        return cuda_status(cudaMemsetAsync(desc->expert_counts, 0, (size_t)desc->n_expert * 4, s));
    if (!desc->x || !desc->ids || !desc->weights || !desc->send_x || !desc->send_expert || !desc->send_weight)
        return LATENT_ERR_INVALID;
    if (!aligned(desc->x, 16) || !aligned(desc->send_x, 16)) return LATENT_ERR_ALIGN;
    const Layout L = ep_layout(desc);
    if (!desc->workspace || desc->workspace_bytes < L.total) return LATENT_ERR_WORKSPACE;
    if (!aligned(desc->workspace, kAlign)) return LATENT_ERR_ALIGN;
    void *ws = desc->workspace;
    RouteArgs ra{};
    ra.ids = desc->ids;
    ra.R = desc->n_tokens * desc->top_k;
    ra.E = desc->n_expert;
    ra.top_k = desc->top_k;
    ra.err = at<uint32_t>(ws, L.err);
    ra.sem = at<uint32_t>(ws, L.sem);
    ra.n_sem = 0;
    ra.counts = at<int32_t>(ws, L.counts);
    ra.offsets = at<int32_t>(ws, L.offsets);
    ra.active = at<int32_t>(ws, L.active);
    ra.n_active = at<int32_t>(ws, L.n_active);
    ra.order = at<int32_t>(ws, L.order);
    ra.pos = at<int32_t>(ws, L.pos);
    ra.block_counts = at<int32_t>(ws, L.block_counts);
    if ((st = cuda_status(launch_route(ra, s)))) return st;
    if ((st = cuda_status(cudaMemcpyAsync(desc->expert_counts, ra.counts, (size_t)desc->n_expert * 4,
                                          cudaMemcpyDeviceToDevice, s))))
        return st;
    EpArgs e{};
    e.E = desc->n_expert;
    e.d = desc->n_embd;
    e.T = desc->n_tokens;
    e.k = desc->top_k;
    e.x_type = desc->x_type;
    e.w_type = desc->w_type;
    e.x = desc->x;
    e.ids = desc->ids;
    e.weights = desc->weights;
    e.offsets = ra.offsets;
    e.order = ra.order;
    e.send_x = desc->send_x;
    e.send_expert = desc->send_expert;
    e.send_weight = desc->send_weight;
    return cuda_status(launch_ep_gather(e, s));
}

namespace latent {
namespace {

int ep_fixed_check(const latent_ep_desc *d, int32_t world, int32_t cap) {
    const int st = ep_validate(d);
    if (st) return st;
    if (world < 1 || d->n_expert % world || cap < 1 || (int64_t)world * cap > (int64_t)1 << 30)
        return LATENT_ERR_SHAPE;
    if (!d->workspace || d->workspace_bytes < ep_layout(d).total) return LATENT_ERR_WORKSPACE;
    if (!aligned(d->workspace, kAlign)) return LATENT_ERR_ALIGN;
    return LATENT_OK;
}

EpArgs ep_args(const latent_ep_desc *d) {
    const Layout L = ep_layout(d);
    EpArgs e{};
    e.E = d->n_expert;
    e.d = d->n_embd;
    e.T = d->n_tokens;
    e.k = d->top_k;
    e.x_type = d->x_type;
    e.w_type = d->w_type;
    e.x = d->x;
    e.ids = d->ids;
    e.weights = d->weights;
    e.offsets = at<int32_t>(d->workspace, L.offsets);
    e.order = at<int32_t>(d->workspace, L.order);
    e.send_x = d->send_x;
    e.send_expert = d->send_expert;
    e.send_weight = d->send_weight;
    e.err = at<uint32_t>(d->workspace, L.err);
    return e;
}

}  // namespace
}  // namespace latent

extern "C" LATENT_API int latent_ep_pack_fixed(const latent_ep_desc *desc, int32_t world, int32_t cap, void *send_rows,
                                               int32_t *send_meta, CUstream_st *stream) {
    int st = ep_fixed_check(desc, world, cap);
    if (st) return st;
    if (!send_rows || !send_meta) return LATENT_ERR_INVALID;
    if (!aligned(send_rows, 16) || !aligned(send_meta, 8)) return LATENT_ERR_ALIGN;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (desc->n_tokens == 0)   // latent_ep_dispatch routed nothing: every row is unused
        return cuda_status(cudaMemsetAsync(send_meta, 0xff, (size_t)world * cap * 8, s));
    if (!desc->send_x || !desc->send_expert || !desc->send_weight) return LATENT_ERR_INVALID;
    if (!aligned(desc->send_x, 16)) return LATENT_ERR_ALIGN;
    return cuda_status(launch_ep_pack_fixed(ep_args(desc), world, cap, send_rows, send_meta, false, s));
}

extern "C" LATENT_API int latent_ep_pack_fixed_merged(const latent_ep_desc *desc, int32_t world, int32_t cap,
                                                      void *send_buf, size_t buf_bytes, size_t *bytes_needed,
                                                      CUstream_st *stream) {
    int st = ep_fixed_check(desc, world, cap);
    if (st) return st;
    const int es = desc->x_type == LATENT_TYPE_F32 ? 4 : 2;
    const size_t need = (size_t)world * ep_merged_block_bytes(cap, desc->n_embd, es);
    if (bytes_needed) *bytes_needed = need;
    if (!send_buf) return LATENT_OK;
    if (buf_bytes < need) return LATENT_ERR_WORKSPACE;
    if (!aligned(send_buf, 16)) return LATENT_ERR_ALIGN;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (desc->n_tokens == 0)   // nothing routed: every row unused (id -1)
        return cuda_status(cudaMemsetAsync(send_buf, 0xff, need, s));
    if (!desc->send_x || !desc->send_expert || !desc->send_weight) return LATENT_ERR_INVALID;
    if (!aligned(desc->send_x, 16)) return LATENT_ERR_ALIGN;
    return cuda_status(launch_ep_pack_fixed(ep_args(desc), world, cap, send_buf, nullptr, true, s));
}

extern "C" LATENT_API int latent_ep_unpack_fixed(const void *recv_buf, int32_t world, int32_t cap, int32_t n_embd,
                                                 int32_t x_type, int32_t expert_base, int32_t n_local, uint32_t flags,
                                                 void *x_out, int32_t *ids_out, float *w_out, uint32_t *err_word,
                                                 CUstream_st *stream) {
    if (world < 1 || cap < 1 || (int64_t)world * cap > (int64_t)1 << 30) return LATENT_ERR_SHAPE;
    if (n_embd < 32 || n_embd % 32 || n_local < 1 || expert_base < 0) return LATENT_ERR_SHAPE;
    if (x_type != LATENT_TYPE_F32 && x_type != LATENT_TYPE_F16 && x_type != LATENT_TYPE_BF16) return LATENT_ERR_DTYPE;
    if (flags & ~(uint32_t)LATENT_FLAG_WEIGHT_BEFORE_DOWN) return LATENT_ERR_INVALID;
    if (!recv_buf || !x_out || !ids_out || !w_out) return LATENT_ERR_INVALID;
    if (!aligned(recv_buf, 16) || !aligned(x_out, 16) || !aligned(ids_out, 4) || !aligned(w_out, 4))
        return LATENT_ERR_ALIGN;
    const int es = x_type == LATENT_TYPE_F32 ? 4 : 2;
    return cuda_status(launch_ep_unpack_fixed(recv_buf, world, cap, n_embd, es, expert_base, n_local,
                                              (flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN) != 0, x_out, ids_out, w_out,
                                              err_word, reinterpret_cast<cudaStream_t>(stream)));
}

extern "C" LATENT_API int latent_ep_combine_fixed(const latent_ep_desc *desc, int32_t world, int32_t cap,
                                                  const float *y_rows, float *out, CUstream_st *stream) {
    int st = ep_fixed_check(desc, world, cap);
    if (st) return st;
    if (desc->n_tokens == 0) return LATENT_OK;
    if (!y_rows || !out || !desc->ids || !desc->weights) return LATENT_ERR_INVALID;
    if (!aligned(y_rows, 16) || !aligned(out, 16)) return LATENT_ERR_ALIGN;
    const Layout L = ep_layout(desc);
    return cuda_status(launch_ep_combine_fixed(ep_args(desc), at<int32_t>(desc->workspace, L.pos), world, cap, y_rows,
                                               out, (desc->flags & LATENT_FLAG_WEIGHT_BEFORE_DOWN) != 0,
                                               reinterpret_cast<cudaStream_t>(stream)));
}

extern "C" LATENT_API int latent_ep_check(const latent_ep_desc *desc, CUstream_st *stream) {
    int st = ep_validate(desc);
    if (st) return st;
    if (desc->n_tokens == 0) return LATENT_OK;
    if (!desc->workspace || desc->workspace_bytes < ep_layout(desc).total) return LATENT_ERR_WORKSPACE;
    if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return LATENT_ERR_CUDA;
    uint32_t err = 0;
    if (cudaMemcpy(&err, at<uint32_t>(desc->workspace, ep_layout(desc).err), sizeof(err), cudaMemcpyDeviceToHost) !=
        cudaSuccess)
        return LATENT_ERR_CUDA;
    if (err & kErrExpertId) return LATENT_ERR_EXPERT_ID;
    if (err & kErrCapacity) return LATENT_ERR_CAPACITY;
    return LATENT_OK;
}

extern "C" LATENT_API int latent_ep_combine(const latent_ep_desc *desc, CUstream_st *stream) {
    int st = ep_validate(desc);
    if (st) return st;
    if (desc->n_tokens == 0) return LATENT_OK;
    if (!desc->y_back || !desc->out || !desc->weights) return LATENT_ERR_INVALID;
    if (!aligned(desc->y_back, 16) || !aligned(desc->out, 16)) return LATENT_ERR_ALIGN;
    const Layout L = ep_layout(desc);
    if (!desc->workspace || desc->workspace_bytes < L.total) return LATENT_ERR_WORKSPACE;
    DecodeArgs a{};
    a.E = desc->n_expert;
    a.d = desc->n_embd;
    a.T = desc->n_tokens;
    a.k = desc->top_k;
    a.w_type = desc->w_type;
    a.flags = desc->flags;
    a.weights = desc->weights;
    a.out = desc->out;
    a.y = const_cast<float *>(desc->y_back);
    a.rt.pos = at<int32_t>(desc->workspace, L.pos);
    return cuda_status(launch_combine(a, reinterpret_cast<cudaStream_t>(stream)));
}

extern "C" LATENT_API int latent_dequantize(const latent_qmatrix *m, int32_t expert, float *out, CUstream_st *stream) {
    if (!m || !out || !m->codes || !m->scales || expert < 0) return LATENT_ERR_INVALID;
    if (m->rows < 1 || m->cols < 32 || m->cols % 32) return LATENT_ERR_SHAPE;
    if (!aligned(m->codes, 16) || !aligned(m->scales, 2) || !aligned(out, 16)) return LATENT_ERR_ALIGN;
    const bool any = m->i8_mask || m->i8_base || m->i8_hi;
    if (any && !(m->i8_mask && m->i8_base && m->i8_hi)) return LATENT_ERR_INVALID;
    return cuda_status(launch_dequant(*m, expert, out, reinterpret_cast<cudaStream_t>(stream)));
}

extern "C" LATENT_API int latent_silu(const float *x, float *y, int64_t n, CUstream_st *stream) {
    if (n < 0 || (n > 0 && (!x || !y))) return LATENT_ERR_INVALID;
    return cuda_status(launch_silu(x, y, n, reinterpret_cast<cudaStream_t>(stream)));
}

extern "C" LATENT_API int latent_pack_tiles(const uint8_t *codes, const uint16_t *scales, int32_t n_expert,
                                            int64_t rows, int64_t cols, uint8_t *dst_codes, uint16_t *dst_scales,
                                            CUstream_st *stream) {
    if (!codes || !scales || !dst_codes || !dst_scales || n_expert < 1) return LATENT_ERR_INVALID;
    if (rows < 1 || cols < 32 || cols % 32 || rows > (1 << 30) || cols > (1 << 30)) return LATENT_ERR_SHAPE;
    if (!aligned(codes, 16) || !aligned(dst_codes, 16) || !aligned(scales, 2) || !aligned(dst_scales, 2))
        return LATENT_ERR_ALIGN;
    const size_t cb = (size_t)n_expert * rows * cols / 2, sb = (size_t)n_expert * rows * (cols / 32) * 2;
    const char *c0 = reinterpret_cast<const char *>(codes), *d0 = reinterpret_cast<const char *>(dst_codes);
    const char *s0 = reinterpret_cast<const char *>(scales), *t0 = reinterpret_cast<const char *>(dst_scales);
    if ((d0 < c0 + cb && c0 < d0 + cb) || (t0 < s0 + sb && s0 < t0 + sb)) return LATENT_ERR_INVALID;  // overlap
    return cuda_status(launch_pack_tiles(codes, scales, n_expert, rows, cols, dst_codes, dst_scales,
                                         reinterpret_cast<cudaStream_t>(stream)));
}
