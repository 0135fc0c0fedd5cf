/*
 * latent_ffn.h -- C ABI of the B200 fused latent expert FFN.
 *
 * Drop-in for LATENT's GGML_OP_LATENT_EXPERT_FFN device op.  The reference
 * op is the host wrapper ggml_cuda_latent_expert_ffn (reference
 * kernels/latent_fused_expert_ffn.cu:134-292) over the structs in
 * kernels/latent_fused_expert_ffn.h:23-59; its CPU semantics are
 * loader/latent_runtime.py:13-73.  Everything here is plain C: pointers,
 * sizes, status codes.  No allocation happens inside any entry point: the
 * caller owns every buffer, including the workspace whose size
 * latent_expert_ffn_workspace_size() reports.  No entry point throws or
 * aborts; all return a latent_status.
 *
 * Factor storage ("stacked" layout, one tensor per factor kind, all experts
 * contiguous -- the per-expert stacking of the reference GGUF writer,
 * loader/write_latent_gguf.py:101-123 and 230-255, with the nibble packing
 * it actually writes).  Each expert matrix [rows][cols] is a sequence of
 * 32-element groups in 256-column tile-major order: tile c (columns
 * 256c .. min(cols, 256c+256)-1) stores its rows one after another, each row
 * its ng_c = min(8, cols/32 - 8c) groups.  Group (row, col) has the
 * expert-local flat index
 *     q = c*rows*8 + row*ng_c + (col - 256c)/32,    c = col/256,
 * so a matrix of at most 256 columns is plain row-major.
 *   codes   uint8  [n_expert][rows*cols/32][16] group q at byte 16q: two 4-bit
 *                                              codes per byte, the even column
 *                                              in the low nibble
 *                                              (loader/latent_loader.py:129)
 *   scales  fp16   [n_expert][rows*cols/32]   scale of group q; scales are
 *                                              >= 0 and the sign bit flags
 *                                              an INT8 group
 *   NF4 group:  value = NF4_LEVEL[code] * float(scale)
 *   INT8 group: value = float(int8(hi << 4 | lo)) * float(|scale|), where lo
 *               is the 4-bit code in `codes` and hi comes from `i8_hi`.
 *   i8_mask uint32 [n_expert][mask_words]     bit q%32 of word q/32 set when
 *                                              group q is INT8;
 *                                              mask_words = ceil(rows*cols/1024)
 *   i8_base uint32 [n_expert][mask_words]     number of INT8 groups in the
 *                                              whole tensor before word w
 *   i8_hi   uint8  [n_int8_groups][16]        high nibbles of the INT8
 *                                              groups in (expert, q) order,
 *                                              same nibble order as codes
 *   i8_blocks int32 [n_blocks][12]           per block b = (e*tiles + c)*row_blocks
 *                                              + s (expert e, 256-column tile c,
 *                                              128-row block s; tiles = ceil(cols/256),
 *                                              row_blocks = ceil(rows/128)): words
 *                                              0..8 cumulative entry offsets of
 *                                              the block's group columns 0..7
 *                                              (word 0 = 0, word 8 = the block's
 *                                              INT8 groups), word 9 the block's
 *                                              first entry in i8_list (a multiple
 *                                              of 4), word 10 its first record in
 *                                              i8_hi, word 11 zero
 *   i8_list uint32 [..]                       one entry per INT8 group:
 *                                              (row in block << 16) | (record -
 *                                              word 10), by column then row; each
 *                                              block's run padded to 4 entries
 * i8_mask/i8_base/i8_hi/i8_blocks/i8_list are NULL when no group is INT8;
 * otherwise all five start on a 16-byte boundary (codes and scales too).  The tile order lets
 * a kernel streaming a row range of one column tile read its codes, scales
 * and INT8 records as three contiguous runs (latent_b200/format.py packs it).
 * cols must be a multiple of 32; the rank dimension may be zero-padded
 * (code 7 = 0.0, scale 1.0), which leaves every result unchanged.
 */
#ifndef LATENT_FFN_H
#define LATENT_FFN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st; /* cudaStream_t */
struct CUevent_st;  /* cudaEvent_t */

#if defined(__GNUC__)
#define LATENT_API __attribute__((visibility("default")))
#else
#define LATENT_API
#endif

#define LATENT_ABI_VERSION 4

typedef enum latent_status {
    LATENT_OK = 0,
    LATENT_ERR_INVALID = 1,     /* NULL pointer or negative size */
    LATENT_ERR_SHAPE = 2,       /* inconsistent or unsupported shape */
    LATENT_ERR_DTYPE = 3,       /* unsupported x / weight / output type */
    LATENT_ERR_ALIGN = 4,       /* buffer not aligned as required */
    LATENT_ERR_EXPERT_ID = 5,   /* an expert id >= n_expert was routed */
    LATENT_ERR_WORKSPACE = 6,   /* workspace missing or too small */
    LATENT_ERR_TIMEOUT = 7,     /* a bounded device-side wait gave up */
    LATENT_ERR_CUDA = 8,        /* a CUDA runtime call failed */
    LATENT_ERR_UNSUPPORTED = 9, /* valid request this build does not serve */
    LATENT_ERR_CAPACITY = 10    /* a fixed-capacity exchange block overflowed */
} latent_status;

typedef enum latent_type {
    LATENT_TYPE_F32 = 0,
    LATENT_TYPE_F16 = 1,
    LATENT_TYPE_BF16 = 2
} latent_type;

enum {
    /* multiply the SwiGLU hidden by the router weight before the down
     * projection (DeepSeek-V4; loader/latent_runtime.py:57-58) instead of in
     * the top-k combine */
    LATENT_FLAG_WEIGHT_BEFORE_DOWN = 1u << 0,
    /* write per-slot rows out[T][k][d] (the ggml op's dst,
     * kernels/latent_fused_expert_ffn.cu:259) instead of the combined
     * out[T][d]; rows of skipped slots (id < 0) are zero */
    LATENT_FLAG_OUT_PER_SLOT = 1u << 1
};

typedef enum latent_path {
    LATENT_PATH_AUTO = 0,    /* pick by routed pairs per expert */
    LATENT_PATH_DECODE = 1,  /* fp32 CUDA-core GEMV chain (rel-L2 <= 1e-5) */
    LATENT_PATH_PREFILL = 2  /* tcgen05 f16 MMA, fp32 accumulate (rel-L2 <= 2e-3) */
} latent_path;

/* One stacked factor tensor (see the layout above).  Mirrors
 * latent_nf4_matrix (reference kernels/latent_fused_expert_ffn.h:23-29),
 * stacked over experts and extended with the INT8 side tables. */
typedef struct latent_qmatrix {
    const uint8_t *codes;
    const uint16_t *scales;
    const uint32_t *i8_mask;
    const uint32_t *i8_base;
    const uint8_t *i8_hi;
    const int32_t *i8_blocks;
    const uint32_t *i8_list;
    int64_t rows;
    int64_t cols;
} latent_qmatrix;

/* One fused expert-FFN call.  Mirrors latent_dispatch_args
 * (reference kernels/latent_fused_expert_ffn.h:40-50) for a whole batch of
 * tokens, with the 15 op sources of ggml_cuda_latent_expert_ffn
 * (kernels/latent_fused_expert_ffn.cu:135-150) as fields. */
typedef struct latent_ffn_desc {
    int32_t n_expert;   /* E */
    int32_t n_embd;     /* d  (multiple of 32) */
    int32_t n_ff;       /* f  (multiple of 32) */
    int32_t rank;       /* r  padded rank (32, 64, 128, 256, 512 or 1024) */
    int32_t n_tokens;   /* T  (0 allowed) */
    int32_t top_k;      /* k */
    int32_t x_type;     /* latent_type of x */
    int32_t w_type;     /* latent_type of weights (F32 or F16) */
    uint32_t flags;     /* LATENT_FLAG_* */
    int32_t path;       /* latent_path */
    const void *x;          /* [T][d] */
    const int32_t *ids;     /* [T][k]; id < 0 skips the slot */
    const void *weights;    /* [T][k] router weights */
    float *out;             /* [T][d], or [T][k][d] with OUT_PER_SLOT */
    latent_qmatrix gate_a;  /* rows d, cols r */
    latent_qmatrix gate_b;  /* rows r, cols f */
    latent_qmatrix up_a;    /* rows d, cols r */
    latent_qmatrix up_b;    /* rows r, cols f */
    latent_qmatrix down_a;  /* rows f, cols r */
    latent_qmatrix down_b;  /* rows r, cols d */
    void *workspace;        /* 256-byte aligned, latent_expert_ffn_workspace_size() bytes */
    size_t workspace_bytes;
} latent_ffn_desc;

/* Expert-parallel dispatch/combine around an NCCL all-to-all (no counterpart
 * in the reference, which has no multi-GPU code).  dispatch routes the
 * batch by global expert id and packs one row per routed slot in expert
 * order -- destination-rank order when experts are contiguous per rank;
 * combine folds the expert outputs that came back (same row order) into
 * out[T][d] with the router weights, in slot order. */
typedef struct latent_ep_desc {
    int32_t n_expert;       /* global E */
    int32_t n_embd;         /* d (multiple of 32) */
    int32_t n_tokens;       /* T */
    int32_t top_k;          /* k */
    int32_t x_type;         /* latent_type of x and send_x */
    int32_t w_type;         /* latent_type of weights */
    uint32_t flags;         /* LATENT_FLAG_WEIGHT_BEFORE_DOWN: combine sums without weights */
    const void *x;          /* [T][d] */
    const int32_t *ids;     /* [T][k] */
    const void *weights;    /* [T][k] */
    void *send_x;           /* out: [T*k][d] rows in expert order (first sum(expert_counts) valid) */
    int32_t *send_expert;   /* out: [T*k] global expert id of each row */
    float *send_weight;     /* out: [T*k] router weight of each row */
    int32_t *expert_counts; /* out: [E] rows per expert */
    const float *y_back;    /* in (combine): [T*k][d] expert outputs in send order */
    float *out;             /* out (combine): [T][d] */
    void *workspace;        /* kept between dispatch and combine */
    size_t workspace_bytes;
} latent_ep_desc;

LATENT_API int latent_ep_workspace_size(const latent_ep_desc *desc, size_t *bytes);
LATENT_API int latent_ep_dispatch(const latent_ep_desc *desc, struct CUstream_st *stream);
LATENT_API int latent_ep_combine(const latent_ep_desc *desc, struct CUstream_st *stream);
/* Synchronises `stream` and reports device-side errors recorded in the EP
 * workspace since the last latent_ep_dispatch (LATENT_ERR_EXPERT_ID, and
 * LATENT_ERR_CAPACITY from latent_ep_pack_fixed). */
LATENT_API int latent_ep_check(const latent_ep_desc *desc, struct CUstream_st *stream);

/* Fixed-capacity exchange blocks (no counterpart in the reference, which has
 * no multi-GPU code).  After latent_ep_dispatch on the same desc and
 * workspace, latent_ep_pack_fixed writes send_rows[world*cap][d] (x's type):
 * block g holds, in routed order, the rows routed to rank g's experts
 * [g*E/world, (g+1)*E/world); send_meta[world*cap][2] int32 holds
 * {global expert id, router weight bits} per row, {-1, 0} for unused rows.
 * cap must be at least the rows any destination receives (T*min(k, E/world)
 * when a token routes no expert twice); a destination with more rows keeps
 * its first cap and records LATENT_ERR_CAPACITY for latent_ep_check, and
 * the rows left out contribute nothing to the combine.  latent_ep_combine_fixed reads the
 * returned blocks y_rows[world*cap][d] fp32 (same placement) and writes
 * out[T][d] = sum_j w[t,j] * y (plain sum with LATENT_FLAG_WEIGHT_BEFORE_DOWN).
 * Neither needs the host to know the per-destination counts. */
LATENT_API int latent_ep_pack_fixed(const latent_ep_desc *desc, int32_t world, int32_t cap, void *send_rows,
                                    int32_t *send_meta, struct CUstream_st *stream);
LATENT_API int latent_ep_combine_fixed(const latent_ep_desc *desc, int32_t world, int32_t cap, const float *y_rows,
                                       float *out, struct CUstream_st *stream);

/* The fixed-capacity blocks with rows and metadata in one buffer, so that
 * one all-to-all carries both: block g (world blocks of equal size) =
 * [cap rows of x (x's type)][cap {global expert id, weight bits} int32 pairs,
 * padded to 16 bytes].  send_buf == NULL: only *bytes_needed is written.
 * latent_ep_unpack_fixed turns the received buffer into the local op's
 * inputs: x_out[world*cap][d], ids_out[world*cap] (id - expert_base for the
 * n_local local experts, -1 for unused rows; an id outside them records
 * LATENT_ERR_EXPERT_ID's bit in *err_word when given) and w_out (the weight
 * with LATENT_FLAG_WEIGHT_BEFORE_DOWN, else 1). */
LATENT_API int latent_ep_pack_fixed_merged(const latent_ep_desc *desc, int32_t world, int32_t cap, void *send_buf,
                                           size_t buf_bytes, size_t *bytes_needed, struct CUstream_st *stream);
LATENT_API int latent_ep_unpack_fixed(const void *recv_buf, int32_t world, int32_t cap, int32_t n_embd, int32_t x_type,
                                      int32_t expert_base, int32_t n_local, uint32_t flags, void *x_out,
                                      int32_t *ids_out, float *w_out, uint32_t *err_word, struct CUstream_st *stream);

/* Dense-fallback experts (reference: the compressor keeps a dense fp16
 * copy `<name>.dense_fallback` of a matrix whose factors miss its error
 * threshold, loader/latent_loader.py:262-265; the dense forward is
 * dense_swiglu_expert, loader/latent_runtime.py:62-73; the reference runtime
 * itself ignores the copy).  A flagged expert is served densely: per kind,
 * its dense matrix when present, else its factor pair as exact fp32 A and B
 * (dequantised once at load).  Use with the latent op on the same batch:
 *   1. latent_dense_experts_prepare: routes the flagged experts' slots into
 *      the workspace and writes ids_latent = ids with those slots set to -1;
 *   2. latent_expert_ffn_forward with ids_latent (writes out);
 *   3. latent_dense_experts_forward: adds the flagged experts' contributions
 *      into out (OUT_PER_SLOT: writes their rows), fp32 accumulation on the
 *      CUDA cores.  Same desc and workspace as step 1. */
typedef struct latent_dense_expert {
    int32_t expert;          /* global expert id */
    int32_t rank;            /* rank of the pairs below (even; unused when all kinds are dense) */
    const void *dense[3];    /* gate [d][f], up [d][f], down [f][d] (dense_type); NULL: the pair */
    const float *a[3];       /* A of the kinds without a dense matrix: [d][r], [d][r], [f][r] fp32 */
    const float *b[3];       /* B: [r][f], [r][f], [r][d] fp32 */
} latent_dense_expert;

typedef struct latent_dense_desc {
    int32_t n_expert;        /* E */
    int32_t n_embd;          /* d (multiple of 32) */
    int32_t n_ff;            /* f (multiple of 32) */
    int32_t n_tokens;        /* T */
    int32_t top_k;           /* k */
    int32_t x_type;          /* latent_type of x */
    int32_t w_type;          /* latent_type of the router weights (F32 or F16) */
    int32_t dense_type;      /* LATENT_TYPE_F16 or F32: element type of the dense matrices */
    uint32_t flags;          /* LATENT_FLAG_WEIGHT_BEFORE_DOWN, LATENT_FLAG_OUT_PER_SLOT */
    int32_t n_dense;         /* flagged experts */
    const latent_dense_expert *experts;  /* host array [n_dense] */
    const int32_t *dense_index;          /* device [E]: index into experts, -1 for latent experts */
    const void *x;           /* [T][d] */
    const int32_t *ids;      /* [T][k] (the caller's ids, not ids_latent) */
    const void *weights;     /* [T][k] */
    float *out;              /* as for latent_expert_ffn_forward */
    void *workspace;         /* 256-byte aligned, latent_dense_workspace_size() bytes */
    size_t workspace_bytes;
} latent_dense_desc;

LATENT_API int latent_dense_workspace_size(const latent_dense_desc *desc, size_t *bytes);
LATENT_API int latent_dense_experts_prepare(const latent_dense_desc *desc, int32_t *ids_latent,
                                            struct CUstream_st *stream);
LATENT_API int latent_dense_experts_forward(const latent_dense_desc *desc, struct CUstream_st *stream);

/* y[M][N] = x[M][K] . w[K][N] in fp32 on the CUDA cores (x F32/F16/BF16,
 * w F32/F16, row-major, K and N even).  The projection utility behind the
 * Python mirror's project (loader/latent_runtime.py:35-36, on dequantised
 * factors) and dense_swiglu_expert (:62-73). */
LATENT_API int latent_dense_matmul(const void *x, int32_t x_type, const void *w, int32_t w_type, float *y, int64_t M,
                                   int64_t K, int64_t N, struct CUstream_st *stream);

/* ggml op adapter: the body of the reference's ggml_cuda_latent_expert_ffn
 * (kernels/latent_fused_expert_ffn.cu:134-292) as library calls.  A ggml
 * tensor is passed as its device data, its ne[4] and its ggml_type value. */
typedef struct latent_ggml_tensor {
    const void *data;
    int64_t ne[4];
    int32_t type;           /* LATENT_GGML_* (the ggml_type enum values) */
} latent_ggml_tensor;
enum { LATENT_GGML_F32 = 0, LATENT_GGML_F16 = 1, LATENT_GGML_I8 = 24, LATENT_GGML_I32 = 26, LATENT_GGML_BF16 = 30 };

/* Load time.  factors[12] = the op's src[3..14] (codes I8 and scales F16 of
 * gate_a, gate_b, up_a, up_b, down_a, down_b) as the reference GGUF writer
 * stores them (loader/write_latent_gguf.py:101-123, :412-436): dims recorded
 * as ne = (n_expert, rows, cols/2) and (n_expert, rows, cols/32), bytes in C
 * order of those dims, A factors [n_in, max_rank], B factors [rank, n_out].
 * Copies them into `dst` (caller-owned device memory, 256-byte aligned) in
 * the library's tile order, padded to one power-of-two rank with zero groups,
 * and fills the layer fields of *desc (n_expert, n_embd, n_ff, rank and the
 * six latent_qmatrix).  dst == NULL: only *bytes_needed is written.
 * Stream-ordered; the sources may be freed once the stream has passed it. */
LATENT_API int latent_ggml_pack_layer(const latent_ggml_tensor *factors, void *dst, size_t dst_bytes,
                                      size_t *bytes_needed, latent_ffn_desc *desc, struct CUstream_st *stream);

/* Per call.  src[3] = the op's x [n_embd, T] (F16, BF16 or F32), ids [k, T]
 * I32, weights [k, T] (F16 or F32); dst F32 [n_embd, k, T] (the op's
 * per-slot output, LATENT_FLAG_OUT_PER_SLOT) or [n_embd, T] (combined by
 * the library).  `layer` comes from latent_ggml_pack_layer.  workspace ==
 * NULL: only *workspace_needed is written; else runs
 * latent_expert_ffn_forward on `stream`. */
LATENT_API int latent_ggml_expert_ffn(const latent_ffn_desc *layer, const latent_ggml_tensor *src,
                                      const latent_ggml_tensor *dst, void *workspace, size_t workspace_bytes,
                                      size_t *workspace_needed, struct CUstream_st *stream);

/* Load-time quantisation of float factors (reference encoders,
 * loader/latent_loader.py:111-158, applied per 32-element group; no
 * counterpart kernel in the reference).  values: n_groups x 32 fp32
 * (row-major groups of a [rows][cols] factor, cols % 32 == 0).  Per group:
 * NF4 codes (absmax, fp32 normalise, nearest level, lowest code on ties,
 * fp16 scale); with snr_db not NaN, a group whose NF4 amplitude SNR
 * ||v|| / max(||v - nf4(v)||, 1e-12) (:173-185; in fp32)
 * is below 10^(snr_db/20) is stored INT8 instead (scale absmax/127,
 * round-half-even, clip +-127); an all-zero group stays NF4.  Writes
 * lo[n_groups][16] (NF4 codes, or the INT8 low nibbles), hi[n_groups][16]
 * (INT8 high nibbles, else 0), the fp16 scale bits, is_int8[n_groups] (0/1)
 * and, when snr is not NULL, each group's NF4 SNR: the GroupedFactor arrays
 * of the Python layer. */
LATENT_API int latent_quantize_groups(const float *values, int64_t n_groups, float snr_db, uint8_t *lo, uint8_t *hi,
                                      uint16_t *scales, uint8_t *is_int8, float *snr, struct CUstream_st *stream);

/* ABI version of the loaded library (LATENT_ABI_VERSION). */
LATENT_API int latent_abi_version(void);

/* Static description of a status code. */
LATENT_API const char *latent_status_string(int status);

/* Workspace bytes latent_expert_ffn_forward needs for this descriptor
 * (pointers may be NULL here).  Replaces the per-call cudaMallocAsync of the
 * reference wrapper (kernels/latent_fused_expert_ffn.cu:246-264). */
LATENT_API int latent_expert_ffn_workspace_size(const latent_ffn_desc *desc, size_t *bytes);

/* Routed SwiGLU expert FFN + top-k combine, stream-ordered on `stream`.
 * Replaces ggml_cuda_latent_expert_ffn (kernels/latent_fused_expert_ffn.cu:134)
 * and latent_fused_expert_dispatch / latent_expert_reduce (:27-132).
 * Semantics: loader/latent_runtime.py:48-59 per routed slot, then
 * out[t] = sum_j w[t][j] * y_j (plain sum with WEIGHT_BEFORE_DOWN).
 * Host-side validation errors return before anything is launched.  A routed
 * id >= n_expert is skipped and recorded in the workspace; read it with
 * latent_expert_ffn_check(). */
LATENT_API int latent_expert_ffn_forward(const latent_ffn_desc *desc, struct CUstream_st *stream);

/* latent_expert_ffn_forward for callers that cannot allocate device memory
 * at call time (a host framework that plans all buffers before running its
 * graph and forbids allocation during it, real-time hosts that reserve all
 * memory up front, processes under a hard GPU memory cap).  No counterpart
 * in the reference op.  It ignores desc->workspace and uses a 16 MiB scratch
 * array that the library keeps in device memory (reserved on every GPU that
 * loads the library, until exit); a call needing more returns
 * LATENT_ERR_WORKSPACE.  The array's address is looked up on every call made
 * outside stream capture; a captured call reuses the last one, so make one
 * call on the device before capturing (else LATENT_ERR_UNSUPPORTED).  All
 * calls share the array: calls that overlap on the GPU race.  Device-side
 * errors are read with latent_expert_ffn_check_noalloc.  Allocates nothing. */
LATENT_API int latent_expert_ffn_forward_noalloc(const latent_ffn_desc *desc, struct CUstream_st *stream);

/* latent_expert_ffn_check for the scratch array of
 * latent_expert_ffn_forward_noalloc on the current device (desc->workspace
 * is ignored): synchronises `stream`, then reports the device-side errors
 * the last no-alloc call recorded. */
LATENT_API int latent_expert_ffn_check_noalloc(const latent_ffn_desc *desc, struct CUstream_st *stream);

/* latent_expert_ffn_forward that also records the caller's events on
 * `stream` around each kernel it launches: events[0] before routing, then one
 * after routing and after every FFN kernel (decode: the routing kernel and
 * the fused chain kernel, so 3 events in all).  A profiling aid with no counterpart in the reference op;
 * results are identical to latent_expert_ffn_forward. */
LATENT_API int latent_expert_ffn_forward_timed(const latent_ffn_desc *desc, struct CUstream_st *stream,
                                               struct CUevent_st *const *events, int n_events);

/* Synchronises `stream` and reports device-side errors recorded by the last
 * forward that used `workspace` (LATENT_ERR_EXPERT_ID, LATENT_ERR_TIMEOUT). */
LATENT_API int latent_expert_ffn_check(const latent_ffn_desc *desc, struct CUstream_st *stream);

/* Failure-path test hook, process-wide, for the decode path's fused kernel
 * (no counterpart in the reference).  wait_ns (1 ms .. 2 s; 0 = the default
 * 2 s) bounds every device-side wait of later launches; with
 * unreachable_dependency != 0 each cross-CTA dependency wait also asks for
 * one completion more than the kernel will ever make, so it runs out, the
 * kernel records LATENT_ERR_TIMEOUT and unwinds without faulting, and the
 * context stays usable.  Call (0, 0) to restore the defaults. */
LATENT_API int latent_debug_set_wait_limit(uint64_t wait_ns, int32_t unreachable_dependency);

/* Dequantize expert `expert` of one stacked factor to fp32 out[rows][cols],
 * bit-exact with dequantize_nf4 / dequantize_int8
 * (reference loader/latent_loader.py:133-145, 161-170). */
LATENT_API int latent_dequantize(const latent_qmatrix *m, int32_t expert, float *out, struct CUstream_st *stream);

/* y = silu(x) elementwise in fp32 (reference loader/latent_runtime.py:39-45). */
LATENT_API int latent_silu(const float *x, float *y, int64_t n, struct CUstream_st *stream);

/* Load-time repack of a stacked factor from the row-major layout of the
 * reference GGUF writer (codes [n_expert][rows][cols/2], fp16 scales
 * [n_expert][rows][cols/32]; loader/write_latent_gguf.py:101-123) into the
 * tile-major layout above.  Device buffers, caller-owned, same sizes as the
 * sources, not overlapping them; 16-byte aligned codes, 2-byte aligned
 * scales.  Scale sign bits pass through unchanged.  No counterpart in the
 * reference, whose kernel reads the row-major layout directly. */
LATENT_API int latent_pack_tiles(const uint8_t *codes, const uint16_t *scales, int32_t n_expert, int64_t rows,
                                 int64_t cols, uint8_t *dst_codes, uint16_t *dst_scales, struct CUstream_st *stream);

/* Adaptive top-k router (reference loader/adaptive_topk.py:29-90,
 * adaptive_topk_inclusive / adaptive_topk_batch).  scores[n_tokens][n_expert]
 * fp32 router scores (e.g. softmax probabilities) -> per token its top_k
 * experts in descending score order (ties: lower expert id first), of which
 * the leading ones are kept while their float32 running sum stays within
 * threshold x the float32 sum of the top_k (compared in float32, as numpy 2
 * evaluates the reference).  ids[n_tokens][top_k] int32: kept expert ids,
 * -1 for dropped slots (the fused op skips them).  weights[n_tokens][top_k]
 * fp32: kept scores divided by their float32 sum with
 * LATENT_ROUTER_RENORMALIZE, else the raw scores; 0 for dropped slots.
 * n_kept[n_tokens] (optional, may be NULL): kept slots per token.  A token
 * whose top_k sum is <= 0 keeps none.  Errors: LATENT_ERR_SHAPE for
 * top_k < 1 or top_k > n_expert (the reference raises ValueError),
 * LATENT_ERR_INVALID for threshold outside (0, 1] (ValueError there) or
 * unknown flags, LATENT_ERR_UNSUPPORTED beyond 1024 experts or top_k 32.
 * NaN scores rank below every number (numpy's sort order), so they are
 * selected only when fewer than top_k numbers remain; a token whose top_k
 * then holds a NaN keeps all top_k slots with NaN weights, as the reference
 * does.  Stream-ordered,
 * allocates nothing; ids/weights feed latent_expert_ffn_forward directly. */
enum { LATENT_ROUTER_RENORMALIZE = 1u << 0, LATENT_ROUTER_SOFTMAX = 1u << 1 };
LATENT_API int latent_router_topk(const float *scores, int32_t n_tokens, int32_t n_expert, int32_t top_k,
                                  double threshold, uint32_t flags, int32_t *ids, float *weights, int32_t *n_kept,
                                  struct CUstream_st *stream);

/* The router in one kernel: latent_router_topk, plus LATENT_ROUTER_SOFTMAX
 * (scores are logits: p = exp(l - max) / sum in fp32 per token, the maximum
 * and the sum by warp reductions; the selection then runs on p) and
 * expert_counts (optional, [n_expert] int32, zeroed by the call): the kept
 * slots per expert, the histogram the fused op's routing builds.  NaN
 * logits give NaN probabilities. */
LATENT_API int latent_router_route(const float *scores, int32_t n_tokens, int32_t n_expert, int32_t top_k,
                                   double threshold, uint32_t flags, int32_t *ids, float *weights, int32_t *n_kept,
                                   int32_t *expert_counts, struct CUstream_st *stream);

#ifdef __cplusplus
}
#endif

#endif /* LATENT_FFN_H */
