/* dsv4cu.h - native C ABI of the B200 (sm_100a) library for the quantized
 * matmul / MoE / sparse-attention-indexer hot path of deepseek-v4-in-c.
 *
 * Two layers are exported from libdsv4cu.so:
 *
 *   1. dsv4_compat.h: the reference's own operator entry points (dsv4_mmq_n,
 *      fp8_n, dsv4_route, dsv4_topk, ...) with HOST pointers, so the reference
 *      engine links against this library unchanged.
 *   2. This header: device-pointer entry points (prefix dsv4cu_) that take a
 *      cudaStream_t and return a status. Every call here is asynchronous on the
 *      given stream unless stated; no call aborts the process.
 *
 * Plain C types only: pointers, ints, floats. A "stream" is a cudaStream_t
 * passed as void*. All pointers are device pointers unless marked (host).
 */
#ifndef DSV4CU_H
#define DSV4CU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
enum {
    DSV4CU_OK = 0,
    DSV4CU_ERR_ARG = -1,          /* invalid argument or shape               */
    DSV4CU_ERR_UNSUPPORTED = -2,  /* format/geometry this build does not cover */
    DSV4CU_ERR_CUDA = -3,         /* a CUDA runtime call or launch failed     */
    DSV4CU_ERR_NOMEM = -4,        /* device allocation failed                 */
    DSV4CU_ERR_TIMEOUT = -5,      /* a bounded device wait expired            */
    DSV4CU_ERR_COMM = -6,         /* collective / peer exchange failed        */
    DSV4CU_ERR_IO = -7            /* pack file missing, malformed or short    */
};

/* Weight storage tags; same values as the reference enum
 * (src/00_base/dsv4.h:81). */
enum { DSV4CU_WF32 = 0, DSV4CU_WBF16 = 1, DSV4CU_WFP8 = 2, DSV4CU_WFP4 = 3 };

/* Packed matrix. Member order and types are those of the reference
 * DSV4QMat (src/00_base/dsv4_weights.h:34-40); here w and s are DEVICE
 * pointers. FP8: w [rows][cols] e4m3, s [ceil(rows/blk_r)][ceil(cols/blk_c)]
 * E8M0. FP4: w [rows][cols/2] (low nibble = even column), s likewise.
 * BF16: w [rows][cols] u16, s unused. */
typedef struct {
    const void *w;
    const void *s;
    int         wdt;
    int         rows, cols;
    int         blk_r, blk_c;
} dsv4cu_qmat;

/* One expert: same member order as the reference DSV4ExpertW
 * (src/00_base/dsv4_weights.h:101-104): w1 (gate) and w3 (up) are
 * [inter][hidden], w2 (down) is [hidden][inter]. */
typedef struct {
    dsv4cu_qmat w1, w3, w2;
} dsv4cu_expert;

/* Last error message of the calling thread (static storage, never NULL). */
const char *dsv4cu_last_error(void);
int dsv4cu_set_error(int code, const char *fmt, ...);

/* Library context: owns a device workspace (grown on demand, or reserved up
 * front with dsv4cu_ctx_reserve so later calls allocate nothing). One context
 * per device; not shared between threads without external locking. */
typedef struct dsv4cu_ctx dsv4cu_ctx;
int  dsv4cu_ctx_create(dsv4cu_ctx **out, int device);
void dsv4cu_ctx_destroy(dsv4cu_ctx *ctx);
int  dsv4cu_ctx_reserve(dsv4cu_ctx *ctx, size_t bytes);
size_t dsv4cu_ctx_workspace_bytes(const dsv4cu_ctx *ctx);
/* Synchronise `stream` and report whether any kernel of this context hit a
 * bounded-wait timeout since the last check (*code = 0: none; otherwise the
 * call returns DSV4CU_ERR_TIMEOUT, clears the word and resets the context's
 * cross-CTA counters, so the next call runs normally). */
int  dsv4cu_ctx_status(dsv4cu_ctx *ctx, void *stream, int *code);
/* Test-only fault, consumed by the next dsv4cu_gemv call on the streamed
 * path: WITHHOLD_STAGE makes its first CTA skip its third weight stage (no
 * copy is issued and nothing arrives on the stage's barrier), so that CTA's
 * consumers' bounded wait expires after 2 s; every role then stops through
 * bounded waits, the call's output is undefined and dsv4cu_ctx_status reports
 * the timeout. 0 cancels. Nothing faults and the context stays usable. */
#define DSV4CU_INJECT_WITHHOLD_STAGE 1
int  dsv4cu_ctx_inject(dsv4cu_ctx *ctx, int what);

/* Workspace bytes a dsv4cu_mmq call of this shape needs. */
size_t dsv4cu_mmq_workspace(const dsv4cu_qmat *m, int nt);

/* y[t*rows + o] = sum_c x[t*cols + c] * W[o][c], t < nt, fp32 in and out.
 * Replaces dsv4_mmq_n (src/10_compute/dsv4_matmul.h:40) on device memory.
 * Every geometry the reference accepts is covered. FP4/FP8 matrices with
 * cols % 128 == 0 and blk_c % 32 == 0 (FP4 weights 32-byte, FP8 16-byte
 * aligned) run on the tcgen05 block-scaled GEMM with 4 exact activation terms
 * (results within ~1e-6 of fp32; a batch row is bit-identical to the same
 * token computed alone); other FP8/FP4 geometries and BF16 use mma.sync
 * kernels, and any remaining block geometry an exact per-element path. */
int dsv4cu_mmq(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *m,
               int nt, void *stream);

/* Decode GEMV: the dsv4cu_mmq product for one or two tokens, streamed at
 * HBM rate. Replaces fp8_n / fp4_n at decode (src/10_compute/
 * dsv4_matmul_fp8.c:49-177, dsv4_matmul_fp4.c:46-162, behind dsv4_mmq_n,
 * src/10_compute/dsv4_matmul.h:40). FP4 matrices with 1x32 scales and
 * cols % 256 == 0, and FP8 matrices with blk_r % 32 == 0, blk_c % 64 == 0
 * and cols % 128 == 0, with rows % 32 == 0, cols <= 8192 and 16-byte aligned
 * weights (and FP4 scales), are read in 32-row x 1 KB tensor-map copies and
 * reduced on the CUDA cores and mma.sync: results within about 1e-6 of fp32,
 * and a token's row has the same bits for nt = 1 and 2 and on every run
 * (they are not the bits of dsv4cu_mmq). Other shapes and nt > 2 run
 * dsv4cu_mmq. */
size_t dsv4cu_gemv_workspace(const dsv4cu_qmat *m, int nt);
int dsv4cu_gemv(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *m,
                int nt, void *stream);
/* dsv4cu_gemv recording events[0..2] (cudaEvent_t) on the stream: [0] and
 * [1] before the streamed GEMV (which splits the activations itself), [2]
 * after it. */
int dsv4cu_gemv_ev(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *m,
                   int nt, void *stream, void **events);

/* ------------------------------------------- tensor-core (tcgen05) GEMM
 * A packed matrix prepared once for the block-scaled tensor-core GEMM: the
 * library keeps its TMA descriptor and a copy of its scale factors in the
 * tensor core's block layout (rows/128 x cols/128 x 512 bytes); the weights
 * stay where they are and must outlive the object. Needs FP4 (weights 32-byte
 * aligned) or FP8 (16-byte aligned), cols % 128 == 0, blk_c % 32 == 0.
 * Replaces the per-tile GEMM of the prefill seam
 * (src/80_prefill/dsv4_prefill_vk_gemm.c:63-137) and dsv4_mmq_n for large nt. */
typedef struct dsv4cu_mat dsv4cu_mat;
int    dsv4cu_mat_create(dsv4cu_mat **out, const dsv4cu_qmat *m, void *stream);
void   dsv4cu_mat_destroy(dsv4cu_mat *m);
size_t dsv4cu_mat_workspace(const dsv4cu_mat *m, int nt, int terms);

/* y[t*rows + o] = sum_c x[t*cols + c] * W[o][c] on the tensor cores
 * (tcgen05.mma kind::mxf8f6f4 with E8M0 block scales). Each fp32 activation
 * is split exactly into `terms` (1..4) e4m3 values with their own per-32
 * E8M0 scales; terms = 3 keeps max|y - y_ref| / max|y_ref| well below 1e-3,
 * terms = 4 is within about 1e-5, terms = 1 is the plain MXFP8 product. */
int dsv4cu_mat_gemm(dsv4cu_ctx *ctx, const dsv4cu_mat *m, float *y, const float *x,
                    int nt, int terms, void *stream);

/* Exact-weight GEMM on the bf16 tensor cores (tcgen05 kind::f16): the
 * prefill GEMM's other numerics mode. Every weight w * 2^e of an FP8 or FP4
 * matrix is a bf16 value exactly and is used as such; the activations enter
 * as `terms` bf16 terms: 1 = x rounded to nearest (max-rel ~1.1e-3 against
 * fp32 activations on Gaussian data, 2^-9 per activation), 2 = hi + lo
 * (~1e-5; twice the MMA work). Apart from that rounding the result is fp32
 * accumulation: against the reference fed the same rounded activations the
 * difference is ~1e-7. Needs cols % 64 == 0, power-of-two scale blocks with
 * blk_c >= 32, 16-byte aligned weights and x. y [nt][rows] fp32. */
size_t dsv4cu_gemm_bf16w_workspace(const dsv4cu_qmat *m, int nt, int terms);
int dsv4cu_gemm_bf16w(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *m, int nt, int terms,
                      void *stream);

/* Where dsv4cu_gemm_bf16w dequantizes the weights (process-wide switch; the
 * results are bit-identical either way). CONVERT: converter warps inside the
 * GEMM, once per 256-token tile. PREDEQUANT: one pass writes the bf16 matrix
 * into the workspace (rows x cols x 2 bytes more), then the GEMM loads it by
 * TMA. AUTO (default): PREDEQUANT when nt x terms > 256. Set it before
 * sizing the workspace. */
enum { DSV4CU_BF16W_AUTO = 0, DSV4CU_BF16W_CONVERT = 1, DSV4CU_BF16W_PREDEQUANT = 2 };
int dsv4cu_gemm_bf16w_set_path(int path);

/* dsv4cu_mat_gemm with an explicit tile configuration: nb B columns per tile
 * (8, 16, 32, 64, 128, 192 or 256; terms x tokens per tile) and kb 128-wide K
 * chunks per pipeline stage (1, 2 or 4; lowered until it divides cols/128).
 * 0 = choose automatically. Built pairs: nb 8/16 with kb 1/2/4, nb 32/64
 * with kb 1/2, nb 128/192/256 with kb 1. */
int dsv4cu_mat_gemm_cfg(dsv4cu_ctx *ctx, const dsv4cu_mat *m, float *y, const float *x,
                        int nt, int terms, int nb, int kb, void *stream);

/* dsv4cu_mat_gemm that also records events[0..2] (cudaEvent_t, created by the
 * caller) on the stream: before the activation split, before the GEMM and
 * after it. For timing the GEMM kernel alone. */
int dsv4cu_mat_gemm_ev(dsv4cu_ctx *ctx, const dsv4cu_mat *m, float *y, const float *x,
                       int nt, int terms, void *stream, void **events);

/* Router for nt tokens; replaces dsv4_route (src/10_compute/dsv4_kernels.h:24).
 * logits [nt][n_experts] (read), scores/orig [nt][n_experts] (written: biased
 * selection scores and sqrt(softplus) scores, either may be NULL), idx/wts
 * [nt][topk]. bias [n_experts] or NULL; tid2eid [vocab][topk] int64 or NULL
 * (hash routing, token_ids [nt] then required). topk <= 16. */
int dsv4cu_route(int *idx, float *wts, float *scores, float *orig,
                 const float *logits, const float *bias, const int64_t *tid2eid,
                 const int *token_ids, int n_experts, int topk,
                 float route_scale, int nt, void *stream);

/* y = silu(min(gate, limit)) * clamp(up, -limit, limit), n elements;
 * replaces dsv4_swiglu (src/10_compute/dsv4_kernels.h:22). */
int dsv4cu_swiglu(float *y, const float *gate, const float *up, int n,
                  float limit, void *stream);

/* A prepared MoE layer: the routed experts and the optional shared expert of
 * one layer, resident in HBM, validated once and given one TMA tensor map per
 * weight matrix. experts: HOST array of n_experts descriptors whose w/s are
 * device pointers (kept by reference: the weights must outlive the layer);
 * shared: HOST pointer to one descriptor or NULL. w1/w3 are [inter][hidden],
 * w2 [hidden][inter]; FP4 (blk_c % 32 == 0) or FP8 (blk_c % 16 == 0), 16-byte
 * aligned weights; hidden and inter multiples of 128. */
typedef struct dsv4cu_moe dsv4cu_moe;

/* Routed experts of one layer read from the reference's pack into HBM (the
 * experts.idx written by tools/pack_trunk.py and read by
 * src/40_io/dsv4_st.c:65-87; shards = model_dir's *.safetensors in name
 * order). Experts first .. first + count - 1 of `layer` are read once (pread
 * into pinned staging, copied on `stream`, synchronised before return) into
 * one device allocation owned by *out, and experts[0 .. count - 1] receive
 * their FP4 e2m1 1x32 E8M0 descriptors (device pointers) for
 * dsv4cu_moe_create. Every record's size is checked against hidden / inter;
 * a missing, malformed or short pack returns DSV4CU_ERR_IO. For expert
 * parallelism rank r loads [r * per_rank, (r + 1) * per_rank). */
typedef struct dsv4cu_expert_store dsv4cu_expert_store;
int  dsv4cu_experts_load(dsv4cu_expert_store **out, dsv4cu_expert *experts, const char *model_dir,
                         const char *index_dir, int layer, int first, int count, int hidden, int inter,
                         void *stream);
void dsv4cu_experts_free(dsv4cu_expert_store *store);
/* Host only: the index's shape, and (when loc != NULL) the six records of
 * (layer, expert) as loc[3 t + {0, 1, 2}] = shard, offset, bytes in the order
 * w1, w1 scales, w2, w2 scales, w3, w3 scales. */
int  dsv4cu_experts_index(const char *index_dir, int *n_layers, int *n_experts, int layer, int expert,
                          int64_t *loc);

/* Dense trunk from the reference's pack into HBM (replaces dsv4_trunk_open,
 * src/50_loader/dsv4_trunk.c:37-131, which reads trunk.bin into host memory;
 * manifest format of src/50_loader/dsv4_trunk_manifest.c:24-110). A tensor
 * record mirrors DSV4TrunkTensor (src/50_loader/dsv4_trunk.h:20-27): off is
 * the byte offset within its layer's run, dtype the safetensors code
 * (1 u8, 2 bf16, 3 f16, 4 f32, 5 e4m3, 6 e8m0, 7 i8, 8 i64), wdt DSV4CU_W*. */
typedef struct {
    int32_t slot;
    int32_t dtype;
    int32_t rows, cols;
    int32_t wdt, blk_r, blk_c;
    int64_t off;
    int64_t nbytes;
} dsv4cu_trunk_tensor;
typedef struct dsv4cu_trunk dsv4cu_trunk;
/* Host only: trunk.idx of `dir`. n_layers always; for layer >= 0 also
 * run[0..2] = file offset, bytes, widened-vector bytes of that layer, its
 * tensor count and up to cap tensor records. A missing or malformed index
 * returns DSV4CU_ERR_IO (bad magic / version, n_layers, layout, layer or
 * tensor line, dtype or format code, a tensor outside its run). */
int  dsv4cu_trunk_manifest(const char *dir, int *n_layers, int layer, int64_t *run, int *n_tensors,
                           dsv4cu_trunk_tensor *tensors, int cap);
/* Layers first .. first + count - 1 (count <= 0: to the last) of trunk.bin
 * into one device arena owned by *out (each run 4 KiB aligned; read in
 * 64 MiB pieces through two pinned buffers, copied on `stream`, synchronised
 * before return). A short read returns DSV4CU_ERR_IO. */
int  dsv4cu_trunk_load(dsv4cu_trunk **out, const char *dir, int first, int count, void *stream);
/* Device address and record of (layer, slot); DSV4CU_ERR_ARG when the layer
 * is not resident or has no such slot. */
int  dsv4cu_trunk_slot(const dsv4cu_trunk *trunk, int layer, int slot, dsv4cu_trunk_tensor *desc, void **dev);
/* A packed matrix's device descriptor: weights from `slot`, shape and format
 * from its record, scales (FP8 / FP4) from slot + 1 (the pack's X / X_S
 * pairing, src/50_loader/dsv4_bind_layer.c:12-23). */
int  dsv4cu_trunk_qmat(const dsv4cu_trunk *trunk, int layer, int slot, dsv4cu_qmat *q);
/* A vector widened to f32 into dst on `stream`, as the reference's bind
 * does (dsv4_widen_f32, src/40_io/dsv4_st.h:117-134): f32 copied, bf16
 * widened exactly, other dtypes DSV4CU_ERR_UNSUPPORTED. */
int  dsv4cu_trunk_widen(const dsv4cu_trunk *trunk, int layer, int slot, float *dst, void *stream);
int64_t dsv4cu_trunk_resident_bytes(const dsv4cu_trunk *trunk);
void dsv4cu_trunk_free(dsv4cu_trunk *trunk);
int  dsv4cu_moe_create(dsv4cu_moe **out, const dsv4cu_expert *experts, int n_experts,
                       const dsv4cu_expert *shared, int hidden, int inter);
void dsv4cu_moe_destroy(dsv4cu_moe *layer);
/* Which kernels a decode of one or two tokens takes. AUTO (the default): the
 * tcgen05 path where every matrix qualifies for it, else the streamed path
 * (one persistent CTA per SM over a queue of 32-row jobs, FP4/FP8 decoded in
 * registers, mma.sync as the reduction). TENSOR / STREAM force one; a layer
 * without that path returns DSV4CU_ERR_UNSUPPORTED. Hash routing, three or
 * more tokens and dsv4cu_moe_prefill always take the tensor-core path. Both
 * paths give the reference's results within the matmul tolerance; each is
 * deterministic. */
#define DSV4CU_MOE_PATH_AUTO   0
#define DSV4CU_MOE_PATH_TENSOR 1
#define DSV4CU_MOE_PATH_STREAM 2
int  dsv4cu_moe_set_path(dsv4cu_moe *layer, int path);
/* Workspace bytes one dsv4cu_moe_decode of this layer needs. */
size_t dsv4cu_moe_workspace(const dsv4cu_moe *layer, int topk, int nt);

/* One MoE layer decode step for nt tokens (the reference dsv4_layer_moe,
 * src/70_decode/dsv4_layer.c:48-117, from the router logits on): route, the
 * routed experts' w1/w3 -> SwiGLU -> w2, the weighted sum in k order, plus the
 * shared expert added unweighted. x [nt][hidden], logits [nt][n_experts],
 * out [nt][hidden]; bias [n_experts] or NULL; tid2eid [vocab][topk] int64 or
 * NULL (hash routing, token_ids [nt] then required). idx_out/wts_out
 * [nt][topk] may be NULL. nt <= 64, topk <= 16. */
int dsv4cu_moe_decode(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out,
                      const float *x, const float *logits, const float *bias,
                      const int64_t *tid2eid, const int *token_ids, int topk,
                      float route_scale, float limit, int nt, int *idx_out,
                      float *wts_out, void *stream);

/* dsv4cu_moe_decode from host buffers x_host [nt][hidden], logits_host
 * [nt][n_experts] and out_host [nt][hidden], enqueued on the stream, nothing
 * synchronised (read out_host after synchronising the stream). With
 * page-locked host buffers (cudaHostAlloc, cudaHostRegister, a framework's
 * pinned allocator) one staging kernel reads the inputs across the bus and the
 * step writes the output into host memory directly; with pageable buffers
 * they are copied through device staging. No bias, hash routing or index
 * outputs. */
int dsv4cu_moe_decode_host(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out_host,
                           const float *x_host, const float *logits_host, int topk,
                           float route_scale, float limit, int nt, void *stream);

/* dsv4cu_moe_decode with CUDA events (cudaEvent_t) recorded around its three
 * launches: events[0] before the router/bucketing prologue, [1] after it,
 * [2] after the w1/w3 kernel (SwiGLU in its epilogue), [3] after the w2
 * kernel (the combine in its epilogue, up to 4 tokens; else a combine kernel).
 * events may be NULL. Used to time each kernel live on the launching stream. */
int dsv4cu_moe_decode_ev(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out,
                         const float *x, const float *logits, const float *bias,
                         const int64_t *tid2eid, const int *token_ids, int topk,
                         float route_scale, float limit, int nt, int *idx_out,
                         float *wts_out, void *stream, void **events);

/* ---- expert-parallel MoE layer (no reference counterpart: it replaces the
 * src/60_cache expert cache with HBM-resident experts spread over ranks;
 * the per-token math is dsv4_layer_moe's, src/70_decode/dsv4_layer.c:48-117).
 *
 * dsv4cu_moe_rows: y[r] = expert ids[r] applied to row r of x (row stride
 * ldx floats, a multiple of 4), no weighting; ids in 0 .. n_experts - 1 or
 * n_experts for the layer's shared expert; id -1 skips the row (y[r] is not
 * written). Any other id out of range gives a zero row and the device status
 * code 26. nrows <= 32768. */
size_t dsv4cu_moe_rows_workspace(const dsv4cu_moe *layer, int nrows);
int dsv4cu_moe_rows(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *y, const float *x, long ldx,
                    const int *ids, int nrows, float limit, void *stream);

/* Dispatch side: the nt * topk (token, slot) pairs of idx [nt][topk] (global
 * expert ids; rank = id / experts_per_rank) become send rows [nt * topk]
 * [hidden + 4] grouped by rank and, inside a rank, in pair order; a row is
 * x[t] then the rank-local expert id as a float and 3 zeros. counts [n_ranks]
 * = rows per rank, pair_slot [nt * topk] = each pair's send row (-1 for an
 * id out of range, which also sets the device status to 31). n_ranks <= 16. */
int dsv4cu_ep_pack(dsv4cu_ctx *ctx, float *send, int *counts, int *pair_slot, const float *x,
                   const int *idx, int nt, int topk, int hidden, int experts_per_rank,
                   int n_ranks, void *stream);

/* recv [nrecv + nt][hidden + 4]: ids[r] = the id column of the nrecv
 * received rows; rows nrecv .. nrecv + nt - 1 are set to x (the own tokens)
 * with id shared_id. */
int dsv4cu_ep_tail(float *recv, int nrecv, const float *x, int nt, int hidden, int shared_id,
                   int *ids, void *stream);

/* out[t] = sum over k in order of wts[t][k] * back[pair_slot[t][k]] (rows of
 * hidden floats), then + shared[t] (may be NULL): the single-device layer's
 * float operations. */
int dsv4cu_ep_combine(float *out, const float *back, const int *pair_slot, const float *wts,
                      const float *shared, int nt, int topk, int hidden, void *stream);

/* ---- one decoder layer's attention on the device (dsv4_layer_attention,
 * src/70_decode/dsv4_layer_attn.c:12-107, and the attention half of
 * dsv4_layer_forward, src/70_decode/dsv4_layer.c:24-36): projections, q / kv
 * norms, RoPE, the KV ring, the compressor, the indexer (ratio 4) with its
 * top-k, sparse attention, the inverse RoPE and the grouped wo_a (one launch)
 * + wo_b, for one token, each step the library's device op. Weights are
 * device pointers kept by reference; dsv4cu_attn_create allocates the
 * layer's state (KV ring + compressed rows, the compressor's ring with its
 * scores at -inf) and scratch. Tokens come in order pos = 0, 1, ...;
 * nothing is synchronised. */
typedef struct {
    int hidden, n_heads, head_dim, q_lora, o_lora, o_groups, qk_rope, sliding_window;
    int index_n_heads, index_head_dim, index_topk;   /* used when compress_ratio == 4 */
    int hc_mult, hc_sinkhorn_iters;                  /* used by dsv4cu_attn_block */
    float rms_eps, hc_eps;
    int compress_ratio;                              /* 0, 4 (compressor + indexer) or another ratio */
    int max_pos;                                     /* rows of the RoPE table; bounds the state */
} dsv4cu_attn_cfg;

typedef struct {
    dsv4cu_qmat wq_a, wq_b, wkv, wo_a, wo_b;         /* FP8 (any dsv4cu_mmq format) */
    dsv4cu_qmat comp_wkv, comp_wgate;                /* compress_ratio != 0 */
    dsv4cu_qmat idx_wq_b, idx_wproj;                 /* compress_ratio == 4 */
    const float *q_norm, *kv_norm, *sink, *comp_ape, *comp_norm;
    const float *attn_norm, *hc_fn, *hc_base, *hc_scale;   /* dsv4cu_attn_block only */
    const float *cs, *sn;                            /* RoPE table [max_pos][qk_rope / 2] */
} dsv4cu_attn_weights;

typedef struct dsv4cu_attn dsv4cu_attn;
int  dsv4cu_attn_create(dsv4cu_attn **out, const dsv4cu_attn_cfg *cfg, const dsv4cu_attn_weights *w);
void dsv4cu_attn_destroy(dsv4cu_attn *a);
/* out [hidden] = the attention of x [hidden] at position pos. */
int  dsv4cu_attn_step(dsv4cu_ctx *ctx, dsv4cu_attn *a, float *out, const float *x, int pos, void *stream);
/* h [hc_mult][hidden] in place: mHC pre-mix, attn_norm, attention, mHC update. */
int  dsv4cu_attn_block(dsv4cu_ctx *ctx, dsv4cu_attn *a, float *h, int pos, void *stream);
int  dsv4cu_attn_n_compressed(const dsv4cu_attn *a);
const float *dsv4cu_attn_kv_cache(const dsv4cu_attn *a);
/* Benchmarking and tests: put the layer at position pos with a synthetic
 * context (seeded values in [-1, 1) in the KV ring, the pos / ratio
 * compressed rows and the compressor's ring), so the next step is pos. */
int  dsv4cu_attn_fill_context(dsv4cu_attn *a, int pos, unsigned long long seed, void *stream);

/* ---- the FFN half of a decoder layer and the whole layer (dsv4_layer_forward,
 * src/70_decode/dsv4_layer.c:18-46): the FFN's mHC pre-mix, ffn_norm, the
 * BF16 router GEMV, the MoE step of dsv4_layer_moe (dsv4cu_moe_decode, or
 * with `ep` set the expert-parallel step dsv4cu_ep_forward over the ranks,
 * whose routing takes no bias or hash table) and the mHC update, for nt <=
 * nt_max tokens (a decode batch: h [nt][hc_mult][hidden] in place;
 * token_ids: device [nt], hash layers only). dsv4cu_layer_step runs
 * dsv4cu_attn_block then the FFN half for one token. Device pointers, kept by
 * reference. */
typedef struct dsv4cu_ep dsv4cu_ep;
typedef struct {
    const dsv4cu_moe *moe;        /* the layer's routed experts + shared expert (this rank's, with ep) */
    dsv4cu_qmat gate;             /* router [n_experts][hidden], BF16 in the engine */
    const float *bias;            /* selection bias [n_experts] or NULL */
    const int64_t *tid2eid;       /* hash layers: [vocab][topk], or NULL */
    const float *ffn_norm, *hc_fn, *hc_base, *hc_scale;
    int hidden, hc_mult, hc_sinkhorn_iters, n_experts, topk, nt_max;
    float rms_eps, hc_eps, route_scale, swiglu_limit;
    dsv4cu_ep *ep;                /* NULL: all experts on this GPU */
} dsv4cu_ffn_desc;
typedef struct dsv4cu_ffn dsv4cu_ffn;
int  dsv4cu_ffn_create(dsv4cu_ffn **out, const dsv4cu_ffn_desc *desc);
void dsv4cu_ffn_destroy(dsv4cu_ffn *f);
int  dsv4cu_ffn_block(dsv4cu_ctx *ctx, dsv4cu_ffn *f, float *h, int nt, const int *token_ids, void *stream);
int  dsv4cu_layer_step(dsv4cu_ctx *ctx, dsv4cu_attn *a, dsv4cu_ffn *f, float *h, int pos, int token_id,
                       void *stream);

/* ---- the expert-parallel layer step on device, ranks joined by NVLink peer
 * memory (replaces dsv4_layer_moe's loop over the src/60_cache expert cache,
 * src/70_decode/dsv4_layer.c:48-117, for experts spread over the GPUs of one
 * box). Rank r holds routed experts [r * experts_per_rank, (r + 1) *
 * experts_per_rank) and the shared expert as one dsv4cu_moe; every rank is the
 * home of its own nt <= nt_max tokens.
 *
 * Set-up, once per rank: dsv4cu_ep_create; dsv4cu_ep_handle writes this
 * rank's DSV4CU_EP_HANDLE_BYTES-byte handle; the caller all-gathers the
 * handles over any transport (MPI, a TCP key-value store, NCCL) into
 * world * DSV4CU_EP_HANDLE_BYTES bytes in rank order and passes them to
 * dsv4cu_ep_connect, which maps the peers' buffers (CUDA IPC; the GPUs must
 * have peer access). Handles of a different geometry are refused with
 * DSV4CU_ERR_COMM.
 *
 * dsv4cu_ep_forward: route the home tokens (logits over experts_per_rank *
 * world experts), store each (token, k) row into its owner's inbox over
 * NVLink, run every received row through its expert and the home tokens
 * through the shared expert on the tensor cores, store the results back,
 * and combine in k order. All ranks call it in lockstep (same number of
 * calls, any nt per rank). It is enqueued on the stream with nothing
 * synchronised (graph-capturable); the cross-rank waits are bounded (2 s) and
 * report through dsv4cu_ctx_status (codes 61 dispatch, 62 return, 63 expert
 * id). out equals the single-device layer bit for bit. events (7 cudaEvent_t
 * or NULL) are recorded around route+plan, dispatch, gather, the expert
 * GEMMs, return and combine. */
#define DSV4CU_EP_HANDLE_BYTES 128
int  dsv4cu_ep_create(dsv4cu_ep **out, int rank, int world, int nt_max, int hidden, int topk,
                      int experts_per_rank);
int  dsv4cu_ep_handle(const dsv4cu_ep *ep, void *blob);
int  dsv4cu_ep_connect(dsv4cu_ep *ep, const void *blobs);
size_t dsv4cu_ep_workspace(const dsv4cu_ep *ep, const dsv4cu_moe *layer, int nt);
int  dsv4cu_ep_forward(dsv4cu_ctx *ctx, dsv4cu_ep *ep, const dsv4cu_moe *layer, float *out,
                       const float *x, const float *logits, int nt, float route_scale, float limit,
                       int *idx_out, float *wts_out, void *stream, void **events);
void dsv4cu_ep_destroy(dsv4cu_ep *ep);

/* Indexer score with fp32 inputs, bit-identical to dsv4_indexer_score
 * (src/10_compute/dsv4_indexer.c:66-90): out[t] = (float)(sum_h relu(q_h.k_t)
 * * w_h) * d^-1/2 h^-1/2, with the reference's double reduction tree. */
int dsv4cu_indexer_score(float *out, const float *q, const float *kv,
                         const float *weights, int n_heads, int head_dim,
                         int n_pos, void *stream);

/* The same score from FP8 inputs: q8 [n_heads][head_dim] e4m3 with one fp32
 * scale per head, k8 [n_pos][k_stride] e4m3 (first head_dim bytes used) with
 * one fp32 scale per position. Bit-identical to dsv4_indexer_score applied to
 * the dequantized values q8*q_scale and k8*k_scale. */
int dsv4cu_indexer_score_fp8(float *out, const uint8_t *q8, const float *q_scale,
                             const uint8_t *k8, const float *k_scale,
                             const float *weights, int n_heads, int head_dim,
                             int n_pos, int k_stride, void *stream);

/* Which kernel dsv4cu_indexer_score_fp8 uses for 64 heads x 128 when every
 * scale is a power of two (both give the same bits): AUTO = exact integer
 * dots on the int8 tensor cores (key rows 16-byte aligned), FP64 = exact
 * dots on the FP64 tensor cores. Process-wide; for comparisons. */
#define DSV4CU_INDEXER_AUTO 0
#define DSV4CU_INDEXER_FP64 1
int dsv4cu_indexer_set_path(int path);

/* The MoE layer over nt tokens at once (prefill, up to 16384 tokens): the
 * reference's prefill union path (src/80_prefill/dsv4_prefill_union.c:30-66,
 * dsv4_prefill_experts.c:23-77, dsv4_prefill_union_run.c:109-121, shared
 * expert dsv4_prefill_moe.c:40-59) with the same arguments as
 * dsv4cu_moe_decode. Tokens are bucketed by expert (tokens ascending inside a
 * bucket) and every bucket runs as tcgen05 block-scaled GEMMs; the fp32
 * activations enter the tensor core as `terms` (1 .. 4) e4m3 terms with
 * per-32 E8M0 scales (4: max-rel error ~1e-6, 3: ~1e-5, 2: ~1e-3; 1 is the
 * plain MXFP8 product, the single-term mode: 64 tokens per 192/256-column
 * tile at 3 / 4 terms, 128 at 2, 256 at 1). Needs a layer whose matrices all
 * qualify for the tensor-core path (FP4/FP8, dims multiples of 128). */
size_t dsv4cu_moe_prefill_workspace(const dsv4cu_moe *layer, int topk, int nt, int terms);
int dsv4cu_moe_prefill(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out, const float *x,
                       const float *logits, const float *bias, const int64_t *tid2eid,
                       const int *token_ids, int topk, float route_scale, float limit,
                       int nt, int terms, int *idx_out, float *wts_out, void *stream);
/* dsv4cu_moe_prefill recording 4 cudaEvent_t (events, may be NULL) on the
 * stream: before routing, before the first GEMM, after the gate/up GEMM and
 * after the last launch. */
int dsv4cu_moe_prefill_ev(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out, const float *x,
                          const float *logits, const float *bias, const int64_t *tid2eid,
                          const int *token_ids, int topk, float route_scale, float limit,
                          int nt, int terms, int *idx_out, float *wts_out, void *stream,
                          void **events);

/* Top-k indices of scores[n], descending, ties to the lower index, k clamped
 * to n; replaces dsv4_topk (src/10_compute/dsv4_topk.c:76-112) without its
 * k <= 1024 bound. Writes min(k, n) indices. */
int dsv4cu_topk(dsv4cu_ctx *ctx, int *idx, const float *scores, int n, int k,
                void *stream);

/* Sparse attention with sinks over gathered rows; replaces dsv4_sparse_attn
 * (src/10_compute/dsv4_attn.c:60-107). q/o [h][d] fp32; kv [n][d] fp32
 * (kv_bf16 = 0) or bf16 (kv_bf16 = 1); idxs [topk] with -1 = masked. */
int dsv4cu_sparse_attn(dsv4cu_ctx *ctx, float *o, const float *q, const void *kv,
                       int kv_bf16, const float *sink, const int *idxs, int h,
                       int d, int topk, float scale, void *stream);

/* Kernel of dsv4cu_sparse_attn: AUTO = one thread-block cluster per 16 heads
 * on the bf16 tensor cores (mma.sync; q and the weights as three bf16 terms
 * each, so only the fp32 accumulation rounds) for a bf16 cache with head_dim
 * 512 or 576 and n_heads % 16 == 0 - 16-CTA clusters where the device fits
 * one per head group, else 8 - and the fp32 chunk kernels otherwise;
 * FP32 = the fp32 chunk kernels always; CLUSTER8 = AUTO with 8-CTA clusters.
 * Process-wide; for comparisons. */
#define DSV4CU_ATTN_AUTO 0
#define DSV4CU_ATTN_FP32 1
#define DSV4CU_ATTN_CLUSTER8 2
int dsv4cu_sparse_attn_set_path(int path);

/* dsv4cu_sparse_attn without a context and without any allocation. No
 * counterpart in the reference (whose dsv4_sparse_attn takes a caller scratch
 * buffer on the host). For callers that must not allocate device memory while
 * they call in (during stream capture, inside an allocator callback, or with
 * all free HBM handed to KV/expert pools). The per-chunk partials live in one
 * 12 MiB array built into the library (per device): shapes whose partials need
 * more ((ceil(topk/32) * h * (d + 2)) * 4 bytes, rounded) return
 * DSV4CU_ERR_UNSUPPORTED; h = 64, d = 576, topk = 2176 fits. All calls on a
 * device share that array and leave their contents in it (nothing needs to
 * start at zero); calls that overlap in time on one device race, so serialise
 * them on one stream. The first call on each device looks up the array's
 * address and may load the library's module there: make it before any stream
 * capture begins. */
int dsv4cu_sparse_attn_noalloc(float *o, const float *q, const void *kv,
                               int kv_bf16, const float *sink, const int *idxs,
                               int h, int d, int topk, float scale, void *stream);

/* Add offset to every idxs[i] >= 0 (dsv4_indexer_offset,
 * src/10_compute/dsv4_indexer.c:92-96). */
int dsv4cu_indexer_offset(int *idxs, int n, int offset, void *stream);

/* RMS norm of nt rows of n floats (dsv4_rmsnorm, src/10_compute/dsv4_ops.c:
 * 26-33): y = w * (x * inv), inv = (float)(1 / sqrt(sum(x^2) / n + eps)) with
 * the sum in double. The result has the reference's bits: the sum runs in
 * parallel with a bound on its distance from the reference's sequential sum,
 * and a row whose inv that bound cannot pin down is replayed in the
 * reference's order. y may alias x. */
int dsv4cu_rmsnorm(float *y, const float *x, const float *w, int n, int nt, float eps, void *stream);

/* Rotary embedding in place (dsv4_rope_apply, src/10_compute/dsv4_rope.c)
 * over v [nt][nh][head_dim]: the last rd dims of each head of token t are
 * rotated by row pos[t] of the device tables cs / sn [n_pos][table_half]
 * (built once on the host with the reference's dsv4_rope_table and copied
 * up), with -sin when inverse. Same float operations as the reference, so the
 * same bits. pos is a device array; a position outside [0, n_pos) leaves that
 * token's heads unchanged and sets status code 41 (dsv4cu_ctx_status). */
int dsv4cu_rope_apply(dsv4cu_ctx *ctx, float *v, int nt, int nh, int head_dim, int rd, const float *cs,
                      const float *sn, const int *pos, int table_half, int n_pos, int inverse, void *stream);

/* mHC pre-mix (dsv4_hc_pre with dsv4_hc_split_sinkhorn,
 * src/10_compute/dsv4_hc.c) for nt tokens: from the residual copies
 * x [nt][hc][hidden] and the block's device weights fn [(2+hc)hc][hc hidden],
 * base [(2+hc)hc], scale [3], writes y [nt][hidden], post [nt][hc],
 * comb [nt][hc][hc] and mixes [nt][(2+hc)hc]. The reference's double dots,
 * sums and float arithmetic in its order; expf is exp in double rounded to
 * float (the reference's glibc expf agrees except within a hair of a rounding
 * midpoint). hc <= 6. */
int dsv4cu_hc_pre(float *y, float *post, float *comb, float *mixes, const float *x, const float *fn,
                  const float *base, const float *scale, int nt, int hc, int hidden, int iters, float norm_eps,
                  float hc_eps, void *stream);

/* One KV compressor step (dsv4_compress_step, src/10_compute/dsv4_compress.c)
 * on device buffers: kv_in / score_in [coff * head_dim] (coff = 2 when ratio
 * is 4, else 1), ape [ratio][coff * head_dim], the layer's ring states
 * kv_state / score_state [coff * ratio][coff * head_dim]. Returns 1 when the
 * window closed and out [head_dim] was written (on the stream), 0 when not,
 * a negative status on bad arguments - the reference's return contract. The
 * reference's double sums in its order; expf as in dsv4cu_hc_pre. */
int dsv4cu_compress_step(float *out, const float *kv_in, const float *score_in, const float *ape, float *kv_state,
                         float *score_state, int pos, int ratio, int head_dim, void *stream);

/* The output head's mHC (hc_head, src/90_cli/dsv4_decode.c:102-125): from
 * x [nt][hc][hidden] and the head's fn [hc][hc hidden], base [hc], scale [1],
 * y [nt][hidden] = sum over j of pre[j] * x[j], pre the head's sigmoid mix.
 * The reference's sequential sums and order; expf as in dsv4cu_hc_pre. Then
 * dsv4cu_rmsnorm and dsv4cu_head complete dsv4_head_from_h. hc <= 6. */
int dsv4cu_hc_head(float *y, const float *x, const float *fn, const float *base, const float *scale, int nt, int hc,
                   int hidden, float norm_eps, float hc_eps, void *stream);

/* mHC residual update (dsv4_hc_post, src/10_compute/dsv4_hc.c) for nt
 * tokens: y [nt][hc][hidden] from the block output x [nt][hidden], the
 * residual copies [nt][hc][hidden], post [nt][hc] and comb [nt][hc][hc], with
 * the reference's double arithmetic in its order - the same bits. y must not
 * alias residual. */
int dsv4cu_hc_post(float *y, const float *x, const float *residual, const float *post, const float *comb,
                   int nt, int hc, int hidden, void *stream);

/* Greedy pick per row of logits [nt][n] into best[nt], with the reference's
 * argmax rule (src/90_cli/dsv4_decode.c:128-133): the first index of the
 * largest value, -0.0 equal to +0.0, NaNs never picked, and 0 when row[0] is
 * NaN. */
int dsv4cu_argmax(int *best, const float *logits, int n, int nt, void *stream);

/* Output head (dsv4_head_from_h, src/90_cli/dsv4_decode.c:138-148, from the
 * normalised hidden state on): logits[nt][head->rows] = dsv4cu_mmq(x, head)
 * - BF16 in the reference, so the reference's bits - then best[nt] as
 * dsv4cu_argmax. */
int dsv4cu_head(dsv4cu_ctx *ctx, float *logits, int *best, const float *x, const dsv4cu_qmat *head, int nt,
                void *stream);

/* --------------------------------------------------- weight packing utility
 * Quantize fp32 [rows][cols] to the reference pack layouts: FP8 e4m3 with one
 * E8M0 scale per 128x128 block, or FP4 e2m1 with one E8M0 scale per 1x32
 * block. Scale = 2^ceil(log2(amax / qmax)) (qmax 448 or 6), values rounded to
 * nearest-even and saturated. */
int dsv4cu_quantize_fp8(uint8_t *w, uint8_t *s, const float *src, int rows,
                        int cols, void *stream);
int dsv4cu_quantize_fp4(uint8_t *w, uint8_t *s, const float *src, int rows,
                        int cols, void *stream);
/* Deterministic N(mean, std) fill from (seed, element index), for synthetic
 * weights and activations. */
int dsv4cu_fill_normal(float *dst, size_t n, uint64_t seed, float mean,
                       float std, void *stream);
/* Round fp32 values to the nearest bf16 value in place (kept as fp32). */
int dsv4cu_round_bf16(float *x, size_t n, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* DSV4CU_H */
