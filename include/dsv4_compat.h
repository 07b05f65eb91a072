/* dsv4_compat.h - the reference engine's operator entry points, implemented
 * by libdsv4cu.so on a B200.
 *
 * Every prototype below is the reference's own, so the reference C host code
 * (src/70_decode, src/80_prefill, src/90_cli, tests/unit) links against this
 * library in place of its CPU kernels without a source change. Pointers are
 * HOST pointers, exactly as in the reference; the library moves data to and
 * from the GPU itself:
 *
 *   - Weights (DSV4QMat.w / .s) are uploaded once per host buffer and kept in
 *     HBM, keyed by host address, byte size and a sampled content fingerprint
 *     (both ends and one word per 4 KiB page), so a cache slot that is
 *     refilled with another expert is re-uploaded. The check is sampled: a
 *     rewrite confined to unsampled bytes is NOT seen unless the caller calls
 *     dsv4cu_host_forget() (one entry) / dsv4cu_host_forget_all(), or turns on
 *     exact checking with dsv4cu_host_verify(1) (every byte hashed per call).
 *   - Activations and results are copied per call.
 *
 * Error behaviour mirrors the reference: an unknown weight format prints the
 * reference's message and aborts (src/10_compute/dsv4_matmul.c:56-60); a
 * device failure in a void entry point prints the CUDA error and aborts, since
 * the reference contract has no error return there. The prefill seam keeps its
 * 0 / -1 return contract (src/80_prefill/dsv4_prefill_vk.h:31-49).
 *
 * When the reference's own headers are included first, their types are used;
 * otherwise layout-identical definitions are provided here.
 */
#ifndef DSV4_COMPAT_H
#define DSV4_COMPAT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef DSV4_WEIGHTS_H
/* src/00_base/dsv4_weights.h:34-40 */
typedef struct {
    const void *w;
    const void *s;
    int         wdt;
    int         rows, cols;
    int         blk_r, blk_c;
} DSV4QMat;
/* src/00_base/dsv4_weights.h:101-104 */
typedef struct {
    DSV4QMat w1, w3;
    DSV4QMat w2;
} DSV4ExpertW;
#endif

#ifndef DSV4_H
/* Opaque here: the CUDA seam reads nothing from the engine config. */
typedef struct dsv4cu_cfg_opaque DSV4Cfg;
enum { DSV4_WF32 = 0, DSV4_WBF16 = 1, DSV4_WFP8 = 2, DSV4_WFP4 = 3 };
#endif

struct DSV4Trunk;
struct DSV4Cache;
typedef struct DSV4PrefillVk DSV4PrefillVk;
/* src/80_prefill/dsv4_prefill_vk.h:29 */
typedef int (*DSV4PrefillVkFillFn)(void *ctx);

/* ---- src/10_compute/dsv4_matmul.h:40-52 ---- */
void dsv4_mmq_n(float *y, const float *x, const DSV4QMat *m, int nt);
void dsv4_mmq(float *y, const float *x, const DSV4QMat *m);
void bf16_n(float *y, const float *x, const uint16_t *W, int in, int out, int nt);
void fp8_n(float *y, const float *x, const uint8_t *W, const uint8_t *S,
           int in, int out, int blk_r, int blk_c, int nt);
void fp4_n(float *y, const float *x, const uint8_t *W, const uint8_t *S,
           int in, int out, int blk_r, int blk_c, int nt);

/* ---- src/10_compute/dsv4_kernels.h:20-57 (the hot-path subset) ---- */
/* src/10_compute/dsv4_kernels.h:20: with dsv4_route, dsv4_swiglu and
 * dsv4_expert_forward, every symbol of src/10_compute/dsv4_ops.c. */
void dsv4_rmsnorm(float *y, const float *x, const float *w, int n, float eps);
void dsv4_swiglu(float *y, const float *gate, const float *up, int n, float limit);
void dsv4_route(int *idx, float *wts, float *scores, float *orig,
                const float *bias, const int64_t *tid2eid, int token_id,
                int n_experts, int topk, float route_scale);
void dsv4_expert_forward(float *out, const float *x, const DSV4ExpertW *e,
                         float *gate, float *up, float *mid, int inter, float limit);
void dsv4_sparse_attn(float *o, const float *q, const float *kv,
                      const float *sink, const int *idxs, int h, int d,
                      int topk, float scale, float *scratch);
int  dsv4_window_idxs(int *idxs, int pos, int win);
void dsv4_indexer_score(float *out, const float *q, const float *kv,
                        const float *weights, int n_heads, int head_dim, int n_pos);
int  dsv4_topk(int *idxs, const float *scores, int n, int k);
void dsv4_indexer_offset(int *idxs, int n, int offset);

/* ---- src/80_prefill/dsv4_prefill_vk.h:31-49: the prefill GPU seam ---- */
int  dsv4_prefill_vk_init(DSV4PrefillVk **out, const DSV4Cfg *cfg,
                          struct DSV4Trunk *tr, struct DSV4Cache *cache);
void dsv4_prefill_vk_free(DSV4PrefillVk *v);
int  dsv4_prefill_vk_gemm(DSV4PrefillVk *v, float *y, const float *x,
                          const DSV4QMat *m, int n);
int  dsv4_prefill_vk_expert_fused(DSV4PrefillVk *v, float *y, const float *x,
                                  const DSV4QMat *w1, const DSV4QMat *w3,
                                  const DSV4QMat *w2, int n, int inter,
                                  float limit, DSV4PrefillVkFillFn fill,
                                  void *fill_ctx);

/* ---- library additions for the host-pointer layer (no reference counterpart) */
/* Drop the HBM copy kept for a host weight buffer / for all of them. */
void dsv4cu_host_forget(const void *host_ptr);
void dsv4cu_host_forget_all(void);
/* 0 (default): sampled content check of mirrored weights; 1: every byte of a
 * mirrored buffer hashed on every call (exact; one pass over the weights). */
void dsv4cu_host_verify(int full);
/* Number of weight buffers currently mirrored in HBM, and their bytes. */
size_t dsv4cu_host_registry_count(void);
size_t dsv4cu_host_registry_bytes(void);

#ifdef __cplusplus
}
#endif

#endif /* DSV4_COMPAT_H */
