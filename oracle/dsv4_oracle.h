/* dsv4_oracle.h - CPU restatement of the reference's hot-path algorithms.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA library is compared
 * against; it is never linked into, loaded by, or called from the product
 * library. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs may load it.
 *
 * Every function restates one reference function (file:line under the
 * reference tree, Entkenntnis/deepseek-v4-in-c). Where the reference result is
 * bit-defined (decoders, router, indexer score, top-k) the restatement uses the
 * same floating-point operations in the same order, so it is bit-identical on
 * the same host libm. Where the reference contract is an L2 bound (the packed
 * matmuls, src/10_compute/dsv4_matmul.h:9-17) the restatement is the scalar
 * double-precision reference of tests/unit/test_matmul.c:54-176.
 *
 * Pinning: tests/test_oracle_pins.py checks every function here against the
 * known-answer fixtures of the reference's own unit tests and, when the
 * reference library oracle/_ref/libdsv4ref.so is present, against the
 * reference's own kernels on seeded random inputs.
 */
#ifndef DSV4_ORACLE_H
#define DSV4_ORACLE_H

#include <stdint.h>

/* Same member order and types as the reference DSV4QMat
 * (src/00_base/dsv4_weights.h:34-40). */
typedef struct {
    const void *w;
    const void *s;
    int         wdt;        /* 0 F32, 1 BF16, 2 FP8, 3 FP4 */
    int         rows, cols;
    int         blk_r, blk_c;
} OrcQMat;

float orc_e8m0(uint8_t b);
float orc_e4m3(uint8_t b);
float orc_e2m1(uint8_t nibble);
float orc_fp4_at(const uint8_t *row, int64_t i);

/* y[t*rows+o] = sum_c x[t*cols+c] * W[o,c]; returns -1 on an unknown format. */
int  orc_mmq_n(float *y, const float *x, const OrcQMat *m, int nt);

void orc_route(int *idx, float *wts, float *scores, float *orig,
               const float *bias, const int64_t *tid2eid, int token_id,
               int n_experts, int topk, float route_scale);
void orc_rope_apply(float *v, int head_dim, int rd, const float *cs, const float *sn, int pos, int table_half,
                    int inverse);
void orc_hc_pre(float *y, float *post, float *comb, float *mixes, const float *x, const float *fn,
                const float *base, const float *scale, int hc, int hidden, int iters, float norm_eps, float hc_eps);
int orc_compress_step(float *out, const float *kv_in, const float *score_in, const float *ape, float *kv_state,
                      float *score_state, int pos, int ratio, int head_dim);
void orc_hc_head(float *y, const float *x, const float *fn, const float *base, const float *scale, int hc,
                 int hidden, float norm_eps, float hc_eps);
void orc_hc_post(float *y, const float *x, const float *residual, const float *post, const float *comb, int hc,
                 int hidden);
void orc_rmsnorm(float *y, const float *x, const float *w, int n, float eps);
void orc_swiglu(float *y, const float *gate, const float *up, int n,
                float limit);
/* w[0]=w1, w[1]=w3, w[2]=w2. */
void orc_expert_forward(float *out, const float *x, const OrcQMat *w,
                        int inter, float limit);
/* One token through router + routed experts + shared expert, combined in k
 * order. experts[e*3 + {0,1,2}] = {w1, w3, w2} of routed expert e. */
void orc_moe_decode(float *out, int *idx_out, float *wts_out, const float *x,
                    const float *logits, const float *bias,
                    const int64_t *tid2eid, int token_id,
                    const OrcQMat *experts, const OrcQMat *shared,
                    int n_experts, int topk, float route_scale, int hidden,
                    int inter, float limit);

double orc_dot_f32d(const float *a, const float *b, int n);
void orc_indexer_score(float *out, const float *q, const float *kv,
                       const float *weights, int n_heads, int head_dim,
                       int n_pos);
int  orc_topk(int *idxs, const float *scores, int n, int k);
void orc_indexer_offset(int *idxs, int n, int offset);
int  orc_window_idxs(int *idxs, int pos, int win);
void orc_sparse_attn(float *o, const float *q, const float *kv,
                     const float *sink, const int *idxs, int h, int d,
                     int topk, float scale);

/* Counting sort of (token, k) pairs by expert; tokens ascending inside a
 * bucket. off has n_experts+1 entries. Returns the number of distinct experts. */
int  orc_expert_buckets(int *count, int *off, int *tok, int *ks,
                        const int *topk_idx, int n, int topk, int n_experts);

#endif /* DSV4_ORACLE_H */
