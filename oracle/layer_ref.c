/* layer_ref.c - test infrastructure only: a harness around the REFERENCE's own
 * attention block (src/70_decode/dsv4_layer_attn.c dsv4_layer_attention, the
 * attention half of dsv4_layer_forward, src/70_decode/dsv4_layer.c:18-36)
 * running on the reference's CPU kernels, so the GPU tests can check the
 * library's device layer step against it. It builds one layer with seeded
 * random weights in the reference's own structs (src/00_base/dsv4_weights.h)
 * and hands their bytes out so the tests upload the very same weights.
 * Compiled by oracle/Makefile into _ref/libdsv4layer.so with the reference's
 * sources read where they lie; nothing here is called by the library. */
#include <execinfo.h>
#include <math.h>
#include <signal.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "dsv4.h"
#include "dsv4_kernels.h"
#include "dsv4_layer.h"
#include "dsv4_matmul.h"
#include "dsv4_weights.h"

enum { LR_WQA, LR_WQB, LR_WKV, LR_WOA, LR_WOB, LR_CWKV, LR_CWGATE, LR_IWQB, LR_IWPROJ, LR_NMAT };
enum { LR_QNORM, LR_KVNORM, LR_SINK, LR_CAPE, LR_CNORM, LR_ATTN_NORM, LR_HC_FN, LR_HC_BASE, LR_HC_SCALE,
       LR_CS, LR_SN, LR_NVEC };

typedef struct {
    DSV4Cfg c;
    DSV4LayerW w;
    DSV4Scratch s;
    DSV4LayerState st;
    int ratios[1];
    int max_pos;
    void *mat_w[LR_NMAT], *mat_s[LR_NMAT];
    DSV4QMat *mat[LR_NMAT];
    float *vec[LR_NVEC];
    int vec_n[LR_NVEC];
    void *arena;                   /* scratch floats */
    int *idxs;
    /* FFN half: n_experts routed FP4 experts + one FP8 shared expert, BF16 gate. */
    int n_experts, topk, inter;
    float route_scale, limit;
    DSV4ExpertW *experts;          /* [n_experts + 1], the shared expert last */
    void **ebuf;                   /* their packed bytes, to free */
    int n_ebuf;
    DSV4QMat gate;
    float *bias, *ffn_norm, *hcf_fn, *hcf_base, *hcf_scale;
    float *macc;                   /* [topk + 1][hidden] expert outputs */
} LR;

static uint64_t lr_next(uint64_t *x)
{
    *x ^= *x << 13;
    *x ^= *x >> 7;
    *x ^= *x << 17;
    return *x;
}

static float lr_normal(uint64_t *x)
{
    const double u1 = ((lr_next(x) >> 11) + 1.0) / 9007199254740993.0;
    const double u2 = (lr_next(x) >> 11) / 9007199254740992.0;
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

static float lr_bf16(float v)
{
    uint32_t u;
    memcpy(&u, &v, 4);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    memcpy(&v, &u, 4);
    return v;
}

/* FP8 e4m3 codes without the NaN codes, 128x128 E8M0 scales 2^-15 .. 2^-10. */
static void lr_fp8(LR *L, int k, DSV4QMat *m, int rows, int cols, uint64_t *rng)
{
    const size_t n = (size_t)rows * cols;
    const int sr = (rows + 127) / 128, sc = (cols + 127) / 128;
    unsigned char *w = (unsigned char *)malloc(n), *s = (unsigned char *)malloc((size_t)sr * sc);
    for (size_t i = 0; i < n; i++) {
        unsigned char b = (unsigned char)lr_next(rng);
        if ((b & 0x7F) == 0x7F) b ^= 1;
        w[i] = b;
    }
    for (int i = 0; i < sr * sc; i++) s[i] = (unsigned char)(112 + lr_next(rng) % 6);
    m->w = w;
    m->s = s;
    m->wdt = DSV4_WFP8;
    m->rows = rows;
    m->cols = cols;
    m->blk_r = 128;
    m->blk_c = 128;
    L->mat_w[k] = w;
    L->mat_s[k] = s;
    L->mat[k] = m;
}

/* BF16 N(0, 0.05). */
static void lr_bf16m(LR *L, int k, DSV4QMat *m, int rows, int cols, uint64_t *rng)
{
    const size_t n = (size_t)rows * cols;
    uint16_t *w = (uint16_t *)malloc(n * 2);
    for (size_t i = 0; i < n; i++) {
        const float v = lr_bf16(0.05f * lr_normal(rng));
        uint32_t u;
        memcpy(&u, &v, 4);
        w[i] = (uint16_t)(u >> 16);
    }
    m->w = w;
    m->s = NULL;
    m->wdt = DSV4_WBF16;
    m->rows = rows;
    m->cols = cols;
    m->blk_r = 0;
    m->blk_c = 0;
    L->mat_w[k] = w;
    L->mat_s[k] = NULL;
    L->mat[k] = m;
}

static float *lr_vecf(LR *L, int k, int n, uint64_t *rng, float mean, float sd, int bf16)
{
    float *v = (float *)malloc((size_t)n * sizeof(float));
    for (int i = 0; i < n; i++) {
        const float x = mean + sd * lr_normal(rng);
        v[i] = bf16 ? lr_bf16(x) : x;
    }
    L->vec[k] = v;
    L->vec_n[k] = n;
    return v;
}

/* dims: hidden, n_heads, head_dim, q_lora, o_lora, o_groups, qk_rope, sliding_window, index_n_heads,
 * index_head_dim, index_topk, hc_mult. ratio: 0, 4 (compressor + indexer) or another compressor ratio. */
/* A crash inside the harness or the reference code prints the native frames
 * before the process ends (the tests then show where). */
static void lr_on_segv(int sig)
{
    void *fr[64];
    const int n = backtrace(fr, 64);
    static const char msg[] = "layer_ref: fatal signal; native frames:\n";
    if (write(2, msg, sizeof msg - 1) < 0) {}
    backtrace_symbols_fd(fr, n, 2);
    signal(sig, SIG_DFL);
    raise(sig);
}

void lr_trap_crashes(void)
{
    signal(SIGSEGV, lr_on_segv);
    signal(SIGBUS, lr_on_segv);
    signal(SIGILL, lr_on_segv);
}

LR *lr_create(const int *dims, int ratio, int max_pos, unsigned long long seed)
{
    LR *L = (LR *)calloc(1, sizeof(LR));
    uint64_t rng = seed * 0x9E3779B97F4A7C15ull + 1;
    DSV4Cfg *c = &L->c;
    c->hidden = dims[0];
    c->n_layers = 1;
    c->rms_eps = 1e-6f;
    c->max_pos = max_pos;
    c->n_heads = dims[1];
    c->n_kv_heads = 1;
    c->head_dim = dims[2];
    c->q_lora = dims[3];
    c->o_lora = dims[4];
    c->o_groups = dims[5];
    c->qk_rope = dims[6];
    c->sliding_window = dims[7];
    c->index_n_heads = dims[8];
    c->index_head_dim = dims[9];
    c->index_topk = dims[10];
    c->hc_mult = dims[11];
    c->hc_sinkhorn_iters = 20;
    c->hc_eps = 1e-6f;
    c->n_compress = 1;
    L->ratios[0] = ratio;
    c->compress_ratios = L->ratios;
    c->compress_rope_theta = 160000.0f;
    L->max_pos = max_pos;
    const int d = c->hidden, H = c->n_heads, hd = c->head_dim, hc = c->hc_mult;

    DSV4LayerW *w = &L->w;
    w->layer = 0;
    w->compress_ratio = ratio;
    w->has_comp = ratio != 0;
    w->has_idx = ratio == 4;
    DSV4AttnW *a = &w->attn;
    lr_fp8(L, LR_WQA, &a->wq_a, c->q_lora, d, &rng);
    lr_fp8(L, LR_WQB, &a->wq_b, H * hd, c->q_lora, &rng);
    lr_fp8(L, LR_WKV, &a->wkv, hd, d, &rng);
    lr_fp8(L, LR_WOA, &a->wo_a, c->o_lora * c->o_groups, H * hd / c->o_groups, &rng);
    lr_fp8(L, LR_WOB, &a->wo_b, d, c->o_lora * c->o_groups, &rng);
    a->q_norm = lr_vecf(L, LR_QNORM, c->q_lora, &rng, 1.0f, 0.1f, 1);
    a->kv_norm = lr_vecf(L, LR_KVNORM, hd, &rng, 1.0f, 0.1f, 1);
    a->sink = lr_vecf(L, LR_SINK, H, &rng, 0.0f, 1.0f, 0);
    w->attn_norm = lr_vecf(L, LR_ATTN_NORM, d, &rng, 1.0f, 0.1f, 1);
    const int mix = (2 + hc) * hc;
    w->hc_attn.fn = lr_vecf(L, LR_HC_FN, mix * hc * d, &rng, 0.0f, 0.02f, 0);
    w->hc_attn.base = lr_vecf(L, LR_HC_BASE, mix, &rng, 0.0f, 0.1f, 0);
    w->hc_attn.scale = lr_vecf(L, LR_HC_SCALE, 3, &rng, 0.5f, 0.1f, 0);
    if (ratio) {
        const int coff = ratio == 4 ? 2 : 1;
        lr_bf16m(L, LR_CWKV, &a->comp.wkv, coff * hd, d, &rng);
        lr_bf16m(L, LR_CWGATE, &a->comp.wgate, coff * hd, d, &rng);
        a->comp.ape = lr_vecf(L, LR_CAPE, ratio * coff * hd, &rng, 0.0f, 0.1f, 0);
        a->comp.norm = lr_vecf(L, LR_CNORM, hd, &rng, 1.0f, 0.1f, 1);
    }
    if (ratio == 4) {
        lr_fp8(L, LR_IWQB, &a->idx.wq_b, c->index_n_heads * c->index_head_dim, c->q_lora, &rng);
        lr_bf16m(L, LR_IWPROJ, &a->idx.weights_proj, c->index_n_heads, d, &rng);
    }
    /* RoPE tables: the compressed layers' table (compress theta, YaRN) or the plain one. */
    const int half = c->qk_rope / 2;
    float *cs = (float *)malloc((size_t)max_pos * half * sizeof(float));
    float *sn = (float *)malloc((size_t)max_pos * half * sizeof(float));
    if (ratio)
        dsv4_rope_table(cs, sn, c->qk_rope, max_pos, 65536, 160000.0, 16.0, 32.0, 1.0);
    else
        dsv4_rope_table(cs, sn, c->qk_rope, max_pos, 0, 10000.0, 1.0, 32.0, 1.0);
    L->vec[LR_CS] = cs;
    L->vec[LR_SN] = sn;
    L->vec_n[LR_CS] = L->vec_n[LR_SN] = max_pos * half;

    if (dsv4_state_init(&L->st, c, 0, max_pos)) return NULL;
    /* Scratch: the buffers dsv4_layer_attention and the block half touch,
     * sized like dsv4_scratch_init (src/70_decode/dsv4_layer.c:120-180). */
    DSV4Scratch *s = &L->s;
    const size_t nidx = (size_t)c->sliding_window + (size_t)c->index_topk;
    const size_t qr_n = d > c->q_lora ? (size_t)d : (size_t)c->q_lora;
    const size_t nf = (size_t)d + (size_t)hc * d + hc + (size_t)hc * hc + (size_t)(2 + hc) * hc + qr_n +
                      (size_t)H * hd * 2 + hd + (size_t)c->o_groups * c->o_lora + (size_t)H * nidx + 4u * hd +
                      (size_t)c->index_n_heads * c->index_head_dim + c->index_n_heads + (size_t)max_pos + 1;
    float *p = (float *)calloc(nf, sizeof(float));
    L->arena = p;
    s->x1 = p;          p += d;
    s->resid = p;       p += (size_t)hc * d;
    s->post = p;        p += hc;
    s->comb = p;        p += (size_t)hc * hc;
    s->mixes = p;       p += (size_t)(2 + hc) * hc;
    s->qr = p;          p += qr_n;
    s->q = p;           p += (size_t)H * hd;
    s->kv = p;          p += hd;
    s->o = p;           p += (size_t)H * hd;
    s->ogrp = p;        p += (size_t)c->o_groups * c->o_lora;
    s->attn_scratch = p; p += (size_t)H * nidx;
    s->comp_kv_in = p;  p += 2u * hd;
    s->comp_sc_in = p;  p += 2u * hd;
    s->idx_q = p;       p += (size_t)c->index_n_heads * c->index_head_dim;
    s->idx_w = p;       p += c->index_n_heads;
    s->idx_scores = p;  p += (size_t)max_pos + 1;
    s->idx_cap = max_pos + 1;
    L->idxs = (int *)calloc(nidx, sizeof(int));
    s->idxs = L->idxs;
    return L;
}

void lr_attn_block(LR *L, float *h, int pos);

static void lr_keep(LR *L, void *p)
{
    L->ebuf = (void **)realloc(L->ebuf, (size_t)(L->n_ebuf + 1) * sizeof(void *));
    L->ebuf[L->n_ebuf++] = p;
}

/* FP4 e2m1 codes (any byte), 1x32 E8M0 scales 2^-8 .. 2^-5. */
static void lr_fp4(LR *L, DSV4QMat *m, int rows, int cols, uint64_t *rng)
{
    const size_t n = (size_t)rows * cols / 2, ns = (size_t)rows * cols / 32;
    unsigned char *w = (unsigned char *)malloc(n), *s = (unsigned char *)malloc(ns);
    for (size_t i = 0; i < n; i++) w[i] = (unsigned char)lr_next(rng);
    for (size_t i = 0; i < ns; i++) s[i] = (unsigned char)(119 + lr_next(rng) % 4);
    *m = (DSV4QMat){w, s, DSV4_WFP4, rows, cols, 1, 32};
    lr_keep(L, w);
    lr_keep(L, s);
}

static void lr_fp8k(LR *L, DSV4QMat *m, int rows, int cols, uint64_t *rng)
{
    const size_t n = (size_t)rows * cols;
    const int sr = (rows + 127) / 128, sc = (cols + 127) / 128;
    unsigned char *w = (unsigned char *)malloc(n), *s = (unsigned char *)malloc((size_t)sr * sc);
    for (size_t i = 0; i < n; i++) {
        unsigned char b = (unsigned char)lr_next(rng);
        if ((b & 0x7F) == 0x7F) b ^= 1;
        w[i] = b;
    }
    for (int i = 0; i < sr * sc; i++) s[i] = (unsigned char)(112 + lr_next(rng) % 6);
    *m = (DSV4QMat){w, s, DSV4_WFP8, rows, cols, 128, 128};
    lr_keep(L, w);
    lr_keep(L, s);
}

/* The FFN half's weights: a BF16 gate, optional selection bias, n_experts FP4
 * experts of inter, the FP8 shared expert, ffn_norm and the FFN's mHC set. */
int lr_ffn_create(LR *L, int n_experts, int topk, int inter, float route_scale, float limit, int with_bias,
                  unsigned long long seed)
{
    uint64_t rng = seed * 0xD1B54A32D192ED03ull + 7;
    const int d = L->c.hidden, hc = L->c.hc_mult, mix = (2 + hc) * hc;
    L->n_experts = n_experts;
    L->topk = topk;
    L->inter = inter;
    L->route_scale = route_scale;
    L->limit = limit;
    L->experts = (DSV4ExpertW *)calloc((size_t)n_experts + 1, sizeof(DSV4ExpertW));
    for (int e = 0; e < n_experts; e++) {
        lr_fp4(L, &L->experts[e].w1, inter, d, &rng);
        lr_fp4(L, &L->experts[e].w3, inter, d, &rng);
        lr_fp4(L, &L->experts[e].w2, d, inter, &rng);
    }
    lr_fp8k(L, &L->experts[n_experts].w1, inter, d, &rng);
    lr_fp8k(L, &L->experts[n_experts].w3, inter, d, &rng);
    lr_fp8k(L, &L->experts[n_experts].w2, d, inter, &rng);
    uint16_t *g = (uint16_t *)malloc((size_t)n_experts * d * 2);
    for (size_t i = 0; i < (size_t)n_experts * d; i++) {
        const float v = lr_bf16(0.05f * lr_normal(&rng));
        uint32_t u;
        memcpy(&u, &v, 4);
        g[i] = (uint16_t)(u >> 16);
    }
    lr_keep(L, g);
    L->gate = (DSV4QMat){g, NULL, DSV4_WBF16, n_experts, d, 0, 0};
    L->bias = NULL;
    if (with_bias) {
        L->bias = (float *)malloc((size_t)n_experts * sizeof(float));
        for (int e = 0; e < n_experts; e++) L->bias[e] = 0.25f * lr_normal(&rng);
        lr_keep(L, L->bias);
    }
    L->ffn_norm = (float *)malloc((size_t)d * sizeof(float));
    for (int i = 0; i < d; i++) L->ffn_norm[i] = lr_bf16(1.0f + 0.1f * lr_normal(&rng));
    lr_keep(L, L->ffn_norm);
    L->hcf_fn = (float *)malloc((size_t)mix * hc * d * sizeof(float));
    for (size_t i = 0; i < (size_t)mix * hc * d; i++) L->hcf_fn[i] = 0.02f * lr_normal(&rng);
    lr_keep(L, L->hcf_fn);
    L->hcf_base = (float *)malloc((size_t)mix * sizeof(float));
    for (int i = 0; i < mix; i++) L->hcf_base[i] = 0.1f * lr_normal(&rng);
    lr_keep(L, L->hcf_base);
    L->hcf_scale = (float *)malloc(3 * sizeof(float));
    for (int i = 0; i < 3; i++) L->hcf_scale[i] = 0.5f + 0.1f * lr_normal(&rng);
    lr_keep(L, L->hcf_scale);
    L->macc = (float *)calloc((size_t)(topk + 1) * d, sizeof(float));
    lr_keep(L, L->macc);
    return 0;
}

/* Matrix m (0 w1, 1 w3, 2 w2) of expert e (e == n_experts: the shared one); e = -1: the gate. */
int lr_expert_qmat(LR *L, int e, int m, DSV4QMat *out)
{
    if (e == -1) {
        *out = L->gate;
        return 1;
    }
    if (!L->experts || e < 0 || e > L->n_experts || m < 0 || m > 2) return 0;
    const DSV4ExpertW *x = &L->experts[e];
    *out = m == 0 ? x->w1 : (m == 1 ? x->w3 : x->w2);
    return 1;
}

const float *lr_ffn_vec(LR *L, int which, int *n)
{
    const int d = L->c.hidden, hc = L->c.hc_mult, mix = (2 + hc) * hc;
    switch (which) {
    case 0: *n = L->bias ? L->n_experts : 0; return L->bias;
    case 1: *n = d; return L->ffn_norm;
    case 2: *n = mix * hc * d; return L->hcf_fn;
    case 3: *n = mix; return L->hcf_base;
    case 4: *n = 3; return L->hcf_scale;
    }
    *n = 0;
    return NULL;
}

/* dsv4_layer_moe (src/70_decode/dsv4_layer.c:48-117) with the routed experts
 * in memory: the gate GEMV, dsv4_route, dsv4_expert_forward per k and for the
 * shared expert (the reference's own functions), then the k-order weighted
 * sum and the shared expert added unweighted, as the reference writes them. */
static void lr_moe(LR *L, float *out, const float *x)
{
    const int d = L->c.hidden, topk = L->topk;
    float *scores = (float *)malloc((size_t)L->n_experts * 2 * sizeof(float));
    float *mid = (float *)malloc((size_t)L->inter * 3 * sizeof(float));
    int idx[DSV4_MAX_TOPK];
    float wts[DSV4_MAX_TOPK];
    dsv4_mmq(scores, x, &L->gate);
    dsv4_route(idx, wts, scores, scores + L->n_experts, L->bias, NULL, 0, L->n_experts, topk, L->route_scale);
    for (int i = 0; i < d; i++) out[i] = 0.0f;
    for (int k = 0; k < topk; k++)
        dsv4_expert_forward(L->macc + (size_t)k * d, x, &L->experts[idx[k]], mid, mid + L->inter,
                            mid + 2 * L->inter, L->inter, L->limit);
    dsv4_expert_forward(L->macc + (size_t)topk * d, x, &L->experts[L->n_experts], mid, mid + L->inter,
                        mid + 2 * L->inter, L->inter, L->limit);
    for (int k = 0; k < topk; k++) {
        const float *acc = L->macc + (size_t)k * d;
        const float wk = wts[k];
        for (int i = 0; i < d; i++) out[i] += wk * acc[i];
    }
    for (int i = 0; i < d; i++) out[i] += L->macc[(size_t)topk * d + i];
    free(scores);
    free(mid);
}

/* The FFN half of dsv4_layer_forward (src/70_decode/dsv4_layer.c:38-46) on h in place. */
void lr_ffn_block(LR *L, float *h)
{
    const DSV4Cfg *c = &L->c;
    const int hc = c->hc_mult, d = c->hidden;
    DSV4Scratch *s = &L->s;
    DSV4HcW hw = {L->hcf_fn, L->hcf_base, L->hcf_scale};
    memcpy(s->resid, h, (size_t)hc * d * sizeof(float));
    dsv4_hc_pre(s->x1, s->post, s->comb, s->mixes, h, &hw, hc, d, c->hc_sinkhorn_iters, c->rms_eps, c->hc_eps);
    dsv4_rmsnorm(s->x1, s->x1, L->ffn_norm, d, c->rms_eps);
    float *out = (float *)malloc((size_t)d * sizeof(float));
    lr_moe(L, out, s->x1);
    dsv4_hc_post(h, out, s->resid, s->post, s->comb, hc, d);
    free(out);
}

/* One whole decoder layer (dsv4_layer_forward) on h in place. */
void lr_layer(LR *L, float *h, int pos)
{
    lr_attn_block(L, h, pos);
    lr_ffn_block(L, h);
}

void lr_free(LR *L)
{
    if (!L) return;
    for (int i = 0; i < L->n_ebuf; i++) free(L->ebuf[i]);
    free(L->ebuf);
    free(L->experts);
    for (int k = 0; k < LR_NMAT; k++) {
        free(L->mat_w[k]);
        free(L->mat_s[k]);
    }
    for (int k = 0; k < LR_NVEC; k++) free(L->vec[k]);
    dsv4_state_free(&L->st);
    free(L->arena);
    free(L->idxs);
    free(L);
}

/* The matrix `which` (its packed bytes stay owned by the harness); 0 if absent. */
int lr_qmat(LR *L, int which, DSV4QMat *out)
{
    if (which < 0 || which >= LR_NMAT || !L->mat[which]) return 0;
    *out = *L->mat[which];
    return 1;
}

const float *lr_vec(LR *L, int which, int *n)
{
    if (which < 0 || which >= LR_NVEC) return NULL;
    *n = L->vec_n[which];
    return L->vec[which];
}

/* dsv4_layer_attention for one token, with the window indices the layer
 * forward computes first (src/70_decode/dsv4_layer.c:32-33). */
void lr_attention(LR *L, float *out, const float *x, int pos)
{
    const int n_idx = dsv4_window_idxs(L->s.idxs, pos, L->c.sliding_window);
    dsv4_layer_attention(out, x, &L->w, &L->c, &L->s, &L->st, L->vec[LR_CS], L->vec[LR_SN], pos, n_idx);
}

/* The attention half of dsv4_layer_forward (src/70_decode/dsv4_layer.c:24-36)
 * on h [hc_mult][hidden] in place. */
void lr_attn_block(LR *L, float *h, int pos)
{
    const DSV4Cfg *c = &L->c;
    const int hc = c->hc_mult, d = c->hidden;
    DSV4Scratch *s = &L->s;
    memcpy(s->resid, h, (size_t)hc * d * sizeof(float));
    dsv4_hc_pre(s->x1, s->post, s->comb, s->mixes, h, &L->w.hc_attn, hc, d, c->hc_sinkhorn_iters, c->rms_eps,
                c->hc_eps);
    dsv4_rmsnorm(s->x1, s->x1, L->w.attn_norm, d, c->rms_eps);
    float *out = (float *)malloc((size_t)d * sizeof(float));
    lr_attention(L, out, s->x1, pos);
    dsv4_hc_post(h, out, s->resid, s->post, s->comb, hc, d);
    free(out);
}

int lr_n_compressed(LR *L) { return L->st.n_compressed; }

const float *lr_kv_cache(LR *L) { return L->st.kv_cache; }
