/* dsv4_oracle.c - CPU restatement of the reference hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see dsv4_oracle.h). Written from the reference's
 * documented behaviour; each function names the reference lines it restates.
 * Build: oracle/Makefile (-O3 -ffp-contract=off, like the reference).
 */
#include "dsv4_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------- decoders ---
 * src/10_compute/dsv4_quant.h:72-86 (E8M0), :99-128 (E4M3-FN), :139-158
 * (E2M1 table and nibble order: the LOW nibble is the even element). */
float orc_e8m0(uint8_t b)
{
    union { uint32_t u; float f; } v;
    if (b == 0xFF) v.u = 0x7FC00000u;        /* NaN, not +inf             */
    else if (b == 0) v.u = 0x00400000u;      /* 2^-127 as an f32 subnormal */
    else v.u = (uint32_t)b << 23;
    return v.f;
}

float orc_e4m3(uint8_t b)
{
    const int sign = (b >> 7) & 1, e = (b >> 3) & 15, m = b & 7;
    float v;
    if (e == 15 && m == 7) v = NAN;                        /* 0x7F / 0xFF  */
    else if (e == 0) v = ldexpf((float)m, -9);             /* subnormals   */
    else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return sign ? -v : v;
}

float orc_e2m1(uint8_t nib)
{
    static const float mag[8] = { 0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f };
    const float v = mag[nib & 7];
    return (nib & 8) ? -v : v;
}

float orc_fp4_at(const uint8_t *row, int64_t i)
{
    const uint8_t byte = row[i >> 1];
    return orc_e2m1((i & 1) ? (uint8_t)(byte >> 4) : (uint8_t)(byte & 15));
}

static double bf16_to_d(uint16_t h)
{
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)h << 16;
    return (double)v.f;
}

/* BF16 row dot in the reference's order: bf16_n (src/10_compute/
 * dsv4_matmul.c:88-113) runs BLOCK_DOT_V (src/10_compute/dsv4_dec_common.h:
 * 45-61), 16 double fma chains a[c] over columns c, c+16, ... below
 * 16*floor(n/16), folded b[j] = (a[j]+a[j+4]) + (a[j+8]+a[j+12]),
 * acc = (b0+b1) + (b2+b3), then the remaining columns fma'd into acc in
 * order. Its scalar twin is BLOCK_DOT_S (tests/unit/test_matmul.c:54-67). */
static double bf16_row_dot(const uint16_t *row, const float *x, int n)
{
    double a[16] = {0};
    int i = 0;
    for (; i + 15 < n; i += 16)
        for (int l = 0; l < 16; l++) a[l] = fma(bf16_to_d(row[i + l]), (double)x[i + l], a[l]);
    double b[4];
    for (int j = 0; j < 4; j++) b[j] = (a[j] + a[j + 4]) + (a[j + 8] + a[j + 12]);
    double acc = (b[0] + b[1]) + (b[2] + b[3]);
    for (; i < n; i++) acc = fma(bf16_to_d(row[i]), (double)x[i], acc);
    return acc;
}

/* ------------------------------------------------------- packed matmul ----
 * Contract: src/10_compute/dsv4_matmul.h:33-43 (y[t*rows+o]). BF16 rows use
 * bf16_row_dot above. FP8/FP4 follow the scalar double reference of
 * tests/unit/test_matmul.c:54-176: every weight decoded exactly, the block dot
 * product in double, one multiply by the block's E8M0 scale per block (as
 * kernel.py does), totals in double, one rounding to float per output. Scale grid indexing follows fp8_n/fp4_n:
 * srow = S + (o / blk_r) * ceil(cols / blk_c)  (dsv4_matmul_fp8.c:158-160,
 * dsv4_matmul_fp4.c:56). FP4 rows are cols/2 bytes (dsv4_weights.h:25-27). */
int orc_mmq_n(float *y, const float *x, const OrcQMat *m, int nt)
{
    const int in = m->cols, out = m->rows;
    if (m->wdt != 1 && m->wdt != 2 && m->wdt != 3) return -1;
    for (int t = 0; t < nt; t++) {
        const float *xt = x + (size_t)t * in;
        float *yt = y + (size_t)t * out;
        for (int o = 0; o < out; o++) {
            if (m->wdt == 1) {
                yt[o] = (float)bf16_row_dot((const uint16_t *)m->w + (size_t)o * in, xt, in);
                continue;
            }
            const int sc = (in + m->blk_c - 1) / m->blk_c;
            const uint8_t *srow = (const uint8_t *)m->s + (size_t)(o / m->blk_r) * sc;
            double total = 0.0;
            int bi = 0;
            for (int c0 = 0; c0 < in; c0 += m->blk_c, bi++) {
                const int n = (in - c0 < m->blk_c) ? (in - c0) : m->blk_c;
                double acc = 0.0;
                if (m->wdt == 2) {
                    const uint8_t *rw = (const uint8_t *)m->w + (size_t)o * in + c0;
                    for (int i = 0; i < n; i++)
                        acc += (double)orc_e4m3(rw[i]) * (double)xt[c0 + i];
                } else {
                    const uint8_t *rw = (const uint8_t *)m->w + (size_t)o * ((size_t)in / 2);
                    for (int i = 0; i < n; i++)
                        acc += (double)orc_fp4_at(rw, (int64_t)c0 + i) * (double)xt[c0 + i];
                }
                total += acc * (double)orc_e8m0(srow[bi]);
            }
            yt[o] = (float)total;
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- router --
 * src/10_compute/dsv4_ops.c:43-46 (softplus with torch's threshold 20) and
 * :117-156 (dsv4_route): orig = sqrtf(softplus(logit)); the bias is added to a
 * copy used for SELECTION only; top-k by repeated argmax with ties to the lower
 * index; weights = orig[idx] / (double sum) * route_scale. Same float ops in
 * the same order, so the result is bit-identical on the same libm. */
static float orc_softplus(float x)
{
    return (x > 20.0f) ? x : log1pf(expf(x));
}

void orc_route(int *idx, float *wts, float *scores, float *orig,
               const float *bias, const int64_t *tid2eid, int token_id,
               int n_experts, int topk, float route_scale)
{
    for (int e = 0; e < n_experts; e++) orig[e] = sqrtf(orc_softplus(scores[e]));
    for (int e = 0; e < n_experts; e++)
        scores[e] = bias ? orig[e] + bias[e] : orig[e];

    if (tid2eid) {
        const int64_t *row = tid2eid + (int64_t)token_id * topk;
        for (int k = 0; k < topk; k++) idx[k] = (int)row[k];
    } else {
        for (int k = 0; k < topk; k++) {
            int best = -1;
            for (int e = 0; e < n_experts; e++) {
                int taken = 0;
                for (int j = 0; j < k; j++) if (idx[j] == e) { taken = 1; break; }
                if (taken) continue;
                if (best < 0 || scores[e] > scores[best]) best = e;
            }
            idx[k] = best;
        }
    }
    double sum = 0.0;
    for (int k = 0; k < topk; k++) { wts[k] = orig[idx[k]]; sum += (double)wts[k]; }
    const float inv = (sum != 0.0) ? (float)(1.0 / sum) : 0.0f;
    for (int k = 0; k < topk; k++) wts[k] = wts[k] * inv * route_scale;
}

/* ---------------------------------------------------------------- SwiGLU --
 * src/10_compute/dsv4_ops.c:61-79: up clamped to [-limit, limit], gate clamped
 * from ABOVE only, silu(g) = g / (1 + expf(-g)); limit <= 0 disables both. */
/* src/10_compute/dsv4_rope.c (dsv4_rope_apply): the last rd dims of v as
 * interleaved (re, im) pairs rotated by table entry (pos, i); inverse uses
 * -sin. Float multiplies and one add or subtract per output, uncontracted. */
void orc_rope_apply(float *v, int head_dim, int rd, const float *cs, const float *sn, int pos, int table_half,
                    int inverse)
{
    float *tail = v + (head_dim - rd);
    const float *c = cs + (size_t)pos * table_half, *s = sn + (size_t)pos * table_half;
    const float sgn = inverse ? -1.0f : 1.0f;
    for (int i = 0; i < rd / 2; i++) {
        const float re = tail[2 * i], im = tail[2 * i + 1];
        const float ci = c[i], si = sgn * s[i];
        tail[2 * i] = re * ci - im * si;
        tail[2 * i + 1] = re * si + im * ci;
    }
}

static float orc_sigmoidf(float x) { return 1.0f / (1.0f + expf(-x)); }

/* src/10_compute/dsv4_hc.c (dsv4_hc_split_sinkhorn): pre = sigmoid + eps,
 * post = 2 sigmoid, comb = row softmax + eps then a column normalise, then
 * iters - 1 rounds of row and column normalising (sums in double, divisors
 * (float)sum + eps). */
static void orc_hc_split_sinkhorn(float *pre, float *post, float *comb, const float *mixes, const float *scale,
                                  const float *base, int hc, int iters, float eps)
{
    for (int j = 0; j < hc; j++) pre[j] = orc_sigmoidf(mixes[j] * scale[0] + base[j]) + eps;
    for (int j = 0; j < hc; j++) post[j] = 2.0f * orc_sigmoidf(mixes[j + hc] * scale[1] + base[j + hc]);
    for (int j = 0; j < hc; j++)
        for (int k = 0; k < hc; k++) {
            const int o = j * hc + k + 2 * hc;
            comb[j * hc + k] = mixes[o] * scale[2] + base[o];
        }
    for (int j = 0; j < hc; j++) {
        float mx = comb[j * hc];
        for (int k = 1; k < hc; k++)
            if (comb[j * hc + k] > mx) mx = comb[j * hc + k];
        double sum = 0.0;
        for (int k = 0; k < hc; k++) {
            const float e = expf(comb[j * hc + k] - mx);
            comb[j * hc + k] = e;
            sum += (double)e;
        }
        const float inv = (float)(1.0 / sum);
        for (int k = 0; k < hc; k++) comb[j * hc + k] = comb[j * hc + k] * inv + eps;
    }
    for (int k = 0; k < hc; k++) {
        double cs = 0.0;
        for (int j = 0; j < hc; j++) cs += (double)comb[j * hc + k];
        const float d = (float)cs + eps;
        for (int j = 0; j < hc; j++) comb[j * hc + k] /= d;
    }
    for (int it = 0; it < iters - 1; it++) {
        for (int j = 0; j < hc; j++) {
            double rs = 0.0;
            for (int k = 0; k < hc; k++) rs += (double)comb[j * hc + k];
            const float d = (float)rs + eps;
            for (int k = 0; k < hc; k++) comb[j * hc + k] /= d;
        }
        for (int k = 0; k < hc; k++) {
            double cs = 0.0;
            for (int j = 0; j < hc; j++) cs += (double)comb[j * hc + k];
            const float d = (float)cs + eps;
            for (int j = 0; j < hc; j++) comb[j * hc + k] /= d;
        }
    }
}

/* src/10_compute/dsv4_hc.c (dsv4_hc_pre): RMS over the whole hc x hidden
 * vector (norm_eps), mixes[m] = (float)dot(fn[m], x) * rsqrt, the Sinkhorn
 * split, then y[d] = (float)(sum over j in order of fma(pre[j], x[j][d])). */
void orc_hc_pre(float *y, float *post, float *comb, float *mixes, const float *x, const float *fn,
                const float *base, const float *scale, int hc, int hidden, int iters, float norm_eps, float hc_eps)
{
    const int hcdim = hc * hidden, mix_hc = (2 + hc) * hc;
    const double sq = orc_dot_f32d(x, x, hcdim);
    const float rsqrt = (float)(1.0 / sqrt(sq / (double)hcdim + (double)norm_eps));
    for (int m = 0; m < mix_hc; m++) mixes[m] = (float)orc_dot_f32d(fn + (size_t)m * hcdim, x, hcdim) * rsqrt;
    float pre[16];
    orc_hc_split_sinkhorn(pre, post, comb, mixes, scale, base, hc, iters, hc_eps);
    for (int d = 0; d < hidden; d++) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc = fma((double)pre[j], (double)x[(size_t)j * hidden + d], acc);
        y[d] = (float)acc;
    }
}

/* src/10_compute/dsv4_compress.c (pool_channel): max over the slots, then
 * e = (double)expf(v - max) over the finite slots, denominator and weighted
 * sum in double in slot order, (float)(acc / denom); 0 when every slot is -inf. */
static float orc_pool_channel(const float *kv, const float *sc, int slots, int kv_stride, int sc_stride, int c)
{
    float mx = -INFINITY;
    for (int s = 0; s < slots; s++) {
        const float v = sc[(size_t)s * sc_stride + c];
        if (v > mx) mx = v;
    }
    if (mx == -INFINITY) return 0.0f;
    double denom = 0.0, acc = 0.0;
    for (int s = 0; s < slots; s++) {
        const float v = sc[(size_t)s * sc_stride + c];
        if (v == -INFINITY) continue;
        const double e = (double)expf(v - mx);
        denom += e;
        acc += e * (double)kv[(size_t)s * kv_stride + c];
    }
    return (float)(acc / denom);
}

/* src/10_compute/dsv4_compress.c (dsv4_compress_step): the token goes into
 * its slot (score + ape[pos % ratio]); when the window closes the slots are
 * pooled per channel - ratio 4 overlaps the previous window (first half of
 * each slot's channels) with the current one (second half), then slides. */
int orc_compress_step(float *out, const float *kv_in, const float *score_in, const float *ape, float *kv_state,
                      float *score_state, int pos, int ratio, int head_dim)
{
    const int overlap = ratio == 4, coff = 1 + overlap, width = coff * head_dim, nslot = coff * ratio;
    const int phase = pos % ratio, slot = overlap ? ratio + phase : phase;
    const float *apr = ape + (size_t)phase * width;
    for (int c = 0; c < width; c++) {
        kv_state[(size_t)slot * width + c] = kv_in[c];
        score_state[(size_t)slot * width + c] = score_in[c] + apr[c];
    }
    if ((pos + 1) % ratio != 0) return 0;
    if (!overlap) {
        for (int c = 0; c < head_dim; c++) out[c] = orc_pool_channel(kv_state, score_state, nslot, width, width, c);
        return 1;
    }
    const int d = head_dim;
    float *gk = malloc(sizeof(float) * 2 * ratio * d), *gs = malloc(sizeof(float) * 2 * ratio * d);
    for (int s = 0; s < ratio; s++) {
        memcpy(gk + (size_t)s * d, kv_state + (size_t)s * width, sizeof(float) * d);
        memcpy(gs + (size_t)s * d, score_state + (size_t)s * width, sizeof(float) * d);
        memcpy(gk + (size_t)(ratio + s) * d, kv_state + (size_t)(ratio + s) * width + d, sizeof(float) * d);
        memcpy(gs + (size_t)(ratio + s) * d, score_state + (size_t)(ratio + s) * width + d, sizeof(float) * d);
    }
    for (int c = 0; c < d; c++) out[c] = orc_pool_channel(gk, gs, 2 * ratio, d, d, c);
    free(gk);
    free(gs);
    memmove(kv_state, kv_state + (size_t)ratio * width, sizeof(float) * ratio * width);
    memmove(score_state, score_state + (size_t)ratio * width, sizeof(float) * ratio * width);
    return 1;
}

/* src/90_cli/dsv4_decode.c:102-125 (hc_head): sq summed in index order
 * (products then adds), rs = (float)(1 / sqrt(sq / hcdim + norm_eps)); per copy
 * j one sequential fma chain over the whole hc x hidden vector, m = (float)acc *
 * rs, pre[j] = 1 / (1 + expf(-(m * scale + base[j]))) + hc_eps; then
 * y[d] = (float)(sum over j in order of pre[j] * x[j][d]). */
void orc_hc_head(float *y, const float *x, const float *fn, const float *base, const float *scale, int hc,
                 int hidden, float norm_eps, float hc_eps)
{
    const int hcdim = hc * hidden;
    double sq = 0.0;
    for (int i = 0; i < hcdim; i++) sq += (double)x[i] * x[i];
    const float rs = (float)(1.0 / sqrt(sq / (double)hcdim + (double)norm_eps));
    float pre[16];
    for (int j = 0; j < hc; j++) {
        const float *row = fn + (size_t)j * hcdim;
        double acc = 0.0;
        for (int i = 0; i < hcdim; i++) acc = fma((double)row[i], (double)x[i], acc);
        const float m = (float)acc * rs;
        pre[j] = 1.0f / (1.0f + expf(-(m * scale[0] + base[j]))) + hc_eps;
    }
    for (int d = 0; d < hidden; d++) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc += (double)pre[j] * (double)x[(size_t)j * hidden + d];
        y[d] = (float)acc;
    }
}

/* src/10_compute/dsv4_hc.c (dsv4_hc_post): for each copy k and dim d,
 * acc = post[k] * x[d] in double, then acc += comb[j][k] * residual[j][d] for
 * j in order (each product exact in double, one rounded add), y = (float)acc. */
void orc_hc_post(float *y, const float *x, const float *residual, const float *post, const float *comb, int hc,
                 int hidden)
{
    for (int k = 0; k < hc; k++)
        for (int d = 0; d < hidden; d++) {
            double acc = (double)post[k] * (double)x[d];
            for (int j = 0; j < hc; j++) acc += (double)comb[j * hc + k] * (double)residual[(size_t)j * hidden + d];
            y[(size_t)k * hidden + d] = (float)acc;
        }
}

/* src/10_compute/dsv4_ops.c:26-33 (dsv4_rmsnorm): the sum of squares in
 * double in index order, mean = sum / n, inv = (float)(1 / sqrt(mean + eps)),
 * y = w * (x * inv) in float. */
void orc_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += (double)x[i] * (double)x[i];
    const double mean = sum / (double)n;
    const float inv = (float)(1.0 / sqrt(mean + (double)eps));
    for (int i = 0; i < n; i++) y[i] = w[i] * (x[i] * inv);
}

void orc_swiglu(float *y, const float *gate, const float *up, int n, float limit)
{
    for (int i = 0; i < n; i++) {
        float u = up[i], g = gate[i];
        if (limit > 0.0f) {
            if (u > limit) u = limit;
            if (u < -limit) u = -limit;
            if (g > limit) g = limit;
        }
        y[i] = (g / (1.0f + expf(-g))) * u;
    }
}

/* src/10_compute/dsv4_ops.c:85-93: w2( swiglu(w1 x, w3 x) ). */
void orc_expert_forward(float *out, const float *x, const OrcQMat *w,
                        int inter, float limit)
{
    float *g = (float *)malloc((size_t)inter * 3 * sizeof(float));
    float *u = g + inter, *mid = u + inter;
    orc_mmq_n(g, x, &w[0], 1);
    orc_mmq_n(u, x, &w[1], 1);
    orc_swiglu(mid, g, u, inter, limit);
    orc_mmq_n(out, mid, &w[2], 1);
    free(g);
}

/* src/70_decode/dsv4_layer.c:48-117 (dsv4_layer_moe, without the gate GEMV:
 * the logits are the input here). Routed outputs are summed IN k ORDER with
 * their weights (:109-113), then the shared expert is added unweighted
 * (:115-116). */
void orc_moe_decode(float *out, int *idx_out, float *wts_out, const float *x,
                    const float *logits, const float *bias,
                    const int64_t *tid2eid, int token_id,
                    const OrcQMat *experts, const OrcQMat *shared,
                    int n_experts, int topk, float route_scale, int hidden,
                    int inter, float limit)
{
    float *scores = (float *)malloc((size_t)n_experts * 2 * sizeof(float));
    float *orig = scores + n_experts;
    float *acc = (float *)malloc((size_t)hidden * (topk + 1) * sizeof(float));
    memcpy(scores, logits, (size_t)n_experts * sizeof(float));
    orc_route(idx_out, wts_out, scores, orig, bias, tid2eid, token_id,
              n_experts, topk, route_scale);
    for (int k = 0; k < topk; k++)
        orc_expert_forward(acc + (size_t)k * hidden, x,
                           experts + (size_t)idx_out[k] * 3, inter, limit);
    float *sh = acc + (size_t)topk * hidden;
    orc_expert_forward(sh, x, shared, inter, limit);
    for (int i = 0; i < hidden; i++) out[i] = 0.0f;
    for (int k = 0; k < topk; k++) {
        const float wk = wts_out[k];
        for (int i = 0; i < hidden; i++) out[i] += wk * acc[(size_t)k * hidden + i];
    }
    for (int i = 0; i < hidden; i++) out[i] += sh[i];
    free(acc);
    free(scores);
}

/* ------------------------------------------------------------- indexer ----
 * src/10_compute/dsv4_dot.h:20-42: four 4-lane double accumulators, i.e. 16
 * fma chains where chain (4m + l) takes elements i = 16j + 4m + l; lanes fold
 * as (a0+a1)+(a2+a3), then (b0+b1)+(b2+b3); the n % 16 tail continues with fma. */
double orc_dot_f32d(const float *a, const float *b, int n)
{
    double p[16];
    for (int l = 0; l < 16; l++) p[l] = 0.0;
    int i = 0;
    for (; i + 15 < n; i += 16)
        for (int l = 0; l < 16; l++)
            p[l] = fma((double)a[i + l], (double)b[i + l], p[l]);
    double bb[4];
    for (int l = 0; l < 4; l++) bb[l] = (p[l] + p[4 + l]) + (p[8 + l] + p[12 + l]);
    double acc = (bb[0] + bb[1]) + (bb[2] + bb[3]);
    for (; i < n; i++) acc = fma((double)a[i], (double)b[i], acc);
    return acc;
}

/* src/10_compute/dsv4_indexer.c:66-90: per position, heads in order 0..H-1,
 * ReLU on the head dot BEFORE the head weight, double accumulation, then
 * (float)total * (d^-1/2 * h^-1/2) computed in float. */
void orc_indexer_score(float *out, const float *q, const float *kv,
                       const float *weights, int n_heads, int head_dim,
                       int n_pos)
{
    const float scale = (1.0f / sqrtf((float)head_dim))
                      * (1.0f / sqrtf((float)n_heads));
    for (int t = 0; t < n_pos; t++) {
        const float *kt = kv + (size_t)t * head_dim;
        double total = 0.0;
        for (int h = 0; h < n_heads; h++) {
            const double dot = orc_dot_f32d(q + (size_t)h * head_dim, kt, head_dim);
            if (dot > 0.0) total += dot * (double)weights[h];
        }
        out[t] = (float)total * scale;
    }
}

/* src/10_compute/dsv4_topk.c:31-112 and its definition tests/unit/
 * test_indexer.c:20-34: the k largest, descending, ties to the LOWER index,
 * k clamped to n. Compared as floats, so -0.0 ties with +0.0. Restated as a
 * sort on (score desc, index asc); unlike the reference heap it has no k<=1024
 * bound (dsv4_topk.c:80-84 aborts above it). NaN scores are outside the
 * contract (the reference ordering is not a total order with NaN). */
static const float *g_sort_scores;
static int topk_cmp(const void *pa, const void *pb)
{
    const int a = *(const int *)pa, b = *(const int *)pb;
    const float sa = g_sort_scores[a], sb = g_sort_scores[b];
    if (sa > sb) return -1;
    if (sa < sb) return 1;
    return (a < b) ? -1 : (a > b);
}

int orc_topk(int *idxs, const float *scores, int n, int k)
{
    if (k > n) k = n;
    if (k <= 0 || n <= 0) return k;
    int *all = (int *)malloc((size_t)n * sizeof(int));
    for (int i = 0; i < n; i++) all[i] = i;
    g_sort_scores = scores;
    qsort(all, (size_t)n, sizeof(int), topk_cmp);
    memcpy(idxs, all, (size_t)k * sizeof(int));
    free(all);
    return k;
}

/* src/10_compute/dsv4_indexer.c:92-96. */
void orc_indexer_offset(int *idxs, int n, int offset)
{
    for (int i = 0; i < n; i++)
        if (idxs[i] >= 0) idxs[i] += offset;
}

/* src/10_compute/dsv4_attn.c:117-127: ring slots of the most recent
 * min(pos+1, win) positions, newest first, -1 for unwritten slots. */
int orc_window_idxs(int *idxs, int pos, int win)
{
    int n = pos + 1;
    if (n > win) n = win;
    for (int k = 0; k < win; k++) idxs[k] = -1;
    for (int k = 0; k < n; k++) idxs[k] = (pos - k) % win;
    return n;
}

/* src/10_compute/dsv4_attn.c:60-107: per head, score = (float)dot_f32d(q, kv)
 * * scale; the max runs over valid slots only; denominator = double sum of
 * expf(s - max) plus expf(sink - max) (the sink is in the denominator only and
 * never in the max); output accumulated in float over slots in order, slots
 * with weight exactly 0 skipped; then multiplied by (float)(1/denom). -1 slots
 * are masked. */
void orc_sparse_attn(float *o, const float *q, const float *kv,
                     const float *sink, const int *idxs, int h, int d,
                     int topk, float scale)
{
    float *s = (float *)malloc((size_t)(topk > 0 ? topk : 1) * sizeof(float));
    for (int i = 0; i < h; i++) {
        const float *qi = q + (size_t)i * d;
        float mx = -INFINITY;
        for (int j = 0; j < topk; j++) {
            const int idx = idxs[j];
            if (idx < 0) { s[j] = -INFINITY; continue; }
            s[j] = (float)orc_dot_f32d(qi, kv + (size_t)idx * d, d) * scale;
            if (s[j] > mx) mx = s[j];
        }
        double denom = 0.0;
        for (int j = 0; j < topk; j++) {
            if (idxs[j] < 0) { s[j] = 0.0f; continue; }
            s[j] = expf(s[j] - mx);
            denom += (double)s[j];
        }
        denom += (double)expf(sink[i] - mx);
        float *oi = o + (size_t)i * d;
        for (int c = 0; c < d; c++) oi[c] = 0.0f;
        for (int j = 0; j < topk; j++) {
            const int idx = idxs[j];
            if (idx < 0) continue;
            const float w = s[j];
            if (w == 0.0f) continue;
            const float *kvj = kv + (size_t)idx * d;
            for (int c = 0; c < d; c++) oi[c] += w * kvj[c];
        }
        const float inv = (float)(1.0 / denom);
        for (int c = 0; c < d; c++) oi[c] *= inv;
    }
    free(s);
}

/* src/80_prefill/dsv4_prefill_union.c:30-52 (union_prepare): count per
 * expert, exclusive prefix offsets, then fill in (t, k) loop order so tokens
 * are ascending inside each bucket. */
int orc_expert_buckets(int *count, int *off, int *tok, int *ks,
                       const int *topk_idx, int n, int topk, int n_experts)
{
    int *fill = (int *)calloc((size_t)n_experts, sizeof(int));
    for (int e = 0; e < n_experts; e++) count[e] = 0;
    for (int t = 0; t < n; t++)
        for (int k = 0; k < topk; k++) count[topk_idx[(size_t)t * topk + k]]++;
    off[0] = 0;
    int distinct = 0;
    for (int e = 0; e < n_experts; e++) {
        off[e + 1] = off[e] + count[e];
        distinct += count[e] > 0;
    }
    for (int t = 0; t < n; t++)
        for (int k = 0; k < topk; k++) {
            const int e = topk_idx[(size_t)t * topk + k];
            const int pos = off[e] + fill[e]++;
            tok[pos] = t;
            ks[pos] = k;
        }
    free(fill);
    return distinct;
}
