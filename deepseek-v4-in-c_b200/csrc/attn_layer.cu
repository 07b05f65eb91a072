// attn_layer.cu - one decoder layer's attention for one token on the device.
//
// dsv4_layer_attention (src/70_decode/dsv4_layer_attn.c:12-107) and the
// attention half of dsv4_layer_forward (src/70_decode/dsv4_layer.c:24-36),
// step by step on device buffers, every step the library's op for it:
//
//   qr = wq_a x; rms(q_norm); q = wq_b qr          dsv4cu_mmq, dsv4cu_rmsnorm
//   per head: unweighted rms, RoPE                 dsv4cu_rmsnorm with unit
//                                                  weights (the reference's
//                                                  per-head formula bit for
//                                                  bit: 1 * (x * inv) = x * inv),
//                                                  dsv4cu_rope_apply
//   kv = wkv x; rms(kv_norm); RoPE; ring row       (same) + one row copy
//   compressor (ratio != 0): BF16 projections,     dsv4cu_compress_step; on an
//     one ring step                                emit: rms(norm), RoPE at the
//                                                  window's first position, the
//                                                  next compressed cache row
//   compressed rows attention may see: ratio 4     dsv4cu_indexer_score over the
//     scores them with the indexer and keeps       compressed rows read with the
//     the top index_topk; other ratios take all    indexer's head_dim as row
//                                                  stride (the reference passes
//                                                  kv_cache + window * head_dim
//                                                  with that stride), dsv4cu_topk,
//                                                  dsv4cu_indexer_offset
//   window indices (dsv4_window_idxs)              epl_window_kernel
//   o = sparse attention; RoPE inverse             dsv4cu_sparse_attn, dsv4cu_rope_apply
//   grouped wo_a, then wo_b                        ONE dsv4cu_mmq launch of the stacked
//                                                  wo_a over the o_groups input
//                                                  slices as columns, the diagonal
//                                                  blocks gathered (a row of a batched
//                                                  product is the single-token row's
//                                                  bits), then dsv4cu_mmq
//
// Shapes are known on the host for every position (the compressor emits at
// (pos + 1) % ratio == 0, so the compressed-row count is a function of pos),
// so nothing is read back: a step is a fixed sequence of launches on the
// stream. Positions must come in order 0, 1, 2, ... (the state is the
// reference's per-layer state: the KV ring, the compressed rows and the
// compressor's ring).
#include <math.h>
#include <string.h>

#include "common.cuh"
#include "ctx.h"

using namespace dsv4cu;

struct dsv4cu_attn {
    dsv4cu_attn_cfg c;
    dsv4cu_attn_weights w;
    int coff, ncomp_max, n_compressed, next_pos;
    void *block;                 // one allocation for the state and the scratch below
    float *kv_cache;             // [(sliding_window + ncomp_max)][head_dim]
    float *comp_kv, *comp_score; // [coff * ratio][coff * head_dim] (score starts at -inf)
    float *ones;                 // [head_dim] unit weights of the per-head norm
    float *qr, *q, *kv, *ckv, *csc, *iq, *iw, *scores, *o, *ogrp_all, *ogrp, *x1, *resid, *post, *comb, *mixes,
        *out;
    int *idxs, *pos_dev;         // [sliding_window + index_topk], [2]: pos, compressed-row rope position
};

namespace {

__global__ void epl_window_kernel(int *__restrict__ idxs, int pos, int win)
{
    // dsv4_window_idxs (src/10_compute/dsv4_attn.c:117-127): slot k holds the
    // ring row of position pos - k for k < min(pos + 1, win), else -1.
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= win) return;
    const int n = min(pos + 1, win);
    idxs[k] = k < n ? (pos - k) % win : -1;
}

__global__ void epl_iota_kernel(int *__restrict__ idxs, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) idxs[i] = i;
}

__global__ void epl_fill_kernel(float *__restrict__ p, long n, float v)
{
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

__global__ void epl_set2_kernel(int *__restrict__ p, int a, int b)
{
    p[0] = a;
    p[1] = b;
}

// ogrp[g * o_lora + r] = all[g][g * o_lora + r]: the diagonal blocks of the
// stacked product (token g = input slice g).
__global__ void epl_diag_kernel(float *__restrict__ ogrp, const float *__restrict__ all, int groups, int o_lora)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= groups * o_lora) return;
    const int g = i / o_lora;
    ogrp[i] = all[(size_t)g * groups * o_lora + i];
}

int epl_check(const dsv4cu_attn_cfg &c, const dsv4cu_attn_weights &w)
{
    const int hd = c.head_dim;
    if (c.hidden <= 0 || c.n_heads <= 0 || hd <= 0 || c.q_lora <= 0 || c.o_lora <= 0 || c.o_groups <= 0 ||
        (c.n_heads * hd) % c.o_groups || c.qk_rope <= 0 || c.qk_rope % 2 || c.qk_rope > hd ||
        c.sliding_window <= 0 || c.hc_mult <= 0 || c.max_pos <= 0 || c.compress_ratio < 0)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_create: bad geometry");
    if (c.compress_ratio == 4 && (c.index_n_heads <= 0 || c.index_head_dim <= 0 || c.index_topk <= 0 ||
                                  c.index_head_dim < c.qk_rope))
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_create: bad indexer geometry");
    auto mat = [](const dsv4cu_qmat &m, int rows, int cols) { return m.w && m.rows == rows && m.cols == cols; };
    if (!mat(w.wq_a, c.q_lora, c.hidden) || !mat(w.wq_b, c.n_heads * hd, c.q_lora) || !mat(w.wkv, hd, c.hidden) ||
        !mat(w.wo_a, c.o_lora * c.o_groups, c.n_heads * hd / c.o_groups) ||
        !mat(w.wo_b, c.hidden, c.o_lora * c.o_groups) || !w.q_norm || !w.kv_norm || !w.sink || !w.cs || !w.sn)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_create: a projection or vector is missing or mis-sized");
    if (c.compress_ratio) {
        const int coff = c.compress_ratio == 4 ? 2 : 1;
        if (!mat(w.comp_wkv, coff * hd, c.hidden) || !mat(w.comp_wgate, coff * hd, c.hidden) || !w.comp_ape ||
            !w.comp_norm)
            return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_create: compressor weights missing or mis-sized");
    }
    if (c.compress_ratio == 4 && (!mat(w.idx_wq_b, c.index_n_heads * c.index_head_dim, c.q_lora) ||
                                  !mat(w.idx_wproj, c.index_n_heads, c.hidden)))
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_create: indexer weights missing or mis-sized");
    return DSV4CU_OK;
}

}  // namespace

extern "C" int dsv4cu_attn_create(dsv4cu_attn **out, const dsv4cu_attn_cfg *cfg, const dsv4cu_attn_weights *w)
{
    if (!out || !cfg || !w) return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_create: NULL argument");
    *out = nullptr;
    int r = epl_check(*cfg, *w);
    if (r) return r;
    dsv4cu_attn *a = new dsv4cu_attn();
    a->c = *cfg;
    a->w = *w;
    const dsv4cu_attn_cfg &c = a->c;
    const int hd = c.head_dim, H = c.n_heads, ratio = c.compress_ratio;
    a->coff = ratio == 4 ? 2 : 1;
    a->ncomp_max = ratio ? c.max_pos / ratio + 1 : 0;
    const int nidx = c.sliding_window + (ratio == 4 ? c.index_topk : a->ncomp_max);
    const size_t cstate = ratio ? (size_t)a->coff * ratio * a->coff * hd : 0;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += dsv4cu_align256(b);
        return o;
    };
    const size_t o_kv = take((size_t)(c.sliding_window + a->ncomp_max) * hd * 4), o_ck = take(cstate * 4),
                 o_cs = take(cstate * 4), o_one = take((size_t)hd * 4), o_qr = take((size_t)c.q_lora * 4),
                 o_q = take((size_t)H * hd * 4), o_kvv = take((size_t)hd * 4), o_ckv = take((size_t)2 * hd * 4),
                 o_csc = take((size_t)2 * hd * 4),
                 o_iq = take((size_t)(ratio == 4 ? c.index_n_heads * c.index_head_dim : 1) * 4),
                 o_iw = take((size_t)(ratio == 4 ? c.index_n_heads : 1) * 4),
                 o_sc = take((size_t)(a->ncomp_max + 1) * 4), o_o = take((size_t)H * hd * 4),
                 o_all = take((size_t)c.o_groups * c.o_groups * c.o_lora * 4),
                 o_og = take((size_t)c.o_groups * c.o_lora * 4), o_x1 = take((size_t)c.hidden * 4),
                 o_res = take((size_t)c.hc_mult * c.hidden * 4), o_post = take((size_t)c.hc_mult * 4),
                 o_comb = take((size_t)c.hc_mult * c.hc_mult * 4),
                 o_mix = take((size_t)(2 + c.hc_mult) * c.hc_mult * 4), o_out = take((size_t)c.hidden * 4),
                 o_idx = take((size_t)nidx * 4), o_pos = take(16);
    if (cudaMalloc(&a->block, off) != cudaSuccess) {
        delete a;
        return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "attn_create: %zu bytes of state", off);
    }
    char *b = (char *)a->block;
    a->kv_cache = (float *)(b + o_kv);
    a->comp_kv = (float *)(b + o_ck);
    a->comp_score = (float *)(b + o_cs);
    a->ones = (float *)(b + o_one);
    a->qr = (float *)(b + o_qr);
    a->q = (float *)(b + o_q);
    a->kv = (float *)(b + o_kvv);
    a->ckv = (float *)(b + o_ckv);
    a->csc = (float *)(b + o_csc);
    a->iq = (float *)(b + o_iq);
    a->iw = (float *)(b + o_iw);
    a->scores = (float *)(b + o_sc);
    a->o = (float *)(b + o_o);
    a->ogrp_all = (float *)(b + o_all);
    a->ogrp = (float *)(b + o_og);
    a->x1 = (float *)(b + o_x1);
    a->resid = (float *)(b + o_res);
    a->post = (float *)(b + o_post);
    a->comb = (float *)(b + o_comb);
    a->mixes = (float *)(b + o_mix);
    a->out = (float *)(b + o_out);
    a->idxs = (int *)(b + o_idx);
    a->pos_dev = (int *)(b + o_pos);
    // The reference's state starts zeroed, with the compressor's scores at -inf.
    if (cudaMemset(b, 0, off) != cudaSuccess) {
        cudaFree(a->block);
        delete a;
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "attn_create: memset");
    }
    epl_fill_kernel<<<(unsigned)((hd + 255) / 256), 256>>>(a->ones, hd, 1.0f);
    if (cstate) epl_fill_kernel<<<(unsigned)((cstate + 255) / 256), 256>>>(a->comp_score, (long)cstate, -INFINITY);
    if (cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(a->block);
        delete a;
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "attn_create: state init");
    }
    *out = a;
    return DSV4CU_OK;
}

extern "C" void dsv4cu_attn_destroy(dsv4cu_attn *a)
{
    if (!a) return;
    cudaFree(a->block);
    delete a;
}

extern "C" int dsv4cu_attn_n_compressed(const dsv4cu_attn *a) { return a ? a->n_compressed : -1; }

namespace {

// Seeded values in [-1, 1) (splitmix64 of the element index).
__global__ void epl_synth_kernel(float *__restrict__ p, long n, unsigned long long seed)
{
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= n) return;
    unsigned long long z = seed + 0x9E3779B97F4A7C15ull * (unsigned long long)(i + 1);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    p[i] = (float)((double)(z >> 11) * (2.0 / 9007199254740992.0) - 1.0);
}

}  // namespace

extern "C" int dsv4cu_attn_fill_context(dsv4cu_attn *a, int pos, unsigned long long seed, void *stream)
{
    if (!a || pos < 0 || pos >= a->c.max_pos) return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_fill_context: pos %d", pos);
    const dsv4cu_attn_cfg &c = a->c;
    cudaStream_t st = (cudaStream_t)stream;
    const int ratio = c.compress_ratio, ncomp = ratio ? pos / ratio : 0;
    if (ncomp > a->ncomp_max) return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_fill_context: beyond the state");
    const long rows = (long)c.sliding_window + ncomp, n = rows * c.head_dim;
    epl_synth_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a->kv_cache, n, seed);
    DSV4CU_LAUNCH_CHECK();
    if (ratio) {
        const long cs = (long)a->coff * ratio * a->coff * c.head_dim;
        epl_synth_kernel<<<(unsigned)((cs + 255) / 256), 256, 0, st>>>(a->comp_kv, cs, seed ^ 0x5151ull);
        epl_synth_kernel<<<(unsigned)((cs + 255) / 256), 256, 0, st>>>(a->comp_score, cs, seed ^ 0xA2A2ull);
        DSV4CU_LAUNCH_CHECK();
    }
    a->n_compressed = ncomp;
    a->next_pos = pos;
    return DSV4CU_OK;
}

extern "C" const float *dsv4cu_attn_kv_cache(const dsv4cu_attn *a) { return a ? a->kv_cache : nullptr; }

extern "C" int dsv4cu_attn_step(dsv4cu_ctx *ctx, dsv4cu_attn *a, float *out, const float *x, int pos, void *stream)
{
    if (!ctx || !a || !out || !x) return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_step: NULL argument");
    if (pos != a->next_pos || pos >= a->c.max_pos)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_step: position %d (expected %d, max_pos %d)", pos, a->next_pos,
                                a->c.max_pos);
    const dsv4cu_attn_cfg &c = a->c;
    const dsv4cu_attn_weights &w = a->w;
    cudaStream_t st = (cudaStream_t)stream;
    const int hd = c.head_dim, rd = c.qk_rope, H = c.n_heads, half = rd / 2, win = c.sliding_window;
    const int ratio = c.compress_ratio;
    const bool emit = ratio && (pos + 1) % ratio == 0;
    epl_set2_kernel<<<1, 1, 0, st>>>(a->pos_dev, pos, emit ? pos + 1 - ratio : 0);
    DSV4CU_LAUNCH_CHECK();
    int r;
#define EPL_TRY(e)            \
    do {                      \
        if ((r = (e))) return r; \
    } while (0)
    // q: learned norm on the latent, then the per-head unweighted norm and RoPE.
    EPL_TRY(dsv4cu_mmq(ctx, a->qr, x, &w.wq_a, 1, stream));
    EPL_TRY(dsv4cu_rmsnorm(a->qr, a->qr, w.q_norm, c.q_lora, 1, c.rms_eps, stream));
    EPL_TRY(dsv4cu_mmq(ctx, a->q, a->qr, &w.wq_b, 1, stream));
    EPL_TRY(dsv4cu_rmsnorm(a->q, a->q, a->ones, hd, H, c.rms_eps, stream));
    EPL_TRY(dsv4cu_rope_apply(ctx, a->q, 1, H, hd, rd, w.cs, w.sn, a->pos_dev, half, c.max_pos, 0, stream));
    // kv: one head into the sliding ring.
    EPL_TRY(dsv4cu_mmq(ctx, a->kv, x, &w.wkv, 1, stream));
    EPL_TRY(dsv4cu_rmsnorm(a->kv, a->kv, w.kv_norm, hd, 1, c.rms_eps, stream));
    EPL_TRY(dsv4cu_rope_apply(ctx, a->kv, 1, 1, hd, rd, w.cs, w.sn, a->pos_dev, half, c.max_pos, 0, stream));
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(a->kv_cache + (size_t)(pos % win) * hd, a->kv, (size_t)hd * 4,
                                    cudaMemcpyDeviceToDevice, st));
    epl_window_kernel<<<(unsigned)((win + 255) / 256), 256, 0, st>>>(a->idxs, pos, win);
    DSV4CU_LAUNCH_CHECK();
    int n_idx = min(pos + 1, win);
    if (ratio) {
        EPL_TRY(dsv4cu_mmq(ctx, a->ckv, x, &w.comp_wkv, 1, stream));
        EPL_TRY(dsv4cu_mmq(ctx, a->csc, x, &w.comp_wgate, 1, stream));
        const int e = dsv4cu_compress_step(a->kv, a->ckv, a->csc, w.comp_ape, a->comp_kv, a->comp_score, pos, ratio,
                                           hd, stream);
        if (e < 0) return e;
        if (e) {
            if (a->n_compressed >= a->ncomp_max)
                return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_step: compressed rows beyond max_pos");
            EPL_TRY(dsv4cu_rmsnorm(a->kv, a->kv, w.comp_norm, hd, 1, c.rms_eps, stream));
            // Stamped with the FIRST position of the window it summarises.
            EPL_TRY(dsv4cu_rope_apply(ctx, a->kv, 1, 1, hd, rd, w.cs, w.sn, a->pos_dev + 1, half, c.max_pos, 0,
                                      stream));
            DSV4CU_CUDA_TRY(cudaMemcpyAsync(a->kv_cache + (size_t)(win + a->n_compressed) * hd, a->kv, (size_t)hd * 4,
                                            cudaMemcpyDeviceToDevice, st));
            a->n_compressed++;
        }
        const int avail = a->n_compressed;
        if (avail > 0) {
            int take = avail;
            int *dst = a->idxs + n_idx;
            if (ratio == 4) {
                const int ih = c.index_n_heads, ihd = c.index_head_dim;
                EPL_TRY(dsv4cu_mmq(ctx, a->iq, a->qr, &w.idx_wq_b, 1, stream));
                EPL_TRY(dsv4cu_rope_apply(ctx, a->iq, 1, ih, ihd, rd, w.cs, w.sn, a->pos_dev, half, c.max_pos, 0,
                                          stream));
                EPL_TRY(dsv4cu_mmq(ctx, a->iw, x, &w.idx_wproj, 1, stream));
                EPL_TRY(dsv4cu_indexer_score(a->scores, a->iq, a->kv_cache + (size_t)win * hd, a->iw, ih, ihd, avail,
                                             stream));
                take = avail < c.index_topk ? avail : c.index_topk;
                EPL_TRY(dsv4cu_topk(ctx, dst, a->scores, avail, take, stream));
            } else {
                epl_iota_kernel<<<(unsigned)((take + 255) / 256), 256, 0, st>>>(dst, take);
                DSV4CU_LAUNCH_CHECK();
            }
            EPL_TRY(dsv4cu_indexer_offset(dst, take, win, stream));
            n_idx += take;
        }
    }
    EPL_TRY(dsv4cu_sparse_attn(ctx, a->o, a->q, a->kv_cache, 0, w.sink, a->idxs, H, hd, n_idx,
                               1.0f / sqrtf((float)hd), stream));
    EPL_TRY(dsv4cu_rope_apply(ctx, a->o, 1, H, hd, rd, w.cs, w.sn, a->pos_dev, half, c.max_pos, 1, stream));
    // Grouped low-rank output projection: the o_groups slices of o are the
    // columns of one product with the stacked wo_a; group g's rows of column g
    // are its result.
    EPL_TRY(dsv4cu_mmq(ctx, a->ogrp_all, a->o, &w.wo_a, c.o_groups, stream));
    const int ng = c.o_groups * c.o_lora;
    epl_diag_kernel<<<(unsigned)((ng + 255) / 256), 256, 0, st>>>(a->ogrp, a->ogrp_all, c.o_groups, c.o_lora);
    DSV4CU_LAUNCH_CHECK();
    EPL_TRY(dsv4cu_mmq(ctx, out, a->ogrp, &w.wo_b, 1, stream));
#undef EPL_TRY
    a->next_pos = pos + 1;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_attn_block(dsv4cu_ctx *ctx, dsv4cu_attn *a, float *h, int pos, void *stream)
{
    if (!ctx || !a || !h) return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_block: NULL argument");
    const dsv4cu_attn_cfg &c = a->c;
    const dsv4cu_attn_weights &w = a->w;
    if (!w.attn_norm || !w.hc_fn || !w.hc_base || !w.hc_scale)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "attn_block: the block's norm and mHC weights are missing");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t wide = (size_t)c.hc_mult * c.hidden;
    int r;
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(a->resid, h, wide * 4, cudaMemcpyDeviceToDevice, st));
    if ((r = dsv4cu_hc_pre(a->x1, a->post, a->comb, a->mixes, h, w.hc_fn, w.hc_base, w.hc_scale, 1, c.hc_mult,
                           c.hidden, c.hc_sinkhorn_iters, c.rms_eps, c.hc_eps, stream)))
        return r;
    if ((r = dsv4cu_rmsnorm(a->x1, a->x1, w.attn_norm, c.hidden, 1, c.rms_eps, stream))) return r;
    if ((r = dsv4cu_attn_step(ctx, a, a->out, a->x1, pos, stream))) return r;
    return dsv4cu_hc_post(h, a->out, a->resid, a->post, a->comb, 1, c.hc_mult, c.hidden, stream);
}
