// layer_step.cu - the FFN half of a decoder layer and the whole layer for one
// token on the device.
//
// dsv4_layer_forward (src/70_decode/dsv4_layer.c:18-46): the attention half
// (dsv4cu_attn_block, attn_layer.cu), then the FFN half - the residual taken
// after the attention half, the FFN's mHC pre-mix, ffn_norm, the router GEMV
// (BF16 gate: the reference's exact double tree), the MoE step
// (dsv4cu_moe_decode: route with bias or hash table, the routed experts and
// the shared expert, the k-order combine of dsv4_layer_moe,
// src/70_decode/dsv4_layer.c:48-117) and the mHC update. All on the stream.
// The FFN half takes a batch of nt tokens (a decode batch: one token of each
// of nt sequences); with an expert-parallel object the MoE step runs over
// the ranks (dsv4cu_ep_forward) instead of on this GPU alone.
#include "common.cuh"
#include "ctx.h"

struct dsv4cu_ffn {
    dsv4cu_ffn_desc d;
    void *block;
    float *resid, *x1, *post, *comb, *mixes, *logits, *out;
    int *token;        // [1] token id for hash routing (dsv4cu_layer_step)
};

namespace {

__global__ void lst_set_kernel(int *p, int v) { *p = v; }

}  // namespace

extern "C" int dsv4cu_ffn_create(dsv4cu_ffn **out, const dsv4cu_ffn_desc *d)
{
    if (!out || !d) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ffn_create: NULL argument");
    *out = nullptr;
    if (!d->moe || !d->gate.w || d->gate.rows != d->n_experts || d->gate.cols != d->hidden || !d->ffn_norm ||
        !d->hc_fn || !d->hc_base || !d->hc_scale || d->hidden <= 0 || d->hc_mult <= 0 || d->topk <= 0 ||
        d->n_experts <= 0 || d->nt_max < 1 || d->nt_max > 64)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ffn_create: missing or mis-sized weights, or nt_max not in 1..64");
    if (d->ep && (d->bias || d->tid2eid))
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "ffn_create: the expert-parallel step routes without bias "
                                                        "or hash table");
    dsv4cu_ffn *f = new dsv4cu_ffn();
    f->d = *d;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += dsv4cu_align256(b);
        return o;
    };
    const int hc = d->hc_mult, hd = d->hidden;
    const size_t n = (size_t)d->nt_max;
    const size_t o_res = take(n * hc * hd * 4), o_x1 = take(n * hd * 4), o_post = take(n * hc * 4),
                 o_comb = take(n * hc * hc * 4), o_mix = take(n * (2 + hc) * hc * 4),
                 o_lg = take(n * d->n_experts * 4), o_out = take(n * hd * 4), o_tok = take(16);
    if (cudaMalloc(&f->block, off) != cudaSuccess) {
        delete f;
        return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "ffn_create: scratch");
    }
    char *b = (char *)f->block;
    f->resid = (float *)(b + o_res);
    f->x1 = (float *)(b + o_x1);
    f->post = (float *)(b + o_post);
    f->comb = (float *)(b + o_comb);
    f->mixes = (float *)(b + o_mix);
    f->logits = (float *)(b + o_lg);
    f->out = (float *)(b + o_out);
    f->token = (int *)(b + o_tok);
    *out = f;
    return DSV4CU_OK;
}

extern "C" void dsv4cu_ffn_destroy(dsv4cu_ffn *f)
{
    if (!f) return;
    cudaFree(f->block);
    delete f;
}

extern "C" int dsv4cu_ffn_block(dsv4cu_ctx *ctx, dsv4cu_ffn *f, float *h, int nt, const int *token_ids,
                                void *stream)
{
    if (!ctx || !f || !h) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ffn_block: NULL argument");
    const dsv4cu_ffn_desc &d = f->d;
    if (nt < 1 || nt > d.nt_max) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ffn_block: nt %d (nt_max %d)", nt, d.nt_max);
    if (d.tid2eid && !token_ids) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ffn_block: hash routing needs token_ids");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t wide = (size_t)nt * d.hc_mult * d.hidden;
    int r;
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(f->resid, h, wide * 4, cudaMemcpyDeviceToDevice, st));
    if ((r = dsv4cu_hc_pre(f->x1, f->post, f->comb, f->mixes, h, d.hc_fn, d.hc_base, d.hc_scale, nt, d.hc_mult,
                           d.hidden, d.hc_sinkhorn_iters, d.rms_eps, d.hc_eps, stream)))
        return r;
    if ((r = dsv4cu_rmsnorm(f->x1, f->x1, d.ffn_norm, d.hidden, nt, d.rms_eps, stream))) return r;
    if ((r = dsv4cu_mmq(ctx, f->logits, f->x1, &d.gate, nt, stream))) return r;
    if (d.ep)
        r = dsv4cu_ep_forward(ctx, d.ep, d.moe, f->out, f->x1, f->logits, nt, d.route_scale, d.swiglu_limit, nullptr,
                              nullptr, stream, nullptr);
    else
        r = dsv4cu_moe_decode(ctx, d.moe, f->out, f->x1, f->logits, d.bias, d.tid2eid, token_ids, d.topk,
                              d.route_scale, d.swiglu_limit, nt, nullptr, nullptr, stream);
    if (r) return r;
    return dsv4cu_hc_post(h, f->out, f->resid, f->post, f->comb, nt, d.hc_mult, d.hidden, stream);
}

extern "C" int dsv4cu_layer_step(dsv4cu_ctx *ctx, dsv4cu_attn *a, dsv4cu_ffn *f, float *h, int pos, int token_id,
                                 void *stream)
{
    if (!f) return dsv4cu_set_error(DSV4CU_ERR_ARG, "layer_step: NULL argument");
    int r = dsv4cu_attn_block(ctx, a, h, pos, stream);
    if (r) return r;
    if (f->d.tid2eid) {
        lst_set_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(f->token, token_id);
        DSV4CU_LAUNCH_CHECK();
    }
    return dsv4cu_ffn_block(ctx, f, h, 1, f->d.tid2eid ? f->token : nullptr, stream);
}
