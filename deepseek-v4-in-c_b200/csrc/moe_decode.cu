// moe_decode.cu - one MoE layer decode step for nt tokens, HBM-resident experts.
//
// Reference: dsv4_layer_moe (src/70_decode/dsv4_layer.c:48-117) from the router
// logits on, with dsv4_route (dsv4_ops.c:117-156), dsv4_expert_forward
// (dsv4_ops.c:85-93) and the k-order combine (dsv4_layer.c:109-116).
//
// Three launches, stream-ordered:
//   prologue  CTA 0 routes every token (one warp per token) and buckets the
//             (token, k) pairs by expert in ascending expert order, tokens
//             ascending inside a bucket (the layout of union_prepare,
//             src/80_prefill/dsv4_prefill_union.c:30-52). The other CTAs split
//             x into the exact f16 hi/lo operand.
//   phase 1   CTA (32-row slice, bucket): w1 and w3 rows of the bucket's expert
//             against every token of the bucket, SwiGLU in the epilogue, and the
//             32 mid values written straight into the hi/lo operand form.
//   phase 2   CTA (16-row slice, bucket): w2 rows against the bucket's mid
//             vectors -> per-pair partial rows. The last CTA of a row slice sums
//             the pairs of every token in k order, then adds the shared expert.
// Every weight byte of the touched experts is read exactly once per step.
//
// The experts are prepared once (dsv4cu_moe_create): descriptors validated and
// copied to the device, and one TMA tensor map per weight matrix (and per FP4
// scale grid) encoded, so the phase kernels stream weights with tensor-map TMA.
#include <stdio.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "gemv.h"
#include "gemv_core.cuh"
#include "moe.h"
#include "router.cuh"
#include "stream_mv.cuh"
#include "tma_gemv.cuh"
#include "tmap.h"

namespace dsv4cu {

constexpr int MOE_MAX_NT = 64;
constexpr int MOE_MAX_TOPK = 16;

struct MoeWs {
    uint16_t *xh, *xl;    // [nt][hidden]
    float *xs;            // [nt][hidden/32]
    int *idx;             // [nt][topk]
    float *wts;           // [nt][topk]
    int *meta;            // [0] n_buckets, [1] bad-route flag
    int *b_expert;        // [nbmax]
    int *b_off;           // [nbmax + 2]
    int *b_tok;           // [npairs] token of each bucket slot (shared slots at the end)
    int *pos;             // [nt][topk] bucket slot of pair (t, k)
    uint16_t *mh, *ml;    // [npairs][inter]
    float *mxs;           // [npairs][inter/32]
    float *ypart;         // [npairs][hidden]
};

// ------------------------------------------------------------- prologue
__global__ void __launch_bounds__(1024) moe_prologue_kernel(
    const float *__restrict__ tab, const float *__restrict__ x, const float *__restrict__ logits, const float *__restrict__ bias,
    const int64_t *__restrict__ tid2eid, const int *__restrict__ token_ids, int n_experts, int topk,
    float route_scale, int hidden, int nt, int has_shared, MoeWs ws, int *__restrict__ idx_out,
    float *__restrict__ wts_out)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    if (blockIdx.x > 0) {
        // x -> f16 hi/lo operand, one warp per (token, 32-element block).
        const int nblk = hidden >> 5;
        for (int gw = (blockIdx.x - 1) * nwarps + warp; gw < nt * nblk; gw += (gridDim.x - 1) * nwarps) {
            const int t = gw / nblk, b = gw - t * nblk, k = b * 32 + lane;
            const float v = x[(size_t)t * hidden + k];
            float a = isfinite(v) ? fabsf(v) : 0.0f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
            int P = 0;
            if (a > 0.0f) {
                int e;
                frexpf(a, &e);
                P = min(125, max(-125, 15 - e));
            }
            const float vs = ldexpf(v, P);
            const __half hh = __float2half_rn(vs);
            const float hf = __half2float(hh);
            const __half lh = isfinite(hf) ? __float2half_rn(vs - hf) : __float2half_rn(0.0f);
            ws.xh[(size_t)t * hidden + k] = __half_as_ushort(hh);
            ws.xl[(size_t)t * hidden + k] = __half_as_ushort(lh);
            if (lane == 0) ws.xs[(size_t)t * nblk + b] = ldexpf(1.0f, -P);
        }
        return;
    }

    // CTA 0: routing, one warp per token.
    for (int t = warp; t < nt; t += nwarps)
        route_token_warp(tab, logits + (size_t)t * n_experts, bias, tid2eid, token_ids ? token_ids[t] : 0,
                         n_experts, topk, route_scale, ws.idx + t * topk, ws.wts + t * topk, nullptr, nullptr);
    __syncthreads();

    // Bucket the pairs by expert. counts[e] then an exclusive scan over experts
    // in ascending order; slots inside a bucket follow (t, k) order.
    __shared__ int cnt[512 + 1];
    __shared__ int boff[512 + 1];
    __shared__ int bad;
    const int npairs = nt * topk;
    for (int e = threadIdx.x; e <= n_experts; e += blockDim.x) cnt[e] = 0;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
        const int e = ws.idx[p];
        if (e < 0 || e >= n_experts) atomicOr(&bad, 1);
        else atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int off = 0, nb = 0;
        for (int e = 0; e < n_experts; e++) {
            boff[e] = off;
            if (cnt[e]) {
                ws.b_expert[nb] = e;
                ws.b_off[nb] = off;
                nb++;
            }
            off += cnt[e];
        }
        ws.b_off[nb] = off;               // end of routed slots
        ws.b_off[nb + 1] = off + (has_shared ? nt : 0);
        ws.meta[0] = nb;
        ws.meta[1] = bad;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
        const int e = ws.idx[p];
        if (e < 0 || e >= n_experts) { ws.pos[p] = -1; continue; }
        int r = 0;
        for (int q = 0; q < p; q++) r += (ws.idx[q] == e);
        const int slot = boff[e] + r;
        ws.pos[p] = slot;
        ws.b_tok[slot] = p / topk;
    }
    if (has_shared)
        for (int t = threadIdx.x; t < nt; t += blockDim.x) ws.b_tok[npairs + t] = t;
    if (idx_out)
        for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
            idx_out[p] = ws.idx[p];
            wts_out[p] = ws.wts[p];
        }
}


}  // namespace dsv4cu

namespace dsv4cu {

// Resolve bucket b of this launch: expert index (n_experts = shared), first
// slot and slot count.
DSV4CU_DEV bool moe_bucket(const MoeWs &ws, const MoeDev &L, int b, int nbmax, int &e, int &s0, int &cnt)
{
    const int nb = ws.meta[0];
    if (b == nbmax) {            // the shared-expert bucket is always the last one
        if (!L.has_shared) return false;
        e = L.n_experts;
        s0 = ws.b_off[nb];
        cnt = ws.b_off[nb + 1] - s0;
        return cnt > 0;
    }
    if (b >= nb) return false;
    e = ws.b_expert[b];
    s0 = ws.b_off[b];
    cnt = ws.b_off[b + 1] - s0;
    return true;
}

DSV4CU_DEV MatArgs mat_of(const dsv4cu_qmat &q)
{
    MatArgs m;
    m.w = (const uint8_t *)q.w;
    m.s = (const uint8_t *)q.s;
    m.rows = q.rows;
    m.cols = q.cols;
    m.blk_r = q.blk_r;
    m.blk_c = q.blk_c;
    m.s_cols = (q.cols + q.blk_c - 1) / q.blk_c;
    m.row_bytes = q.wdt == DSV4CU_WFP4 ? q.cols / 2 : q.cols;
    return m;
}

DSV4CU_DEV Stream moe_stream(const MoeDev &L, int e, int mat, int row0, int kb0)
{
    const dsv4cu_expert &ex = L.experts[e];
    Stream st;
    st.m = mat_of(mat == 0 ? ex.w1 : (mat == 1 ? ex.w3 : ex.w2));
    st.tw = L.maps + 6 * e + 2 * mat;
    st.ts = L.staged[3 * e + mat] ? L.maps + 6 * e + 2 * mat + 1 : nullptr;
    st.row0 = row0;
    st.kb0 = kb0;
    return st;
}

// ---------------------------------------------------------------- phases
// Both phases run on a 1-D grid of CTAs of 8 consumer warps + 1 TMA producer
// warp (tma_gemv.cuh), sized for three CTAs per SM so the whole grid of a
// decode step is resident in one wave. A CTA owns a row block of one bucket's
// matrix; the block is sized by the weight format so every CTA streams the
// same bytes: FP4 rows are half the bytes of FP8 rows, so FP4 blocks are twice
// as tall, and the 8 warps cover them as 16-row x full-K streams (tall block)
// or 16-row x K-half streams (short block).
constexpr int P1_ROWS_FP4 = 64, P1_ROWS_FP8 = 32;    // phase 1: rows of w1 (and of w3) per CTA
constexpr int P2_ROWS_FP4 = 128, P2_ROWS_FP8 = 64;   // phase 2: w2 rows per CTA
constexpr int MOE_STAGES = 2;
using MoeSmem = TmaSmem<MOE_STAGES>;
constexpr int MOE_THREADS = 288;

// CTA id -> (bucket, first row, rows) over the routed buckets then the shared one.
DSV4CU_DEV bool moe_cta_work(int cta, int nbmax, int rows_total, int rows_routed, int rows_shared,
                             int &bucket, int &row0, int &nrows)
{
    const int per_routed = rows_total / rows_routed;
    if (cta < nbmax * per_routed) {
        bucket = cta / per_routed;
        row0 = (cta - bucket * per_routed) * rows_routed;
        nrows = rows_routed;
        return true;
    }
    cta -= nbmax * per_routed;
    if (cta >= rows_total / rows_shared) return false;
    bucket = nbmax;
    row0 = cta * rows_shared;
    nrows = rows_shared;
    return true;
}

template <int NT>
DSV4CU_DEV void moe_run_streams(int fmt, unsigned char *dsmem, const Stream *streams, int L, const XArgs &xa, int nv,
                                float (&acc)[NT][2], int *err)
{
    if (fmt == DSV4CU_WFP4)
        tma_gemv_streams<DSV4CU_WFP4, NT, MOE_STAGES>(dsmem, streams, L, xa, nv, acc, err);
    else
        tma_gemv_streams<DSV4CU_WFP8, NT, MOE_STAGES>(dsmem, streams, L, xa, nv, acc, err);
}

template <int NT>
__global__ void __launch_bounds__(MOE_THREADS, NT == 1 ? 3 : 2)
    moe_gate_up_kernel(MoeWs ws, MoeDev Ld, int nbmax, int hidden, int inter, float limit, int *status)
{
    extern __shared__ __align__(128) unsigned char dsmem[];
    __shared__ Stream streams[8];
    __shared__ float red[2][4][2][NT][16];   // [mat][row group][K part][token][row]
    __shared__ float mid[NT][64];
    int bucket, row0, rows;
    if (!moe_cta_work(blockIdx.x, nbmax, inter, P1_ROWS_FP4, P1_ROWS_FP8, bucket, row0, rows)) return;
    int e, s0, cnt;
    if (!moe_bucket(ws, Ld, bucket, nbmax, e, s0, cnt)) return;
    const int fmt = Ld.experts[e].w1.wdt;
    // A bucket of the other format than its grid slot was laid out for covers
    // the slot in blocks of its own height.
    const int want = min(rows, (fmt == DSV4CU_WFP4) ? P1_ROWS_FP4 : P1_ROWS_FP8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = status;

    for (int r0 = row0; r0 < row0 + rows; r0 += want) {
        const int nrow = want;                        // 64 (full-K streams) or 32 (K halves)
        const int nk = nrow == 64 ? 1 : 2;
        if (threadIdx.x < 8) {
            const int w = threadIdx.x, mat = w >> 2;
            const int rg = nk == 1 ? (w & 3) : ((w >> 1) & 1), kp = nk == 1 ? 0 : (w & 1);
            const int rb = Ld.experts[e].w1.wdt == DSV4CU_WFP4 ? hidden / 2 : hidden;
            streams[w] = moe_stream(Ld, e, mat, r0 + rg * 16, kp * (rb / nk));
        }
        __syncthreads();
        const int L = streams[0].m.row_bytes / nk;
        for (int c0 = 0; c0 < cnt; c0 += NT) {
            const int nv = min(NT, cnt - c0);
            XArgs xa;
            xa.xh = ws.xh;
            xa.xl = ws.xl;
            xa.xs = ws.xs;
            xa.ldx = hidden;
            xa.tok = ws.b_tok + s0 + c0;
            float acc[NT][2];
#pragma unroll
            for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.0f;
            moe_run_streams<NT>(fmt, dsmem, streams, L, xa, nv, acc, err);
            if (warp < 8) {
                const int mat = warp >> 2;
                const int rg = nk == 1 ? (warp & 3) : ((warp >> 1) & 1), kp = nk == 1 ? 0 : (warp & 1);
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    const float v0 = quad_sum(acc[t][0]), v1 = quad_sum(acc[t][1]);
                    if ((lane & 3) == 0) {
                        red[mat][rg][kp][t][lane >> 2] = v0;
                        red[mat][rg][kp][t][(lane >> 2) + 8] = v1;
                    }
                }
            }
            __syncthreads();
            // SwiGLU (dsv4_ops.c:61-79): up clamped both ways, gate from above only.
            if (threadIdx.x < nv * nrow) {
                const int t = threadIdx.x / nrow, r = threadIdx.x - t * nrow, rg = r >> 4, rr = r & 15;
                float g = red[0][rg][0][t][rr], u = red[1][rg][0][t][rr];
                if (nk == 2) {
                    g += red[0][rg][1][t][rr];
                    u += red[1][rg][1][t][rr];
                }
                if (limit > 0.0f) {
                    u = fminf(fmaxf(u, -limit), limit);
                    g = fminf(g, limit);
                }
                mid[t][r] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
            }
            __syncthreads();
            // mid -> f16 hi/lo operand for phase 2: one warp per (token, 32 rows).
            if (warp < nv * (nrow >> 5)) {
                const int t = warp / (nrow >> 5), half = warp - t * (nrow >> 5), slot = s0 + c0 + t;
                const int rr = half * 32 + lane, row = r0 + rr;
                const float v = mid[t][rr];
                float a = isfinite(v) ? fabsf(v) : 0.0f;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
                int P = 0;
                if (a > 0.0f) {
                    int ex2;
                    frexpf(a, &ex2);
                    P = min(125, max(-125, 15 - ex2));
                }
                const float vs = ldexpf(v, P);
                const __half hh = __float2half_rn(vs);
                const float hf = __half2float(hh);
                const __half lh = isfinite(hf) ? __float2half_rn(vs - hf) : __float2half_rn(0.0f);
                ws.mh[(size_t)slot * inter + row] = __half_as_ushort(hh);
                ws.ml[(size_t)slot * inter + row] = __half_as_ushort(lh);
                if (lane == 0) ws.mxs[(size_t)slot * (inter >> 5) + (row >> 5)] = ldexpf(1.0f, -P);
            }
            __syncthreads();
        }
    }
}

// Combine of one 64-row slice of the output: the routed pairs of every token
// IN k ORDER (dsv4_layer.c:109-113), then the shared expert unweighted (:115).
DSV4CU_DEV void moe_combine_slice(const MoeWs &ws, int row0, int nt, int topk, int hidden, int has_shared,
                                  float *__restrict__ out)
{
    const int nb = ws.meta[0];
    for (int i = threadIdx.x; i < nt * 64; i += blockDim.x) {
        const int t = i >> 6, row = row0 + (i & 63);
        float o = 0.0f;
        for (int k = 0; k < topk; k++) {
            const int slot = __ldcg(ws.pos + t * topk + k);
            if (slot < 0) continue;
            o = __fadd_rn(o, __fmul_rn(__ldcg(ws.wts + t * topk + k),
                                       __ldcg(ws.ypart + (size_t)slot * hidden + row)));
        }
        if (has_shared)
            o = __fadd_rn(o, __ldcg(ws.ypart + (size_t)(__ldcg(ws.b_off + nb) + t) * hidden + row));
        out[(size_t)t * hidden + row] = o;
    }
}

// counters[s] counts the CTAs that have written 64-row slice s; the last of
// the (nbmax + has_shared) contributions combines the slice and resets it.
template <int NT>
__global__ void __launch_bounds__(MOE_THREADS, NT == 1 ? 3 : 2)
    moe_down_kernel(MoeWs ws, MoeDev Ld, int nbmax, int hidden, int inter, int nt, int topk,
                    float *__restrict__ out, int *__restrict__ counters, int *status)
{
    extern __shared__ __align__(128) unsigned char dsmem[];
    __shared__ Stream streams[8];
    __shared__ float red[8][2][NT][16];
    __shared__ int last[2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int bucket, row0, rows;
    if (!moe_cta_work(blockIdx.x, nbmax, hidden, P2_ROWS_FP4, P2_ROWS_FP8, bucket, row0, rows)) return;
    int e, s0, cnt;
    int *err = status;
    if (moe_bucket(ws, Ld, bucket, nbmax, e, s0, cnt)) {
        const int fmt = Ld.experts[e].w2.wdt;
        const int want = min(rows, (fmt == DSV4CU_WFP4) ? P2_ROWS_FP4 : P2_ROWS_FP8);
        for (int r0 = row0; r0 < row0 + rows; r0 += want) {
            const int nrow = want;                    // 128 (full-K streams) or 64 (K halves)
            const int nk = nrow == 128 ? 1 : 2;
            if (threadIdx.x < 8) {
                const int w = threadIdx.x;
                const int rg = nk == 1 ? w : (w >> 1), kp = nk == 1 ? 0 : (w & 1);
                const int rb = fmt == DSV4CU_WFP4 ? inter / 2 : inter;
                streams[w] = moe_stream(Ld, e, 2, r0 + rg * 16, kp * (rb / nk));
            }
            __syncthreads();
            const int L = streams[0].m.row_bytes / nk;
            for (int c0 = 0; c0 < cnt; c0 += NT) {
                const int nv = min(NT, cnt - c0);
                XArgs xa;
                xa.xh = ws.mh + (size_t)(s0 + c0) * inter;
                xa.xl = ws.ml + (size_t)(s0 + c0) * inter;
                xa.xs = ws.mxs + (size_t)(s0 + c0) * (inter >> 5);
                xa.ldx = inter;
                xa.tok = nullptr;
                float acc[NT][2];
#pragma unroll
                for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.0f;
                moe_run_streams<NT>(fmt, dsmem, streams, L, xa, nv, acc, err);
                if (warp < 8) {
                    const int rg = nk == 1 ? warp : (warp >> 1), kp = nk == 1 ? 0 : (warp & 1);
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        const float v0 = quad_sum(acc[t][0]), v1 = quad_sum(acc[t][1]);
                        if ((lane & 3) == 0) {
                            red[rg][kp][t][lane >> 2] = v0;
                            red[rg][kp][t][(lane >> 2) + 8] = v1;
                        }
                    }
                }
                __syncthreads();
                for (int i = threadIdx.x; i < nv * nrow; i += blockDim.x) {
                    const int t = i / nrow, r = i - t * nrow, rg = r >> 4, rr = r & 15;
                    float v = red[rg][0][t][rr];
                    if (nk == 2) v += red[rg][1][t][rr];
                    ws.ypart[(size_t)(s0 + c0 + t) * hidden + r0 + r] = v;
                }
                __syncthreads();
            }
        }
    }
    // Every CTA (idle ones included) reports each 64-row slice it covers.
    __threadfence();
    const int nslice = rows >> 6;
    if (threadIdx.x < nslice) {
        const int sl = (row0 >> 6) + threadIdx.x;
        last[threadIdx.x] = (atomicAdd(&counters[sl], 1) == nbmax + Ld.has_shared - 1);
    }
    __syncthreads();
    for (int i = 0; i < nslice; i++) {
        if (!last[i]) continue;
        __threadfence();
        moe_combine_slice(ws, row0 + i * 64, nt, topk, hidden, Ld.has_shared, out);
        if (threadIdx.x == 0) counters[(row0 >> 6) + i] = 0;
    }
}

static size_t moe_ws_layout(int nt, int topk, int n_experts, int hidden, int inter, int has_shared,
                            char *base, MoeWs *w)
{
    const size_t npairs = (size_t)nt * topk + (has_shared ? nt : 0);
    const size_t nbmax = (size_t)min(nt * topk, n_experts);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = base ? base + off : nullptr;
        off += dsv4cu_align256(bytes);
        return p;
    };
    MoeWs t;
    t.xh = (uint16_t *)take((size_t)nt * hidden * 2);
    t.xl = (uint16_t *)take((size_t)nt * hidden * 2);
    t.xs = (float *)take((size_t)nt * (hidden / 32) * 4);
    t.idx = (int *)take((size_t)nt * topk * 4);
    t.wts = (float *)take((size_t)nt * topk * 4);
    t.meta = (int *)take(16);
    t.b_expert = (int *)take(nbmax * 4 + 4);
    t.b_off = (int *)take((nbmax + 2) * 4);
    t.b_tok = (int *)take(npairs * 4);
    t.pos = (int *)take((size_t)nt * topk * 4);
    t.mh = (uint16_t *)take(npairs * inter * 2);
    t.ml = (uint16_t *)take(npairs * inter * 2);
    t.mxs = (float *)take(npairs * (inter / 32) * 4);
    t.ypart = (float *)take(npairs * hidden * 4);
    if (w) *w = t;
    return off;
}

size_t moe_decode_workspace(int nt, int topk, int n_experts, int hidden, int inter, int has_shared)
{
    return moe_ws_layout(nt, topk, n_experts, hidden, inter, has_shared, nullptr, nullptr);
}

int moe_decode_run(const dsv4cu_moe *layer, float *out, const float *x, const float *logits, const float *bias,
                   const int64_t *tid2eid, const int *token_ids, int topk, float route_scale, float limit, int nt,
                   int *idx_out, float *wts_out, void *wsp, int *counters, int *status, cudaStream_t st,
                   cudaEvent_t *ev)
{
    const int n_experts = layer->n_experts, hidden = layer->hidden, inter = layer->inter;
    const int has_shared = layer->has_shared;
    MoeWs ws;
    moe_ws_layout(nt, topk, n_experts, hidden, inter, has_shared, (char *)wsp, &ws);
    const int nbmax = min(nt * topk, n_experts);
    const int xblocks = min(64, max(1, nt * (hidden / 32) / 32));
    const float *tab = router_table_get();
    if (!tab) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "moe_decode: router table setup failed");
    const int smem = MoeSmem::BYTES;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
    moe_prologue_kernel<<<1 + xblocks, 1024, 0, st>>>(tab, x, logits, bias, tid2eid, token_ids, n_experts,
                                                      topk, route_scale, hidden, nt, has_shared, ws,
                                                      idx_out, wts_out);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));
    const int g1 = nbmax * (inter / P1_ROWS_FP4) + (has_shared ? inter / P1_ROWS_FP8 : 0);
    const int g2 = nbmax * (hidden / P2_ROWS_FP4) + (has_shared ? hidden / P2_ROWS_FP8 : 0);
    if (nt == 1) {
        DSV4CU_CUDA_TRY(cudaFuncSetAttribute(moe_gate_up_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        moe_gate_up_kernel<1><<<g1, MOE_THREADS, smem, st>>>(ws, layer->view, nbmax, hidden, inter, limit, status);
    } else {
        DSV4CU_CUDA_TRY(cudaFuncSetAttribute(moe_gate_up_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        moe_gate_up_kernel<4><<<g1, MOE_THREADS, smem, st>>>(ws, layer->view, nbmax, hidden, inter, limit, status);
    }
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[2], st));
    if (nt == 1) {
        DSV4CU_CUDA_TRY(cudaFuncSetAttribute(moe_down_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        moe_down_kernel<1><<<g2, MOE_THREADS, smem, st>>>(ws, layer->view, nbmax, hidden, inter, nt, topk, out,
                                                          counters, status);
    } else {
        DSV4CU_CUDA_TRY(cudaFuncSetAttribute(moe_down_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        moe_down_kernel<4><<<g2, MOE_THREADS, smem, st>>>(ws, layer->view, nbmax, hidden, inter, nt, topk, out,
                                                          counters, status);
    }
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[3], st));
    return DSV4CU_OK;
}

// Host-side validation of one expert: shapes, a format the kernels stream,
// and a TMA-streamable weight layout.
static int expert_check(const dsv4cu_expert &e, int hidden, int inter, const char *what)
{
    const dsv4cu_qmat *ms[3] = {&e.w1, &e.w3, &e.w2};
    const int rows[3] = {inter, inter, hidden}, cols[3] = {hidden, hidden, inter};
    for (int i = 0; i < 3; i++) {
        const dsv4cu_qmat &q = *ms[i];
        if (q.rows != rows[i] || q.cols != cols[i] || !q.w || !q.s)
            return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_create: %s matrix %d shape %dx%d, want %dx%d", what, i,
                                    q.rows, q.cols, rows[i], cols[i]);
        const bool fmt_ok = (q.wdt == DSV4CU_WFP4 && q.blk_c > 0 && q.blk_c % 32 == 0 && q.blk_r > 0) ||
                            (q.wdt == DSV4CU_WFP8 && q.blk_c > 0 && q.blk_c % 16 == 0 && q.blk_r > 0);
        if (!fmt_ok)
            return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_create: %s matrix %d format %d blk %dx%d", what, i,
                                    q.wdt, q.blk_r, q.blk_c);
        if (!tmap_weights_ok(&q))
            return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED,
                                    "moe_create: %s matrix %d: rows must be >= 128 bytes, a multiple of 16, on a "
                                    "16-byte aligned base", what, i);
    }
    if (e.w1.wdt != e.w3.wdt) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_create: %s w1/w3 formats differ", what);
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

// Whether a decode of nt tokens takes the streamed path: chosen explicitly,
// or by default only where the tensor-core path is missing (it is the faster
// of the two for the layer shapes measured). Buckets of the streamed path
// hold at most nt tokens, which hash routing (rows may repeat an expert)
// breaks.
static bool use_stream(const dsv4cu_moe *L, int nt, bool hash)
{
    if (!L->smv_ok || nt > SMV_MAXT || hash || L->path == DSV4CU_MOE_PATH_TENSOR) return false;
    return L->path == DSV4CU_MOE_PATH_STREAM || !L->mx_ok;
}

extern "C" int dsv4cu_moe_create(dsv4cu_moe **out, const dsv4cu_expert *experts, int n_experts,
                                 const dsv4cu_expert *shared, int hidden, int inter)
{
    if (!out || !experts) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_create: NULL argument");
    *out = nullptr;
    if (n_experts < 1 || n_experts > 32 * RMAX_PER_LANE)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_create: n_experts %d", n_experts);
    if (hidden % 128 || inter % 128 || hidden <= 0 || inter <= 0)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_create: hidden and inter must be multiples of 128");
    if (hidden / 64 > DSV4CU_MAX_COUNTERS) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_create: hidden too large");
    for (int e = 0; e < n_experts; e++) {
        char what[32];
        snprintf(what, sizeof what, "expert %d", e);
        int r = expert_check(experts[e], hidden, inter, what);
        if (r) return r;
    }
    if (shared) {
        int r = expert_check(*shared, hidden, inter, "shared expert");
        if (r) return r;
    }
    const int ne1 = n_experts + 1;
    std::vector<dsv4cu_expert> hexp(experts, experts + n_experts);
    hexp.push_back(shared ? *shared : experts[0]);
    std::vector<CUtensorMap> maps((size_t)6 * ne1);
    std::vector<int> staged((size_t)3 * ne1, 0);
    memset(maps.data(), 0, maps.size() * sizeof(CUtensorMap));
    for (int e = 0; e < ne1; e++) {
        const dsv4cu_qmat *ms[3] = {&hexp[e].w1, &hexp[e].w3, &hexp[e].w2};
        for (int m = 0; m < 3; m++) {
            int r = tmap_encode(ms[m], &maps[6 * e + 2 * m], &maps[6 * e + 2 * m + 1], &staged[3 * e + m]);
            if (r) return r;
        }
    }
    const size_t b_exp = dsv4cu_align256(hexp.size() * sizeof(dsv4cu_expert));
    const size_t b_map = dsv4cu_align256(maps.size() * sizeof(CUtensorMap));
    const size_t b_stg = dsv4cu_align256(staged.size() * sizeof(int));
    void *blk = nullptr;
    cudaError_t ce = cudaMalloc(&blk, b_exp + b_map + b_stg);
    if (ce != cudaSuccess) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "moe_create: %s", cudaGetErrorString(ce));
    char *p = (char *)blk;
    ce = cudaMemcpy(p, hexp.data(), hexp.size() * sizeof(dsv4cu_expert), cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemcpy(p + b_exp, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemcpy(p + b_exp + b_map, staged.data(), staged.size() * sizeof(int), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        cudaFree(blk);
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "moe_create: %s", cudaGetErrorString(ce));
    }
    dsv4cu_moe *L = new dsv4cu_moe;
    L->n_experts = n_experts;
    L->hidden = hidden;
    L->inter = inter;
    L->has_shared = shared != nullptr;
    cudaGetDevice(&L->device);
    L->dev_block = blk;
    L->view.experts = (const dsv4cu_expert *)p;
    L->view.maps = (const CUtensorMap *)(p + b_exp);
    L->view.staged = (const int *)(p + b_exp + b_map);
    L->view.n_experts = n_experts;
    L->view.has_shared = L->has_shared;
    L->mx_ok = 0;
    L->mx_block = nullptr;
    L->smv_ok = 0;
    L->path = DSV4CU_MOE_PATH_AUTO;
    L->smv_block = nullptr;
    L->smv_maps = nullptr;
    if (smv_moe_layer_ok(hexp.data(), n_experts, hidden, inter)) {
        const int rs = smv_moe_prepare(L, hexp.data());
        if (rs) {
            cudaFree(blk);
            delete L;
            return rs;
        }
    }
    const int r = moe_mx_prepare(L, hexp.data());
    if (r && r != DSV4CU_ERR_UNSUPPORTED) {
        cudaFree(L->smv_block);
        cudaFree(blk);
        delete L;
        return r;
    }
    *out = L;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_moe_set_path(dsv4cu_moe *L, int path)
{
    if (!L) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_set_path: NULL layer");
    if (path == DSV4CU_MOE_PATH_TENSOR && !L->mx_ok)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_set_path: layer has no tensor-core path");
    if (path == DSV4CU_MOE_PATH_STREAM && !L->smv_ok)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_set_path: layer has no streamed path");
    if (path < DSV4CU_MOE_PATH_AUTO || path > DSV4CU_MOE_PATH_STREAM)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_set_path: path %d", path);
    L->path = path;
    return DSV4CU_OK;
}

extern "C" void dsv4cu_moe_destroy(dsv4cu_moe *L)
{
    if (!L) return;
    moe_mx_release(L);
    cudaFree(L->smv_block);
    cudaFree(L->dev_block);
    delete L;
}

extern "C" size_t dsv4cu_moe_workspace(const dsv4cu_moe *L, int topk, int nt)
{
    if (!L) return 0;
    const size_t a = moe_decode_workspace(nt, topk, L->n_experts, L->hidden, L->inter, L->has_shared);
    const size_t b = L->mx_ok ? moe_mx_workspace(L, topk, nt) : 0;
    const size_t c = use_stream(L, nt, false) ? smv_moe_workspace(L, topk, nt) : 0;
    return a > b ? (a > c ? a : c) : (b > c ? b : c);
}

extern "C" int dsv4cu_moe_decode_ev(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out, const float *x,
                                    const float *logits, const float *bias, const int64_t *tid2eid,
                                    const int *token_ids, int topk, float route_scale, float limit, int nt,
                                    int *idx_out, float *wts_out, void *stream, void **events)
{
    if (!ctx || !layer || !out || !x || !logits) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: NULL argument");
    if ((idx_out == nullptr) != (wts_out == nullptr))
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: idx_out and wts_out go together");
    if (tid2eid && !token_ids) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: hash routing needs token_ids");
    if (nt < 1 || nt > MOE_MAX_NT) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_decode: nt %d not in 1..%d", nt, MOE_MAX_NT);
    if (topk < 1 || topk > MOE_MAX_TOPK || topk > layer->n_experts)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: topk %d", topk);
    void *ws = nullptr;
    if (use_stream(layer, nt, tid2eid != nullptr)) {
        int r = dsv4cu_ws_get(ctx, smv_moe_workspace(layer, topk, nt), &ws);
        if (r) return r;
        return smv_moe_decode(layer, out, x, logits, bias, tid2eid, token_ids, topk, route_scale, limit, nt, idx_out,
                              wts_out, ws, ctx->status, ctx->sm_count, (cudaStream_t)stream, (cudaEvent_t *)events);
    }
    if (layer->mx_ok) {
        int r = dsv4cu_ws_get(ctx, moe_mx_workspace(layer, topk, nt), &ws);
        if (r) return r;
        return moe_mx_decode(layer, out, x, logits, bias, tid2eid, token_ids, topk, route_scale, limit, nt, idx_out,
                             wts_out, ws, ctx->counters, ctx->status, ctx->sm_count, (cudaStream_t)stream,
                             (cudaEvent_t *)events);
    }
    int r = dsv4cu_ws_get(ctx, moe_decode_workspace(nt, topk, layer->n_experts, layer->hidden, layer->inter,
                                                    layer->has_shared), &ws);
    if (r) return r;
    return moe_decode_run(layer, out, x, logits, bias, tid2eid, token_ids, topk, route_scale, limit, nt, idx_out,
                          wts_out, ws, ctx->counters, ctx->status, (cudaStream_t)stream, (cudaEvent_t *)events);
}

extern "C" int dsv4cu_moe_decode(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out, const float *x,
                                 const float *logits, const float *bias, const int64_t *tid2eid,
                                 const int *token_ids, int topk, float route_scale, float limit, int nt,
                                 int *idx_out, float *wts_out, void *stream)
{
    return dsv4cu_moe_decode_ev(ctx, layer, out, x, logits, bias, tid2eid, token_ids, topk, route_scale, limit, nt,
                                idx_out, wts_out, stream, nullptr);
}

extern "C" size_t dsv4cu_moe_prefill_workspace(const dsv4cu_moe *L, int topk, int nt, int terms)
{
    return (L && L->mx_ok) ? moe_mx_prefill_workspace(L, topk, nt, terms) : 0;
}

extern "C" int dsv4cu_moe_prefill_ev(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out, const float *x,
                                     const float *logits, const float *bias, const int64_t *tid2eid,
                                     const int *token_ids, int topk, float route_scale, float limit, int nt,
                                     int terms, int *idx_out, float *wts_out, void *stream, void **events)
{
    if (!ctx || !layer || !out || !x || !logits) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_prefill: NULL argument");
    if ((idx_out == nullptr) != (wts_out == nullptr))
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_prefill: idx_out and wts_out go together");
    if (tid2eid && !token_ids) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_prefill: hash routing needs token_ids");
    if (nt < 1) return nt == 0 ? DSV4CU_OK : dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_prefill: nt %d", nt);
    if (topk < 1 || topk > MOE_MAX_TOPK || topk > layer->n_experts)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_prefill: topk %d", topk);
    if (!layer->mx_ok)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED,
                                "moe_prefill: the layer's matrices do not qualify for the tensor-core path");
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, moe_mx_prefill_workspace(layer, topk, nt, terms), &ws);
    if (r) return r;
    return moe_mx_prefill(layer, out, x, logits, bias, tid2eid, token_ids, topk, route_scale, limit, nt, terms,
                          idx_out, wts_out, ws, ctx->status, ctx->sm_count, (cudaStream_t)stream,
                          (cudaEvent_t *)events);
}

extern "C" int dsv4cu_moe_prefill(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out, const float *x,
                                  const float *logits, const float *bias, const int64_t *tid2eid,
                                  const int *token_ids, int topk, float route_scale, float limit, int nt, int terms,
                                  int *idx_out, float *wts_out, void *stream)
{
    return dsv4cu_moe_prefill_ev(ctx, layer, out, x, logits, bias, tid2eid, token_ids, topk, route_scale, limit, nt,
                                 terms, idx_out, wts_out, stream, nullptr);
}

extern "C" size_t dsv4cu_moe_rows_workspace(const dsv4cu_moe *L, int nrows)
{
    return (L && L->mx_ok && nrows > 0) ? moe_mx_rows_workspace(L, nrows, nrows) : 0;
}

extern "C" int dsv4cu_moe_rows(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *y, const float *x, long ldx,
                               const int *ids, int nrows, float limit, void *stream)
{
    if (!ctx || !layer || !y || !x || !ids) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_rows: NULL argument");
    if (nrows < 1) return nrows == 0 ? DSV4CU_OK : dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_rows: nrows %d", nrows);
    if (ldx < layer->hidden || ldx % 4)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_rows: ldx %ld (hidden %d, multiple of 4)", ldx, layer->hidden);
    if (!layer->mx_ok)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED,
                                "moe_rows: the layer's matrices do not qualify for the tensor-core path");
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, moe_mx_rows_workspace(layer, nrows, nrows), &ws);
    if (r) return r;
    return moe_mx_rows(layer, y, x, ldx, ids, nrows, nrows, limit, ws, ctx->status, ctx->sm_count,
                       (cudaStream_t)stream);
}

// Device address of a page-locked, mapped host buffer (cudaHostAlloc /
// cudaHostRegister with unified addressing), or NULL for pageable memory.
static const void *mapped_host(const void *p)
{
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return (a.type == cudaMemoryTypeHost && a.devicePointer) ? a.devicePointer : nullptr;
}

// x and the logits from mapped host memory into device staging in one
// coalesced pass (every load in flight at once), after the previous kernel on
// the stream has finished (it may have written these host buffers).
__global__ void __launch_bounds__(1024) stage_in_kernel(float4 *__restrict__ dx, const float4 *__restrict__ hx,
                                                        long nx4, float *__restrict__ dl,
                                                        const float *__restrict__ hl, long nl)
{
    pdl_wait();
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x, stride = (long)gridDim.x * blockDim.x;
    for (long j = i; j < nx4; j += stride) dx[j] = hx[j];
    for (long j = i; j < nl; j += stride) dl[j] = hl[j];
    pdl_trigger();
}

// Workspace and launch of the decode path a layer takes for nt tokens
// without bias, hash routing or index outputs.
static size_t decode_plain_workspace(const dsv4cu_moe *layer, int topk, int nt)
{
    if (use_stream(layer, nt, false)) return smv_moe_workspace(layer, topk, nt);
    if (layer->mx_ok) return moe_mx_workspace(layer, topk, nt);
    return moe_decode_workspace(nt, topk, layer->n_experts, layer->hidden, layer->inter, layer->has_shared);
}
static int decode_plain(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out, const float *x, const float *lg,
                        int topk, float route_scale, float limit, int nt, void *ws, cudaStream_t st)
{
    if (use_stream(layer, nt, false))
        return smv_moe_decode(layer, out, x, lg, nullptr, nullptr, nullptr, topk, route_scale, limit, nt, nullptr,
                              nullptr, ws, ctx->status, ctx->sm_count, st, nullptr);
    if (layer->mx_ok)
        return moe_mx_decode(layer, out, x, lg, nullptr, nullptr, nullptr, topk, route_scale, limit, nt, nullptr,
                             nullptr, ws, ctx->counters, ctx->status, ctx->sm_count, st, nullptr);
    return moe_decode_run(layer, out, x, lg, nullptr, nullptr, nullptr, topk, route_scale, limit, nt, nullptr, nullptr,
                          ws, ctx->counters, ctx->status, st, nullptr);
}

// Host buffers in and out, all on the stream, nothing synchronised. With
// page-locked host buffers on the streamed or tensor-core path one staging
// kernel reads x and the logits across the bus and the combine writes the
// output straight into host memory (no copy operations between the step's
// launches); otherwise x and logits are copied into staging after the step's
// workspace and the output is copied back.
extern "C" int dsv4cu_moe_decode_host(dsv4cu_ctx *ctx, const dsv4cu_moe *layer, float *out_host,
                                      const float *x_host, const float *logits_host, int topk, float route_scale,
                                      float limit, int nt, void *stream)
{
    if (!ctx || !layer || !out_host || !x_host || !logits_host)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode_host: NULL argument");
    if (nt < 1 || nt > MOE_MAX_NT) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_decode_host: nt %d", nt);
    if (topk < 1 || topk > MOE_MAX_TOPK || topk > layer->n_experts)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode_host: topk %d", topk);
    const size_t need = decode_plain_workspace(layer, topk, nt);
    const size_t xb = (size_t)nt * layer->hidden * 4, lb = (size_t)nt * layer->n_experts * 4;
    const size_t base = dsv4cu_align256(need);
    cudaStream_t st = (cudaStream_t)stream;
    if ((layer->mx_ok || use_stream(layer, nt, false)) && xb % 16 == 0) {
        const void *mx = mapped_host(x_host), *ml = mapped_host(logits_host), *mo = mapped_host(out_host);
        if (mx && ml && mo && ((uintptr_t)mx & 15u) == 0) {
            void *ws = nullptr;
            int r = dsv4cu_ws_get(ctx, base + dsv4cu_align256(xb) + dsv4cu_align256(lb), &ws);
            if (r) return r;
            float *dx = (float *)((char *)ws + base);
            float *dl = (float *)((char *)dx + dsv4cu_align256(xb));
            const long nx4 = (long)(xb / 16), nl = (long)(lb / 4);
            const long work = nx4 > nl ? nx4 : nl;
            const unsigned blocks = (unsigned)((work + 1023) / 1024 < 32 ? (work + 1023) / 1024 : 32);
            DSV4CU_CUDA_TRY(launch_pdl(stage_in_kernel, dim3(blocks), dim3(1024), 0, st, (float4 *)dx,
                                       (const float4 *)mx, nx4, dl, (const float *)ml, nl));
            return decode_plain(ctx, layer, (float *)mo, dx, dl, topk, route_scale, limit, nt, ws, st);
        }
    }
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, base + dsv4cu_align256(xb) * 2 + dsv4cu_align256(lb), &ws);
    if (r) return r;
    float *dx = (float *)((char *)ws + base);
    float *dl = (float *)((char *)dx + dsv4cu_align256(xb));
    float *dout = (float *)((char *)dl + dsv4cu_align256(lb));
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(dx, x_host, xb, cudaMemcpyHostToDevice, st));
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(dl, logits_host, lb, cudaMemcpyHostToDevice, st));
    r = decode_plain(ctx, layer, dout, dx, dl, topk, route_scale, limit, nt, ws, st);
    if (r) return r;
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(out_host, dout, xb, cudaMemcpyDeviceToHost, st));
    return DSV4CU_OK;
}
