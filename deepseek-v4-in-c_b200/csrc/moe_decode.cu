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
#include <stdio.h>

#include "common.cuh"
#include "ctx.h"
#include "gemv.h"
#include "gemv_core.cuh"
#include "router.cuh"

namespace dsv4cu {

constexpr int MOE_MAX_NT = 64;
constexpr int MOE_MAX_TOPK = 16;

struct MoeWs {
    uint16_t *xh, *xl;    // [nt][hidden]
    float *xs;            // [nt][hidden/32]
    int *idx;             // [nt][topk]
    float *wts;           // [nt][topk]
    int *meta;            // [0] n_buckets, [1] error flag
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
    const float *__restrict__ x, const float *__restrict__ logits, const float *__restrict__ bias,
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
    for (int t = warp; t < nt; t += nwarps) {
        route_token_warp(logits + (size_t)t * n_experts, bias, tid2eid,
                         token_ids ? token_ids[t] : 0, n_experts, topk, route_scale,
                         ws.idx + t * topk, ws.wts + t * topk, nullptr, nullptr);
    }
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

// Resolve bucket b of this launch: expert descriptor, first slot, slot count.
DSV4CU_DEV bool mat_ok(const dsv4cu_qmat &q, int rows, int cols)
{
    if (q.rows != rows || q.cols != cols || !q.w || !q.s || q.blk_r <= 0 || q.blk_c <= 0) return false;
    if ((uintptr_t)q.w & 15u) return false;   // 16-byte weight loads
    if (q.wdt == DSV4CU_WFP4) return q.blk_c % 32 == 0;
    if (q.wdt == DSV4CU_WFP8) return q.blk_c % 16 == 0;
    return false;
}

DSV4CU_DEV bool expert_ok(const dsv4cu_expert &e, int hidden, int inter)
{
    return mat_ok(e.w1, inter, hidden) && mat_ok(e.w3, inter, hidden) && mat_ok(e.w2, hidden, inter) &&
           e.w1.wdt == e.w3.wdt;
}

DSV4CU_DEV bool moe_bucket(const MoeWs &ws, int b, int nbmax, const dsv4cu_expert *experts,
                           const dsv4cu_expert &shared, int has_shared, int hidden, int inter,
                           const dsv4cu_expert *&ex, int &s0, int &cnt)
{
    const int nb = ws.meta[0];
    if (b == nbmax) {            // the shared-expert bucket is always the last one
        if (!has_shared) return false;
        ex = &shared;
        s0 = ws.b_off[nb];
        cnt = ws.b_off[nb + 1] - s0;
        return cnt > 0;
    }
    if (b >= nb) return false;
    ex = experts + ws.b_expert[b];
    s0 = ws.b_off[b];
    cnt = ws.b_off[b + 1] - s0;
    // Routed descriptors live in device memory and are checked here: a
    // descriptor whose shape or format this kernel cannot read is skipped and
    // flagged (meta[1] bit 1), never read out of shape.
    if (!expert_ok(*ex, hidden, inter)) {
        atomicOr(ws.meta + 1, 2);
        return false;
    }
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

template <int FMT, int NT>
DSV4CU_DEV void moe_gate_up_body(const dsv4cu_expert &ex, int row0, const XArgs &xa, int nvalid,
                                 float (*red)[2][2][4][16], int warp)
{
    // warp -> (matrix w1|w3, 16-row half, K half)
    const int mat = (warp >> 2) & 1, rs = (warp >> 1) & 1, kh = warp & 1;
    const MatArgs m = mat_of(mat ? ex.w3 : ex.w1);
    const int ns = (m.row_bytes + 63) >> 6;
    const int sb = kh * ns / 2, se = (kh + 1) * ns / 2;
    float acc[NT][2];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.0f;
    gemv_tile16<FMT, NT, 2>(m, row0 + rs * 16, sb, se, xa, nvalid, acc);
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < NT; t++) {
        const float s0 = quad_sum(acc[t][0]), s1 = quad_sum(acc[t][1]);
        if ((lane & 3) == 0) {
            red[mat][rs][kh][t][lane >> 2] = s0;
            red[mat][rs][kh][t][(lane >> 2) + 8] = s1;
        }
    }
}

// grid (inter/32, nbmax + 1), block 256 (8 warps).
__global__ void __launch_bounds__(256) moe_gate_up_kernel(MoeWs ws, const dsv4cu_expert *__restrict__ experts,
                                                          dsv4cu_expert shared, int has_shared, int nbmax,
                                                          int hidden, int inter, float limit)
{
    __shared__ float red[2][2][2][4][16];   // [mat][row half][K half][token][row]
    __shared__ float mid[4][32];
    const dsv4cu_expert *ex;
    int s0, cnt;
    if (!moe_bucket(ws, blockIdx.y, nbmax, experts, shared, has_shared, hidden, inter, ex, s0, cnt)) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * 32;
    const int fmt = ex->w1.wdt;

    for (int c0 = 0; c0 < cnt; c0 += 4) {
        const int nv = min(4, cnt - c0);
        XArgs xa;
        xa.xh = ws.xh;
        xa.xl = ws.xl;
        xa.xs = ws.xs;
        xa.ldx = hidden;
        xa.tok = ws.b_tok + s0 + c0;
        if (fmt == DSV4CU_WFP4) {
            if (nv == 1) moe_gate_up_body<DSV4CU_WFP4, 1>(*ex, row0, xa, nv, red, warp);
            else moe_gate_up_body<DSV4CU_WFP4, 4>(*ex, row0, xa, nv, red, warp);
        } else {
            if (nv == 1) moe_gate_up_body<DSV4CU_WFP8, 1>(*ex, row0, xa, nv, red, warp);
            else moe_gate_up_body<DSV4CU_WFP8, 4>(*ex, row0, xa, nv, red, warp);
        }
        __syncthreads();
        // SwiGLU (dsv4_ops.c:61-79): up clamped both ways, gate from above only.
        if (threadIdx.x < nv * 32) {
            const int t = threadIdx.x >> 5, r = threadIdx.x & 31, rs = r >> 4, rr = r & 15;
            const float g0 = red[0][rs][0][t][rr] + red[0][rs][1][t][rr];
            const float u0 = red[1][rs][0][t][rr] + red[1][rs][1][t][rr];
            float g = g0, u = u0;
            if (limit > 0.0f) {
                u = fminf(fmaxf(u, -limit), limit);
                g = fminf(g, limit);
            }
            mid[t][r] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
        }
        __syncthreads();
        // mid -> f16 hi/lo operand for phase 2; one warp per token, lane = row.
        if (warp < nv) {
            const int t = warp, slot = s0 + c0 + t;
            const float v = mid[t][lane];
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
            ws.mh[(size_t)slot * inter + row0 + lane] = __half_as_ushort(hh);
            ws.ml[(size_t)slot * inter + row0 + lane] = __half_as_ushort(lh);
            if (lane == 0) ws.mxs[(size_t)slot * (inter >> 5) + (row0 >> 5)] = ldexpf(1.0f, -P);
        }
        __syncthreads();
    }
}

template <int FMT, int NT>
DSV4CU_DEV void moe_down_body(const dsv4cu_qmat &q, int row0, const XArgs &xa, int nvalid,
                              float (*red)[4][16], int warp, int nw)
{
    const MatArgs m = mat_of(q);
    const int ns = (m.row_bytes + 63) >> 6;
    const int sb = warp * ns / nw, se = (warp + 1) * ns / nw;
    float acc[NT][2];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.0f;
    gemv_tile16<FMT, NT, 2>(m, row0, sb, se, xa, nvalid, acc);
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < NT; t++) {
        const float s0 = quad_sum(acc[t][0]), s1 = quad_sum(acc[t][1]);
        if ((lane & 3) == 0) {
            red[warp][t][lane >> 2] = s0;
            red[warp][t][(lane >> 2) + 8] = s1;
        }
    }
}

// grid (hidden/16, nbmax + 1), block 128 (4 warps splitting K).
__global__ void __launch_bounds__(128) moe_down_kernel(MoeWs ws, const dsv4cu_expert *__restrict__ experts,
                                                       dsv4cu_expert shared, int has_shared, int nbmax,
                                                       int hidden, int inter, int nt, int topk,
                                                       float *__restrict__ out, int *__restrict__ counters)
{
    __shared__ float red[4][4][16];
    __shared__ int last;
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int row0 = blockIdx.x * 16;
    const dsv4cu_expert *ex;
    int s0, cnt;
    if (moe_bucket(ws, blockIdx.y, nbmax, experts, shared, has_shared, hidden, inter, ex, s0, cnt)) {
        const int fmt = ex->w2.wdt;
        for (int c0 = 0; c0 < cnt; c0 += 4) {
            const int nv = min(4, cnt - c0);
            XArgs xa;
            xa.xh = ws.mh + (size_t)(s0 + c0) * inter;
            xa.xl = ws.ml + (size_t)(s0 + c0) * inter;
            xa.xs = ws.mxs + (size_t)(s0 + c0) * (inter >> 5);
            xa.ldx = inter;
            xa.tok = nullptr;
            if (fmt == DSV4CU_WFP4) {
                if (nv == 1) moe_down_body<DSV4CU_WFP4, 1>(ex->w2, row0, xa, nv, red, warp, nw);
                else moe_down_body<DSV4CU_WFP4, 4>(ex->w2, row0, xa, nv, red, warp, nw);
            } else {
                if (nv == 1) moe_down_body<DSV4CU_WFP8, 1>(ex->w2, row0, xa, nv, red, warp, nw);
                else moe_down_body<DSV4CU_WFP8, 4>(ex->w2, row0, xa, nv, red, warp, nw);
            }
            __syncthreads();
            if (threadIdx.x < nv * 16) {
                const int t = threadIdx.x >> 4, r = threadIdx.x & 15;
                float s = 0.0f;
                for (int w = 0; w < nw; w++) s += red[w][t][r];
                ws.ypart[(size_t)(s0 + c0 + t) * hidden + row0 + r] = s;
            }
            __syncthreads();
        }
    }
    // The last CTA of this 16-row slice combines, in k order, then the shared expert.
    __threadfence();
    if (threadIdx.x == 0) last = (atomicAdd(&counters[blockIdx.x], 1) == (int)gridDim.y - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int nb = ws.meta[0];
    for (int i = threadIdx.x; i < nt * 16; i += blockDim.x) {
        const int t = i >> 4, row = row0 + (i & 15);
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
    if (threadIdx.x == 0) counters[blockIdx.x] = 0;
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

int moe_decode_run(float *out, const float *x, const float *logits, const float *bias,
                   const int64_t *tid2eid, const int *token_ids, const dsv4cu_expert *experts,
                   int n_experts, const dsv4cu_expert *shared, int topk, float route_scale, int hidden,
                   int inter, float limit, int nt, int *idx_out, float *wts_out, void *wsp,
                   int *counters, cudaStream_t st, cudaEvent_t *ev = nullptr)
{
    const int has_shared = shared != nullptr;
    MoeWs ws;
    moe_ws_layout(nt, topk, n_experts, hidden, inter, has_shared, (char *)wsp, &ws);
    const int nbmax = min(nt * topk, n_experts);
    const int xblocks = min(64, max(1, nt * (hidden / 32) / 32));
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
    moe_prologue_kernel<<<1 + xblocks, 1024, 0, st>>>(x, logits, bias, tid2eid, token_ids, n_experts,
                                                      topk, route_scale, hidden, nt, has_shared, ws,
                                                      idx_out, wts_out);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));
    dsv4cu_expert sh{};
    if (has_shared) sh = *shared;
    moe_gate_up_kernel<<<dim3(inter / 32, nbmax + 1), 256, 0, st>>>(ws, experts, sh, has_shared, nbmax,
                                                                    hidden, inter, limit);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[2], st));
    moe_down_kernel<<<dim3(hidden / 16, nbmax + 1), 128, 0, st>>>(ws, experts, sh, has_shared, nbmax,
                                                                  hidden, inter, nt, topk, out, counters);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[3], st));
    return DSV4CU_OK;
}

size_t moe_decode_workspace(int nt, int topk, int n_experts, int hidden, int inter, int has_shared)
{
    return moe_ws_layout(nt, topk, n_experts, hidden, inter, has_shared, nullptr, nullptr);
}

static bool moe_mat_ok(const dsv4cu_qmat &q, int rows, int cols)
{
    if (q.rows != rows || q.cols != cols || !q.w || !q.s || ((uintptr_t)q.w & 15u)) return false;
    if (q.wdt == DSV4CU_WFP4) return q.blk_c > 0 && q.blk_c % 32 == 0 && q.blk_r > 0;
    if (q.wdt == DSV4CU_WFP8) return q.blk_c > 0 && q.blk_c % 16 == 0 && q.blk_r > 0;
    return false;
}

int moe_decode_check(const dsv4cu_expert *shared, int n_experts, int topk, int hidden, int inter, int nt)
{
    if (nt < 1 || nt > MOE_MAX_NT) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_decode: nt %d not in 1..%d", nt, MOE_MAX_NT);
    if (topk < 1 || topk > MOE_MAX_TOPK) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: topk %d", topk);
    if (n_experts < topk || n_experts > 32 * RMAX_PER_LANE) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: n_experts %d", n_experts);
    if (hidden % 32 || inter % 32 || hidden <= 0 || inter <= 0)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_decode: hidden/inter must be multiples of 32");
    if (hidden / 16 > DSV4CU_MAX_COUNTERS) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_decode: hidden too large");
    if (shared) {
        if (!moe_mat_ok(shared->w1, inter, hidden) || !moe_mat_ok(shared->w3, inter, hidden) ||
            !moe_mat_ok(shared->w2, hidden, inter) || shared->w1.wdt != shared->w3.wdt)
            return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: shared expert shapes/formats");
    }
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_moe_decode_ev(dsv4cu_ctx *ctx, float *out, const float *x, const float *logits,
                                    const float *bias, const int64_t *tid2eid, const int *token_ids,
                                    const dsv4cu_expert *experts, int n_experts, const dsv4cu_expert *shared,
                                    int topk, float route_scale, int hidden, int inter, float limit, int nt,
                                    int *idx_out, float *wts_out, void *stream, void **events)
{
    if (!ctx || !out || !x || !logits || !experts) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: NULL argument");
    if ((idx_out == nullptr) != (wts_out == nullptr)) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: idx_out and wts_out go together");
    if (tid2eid && !token_ids) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_decode: hash routing needs token_ids");
    int r = moe_decode_check(shared, n_experts, topk, hidden, inter, nt);
    if (r) return r;
    void *ws = nullptr;
    r = dsv4cu_ws_get(ctx, moe_decode_workspace(nt, topk, n_experts, hidden, inter, shared != nullptr), &ws);
    if (r) return r;
    return moe_decode_run(out, x, logits, bias, tid2eid, token_ids, experts, n_experts, shared, topk,
                          route_scale, hidden, inter, limit, nt, idx_out, wts_out, ws, ctx->counters,
                          (cudaStream_t)stream, (cudaEvent_t *)events);
}

extern "C" int dsv4cu_moe_decode(dsv4cu_ctx *ctx, float *out, const float *x, const float *logits,
                                 const float *bias, const int64_t *tid2eid, const int *token_ids,
                                 const dsv4cu_expert *experts, int n_experts, const dsv4cu_expert *shared,
                                 int topk, float route_scale, int hidden, int inter, float limit, int nt,
                                 int *idx_out, float *wts_out, void *stream)
{
    return dsv4cu_moe_decode_ev(ctx, out, x, logits, bias, tid2eid, token_ids, experts, n_experts, shared,
                                topk, route_scale, hidden, inter, limit, nt, idx_out, wts_out, stream, nullptr);
}
