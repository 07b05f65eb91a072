// moe_mx.cu - one MoE layer decode step on the tcgen05 block-scaled GEMM.
//
// Reference: dsv4_layer_moe (src/70_decode/dsv4_layer.c:48-117) from the router
// logits on, with dsv4_route (dsv4_ops.c:117-156), dsv4_expert_forward
// (dsv4_ops.c:85-93), dsv4_swiglu (dsv4_ops.c:61-79) and the k-order combine
// (dsv4_layer.c:109-116).
//
// Five launches, stream-ordered:
//   prep     every CTA routes the tokens (one warp per token) and buckets the
//            (token, k) pairs by expert in ascending expert order with tokens
//            ascending inside a bucket (the layout of union_prepare,
//            src/80_prefill/dsv4_prefill_union.c:30-52), the shared expert's
//            bucket last, and cuts the buckets into column tiles of tpt slots;
//            CTA 0 publishes the tables, all CTAs write the gate/up B operand
//            (the slots' tokens as e4m3 terms).
//   gate/up  mx_kernel over (column tile, 128-row tile, w1 | w3): per-slot
//            gate and up rows.
//   swiglu   SwiGLU of every slot written as e4m3 terms: the down B operand.
//   down     mx_kernel over (column tile, 128-row tile of w2): per-slot rows.
//   combine  per token the routed pairs in k order with the routing weights,
//            plus the shared expert unweighted.
// Every weight byte of the touched experts is read once per step per column
// tile (one column tile per expert at batch 1). No step depends on the order
// in which CTAs finish: the results are the same on every run.
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "moe.h"
#include "mx_kernel.cuh"
#include "mxgemm.h"
#include "router.cuh"

namespace dsv4cu {

constexpr int MX_TERMS = 4;         // activation terms (results within ~1e-6 of fp32)
constexpr int MXMOE_MAX_NT = 64;
constexpr int MXMOE_MAX_TOPK = 16;
constexpr int MXMOE_FUSE_COMBINE_NT = 4;   // tokens a fused-combine thread loops over at most

// Workspace of one step.
struct MxMoeWs {
    int *idx;            // [nt][topk]
    float *wts;          // [nt][topk]
    int *pos;            // [nt][topk] bucket slot of pair (t, k), -1 = dropped
    int *meta;           // [0] routed buckets, [1] bad-route flag, [2] column tiles
    int *b_expert;       // [nbmax]
    int *b_off;          // [nbmax + 2]
    int *b_tok;          // [npairs] token of each slot (shared slots last)
    int *c_slot0, *c_cnt, *c_expert;   // [max_tiles] column tiles
    uint8_t *xq1, *sfb1; // gate/up B operand and its scale blocks
    uint8_t *xq2, *sfb2; // down B operand and its scale blocks
    float *gu;           // [npairs][2][inter] gate (w1) and up (w3) rows of each slot
    float *ypart;        // [npairs][hidden] down projection of each slot
    // Arrival counters of the fused epilogues, zeroed by the decode prep
    // kernel: [max_tiles][inter / 128] gate/up pairs (w1 and w3 tile of one
    // column tile and row tile), then [hidden / 128] down row tiles.
    int *pcnt;
    int npcnt;
};

struct MxMoeShape {
    int nt, topk, n_experts, hidden, inter, has_shared;
    int NB, tpt, KB, nbb, max_tiles, npairs, nbmax;
};

static MxMoeShape mxmoe_shape(const dsv4cu_moe *L, int topk, int nt, int sms)
{
    MxMoeShape s;
    s.nt = nt;
    s.topk = topk;
    s.n_experts = L->n_experts;
    s.hidden = L->hidden;
    s.inter = L->inter;
    s.has_shared = L->has_shared;
    // A bucket never holds more than nt slots: size the column tile for that.
    if (nt <= 2) { s.NB = 8; s.KB = 4; }
    else if (nt <= 4) { s.NB = 16; s.KB = 4; }
    else { s.NB = 32; s.KB = 2; }
    s.tpt = s.NB <= 16 ? s.NB / MX_TERMS : (s.NB / MX_TERMS) / 8 * 8;
    s.nbb = (s.NB + 127) / 128;
    s.npairs = nt * topk + (s.has_shared ? nt : 0);
    s.nbmax = min(nt * topk, s.n_experts);
    // sum over buckets of ceil(cnt / tpt) <= slots / tpt + buckets
    s.max_tiles = (nt * topk) / s.tpt + s.nbmax + (s.has_shared ? nt / s.tpt + 1 : 0) + 1;
    (void)sms;
    return s;
}

static size_t mxmoe_layout(const MxMoeShape &s, char *base, MxMoeWs *w)
{
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = base ? base + off : nullptr;
        off += dsv4cu_align256(bytes);
        return p;
    };
    MxMoeWs t;
    t.idx = (int *)take((size_t)s.nt * s.topk * 4);
    t.wts = (float *)take((size_t)s.nt * s.topk * 4);
    t.pos = (int *)take((size_t)s.nt * s.topk * 4);
    t.meta = (int *)take(64);
    t.b_expert = (int *)take((size_t)s.nbmax * 4 + 4);
    t.b_off = (int *)take(((size_t)s.nbmax + 2) * 4);
    t.b_tok = (int *)take((size_t)s.npairs * 4);
    t.c_slot0 = (int *)take((size_t)s.max_tiles * 4);
    t.c_cnt = (int *)take((size_t)s.max_tiles * 4);
    t.c_expert = (int *)take((size_t)s.max_tiles * 4);
    t.xq1 = (uint8_t *)take((size_t)s.max_tiles * s.NB * s.hidden);
    t.sfb1 = (uint8_t *)take((size_t)s.max_tiles * (s.hidden / 128) * s.nbb * 512);
    t.xq2 = (uint8_t *)take((size_t)s.max_tiles * s.NB * s.inter);
    t.sfb2 = (uint8_t *)take((size_t)s.max_tiles * (s.inter / 128) * s.nbb * 512);
    t.gu = (float *)take((size_t)s.npairs * 2 * s.inter * 4);
    t.ypart = (float *)take((size_t)s.npairs * s.hidden * 4);
    t.npcnt = s.max_tiles * (s.inter / 128) + s.hidden / 128;
    t.pcnt = (int *)take((size_t)t.npcnt * 4);
    if (w) *w = t;
    return off;
}

// ------------------------------------------------------------ prep kernel
// Exclusive prefix sum of a[0..n) in shared memory by one warp (n <= 32 * 32);
// returns the total to every lane.
DSV4CU_DEV int warp_scan_excl(int *a, int n)
{
    const int lane = threadIdx.x & 31, seg = (n + 31) >> 5;
    const int b0 = min(n, lane * seg), b1 = min(n, b0 + seg);
    int loc = 0;
    for (int i = b0; i < b1; i++) loc += a[i];
    int inc = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += v;
    }
    int run = inc - loc;
    for (int i = b0; i < b1; i++) {
        const int v = a[i];
        a[i] = run;
        run += v;
    }
    return __shfl_sync(0xFFFFFFFFu, inc, 31);
}

constexpr int PREP_MAX_PAIRS = MXMOE_MAX_NT * MXMOE_MAX_TOPK;            // 1024
constexpr int PREP_MAX_SLOTS = PREP_MAX_PAIRS + MXMOE_MAX_NT;
constexpr int PREP_MAX_EXPERTS = 32 * RMAX_PER_LANE;                      // 512
constexpr int PREP_MAX_TILES = PREP_MAX_PAIRS / 2 + PREP_MAX_EXPERTS + MXMOE_MAX_NT + 2;

// One 128-wide chunk c of a source row of length K, split into `terms`
// e4m3 terms, written as columns j * tpt + tl of column tile i of a B operand
// (rows [tile][NB][K], scale blocks [tile][K / 128][NBB][512]). Whole warp.
DSV4CU_DEV void mxmoe_split_row_chunk(const float *__restrict__ src, int K, int c, int i, int tl, int terms, int tpt,
                                      int NB, int nbb, uint8_t *__restrict__ xq, uint8_t *__restrict__ sfb)
{
    const int lane = threadIdx.x & 31;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = src[c * 128 + 4 * lane + k];
    uint32_t q[4];
    uint8_t sb[4];
    mx_split128(v, terms, q, sb);
    uint8_t *row[4], *sf[4];
    int step[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int n = j * tpt + tl;
        row[j] = xq + ((size_t)i * NB + n) * K + c * 128;
        sf[j] = sfb + ((size_t)i * (K >> 7) + c) * nbb * 512 + mx_sfb_offset(n, 0);
        step[j] = 1;
    }
    mx_store128(q, sb, terms, row, sf, step);
}

// Every CTA routes all nt tokens (one warp per token), buckets the (token, k)
// pairs by expert in ascending expert order with tokens ascending inside a
// bucket (the layout of union_prepare, src/80_prefill/dsv4_prefill_union.c:
// 30-52), shared expert's bucket last, and cuts the buckets into column tiles
// of tpt slots - all in shared memory, identically in every CTA. CTA 0
// publishes the tables; then all CTAs write their share of the gate/up B
// operand: one warp per (column tile, column, 32-wide K block).
constexpr int PREP_THREADS = 512;     // 128 registers a thread: the tables stay out of local memory

__global__ void __launch_bounds__(PREP_THREADS) mxmoe_prep_kernel(
    const float *__restrict__ tab, const float *__restrict__ x, const float *__restrict__ logits,
    const float *__restrict__ bias, const int64_t *__restrict__ tid2eid, const int *__restrict__ token_ids,
    int n_experts, int topk, float route_scale, int nt, int hidden, int has_shared, int terms, int tpt, int NB,
    MxMoeWs ws, int *__restrict__ idx_out, float *__restrict__ wts_out)
{
    __shared__ int s_idx[PREP_MAX_PAIRS];
    __shared__ float s_wts[PREP_MAX_PAIRS];
    __shared__ int s_pos[PREP_MAX_PAIRS];
    // Scratch: router scores first (2 x 1024 floats), then per-expert tables.
    __shared__ __align__(16) int s_scratch[2048];
    __shared__ int s_cnt[PREP_MAX_EXPERTS + 2];
    __shared__ int s_bexp[PREP_MAX_EXPERTS + 2], s_boff[PREP_MAX_EXPERTS + 3];
    __shared__ int s_btok[PREP_MAX_SLOTS];
    __shared__ int s_tslot[PREP_MAX_TILES], s_tcnt[PREP_MAX_TILES], s_texp[PREP_MAX_TILES];
    __shared__ int s_sorted[32];
    __shared__ int s_nb, s_ntiles, s_bad;
    int *s_off = s_scratch, *s_bid = s_scratch + 514, *s_btiles = s_scratch + 1028;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int npairs = nt * topk;
    pdl_wait();       // x and the logits come from the previous kernel
    pdl_trigger();

    // ---- routing (dsv4_route, src/10_compute/dsv4_ops.c:117-156)
    bool warp_route = tid2eid != nullptr || nt * n_experts > (int)blockDim.x;
    if (!warp_route) {
        // Small batches: one thread per (token, expert). Without NaN scores,
        // repeated arg-max with strict '>' in increasing index order selects
        // exactly the experts of rank < topk under (score desc, index asc),
        // in that rank order.
        float *r_s = (float *)s_scratch, *r_o = (float *)s_scratch + 1024;
        const int t = threadIdx.x / n_experts, e = threadIdx.x - t * n_experts;
        const bool act = t < nt;
        bool nan = false;
        if (act) {
            const float o = router_score(logits[(size_t)t * n_experts + e], tab);
            const float sv = bias ? __fadd_rn(o, bias[e]) : o;
            r_o[threadIdx.x] = o;
            r_s[threadIdx.x] = sv;
            nan = isnan(sv);
        }
        warp_route = __syncthreads_or(nan);
        if (!warp_route) {
            // Rank of (t, e) among its token's scores, `per` adjacent threads
            // counting a quarter / half of the experts each (4-wide loads).
            const int items = nt * n_experts;
            int per = 1;
            while (per < 4 && items * per * 2 <= (int)blockDim.x && n_experts % (8 * per) == 0) per *= 2;
            const int item = threadIdx.x / per, part = threadIdx.x % per;
            if (item < items) {
                const int ti = item / n_experts, ei = item - ti * n_experts, span = n_experts / per;
                const float v = r_s[item];
                const float *row = r_s + ti * n_experts + part * span;
                const int q0 = part * span;
                int r = 0;
                if (span % 4 == 0) {
#pragma unroll 2
                    for (int q = 0; q < span; q += 4) {
                        const float4 w = *reinterpret_cast<const float4 *>(row + q);
                        const int qq = q0 + q;
                        r += (w.x > v) || (w.x == v && qq < ei);
                        r += (w.y > v) || (w.y == v && qq + 1 < ei);
                        r += (w.z > v) || (w.z == v && qq + 2 < ei);
                        r += (w.w > v) || (w.w == v && qq + 3 < ei);
                    }
                } else {
                    for (int q = 0; q < span; q++) r += (row[q] > v) || (row[q] == v && q0 + q < ei);
                }
                for (int o2 = 1; o2 < per; o2 <<= 1) r += __shfl_xor_sync(__activemask(), r, o2);
                if (part == 0 && r < topk) s_idx[ti * topk + r] = ei;
            }
            __syncthreads();
            if ((int)threadIdx.x < nt) {
                // Weights from the unbiased scores; double sum in k order.
                const int tt = threadIdx.x;
                double sum = 0.0;
                for (int k = 0; k < topk; k++) sum = __dadd_rn(sum, (double)r_o[tt * n_experts + s_idx[tt * topk + k]]);
                const float inv = (sum != 0.0) ? (float)__drcp_rn(sum) : 0.0f;
                for (int k = 0; k < topk; k++)
                    s_wts[tt * topk + k] =
                        __fmul_rn(__fmul_rn(r_o[tt * n_experts + s_idx[tt * topk + k]], inv), route_scale);
            }
        }
        __syncthreads();
    }
    if (warp_route) {
        // Hash layers, NaN scores, larger batches: one warp per token.
        for (int t = warp; t < nt; t += nwarps)
            route_token_warp(tab, logits + (size_t)t * n_experts, bias, tid2eid, token_ids ? token_ids[t] : 0,
                             n_experts, topk, route_scale, s_idx + t * topk, s_wts + t * topk, nullptr, nullptr);
        __syncthreads();
    }

    // ---- buckets and column tiles
    if (npairs <= 32) {
        // One warp sorts the pairs by (expert, pair index): slot = rank.
        if (warp == 0) {
            const int p = lane;
            const bool live = p < npairs;
            const int e0 = live ? s_idx[p] : -1;
            const bool ok = live && e0 >= 0 && e0 < n_experts;
            const int key = ok ? e0 : 0x7FFFFFFF;
            int rank = 0;
#pragma unroll 1
            for (int q = 0; q < npairs; q++) {      // a short loop: this code runs once per launch
                const int kq = __shfl_sync(0xFFFFFFFFu, key, q);
                rank += kq < key || (kq == key && q < p);
            }
            const int routed = __popc(__ballot_sync(0xFFFFFFFFu, ok));
            const bool bad = __any_sync(0xFFFFFFFFu, live && !ok);
            if (ok) {
                s_pos[p] = rank;
                s_btok[rank] = p / topk;
                s_sorted[rank] = e0;
            } else if (live) {
                s_pos[p] = -1;
            }
            __syncwarp();
            const int el = lane < routed ? s_sorted[lane] : -1;
            const bool head = lane < routed && (lane == 0 || s_sorted[lane - 1] != el);
            const unsigned hm = __ballot_sync(0xFFFFFFFFu, head);
            const int nb = __popc(hm);
            if (head) {
                const int bi = __popc(hm & ((1u << lane) - 1u));
                s_bexp[bi] = el;
                s_boff[bi] = lane;
            }
            if (has_shared)
                for (int t = lane; t < nt; t += 32) s_btok[routed + t] = t;
            __syncwarp();
            if (lane == 0) {
                s_nb = nb;
                s_bad = bad;
                s_boff[nb] = routed;
                s_boff[nb + 1] = routed + (has_shared ? nt : 0);
                int n = 0;
                for (int b = 0; b < nb + (has_shared ? 1 : 0); b++) {
                    const int s0 = s_boff[b], c = s_boff[b + 1] - s0, e = b < nb ? s_bexp[b] : n_experts;
                    for (int j = 0; j < c && n < PREP_MAX_TILES; j += tpt, n++) {
                        s_tslot[n] = s0 + j;
                        s_tcnt[n] = min(tpt, c - j);
                        s_texp[n] = e;
                    }
                }
                s_ntiles = n;
            }
        }
    } else {
    for (int e = threadIdx.x; e <= n_experts; e += blockDim.x) s_cnt[e] = 0;
    if (threadIdx.x == 0) s_bad = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
        const int e = s_idx[p];
        if (e < 0 || e >= n_experts) atomicOr(&s_bad, 1);
        else atomicAdd(&s_cnt[e], 1);
    }
    __syncthreads();
    if (warp == 0) {
        // Slot offsets per expert, bucket index per expert (experts with pairs).
        for (int e = lane; e < n_experts; e += 32) {
            s_off[e] = s_cnt[e];
            s_bid[e] = s_cnt[e] > 0;
        }
        __syncwarp();
        const int routed = warp_scan_excl(s_off, n_experts);
        const int nb = warp_scan_excl(s_bid, n_experts);
        __syncwarp();
        for (int e = lane; e < n_experts; e += 32)
            if (s_cnt[e]) {
                s_bexp[s_bid[e]] = e;
                s_boff[s_bid[e]] = s_off[e];
            }
        if (lane == 0) {
            s_nb = nb;
            s_boff[nb] = routed;
            s_boff[nb + 1] = routed + (has_shared ? nt : 0);
        }
        // Rank of each pair inside its bucket: pairs are in (t, k) order, so a
        // running count per expert over 32-pair chunks keeps tokens ascending.
        for (int e = lane; e < n_experts; e += 32) s_cnt[e] = 0;
        __syncwarp();
        for (int c0 = 0; c0 < npairs; c0 += 32) {
            const int p = c0 + lane;
            const int e = p < npairs ? s_idx[p] : -1;
            const bool ok = e >= 0 && e < n_experts;
            const unsigned same = __match_any_sync(0xFFFFFFFFu, ok ? e : -1);
            const int before = __popc(same & ((1u << lane) - 1u));
            const int base = ok ? s_cnt[e] : 0;
            __syncwarp();
            if (ok) {
                const int slot = s_off[e] + base + before;
                s_pos[p] = slot;
                s_btok[slot] = p / topk;
                if (before == __popc(same) - 1) s_cnt[e] = base + before + 1;   // last lane of the group
            } else if (p < npairs) {
                s_pos[p] = -1;
            }
            __syncwarp();
        }
        if (has_shared)
            for (int t = lane; t < nt; t += 32) s_btok[routed + t] = t;
        // Column tiles per bucket (shared expert's bucket last), then offsets.
        __syncwarp();
        const int nbk = s_nb + (has_shared ? 1 : 0);
        for (int b = lane; b < nbk; b += 32) s_btiles[b] = (s_boff[b + 1] - s_boff[b] + tpt - 1) / tpt;
        __syncwarp();
        const int ntiles = warp_scan_excl(s_btiles, nbk);
        __syncwarp();
        for (int b = lane; b < nbk; b += 32) {
            const int s0 = s_boff[b], c = s_boff[b + 1] - s0, e = b < s_nb ? s_bexp[b] : n_experts;
            for (int j = 0, n = s_btiles[b]; j < c; j += tpt, n++) {
                s_tslot[n] = s0 + j;
                s_tcnt[n] = min(tpt, c - j);
                s_texp[n] = e;
            }
        }
        if (lane == 0) s_ntiles = ntiles;
    }
    }
    __syncthreads();
    const int nb = s_nb, ntiles = s_ntiles, nslots = npairs + (has_shared ? nt : 0);

    if (blockIdx.x == 0) {
        for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
            ws.idx[p] = s_idx[p];
            ws.wts[p] = s_wts[p];
            ws.pos[p] = s_pos[p];
            if (idx_out) {
                idx_out[p] = s_idx[p];
                wts_out[p] = s_wts[p];
            }
        }
        for (int i = threadIdx.x; i < nslots; i += blockDim.x) ws.b_tok[i] = s_btok[i];
        for (int b = threadIdx.x; b < nb; b += blockDim.x) ws.b_expert[b] = s_bexp[b];
        for (int b = threadIdx.x; b < nb + 2; b += blockDim.x) ws.b_off[b] = s_boff[b];
        for (int i = threadIdx.x; i < ntiles; i += blockDim.x) {
            ws.c_slot0[i] = s_tslot[i];
            ws.c_cnt[i] = s_tcnt[i];
            ws.c_expert[i] = s_texp[i];
        }
        if (threadIdx.x == 0) {
            ws.meta[0] = nb;
            ws.meta[1] = s_bad;
            ws.meta[2] = ntiles;
        }
        for (int i = threadIdx.x; i < ws.npcnt; i += blockDim.x) ws.pcnt[i] = 0;
    }

    // Gate/up B operand: one warp per (column tile, slot, 128-wide K chunk)
    // writes all terms of that chunk. Columns past the tile's slots are left as
    // they are: they only feed accumulator columns that are never read.
    const int kc = hidden >> 7, nbb = (NB + 127) / 128;
    const long tasks = (long)ntiles * tpt * kc;
    for (long task = (long)blockIdx.x * nwarps + warp; task < tasks; task += (long)gridDim.x * nwarps) {
        const int it = (int)(task / kc), c = (int)(task - (long)it * kc);
        const int i = it / tpt, tl = it - i * tpt;
        if (tl >= s_tcnt[i]) continue;
        const int tok = s_btok[s_tslot[i] + tl];
        mxmoe_split_row_chunk(x + (size_t)tok * hidden, hidden, c, i, tl, terms, tpt, NB, nbb, ws.xq1, ws.sfb1);
    }
}

// ------------------------------------------------------------ policies
struct MxMoeCommon {
    MoeMxDev L;
    MxMoeWs ws;
    int nb, nbb, tpt, terms, hidden, inter;
    int *err;
    int max_tiles, n_mats;   // bounds of the column-tile table and of the matrix index (3 x experts)
    int once;                // every bucket fits one column tile: each weight tile is read once
    // Fused epilogues (decode): the CTA that completes a (column tile, row
    // tile) pair of w1 / w3 applies SwiGLU and writes the down B operand; the
    // one that completes a down row tile over all column tiles combines it.
    int fuse_swiglu, fuse_combine;
    int shared_first;        // the shared expert is exactly the last column tile: its gate/up tiles go first
    float limit;
    int nt, topk, has_shared;
    float *out;
};

// SwiGLU (dsv4_ops.c:61-79: up clamped both ways, gate from above only) of
// rows [128 c, 128 c + 128) of one slot, split into e4m3 terms (mx_split128)
// as column tl of column tile i of the down projection's B operand. Whole
// warp; lane l takes rows 4 l .. 4 l + 3. The gate/up rows are read from L2.
DSV4CU_DEV void mxmoe_swiglu_chunk(const MxMoeWs &ws, int slot, int i, int tl, int c, int inter, int terms, int tpt,
                                   int NB, float limit)
{
    const int lane = threadIdx.x & 31, kc = inter >> 7, nbb = (NB + 127) / 128;
    const float *g = ws.gu + (size_t)slot * 2 * inter + c * 128 + 4 * lane, *u = g + inter;
    const float4 g4 = __ldcg(reinterpret_cast<const float4 *>(g)), u4 = __ldcg(reinterpret_cast<const float4 *>(u));
    const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float gg = gv[k], uu = uv[k];
        if (limit > 0.0f) {
            uu = fminf(fmaxf(uu, -limit), limit);
            gg = fminf(gg, limit);
        }
        v[k] = __fmul_rn(__fdiv_rn(gg, __fadd_rn(1.0f, expf(-gg))), uu);
    }
    uint32_t q[4];
    uint8_t sb[4];
    mx_split128(v, terms, q, sb);
    uint8_t *row[4], *sf[4];
    int step[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int n = j * tpt + tl;
        row[j] = ws.xq2 + ((size_t)i * NB + n) * inter + c * 128;
        sf[j] = ws.sfb2 + ((size_t)i * kc + c) * nbb * 512 + mx_sfb_offset(n, 0);
        step[j] = 1;
    }
    mx_store128(q, sb, terms, row, sf, step);
}

// Output row `row` of token t: the routed pairs IN k ORDER with the routing
// weights (dsv4_layer.c:109-113), then the shared expert unweighted (:115).
// The slot rows are read from L2.
DSV4CU_DEV float mxmoe_combine_one(const MxMoeWs &ws, int t, int topk, int hidden, int has_shared, int row)
{
    float o = 0.0f;
    for (int k = 0; k < topk; k++) {
        const int slot = ws.pos[t * topk + k];
        if (slot >= 0) o = __fadd_rn(o, __fmul_rn(ws.wts[t * topk + k], __ldcg(ws.ypart + (size_t)slot * hidden + row)));
    }
    if (has_shared) o = __fadd_rn(o, __ldcg(ws.ypart + (size_t)(ws.b_off[ws.meta[0]] + t) * hidden + row));
    return o;
}

DSV4CU_DEV MxTile mxmoe_tile(const MxMoeCommon &c, int i, int m, int rt, int kc, const uint8_t *sfb)
{
    MxTile T;
    const int fp4 = c.L.fp4[m];
    T.ta = c.L.maps + m;
    T.sfa = c.L.sfa[m] + (size_t)rt * kc * 512;
    T.sfb = sfb + (size_t)i * kc * c.nbb * 512;
    T.idesc = umma::idesc_mx(fp4 ? umma::FMT_E2M1 : umma::FMT_E4M3, umma::FMT_E4M3, 128, c.nb);
    T.a_tx = fp4 ? 128 * 64 : 128 * 128;
    T.a_row = rt * 128;
    T.b_row = i * c.nb;
    T.k0 = 0;
    T.kc = kc;
    T.nseg = 1;
    T.kst = 1;
    T.once = c.once;
    return T;
}

// Gate/up tiles, t = (i * RT + rt) * 2 + mat: column tile i, 128-row tile rt
// of w1 (mat 0) or w3 (mat 1). Results go to the per-slot gate/up rows.
// When the shared expert fills exactly one column tile (the last), its 2 RT
// tiles come first: their weights do not depend on the routing, so a CTA
// whose first tile is one of them fills its stage ring before the wait for
// the routing kernel (kPrefetchA), while that kernel still runs.
struct MoeGateUp {
    struct Params {
        MxMoeCommon c;
    };
    static constexpr bool kPrefetchA = true;
    DSV4CU_DEV static int shared_first(const Params &p) { return p.c.shared_first ? 2 * (p.c.inter >> 7) : 0; }
    DSV4CU_DEV static int ntiles_pre(const Params &p) { return shared_first(p); }
    DSV4CU_DEV static MxTile tile_pre(const Params &p, int t)   // A side only (column tile unknown yet)
    {
        return mxmoe_tile(p.c, 0, p.c.n_mats - 3 + (t & 1), t >> 1, p.c.hidden >> 7, p.c.ws.sfb1);
    }
    DSV4CU_DEV static int ntiles(const Params &p) { return p.c.ws.meta[2] * 2 * (p.c.inter >> 7); }
    DSV4CU_DEV static int *err(const Params &p) { return p.c.err; }
    DSV4CU_DEV static int terms(const Params &p) { return p.c.terms; }
    DSV4CU_DEV static int tpt(const Params &p) { return p.c.tpt; }
    DSV4CU_DEV static MxTile tile(const Params &p, int t)
    {
        const int RT = p.c.inter >> 7, sh = shared_first(p);
        int mat, i, rt;
        if (t < sh) {                       // the shared expert's column tile, the last one
            mat = t & 1;
            rt = t >> 1;
            i = p.c.ws.meta[2] - 1;
        } else {
            const int u = t - sh, pr = u >> 1;
            mat = u & 1;
            i = pr / RT;
            rt = pr - i * RT;
        }
        MxTile T = mxmoe_tile(p.c, i, 3 * p.c.ws.c_expert[i] + mat, rt, p.c.hidden >> 7, p.c.ws.sfb1);
        T.id0 = i;
        T.id1 = mat;
        T.id2 = rt;
        T.id3 = 0;
        return T;
    }
    DSV4CU_DEV static void store(const Params &p, const MxTile &T, int row_l, int tl, float v, int)
    {
        if (tl < p.c.tpt && tl < p.c.ws.c_cnt[T.id0]) {
            const int slot = p.c.ws.c_slot0[T.id0] + tl;
            p.c.ws.gu[((size_t)slot * 2 + T.id1) * p.c.inter + T.id2 * 128 + row_l] = v;
        }
    }
    // Fused SwiGLU: the second of the (w1, w3) tiles of a column tile and row
    // tile to finish turns their rows into the down operand's chunk T.id2.
    DSV4CU_DEV static void finish(const Params &p, const MxTile &T, int row_l, int *words)
    {
        if (!p.c.fuse_swiglu) return;
        __threadfence();
        epi_sync();
        if (row_l == 0) words[0] = atomicAdd(p.c.ws.pcnt + T.id0 * (p.c.inter >> 7) + T.id2, 1) == 1;
        epi_sync();
        if (!words[0]) return;
        __threadfence();
        const int i = T.id0, n = min(p.c.tpt, p.c.ws.c_cnt[i]);
        for (int tl = row_l >> 5; tl < n; tl += 4)
            mxmoe_swiglu_chunk(p.c.ws, p.c.ws.c_slot0[i] + tl, i, tl, T.id2, p.c.inter, p.c.terms, p.c.tpt, p.c.nb,
                               p.c.limit);
    }
    DSV4CU_DEV static void finish_all(const Params &, int, int, int *) {}
};

// Down tiles, t = i * RTH + rt. Results go to the per-slot output rows.
struct MoeDown {
    struct Params {
        MxMoeCommon c;
    };
    // The tile list (the routing kernel's tables) is complete before this
    // kernel can start (its predecessors waited for that kernel), so the first
    // weight tiles are requested before the wait for the SwiGLU operand, while
    // the gate/up kernel's last CTAs still run. Table entries are clamped to
    // their bounds.
    static constexpr bool kPrefetchA = true;
    DSV4CU_DEV static int ntiles_pre(const Params &p) { return ntiles(p); }
    DSV4CU_DEV static MxTile tile_pre(const Params &p, int t) { return tile(p, t); }
    DSV4CU_DEV static int ntiles(const Params &p)
    {
        return min(p.c.ws.meta[2], p.c.max_tiles) * (p.c.hidden >> 7);
    }
    DSV4CU_DEV static int *err(const Params &p) { return p.c.err; }
    DSV4CU_DEV static int terms(const Params &p) { return p.c.terms; }
    DSV4CU_DEV static int tpt(const Params &p) { return p.c.tpt; }
    DSV4CU_DEV static MxTile tile(const Params &p, int t)
    {
        const int RTH = p.c.hidden >> 7;
        const int i = t / RTH, rt = t - i * RTH;
        const int m = min(3 * p.c.ws.c_expert[i] + 2, p.c.n_mats - 1);
        MxTile T = mxmoe_tile(p.c, i, m < 0 ? 2 : m, rt, p.c.inter >> 7, p.c.ws.sfb2);
        T.id0 = i;
        T.id1 = 0;
        T.id2 = rt;
        T.id3 = 0;
        return T;
    }
    DSV4CU_DEV static void store(const Params &p, const MxTile &T, int row_l, int tl, float v, int)
    {
        if (tl < p.c.tpt && tl < p.c.ws.c_cnt[T.id0]) {
            const int slot = p.c.ws.c_slot0[T.id0] + tl;
            p.c.ws.ypart[(size_t)slot * p.c.hidden + T.id2 * 128 + row_l] = v;
        }
    }
    // Fused combine: the last column tile to finish row tile T.id2 writes
    // those output rows of every token.
    DSV4CU_DEV static void finish(const Params &p, const MxTile &T, int row_l, int *words)
    {
        if (!p.c.fuse_combine) return;
        __threadfence();
        epi_sync();
        if (row_l == 0) {
            const int cols = min(p.c.ws.meta[2], p.c.max_tiles);
            words[0] = atomicAdd(p.c.ws.pcnt + p.c.max_tiles * (p.c.inter >> 7) + T.id2, 1) == cols - 1;
        }
        epi_sync();
        if (!words[0]) return;
        __threadfence();
        const int row = T.id2 * 128 + row_l;
        for (int t = 0; t < p.c.nt; t++)
            p.c.out[(size_t)t * p.c.hidden + row] = mxmoe_combine_one(p.c.ws, t, p.c.topk, p.c.hidden, p.c.has_shared, row);
    }
    DSV4CU_DEV static void finish_all(const Params &, int, int, int *) {}
};

// SwiGLU of every slot (mxmoe_swiglu_chunk) as its own launch, for the steps
// whose gate/up epilogue does not fuse it: one warp per (column tile, slot,
// group of cpt 128-wide chunks).
__global__ void __launch_bounds__(256) mxmoe_swiglu_kernel(MxMoeWs ws, int inter, int terms, int tpt, int NB,
                                                           float limit, int cpt, int max_items)
{
    // The down kernel may launch at once: it fetches weights until it needs
    // this kernel's output.
    pdl_trigger();
    pdl_wait();
    const int gw = (int)((blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5);
    const int kc = inter >> 7, ntiles = ws.meta[2], groups = kc / cpt;
    if (gw >= max_items) return;
    const int it = gw / groups, grp = gw - it * groups, i = it / tpt, tl = it - i * tpt;
    if (i >= ntiles || tl >= ws.c_cnt[i]) return;
    const int slot = ws.c_slot0[i] + tl;
    for (int c = grp * cpt; c < (grp + 1) * cpt; c++) mxmoe_swiglu_chunk(ws, slot, i, tl, c, inter, terms, tpt, NB, limit);
}

// Output rows: per token the routed pairs IN k ORDER with the routing
// weights (dsv4_layer.c:109-113), then the shared expert unweighted (:115).
__global__ void __launch_bounds__(256) mxmoe_combine_kernel(MxMoeWs ws, int nt, int topk, int hidden,
                                                            int has_shared, float *__restrict__ out)
{
    pdl_wait();
    pdl_trigger();
    // Four consecutive output rows per thread (16-byte loads of the slot rows).
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    const int h4 = hidden >> 2;
    if (i >= (long)nt * h4) return;
    const int t = (int)(i / h4), row = (int)(i - (long)t * h4) * 4;
    int slot[MXMOE_MAX_TOPK + 1];
    float w[MXMOE_MAX_TOPK];
#pragma unroll
    for (int k = 0; k < MXMOE_MAX_TOPK; k++) {
        slot[k] = k < topk ? ws.pos[t * topk + k] : -1;
        w[k] = k < topk ? ws.wts[t * topk + k] : 0.0f;
    }
    slot[MXMOE_MAX_TOPK] = has_shared ? ws.b_off[ws.meta[0]] + t : -1;
    float4 y[MXMOE_MAX_TOPK + 1];
#pragma unroll
    for (int k = 0; k <= MXMOE_MAX_TOPK; k++)
        y[k] = slot[k] >= 0 ? *reinterpret_cast<const float4 *>(ws.ypart + (size_t)slot[k] * hidden + row)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
#pragma unroll
    for (int k = 0; k < MXMOE_MAX_TOPK; k++)
        if (slot[k] >= 0) {
            o0 = __fadd_rn(o0, __fmul_rn(w[k], y[k].x));
            o1 = __fadd_rn(o1, __fmul_rn(w[k], y[k].y));
            o2 = __fadd_rn(o2, __fmul_rn(w[k], y[k].z));
            o3 = __fadd_rn(o3, __fmul_rn(w[k], y[k].w));
        }
    if (has_shared) {
        const float4 sh = y[MXMOE_MAX_TOPK];
        o0 = __fadd_rn(o0, sh.x);
        o1 = __fadd_rn(o1, sh.y);
        o2 = __fadd_rn(o2, sh.z);
        o3 = __fadd_rn(o3, sh.w);
    }
    float *o = out + (size_t)t * hidden + row;
    o[0] = o0;
    o[1] = o1;
    o[2] = o2;
    o[3] = o3;
}

// ------------------------------------------------------------ host side
template <int NB, int KB, class P>
static int mxmoe_launch(const CUtensorMap &tb, const typename P::Params &p, int grid, cudaStream_t st)
{
    int r = mx_kernel_prepare<NB, KB, P>();
    if (r) return r;
    DSV4CU_CUDA_TRY(launch_pdl(mx_kernel<NB, KB, P>, dim3(grid), dim3(MX_THREADS), MxCfg<NB, KB>::SMEM, st, tb, p));
    return DSV4CU_OK;
}

template <class P>
static int mxmoe_dispatch(int NB, int KB, const CUtensorMap &tb, const typename P::Params &p, int grid,
                          cudaStream_t st)
{
    switch (NB * 8 + KB) {
    case 8 * 8 + 4: return mxmoe_launch<8, 4, P>(tb, p, grid, st);
    case 8 * 8 + 2: return mxmoe_launch<8, 2, P>(tb, p, grid, st);
    case 16 * 8 + 4: return mxmoe_launch<16, 4, P>(tb, p, grid, st);
    case 16 * 8 + 2: return mxmoe_launch<16, 2, P>(tb, p, grid, st);
    case 8 * 8 + 1: return mxmoe_launch<8, 1, P>(tb, p, grid, st);
    case 16 * 8 + 1: return mxmoe_launch<16, 1, P>(tb, p, grid, st);
    case 32 * 8 + 2: return mxmoe_launch<32, 2, P>(tb, p, grid, st);
    case 32 * 8 + 1: return mxmoe_launch<32, 1, P>(tb, p, grid, st);
    case 192 * 8 + 1: return mxmoe_launch<192, 1, P>(tb, p, grid, st);
    case 256 * 8 + 1: return mxmoe_launch<256, 1, P>(tb, p, grid, st);
    default: return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe: no kernel for %d columns x %d chunks", NB, KB);
    }
}


size_t moe_mx_workspace(const dsv4cu_moe *L, int topk, int nt)
{
    return mxmoe_layout(mxmoe_shape(L, topk, nt, L->sms), nullptr, nullptr);
}

// Loads every tile variant the layer's calls may pick (the shared-memory
// limit is set and the kernel loaded), so a step that first needs a variant
// does not pay for it.
template <class P>
static int mxmoe_prepare_variants()
{
    int r = 0;
    if (!r) r = mx_kernel_prepare<8, 4, P>();
    if (!r) r = mx_kernel_prepare<8, 2, P>();
    if (!r) r = mx_kernel_prepare<8, 1, P>();
    if (!r) r = mx_kernel_prepare<16, 4, P>();
    if (!r) r = mx_kernel_prepare<16, 2, P>();
    if (!r) r = mx_kernel_prepare<16, 1, P>();
    if (!r) r = mx_kernel_prepare<32, 2, P>();
    if (!r) r = mx_kernel_prepare<32, 1, P>();
    if (!r) r = mx_kernel_prepare<192, 1, P>();
    if (!r) r = mx_kernel_prepare<256, 1, P>();
    return r;
}

int moe_mx_prepare(dsv4cu_moe *L, const dsv4cu_expert *hexp)
{
    {
        int r = mxmoe_prepare_variants<MoeGateUp>();
        if (!r) r = mxmoe_prepare_variants<MoeDown>();
        if (r) return r;
    }
    L->mx_ok = 0;
    L->mx_block = nullptr;
    L->sms = 148;
    cudaDeviceGetAttribute(&L->sms, cudaDevAttrMultiProcessorCount, L->device);
    const int nm = 3 * (L->n_experts + 1);
    std::vector<const dsv4cu_qmat *> qs(nm);
    for (int e = 0; e <= L->n_experts; e++) {
        qs[3 * e] = &hexp[e].w1;
        qs[3 * e + 1] = &hexp[e].w3;
        qs[3 * e + 2] = &hexp[e].w2;
    }
    size_t sf_total = 0;
    for (int m = 0; m < nm; m++) {
        if (!mx_supported(qs[m])) return DSV4CU_ERR_UNSUPPORTED;   // the CUDA-core path serves this layer
        sf_total += dsv4cu_align256(mx_sfa_bytes(qs[m]));
    }
    // One block: [maps][pointer table][fp4 flags][scale blocks].
    const size_t b_map = dsv4cu_align256((size_t)nm * sizeof(CUtensorMap));
    const size_t b_ptr = dsv4cu_align256((size_t)nm * sizeof(void *));
    const size_t b_fmt = dsv4cu_align256((size_t)nm * sizeof(int));
    char *blk = nullptr;
    cudaError_t ce = cudaMalloc((void **)&blk, b_map + b_ptr + b_fmt + sf_total);
    if (ce != cudaSuccess) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "moe_create: %s", cudaGetErrorString(ce));
    std::vector<CUtensorMap> maps(nm);
    std::vector<const uint8_t *> ptrs(nm);
    std::vector<int> fp4(nm);
    char *sf = blk + b_map + b_ptr + b_fmt;
    int r = DSV4CU_OK;
    for (int m = 0; m < nm && !r; m++) {
        MxMat mm;
        r = mx_prepare(&mm, qs[m], (uint8_t *)sf, 0);
        if (r) break;
        maps[m] = mm.ta;
        ptrs[m] = (const uint8_t *)sf;
        fp4[m] = mm.fp4;
        sf += dsv4cu_align256(mx_sfa_bytes(qs[m]));
    }
    if (!r) {
        ce = cudaMemcpy(blk, maps.data(), nm * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
        if (ce == cudaSuccess) ce = cudaMemcpy(blk + b_map, ptrs.data(), nm * sizeof(void *), cudaMemcpyHostToDevice);
        if (ce == cudaSuccess)
            ce = cudaMemcpy(blk + b_map + b_ptr, fp4.data(), nm * sizeof(int), cudaMemcpyHostToDevice);
        if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
        if (ce != cudaSuccess) r = dsv4cu_set_error(DSV4CU_ERR_CUDA, "moe_create: %s", cudaGetErrorString(ce));
    }
    if (r) {
        cudaFree(blk);
        return r == DSV4CU_ERR_UNSUPPORTED ? DSV4CU_ERR_CUDA : r;
    }
    L->mx_block = blk;
    L->mx.maps = (const CUtensorMap *)blk;
    L->mx.sfa = (const uint8_t *const *)(blk + b_map);
    L->mx.fp4 = (const int *)(blk + b_map + b_ptr);
    L->mx_ok = 1;
    return DSV4CU_OK;
}

void moe_mx_release(dsv4cu_moe *L)
{
    if (L && L->mx_block) cudaFree(L->mx_block);
    if (L) {
        L->mx_block = nullptr;
        L->mx_ok = 0;
    }
}

// The four launches after the B operand of gate/up is in place: gate/up,
// SwiGLU split, down, combine.
// y[r] = the expert output of slot pos[r] (per-row mode of the layer, no combine);
// rows whose caller id is -1 (skip) are left unwritten.
__global__ void __launch_bounds__(256) mxmoe_rows_out_kernel(MxMoeWs ws, int nrows, int hidden, float *__restrict__ y,
                                                             const int *__restrict__ ids)
{
    pdl_wait();
    pdl_trigger();
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    const int h4 = hidden >> 2;
    if (i >= (long)nrows * h4) return;
    const int r = (int)(i / h4), c = (int)(i - (long)r * h4) * 4;
    if (ids && ids[r] == -1) return;
    const int slot = ws.pos[r];
    const float4 v = slot >= 0 ? *reinterpret_cast<const float4 *>(ws.ypart + (size_t)slot * hidden + c)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4 *>(y + (size_t)r * hidden + c) = v;
}

// rows_mode: out receives each row's expert output (the pairs are rows,
// topk = 1) instead of the weighted combine.
static int mxmoe_gemms(const dsv4cu_moe *L, const MxMoeShape &s, const MxMoeWs &ws, int terms, float limit,
                       float *out, int *status, int sms, cudaStream_t st, cudaEvent_t *ev, bool rows_mode = false,
                       const int *row_ids = nullptr, bool fused = false)
{
    const int RT = s.inter / 128, RTH = s.hidden / 128, nt = s.nt, topk = s.topk;
    MxMoeCommon c;
    c.L = L->mx;
    c.ws = ws;
    c.nb = s.NB;
    c.nbb = s.nbb;
    c.tpt = s.tpt;
    c.terms = terms;
    c.hidden = s.hidden;
    c.inter = s.inter;
    c.err = status;
    c.max_tiles = s.max_tiles;
    c.n_mats = 3 * (L->n_experts + 1);
    c.once = s.nt <= s.tpt;   // a bucket holds at most nt slots
    // Decode (the prep kernel zeroes the arrival counters): SwiGLU in the
    // gate/up epilogue; the combine in the down epilogue while one thread's
    // loop over the tokens stays short.
    c.fuse_swiglu = fused && !rows_mode;
    c.fuse_combine = c.fuse_swiglu && nt <= MXMOE_FUSE_COMBINE_NT;
    c.shared_first = fused && s.has_shared && s.nt <= s.tpt;
    c.limit = limit;
    c.nt = nt;
    c.topk = topk;
    c.has_shared = s.has_shared;
    c.out = out;
    // Persistent grids: the tile count is known only on the device.
    const int g1 = min(sms, s.max_tiles * 2 * RT), g2 = min(sms, s.max_tiles * RTH);

    CUtensorMap tb1, tb2;
    int r = mx_cached_bmap(&tb1, ws.xq1, (uint64_t)s.hidden, (uint64_t)s.max_tiles * s.NB, (uint32_t)s.NB);
    if (!r) r = mx_cached_bmap(&tb2, ws.xq2, (uint64_t)s.inter, (uint64_t)s.max_tiles * s.NB, (uint32_t)s.NB);
    if (r) return r;

    MoeGateUp::Params pg;
    pg.c = c;
    int kb1 = s.KB;
    while (kb1 > 1 && (s.hidden / 128) % kb1) kb1 >>= 1;
    r = mxmoe_dispatch<MoeGateUp>(s.NB, kb1, tb1, pg, g1, st);
    if (r) return r;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[2], st));
    if (!c.fuse_swiglu) {
        // Few slots (decode): one chunk per warp; many (prefill): whole rows.
        const int cpt = s.npairs > 1024 ? s.inter / 128 : 1;
        const int items = s.max_tiles * s.tpt * (s.inter / 128 / cpt);
        DSV4CU_CUDA_TRY(launch_pdl(mxmoe_swiglu_kernel, dim3((items * 32 + 255) / 256), dim3(256), 0, st, ws, s.inter,
                                   terms, s.tpt, s.NB, limit, cpt, items));
    }

    MoeDown::Params pd;
    pd.c = c;
    int kb2 = s.KB;
    while (kb2 > 1 && (s.inter / 128) % kb2) kb2 >>= 1;
    r = mxmoe_dispatch<MoeDown>(s.NB, kb2, tb2, pd, g2, st);
    if (r) return r;
    if (rows_mode)
        DSV4CU_CUDA_TRY(launch_pdl(mxmoe_rows_out_kernel, dim3((unsigned)(((long)nt * (s.hidden / 4) + 255) / 256)),
                                   dim3(256), 0, st, ws, nt, s.hidden, out, row_ids));
    else if (!c.fuse_combine)   // else the down kernel's epilogue writes out
        DSV4CU_CUDA_TRY(launch_pdl(mxmoe_combine_kernel, dim3((unsigned)(((long)nt * (s.hidden / 4) + 255) / 256)),
                                   dim3(256), 0, st, ws, nt, topk, s.hidden, s.has_shared, out));
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[3], st));
    return DSV4CU_OK;
}

int moe_mx_decode(const dsv4cu_moe *L, float *out, const float *x, const float *logits, const float *bias,
                  const int64_t *tid2eid, const int *token_ids, int topk, float route_scale, float limit, int nt,
                  int *idx_out, float *wts_out, void *wsp, int *counters, int *status, int sms, cudaStream_t st,
                  cudaEvent_t *ev)
{
    if (nt > MXMOE_MAX_NT || topk > MXMOE_MAX_TOPK || L->n_experts > PREP_MAX_EXPERTS)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_decode: nt %d / topk %d / experts %d beyond 64 / 16 / 512",
                                nt, topk, L->n_experts);
    const MxMoeShape s = mxmoe_shape(L, topk, nt, L->sms);
    MxMoeWs ws;
    mxmoe_layout(s, (char *)wsp, &ws);
    (void)counters;
    const float *tab = router_table_get();
    if (!tab) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "moe_decode: router table setup failed");

    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
    {
        // Every SM takes part in the split; each CTA repeats the (cheap) routing.
        const long tasks = (long)s.max_tiles * s.tpt * (s.hidden / 128);
        const int grid = (int)min((long)sms, max(1L, (tasks + PREP_THREADS / 32 - 1) / (PREP_THREADS / 32)));
        DSV4CU_CUDA_TRY(launch_pdl(mxmoe_prep_kernel, dim3(grid), dim3(PREP_THREADS), 0, st, tab, x, logits, bias, tid2eid,
                                   token_ids, s.n_experts, topk, route_scale, nt, s.hidden, s.has_shared, MX_TERMS,
                                   s.tpt, s.NB, ws, idx_out, wts_out));
    }
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));

    return mxmoe_gemms(L, s, ws, MX_TERMS, limit, out, status, sms, st, ev, false, nullptr, true);
}


// ============================================================ prefill
// The MoE layer over many tokens (the reference's prefill union path:
// union_prepare, src/80_prefill/dsv4_prefill_union.c:30-66, bucketing as in
// dsv4_prefill_expert_bucket, src/80_prefill/dsv4_prefill_experts.c:23-77,
// k-order combine, src/80_prefill/dsv4_prefill_union_run.c:109-121, shared
// expert over every token, src/80_prefill/dsv4_prefill_moe.c:40-59). The GEMM,
// SwiGLU and combine launches are those of the decode step with wide column
// tiles; routing and bucketing run as separate grid-wide kernels:
//   route    one warp per token;
//   count    per chunk of PF_CHUNK pairs, a per-expert histogram;
//   offsets  one CTA: per expert the chunk offsets and total, the bucket
//            offsets (ascending expert order), the column tiles;
//   scatter  per chunk, pairs ranked in (token, k) order inside their expert,
//            so a bucket holds its tokens ascending - a stable counting sort.
constexpr int PF_CHUNK = 1024;
constexpr int PF_MAX_NT = 16384;

struct PfWs {
    int *chunk_cnt;      // [nchunks][n_experts]: counts, then exclusive offsets inside each expert
    int *e_off;          // [n_experts + 1]
};

__global__ void __launch_bounds__(256) mxpf_route_kernel(const float *__restrict__ tab,
                                                         const float *__restrict__ logits,
                                                         const float *__restrict__ bias,
                                                         const int64_t *__restrict__ tid2eid,
                                                         const int *__restrict__ token_ids, int n_experts, int topk,
                                                         float route_scale, int nt, MxMoeWs ws,
                                                         int *__restrict__ idx_out, float *__restrict__ wts_out)
{
    pdl_wait();
    pdl_trigger();
    const int t = (int)((blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5);
    if (t >= nt) return;
    route_token_warp(tab, logits + (size_t)t * n_experts, bias, tid2eid, token_ids ? token_ids[t] : 0, n_experts,
                     topk, route_scale, ws.idx + (size_t)t * topk, ws.wts + (size_t)t * topk, nullptr, nullptr);
    __syncwarp();
    if ((threadIdx.x & 31) < topk && idx_out) {
        const int k = threadIdx.x & 31;
        idx_out[(size_t)t * topk + k] = ws.idx[(size_t)t * topk + k];
        wts_out[(size_t)t * topk + k] = ws.wts[(size_t)t * topk + k];
    }
}

__global__ void __launch_bounds__(1024) mxpf_count_kernel(MxMoeWs ws, PfWs pf, int npairs, int n_experts)
{
    __shared__ int h[PREP_MAX_EXPERTS];
    pdl_wait();
    pdl_trigger();
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) h[e] = 0;
    __syncthreads();
    const int p = blockIdx.x * PF_CHUNK + threadIdx.x;
    if (threadIdx.x < PF_CHUNK && p < npairs) {
        const int e = ws.idx[p];
        if (e >= 0 && e < n_experts) atomicAdd(&h[e], 1);
        else atomicOr(ws.meta + 1, 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) pf.chunk_cnt[(size_t)blockIdx.x * n_experts + e] = h[e];
}

__global__ void __launch_bounds__(1024) mxpf_offsets_kernel(MxMoeWs ws, PfWs pf, int nchunks, int n_experts, int nt,
                                                            int has_shared, int tpt, int max_tiles)
{
    __shared__ int tot[PREP_MAX_EXPERTS + 2], bid[PREP_MAX_EXPERTS + 2], ntl[PREP_MAX_EXPERTS + 2];
    __shared__ int s_nb, s_routed;
    pdl_wait();
    pdl_trigger();
    // Per expert: exclusive offsets over the chunks, and the total.
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
        int run = 0;
        for (int c = 0; c < nchunks; c++) {
            int *q = pf.chunk_cnt + (size_t)c * n_experts + e;
            const int v = *q;
            *q = run;
            run += v;
        }
        tot[e] = run;
        bid[e] = run > 0;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        int *off = ntl;      // scratch: expert offsets
        for (int e = threadIdx.x; e < n_experts; e += 32) off[e] = tot[e];
        __syncwarp();
        const int routed = warp_scan_excl(off, n_experts);
        const int nb = warp_scan_excl(bid, n_experts);
        __syncwarp();
        for (int e = threadIdx.x; e < n_experts; e += 32) {
            pf.e_off[e] = off[e];
            if (tot[e]) {
                ws.b_expert[bid[e]] = e;
                ws.b_off[bid[e]] = off[e];
            }
        }
        if (threadIdx.x == 0) {
            pf.e_off[n_experts] = routed;
            ws.b_off[nb] = routed;
            ws.b_off[nb + 1] = routed + (has_shared ? nt : 0);
            ws.meta[0] = nb;
            s_nb = nb;
            s_routed = routed;
        }
    }
    __syncthreads();
    const int nb = s_nb, nbk = nb + (has_shared ? 1 : 0);
    // Column tiles: per bucket ceil(count / tpt), then offsets.
    for (int b = threadIdx.x; b < nbk; b += blockDim.x) {
        const int c = b < nb ? tot[ws.b_expert[b]] : nt;
        ntl[b] = (c + tpt - 1) / tpt;
    }
    __syncthreads();
    __shared__ int s_ntiles;
    if (threadIdx.x < 32) {
        const int n = warp_scan_excl(ntl, nbk);
        if (threadIdx.x == 0) s_ntiles = min(n, max_tiles);
    }
    __syncthreads();
    for (int b = threadIdx.x; b < nbk; b += blockDim.x) {
        const int e = b < nb ? ws.b_expert[b] : n_experts;
        const int s0 = b < nb ? ws.b_off[b] : s_routed, c = b < nb ? tot[e] : nt;
        for (int j = 0, n = ntl[b]; j < c && n < max_tiles; j += tpt, n++) {
            ws.c_slot0[n] = s0 + j;
            ws.c_cnt[n] = min(tpt, c - j);
            ws.c_expert[n] = b < nb ? e : n_experts;
        }
    }
    if (threadIdx.x == 0) ws.meta[2] = s_ntiles;
}

__global__ void __launch_bounds__(1024) mxpf_scatter_kernel(MxMoeWs ws, PfWs pf, int npairs, int n_experts, int topk,
                                                            int nt, int has_shared)
{
    __shared__ int run[PREP_MAX_EXPERTS];
    pdl_wait();
    pdl_trigger();
    const int c = blockIdx.x, lane = threadIdx.x & 31;
    if (threadIdx.x < 32) {
        for (int e = lane; e < n_experts; e += 32)
            run[e] = pf.e_off[e] + pf.chunk_cnt[(size_t)c * n_experts + e];
        __syncwarp();
        for (int c0 = 0; c0 < PF_CHUNK; c0 += 32) {
            const int p = c * PF_CHUNK + c0 + lane;
            const int e = p < npairs ? ws.idx[p] : -1;
            const bool ok = e >= 0 && e < n_experts;
            const unsigned same = __match_any_sync(0xFFFFFFFFu, ok ? e : -1);
            const int before = __popc(same & ((1u << lane) - 1u));
            const int base = ok ? run[e] : 0;
            __syncwarp();
            if (ok) {
                const int slot = base + before;
                ws.pos[p] = slot;
                ws.b_tok[slot] = p / topk;
                if (before == __popc(same) - 1) run[e] = base + before + 1;
            } else if (p < npairs) {
                ws.pos[p] = -1;
            }
            __syncwarp();
        }
    }
    if (has_shared && c == 0)
        for (int t = threadIdx.x; t < nt; t += blockDim.x) ws.b_tok[pf.e_off[n_experts] + t] = t;
}

// Gate/up B operand of the prefill: one warp per (column tile, slot) walks
// the token's row chunk by chunk (the table lookups are paid once per row).
__global__ void __launch_bounds__(256) mxpf_split_kernel(const float *__restrict__ x, int hidden, long ldx, MxMoeWs ws,
                                                         int terms, int tpt, int NB, long max_tasks)
{
    pdl_wait();
    pdl_trigger();
    const long task = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
    if (task >= max_tasks) return;
    const int i = (int)(task / tpt), tl = (int)(task - (long)i * tpt);
    if (i >= ws.meta[2] || tl >= ws.c_cnt[i]) return;
    const int tok = ws.b_tok[ws.c_slot0[i] + tl], nbb = (NB + 127) / 128;
    for (int c = 0; c < (hidden >> 7); c++)
        mxmoe_split_row_chunk(x + (size_t)tok * ldx, hidden, c, i, tl, terms, tpt, NB, nbb, ws.xq1, ws.sfb1);
}

static MxMoeShape mxpf_shape(const dsv4cu_moe *L, int topk, int nt, int terms)
{
    MxMoeShape s;
    s.nt = nt;
    s.topk = topk;
    s.n_experts = L->n_experts;
    s.hidden = L->hidden;
    s.inter = L->inter;
    s.has_shared = L->has_shared;
    s.NB = terms == 3 ? 192 : 256;         // 64 tokens per tile at 3 and 4 terms, 128 at 2, 256 at 1
    s.KB = 1;
    s.tpt = (s.NB / terms) / 8 * 8;
    s.nbb = (s.NB + 127) / 128;
    s.npairs = nt * topk + (s.has_shared ? nt : 0);
    s.nbmax = min(nt * topk, s.n_experts);
    s.max_tiles = (nt * topk) / s.tpt + s.nbmax + (s.has_shared ? nt / s.tpt + 1 : 0) + 1;
    return s;
}

static size_t mxpf_layout(const MxMoeShape &s, char *base, MxMoeWs *w, PfWs *pf)
{
    size_t off = mxmoe_layout(s, base, w);
    const int nchunks = (s.nt * s.topk + PF_CHUNK - 1) / PF_CHUNK;
    auto take = [&](size_t bytes) {
        char *p = base ? base + off : nullptr;
        off += dsv4cu_align256(bytes);
        return p;
    };
    PfWs t;
    t.chunk_cnt = (int *)take((size_t)nchunks * s.n_experts * 4);
    t.e_off = (int *)take(((size_t)s.n_experts + 1) * 4);
    if (pf) *pf = t;
    return off;
}

size_t moe_mx_prefill_workspace(const dsv4cu_moe *L, int topk, int nt, int terms)
{
    return mxpf_layout(mxpf_shape(L, topk, nt, terms), nullptr, nullptr, nullptr);
}

int moe_mx_prefill(const dsv4cu_moe *L, float *out, const float *x, const float *logits, const float *bias,
                   const int64_t *tid2eid, const int *token_ids, int topk, float route_scale, float limit, int nt,
                   int terms, int *idx_out, float *wts_out, void *wsp, int *status, int sms, cudaStream_t st,
                   cudaEvent_t *ev)
{
    if (nt > PF_MAX_NT || topk > MXMOE_MAX_TOPK || L->n_experts > PREP_MAX_EXPERTS)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_prefill: nt %d / topk %d / experts %d beyond %d / 16 / 512",
                                nt, topk, L->n_experts, PF_MAX_NT);
    if (terms < 1 || terms > 4) return dsv4cu_set_error(DSV4CU_ERR_ARG, "moe_prefill: terms must be 1 .. 4");
    const MxMoeShape s = mxpf_shape(L, topk, nt, terms);
    MxMoeWs ws;
    PfWs pf;
    mxpf_layout(s, (char *)wsp, &ws, &pf);
    const float *tab = router_table_get();
    if (!tab) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "moe_prefill: router table setup failed");
    const int npairs = nt * topk, nchunks = (npairs + PF_CHUNK - 1) / PF_CHUNK;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
    DSV4CU_CUDA_TRY(cudaMemsetAsync(ws.meta, 0, 64, st));
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_route_kernel, dim3((nt * 32 + 255) / 256), dim3(256), 0, st, tab, logits, bias,
                               tid2eid, token_ids, s.n_experts, topk, route_scale, nt, ws, idx_out, wts_out));
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_count_kernel, dim3(nchunks), dim3(1024), 0, st, ws, pf, npairs, s.n_experts));
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_offsets_kernel, dim3(1), dim3(1024), 0, st, ws, pf, nchunks, s.n_experts, nt,
                               s.has_shared, s.tpt, s.max_tiles));
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_scatter_kernel, dim3(nchunks), dim3(1024), 0, st, ws, pf, npairs, s.n_experts, topk,
                               nt, s.has_shared));
    const long tasks = (long)s.max_tiles * s.tpt;
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_split_kernel, dim3((unsigned)((tasks * 32 + 255) / 256)), dim3(256), 0, st, x,
                               s.hidden, (long)s.hidden, ws, terms, s.tpt, s.NB, tasks));
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));
    return mxmoe_gemms(L, s, ws, terms, limit, out, status, sms, st, ev);
}


// ------------------------------------------------------------ per-row experts
// Row r of x (row stride ldx) through expert ids[r] (0 .. n_experts - 1, or
// n_experts for the shared expert), no weighting: the local compute of the
// expert-parallel layer. The prefill bucketing runs with the shared expert as
// one more bucket and one pair per row; each row's result is the same bits
// as the layer's decode / prefill paths give that (token, expert) pair.
// Tile width from the rows per expert: a few rows per expert (decode-like
// batches) stream weights best through the narrow decode tiles, many rows
// (prefill-like) through 256-column tiles.
// live_rows: the rows expected to carry an expert (the rest skipped with id
// -1); it picks the tile width, nrows bounds every buffer.
static MxMoeShape mxrows_shape(const dsv4cu_moe *L, int nrows, int live_rows)
{
    MxMoeShape s = mxpf_shape(L, 1, nrows, MX_TERMS);
    s.n_experts = L->n_experts + (L->has_shared ? 1 : 0);
    s.has_shared = 0;
    s.npairs = nrows;
    s.nbmax = min(nrows, s.n_experts);
    const int live = max(1, min(live_rows, nrows));
    const int avg = (live + min(live, s.n_experts) - 1) / max(1, min(live, s.n_experts));
    if (avg <= 2) {
        s.NB = 8;
        s.KB = 4;
    } else if (avg <= 4) {
        s.NB = 16;
        s.KB = 4;
    } else if (avg <= 16) {
        s.NB = 32;
        s.KB = 2;
    }
    s.tpt = s.NB <= 16 ? s.NB / MX_TERMS : (s.NB / MX_TERMS) / 8 * 8;
    s.nbb = (s.NB + 127) / 128;
    s.max_tiles = nrows / s.tpt + s.nbmax + 1;
    return s;
}

__global__ void __launch_bounds__(256) mxrows_ids_kernel(const int *__restrict__ ids, int nrows, int n_buckets,
                                                         MxMoeWs ws, int *status)
{
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= nrows) return;
    const int e = ids[r];
    const bool ok = e >= 0 && e < n_buckets;
    ws.idx[r] = ok ? e : -1;
    ws.wts[r] = 1.0f;
    if (!ok && e != -1) atomicCAS(status, 0, MXE_BAD_EXPERT);     // -1: a skipped row
}

size_t moe_mx_rows_workspace(const dsv4cu_moe *L, int nrows, int live_rows)
{
    return mxpf_layout(mxrows_shape(L, nrows, live_rows), nullptr, nullptr, nullptr);
}

int moe_mx_rows(const dsv4cu_moe *L, float *y, const float *x, long ldx, const int *ids, int nrows, int live_rows,
                float limit, void *wsp, int *status, int sms, cudaStream_t st)
{
    if (nrows > PF_MAX_NT * 2 || L->n_experts + 1 > PREP_MAX_EXPERTS)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_rows: %d rows / %d experts beyond %d / %d", nrows,
                                L->n_experts, PF_MAX_NT * 2, PREP_MAX_EXPERTS - 1);
    const MxMoeShape s = mxrows_shape(L, nrows, live_rows);
    MxMoeWs ws;
    PfWs pf;
    mxpf_layout(s, (char *)wsp, &ws, &pf);
    const int nchunks = (nrows + PF_CHUNK - 1) / PF_CHUNK;
    DSV4CU_CUDA_TRY(cudaMemsetAsync(ws.meta, 0, 64, st));
    DSV4CU_CUDA_TRY(launch_pdl(mxrows_ids_kernel, dim3((nrows + 255) / 256), dim3(256), 0, st, ids, nrows,
                               s.n_experts, ws, status));
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_count_kernel, dim3(nchunks), dim3(1024), 0, st, ws, pf, nrows, s.n_experts));
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_offsets_kernel, dim3(1), dim3(1024), 0, st, ws, pf, nchunks, s.n_experts, nrows, 0,
                               s.tpt, s.max_tiles));
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_scatter_kernel, dim3(nchunks), dim3(1024), 0, st, ws, pf, nrows, s.n_experts, 1,
                               nrows, 0));
    const long tasks = (long)s.max_tiles * s.tpt;
    DSV4CU_CUDA_TRY(launch_pdl(mxpf_split_kernel, dim3((unsigned)((tasks * 32 + 255) / 256)), dim3(256), 0, st, x,
                               s.hidden, ldx, ws, MX_TERMS, s.tpt, s.NB, tasks));
    return mxmoe_gemms(L, s, ws, MX_TERMS, limit, y, status, sms, st, nullptr, true, ids);
}

}  // namespace dsv4cu
