// moe_stream.cu - the MoE layer decode step for one or two tokens on the
// streamed GEMV core (stream_mv.cuh).
//
// Reference: dsv4_layer_moe (src/70_decode/dsv4_layer.c:48-117) from the router
// logits on, with dsv4_route (dsv4_ops.c:117-156), dsv4_expert_forward
// (dsv4_ops.c:85-93), dsv4_swiglu (dsv4_ops.c:61-79) and the k-order combine
// (dsv4_layer.c:109-116).
//
// Three launches, chained by programmatic dependent launch:
//   prep     CTA 0 routes every token (one warp per token, the reference's
//            float operations) and buckets the (token, k) pairs by expert in
//            ascending expert order, tokens ascending inside a bucket (the
//            layout of union_prepare, src/80_prefill/dsv4_prefill_union.c:
//            30-52), the shared expert's bucket after them; it also zeroes the
//            step's counters. The other CTAs split x into the f16 hi / lo
//            operand.
//   stream   one persistent CTA per SM over a queue of jobs:
//              A jobs (bucket, 32 rows of w1 and of w3): SwiGLU of the 32 gate
//                and up values of every token of the bucket, written as the
//                down operand (32 values = one activation block);
//              B jobs (bucket, 64 rows of w2): the bucket's output rows.
//            The queue holds every A job (the shared expert's first: its
//            weights are known before routing, so the first CTAs fetch them
//            while prep runs), then every B job. A B job's operand is copied
//            once every A job of its bucket is done (bounded wait); CTAs take
//            jobs in queue order, so that wait is short.
//   combine  per token the routed pairs in k order with the routing weights,
//            then the shared expert unweighted.
// Every weight byte of the touched experts is read once per step. Each output
// value is summed in one fixed order, so results are identical run to run.
#include <stdio.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "moe.h"
#include "router.cuh"
#include "stream_mv.cuh"

namespace dsv4cu {

constexpr int SMV_MOE_MAX_TOPK = 16;

struct SmvMoeWs {
    uint16_t *xh, *xl;      // [nt][hidden] activation operand
    float *xs;              // [nt][hidden / 32]
    int *idx;               // [nt][topk]
    float *wts;             // [nt][topk]
    int *pos;               // [nt][topk] slot of pair (t, k), -1 = dropped
    int *meta;              // [0] routed buckets nb, [1] bad-route flag
    int *b_expert;          // [nbmax]
    int *b_off;             // [nbmax + 2]: bucket b holds slots b_off[b] .. b_off[b + 1] - 1;
                            // the shared bucket (index nb) follows the routed ones
    int *b_tok;             // [nslots] token of each slot
    uint16_t *hh, *hl;      // [nslots][inter] SwiGLU output as the down operand
    float *hs;              // [nslots][inter / 32]
    float *ypart;           // [nslots][hidden] output row of each slot
    int *ctr;               // [0] job queue, [1 + b] finished A jobs of bucket b
};

struct SmvMoeShape {
    int nt, topk, n_experts, hidden, inter, has_shared, npairs, nslots, nbmax;
};

static SmvMoeShape smv_moe_shape(const dsv4cu_moe *L, int topk, int nt)
{
    SmvMoeShape s;
    s.nt = nt;
    s.topk = topk;
    s.n_experts = L->n_experts;
    s.hidden = L->hidden;
    s.inter = L->inter;
    s.has_shared = L->has_shared;
    s.npairs = nt * topk;
    s.nslots = s.npairs + (s.has_shared ? nt : 0);
    s.nbmax = min(s.npairs, s.n_experts);
    return s;
}

static size_t smv_moe_layout(const SmvMoeShape &s, char *base, SmvMoeWs *w)
{
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *p = base ? base + off : nullptr;
        off += dsv4cu_align256(bytes);
        return p;
    };
    SmvMoeWs t;
    t.xh = (uint16_t *)take((size_t)s.nt * s.hidden * 2);
    t.xl = (uint16_t *)take((size_t)s.nt * s.hidden * 2);
    t.xs = (float *)take((size_t)s.nt * (s.hidden / 32) * 4);
    t.idx = (int *)take((size_t)s.npairs * 4);
    t.wts = (float *)take((size_t)s.npairs * 4);
    t.pos = (int *)take((size_t)s.npairs * 4);
    t.meta = (int *)take(64);
    t.b_expert = (int *)take((size_t)s.nbmax * 4 + 4);
    t.b_off = (int *)take(((size_t)s.nbmax + 2) * 4);
    t.b_tok = (int *)take((size_t)s.nslots * 4);
    t.hh = (uint16_t *)take((size_t)s.nslots * s.inter * 2);
    t.hl = (uint16_t *)take((size_t)s.nslots * s.inter * 2);
    t.hs = (float *)take((size_t)s.nslots * (s.inter / 32) * 4);
    t.ypart = (float *)take((size_t)s.nslots * s.hidden * 4);
    t.ctr = (int *)take(((size_t)s.nbmax + 4) * 4);
    if (w) *w = t;
    return off;
}

// ------------------------------------------------------------------ prep
__global__ void __launch_bounds__(256) smv_moe_prep_kernel(
    const float *__restrict__ tab, const float *__restrict__ x, const float *__restrict__ logits,
    const float *__restrict__ bias, const int64_t *__restrict__ tid2eid, const int *__restrict__ token_ids,
    int n_experts, int topk, float route_scale, int hidden, int nt, int has_shared, int nbmax, SmvMoeWs ws,
    int *__restrict__ idx_out, float *__restrict__ wts_out)
{
    // The stream kernel may launch at once: it fetches the shared expert's
    // weights, which do not depend on this kernel, and waits for the rest.
    pdl_trigger();
    // x and the logits may come from the previous kernel, which may also still
    // be reading this workspace.
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    if (blockIdx.x > 0) {
        // x -> f16 hi / lo operand, one warp per (token, 32-element block).
        const int nblk = hidden >> 5;
        for (int gw = (blockIdx.x - 1) * nwarps + warp; gw < nt * nblk; gw += (gridDim.x - 1) * nwarps) {
            const int t = gw / nblk, b = gw - t * nblk;
            const size_t i = (size_t)t * hidden + b * 32 + lane;
            uint16_t hi, lo;
            float fac;
            smv_split32(x[i], hi, lo, fac);
            ws.xh[i] = hi;
            ws.xl[i] = lo;
            if (lane == 0) ws.xs[(size_t)t * nblk + b] = fac;
        }
        return;
    }

    // CTA 0: routing, one warp per token (dsv4_route, dsv4_ops.c:117-156),
    // into shared memory.
    constexpr int MAXP = SMV_MAXT * SMV_MOE_MAX_TOPK;
    __shared__ int sidx[MAXP];
    __shared__ float swts[MAXP];
    __shared__ int cnt[512];
    __shared__ int boff[512];
    __shared__ int wtot[2][8];
    __shared__ int bad;
    const int npairs = nt * topk;
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
    if (threadIdx.x == 0) bad = 0;
    for (int i = threadIdx.x; i < nbmax + 4; i += blockDim.x) ws.ctr[i] = 0;
    for (int t = warp; t < nt; t += nwarps)
        route_token_warp(tab, logits + (size_t)t * n_experts, bias, tid2eid, token_ids ? token_ids[t] : 0,
                         n_experts, topk, route_scale, sidx + t * topk, swts + t * topk, nullptr, nullptr);
    __syncthreads();

    // Buckets: per-expert counts, then one block scan over the experts
    // (two per thread, n_experts <= 512) gives each expert its first slot and
    // each touched expert its bucket, in ascending expert order; slots inside
    // a bucket follow (t, k) order, so tokens ascend.
    for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
        const int e = sidx[p];
        ws.idx[p] = e;
        ws.wts[p] = swts[p];
        if (idx_out) {
            idx_out[p] = e;
            wts_out[p] = swts[p];
        }
        if (e < 0 || e >= n_experts) atomicOr(&bad, 1);
        else atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    const int e0 = 2 * threadIdx.x;
    const int c0 = e0 < n_experts ? cnt[e0] : 0, c1 = e0 + 1 < n_experts ? cnt[e0 + 1] : 0;
    const int sc = c0 + c1, sg = (c0 > 0) + (c1 > 0);
    int ic = sc, ig = sg;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int uc = __shfl_up_sync(0xFFFFFFFFu, ic, d), ug = __shfl_up_sync(0xFFFFFFFFu, ig, d);
        if (lane >= d) {
            ic += uc;
            ig += ug;
        }
    }
    if (lane == 31) {
        wtot[0][warp] = ic;
        wtot[1][warp] = ig;
    }
    __syncthreads();
    int oc = ic - sc, og = ig - sg, tc = 0, tg = 0;
    for (int w = 0; w < nwarps; w++) {
        if (w < warp) {
            oc += wtot[0][w];
            og += wtot[1][w];
        }
        tc += wtot[0][w];
        tg += wtot[1][w];
    }
    if (e0 < n_experts) boff[e0] = oc;
    if (e0 + 1 < n_experts) boff[e0 + 1] = oc + c0;
    if (c0) {
        ws.b_expert[og] = e0;
        ws.b_off[og] = oc;
    }
    if (c1) {
        ws.b_expert[og + (c0 > 0)] = e0 + 1;
        ws.b_off[og + (c0 > 0)] = oc + c0;
    }
    if (threadIdx.x == 0) {
        ws.b_off[tg] = tc;
        ws.b_off[tg + 1] = tc + (has_shared ? nt : 0);
        ws.meta[0] = tg;
        ws.meta[1] = bad;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
        const int e = sidx[p];
        if (e < 0 || e >= n_experts) {
            ws.pos[p] = -1;
            continue;
        }
        int r = 0;
        for (int q = 0; q < p; q++) r += (sidx[q] == e);
        const int slot = boff[e] + r;
        ws.pos[p] = slot;
        ws.b_tok[slot] = p / topk;
    }
    if (has_shared)
        for (int t = threadIdx.x; t < nt; t += blockDim.x) ws.b_tok[tc + t] = t;
}

// ------------------------------------------------------------- the stream
struct SmvMoeParams {
    SmvGeom geom;
    SmvMoeWs ws;
    const dsv4cu_expert *experts;   // [n_experts + 1], shared last
    const CUtensorMap *maps;        // [(n_experts + 1) * 3][2]: weight map, FP4 scale map
    int nt, hidden, inter, has_shared, n_experts;
    float limit;
    int *status;
};

// Queue order: A jobs (inter / 32 per bucket), then B jobs (hidden / 64 per
// bucket); buckets in order o = 0 .. nbt - 1 with the shared expert first.
struct SmvMoeJob {
    int phase, o, rg;
};
DSV4CU_DEV SmvMoeJob smv_moe_job(int j, int ja_per, int jb_per, int nbt)
{
    SmvMoeJob r;
    const int ja = nbt * ja_per;
    if (j < ja) {
        r.phase = 0;
        r.o = j / ja_per;
        r.rg = j - r.o * ja_per;
    } else {
        j -= ja;
        r.phase = 1;
        r.o = j / jb_per;
        r.rg = j - r.o * jb_per;
    }
    return r;
}
// Bucket index of order position o (the shared bucket is index nb).
DSV4CU_DEV int smv_moe_bucket(int o, int nb, int has_shared) { return has_shared ? (o == 0 ? nb : o - 1) : o; }

// Key of an x operand: the token rows (at most 2) and their count.
DSV4CU_DEV long long smv_moe_xkey(const int *rows, int cnt)
{
    long long k = cnt;
    for (int i = 0; i < cnt; i++) k |= (long long)(rows[i] + 1) << (8 + 24 * i);
    return k;
}

// Producer state across jobs. pend: the first job's operand (x of tokens
// 0 .. nt - 1, buffer 0) is still to be copied, after the dependency wait.
struct SmvMoeProd {
    int slot;
    uint32_t ph;
    int jl;               // CTA-local job sequence number
    bool pend;
    SmvBufState bs;
    SmvDrain dr;
};

// The deferred operand of the first job (producer thread): wait for the
// previous kernel (prep), then copy.
template <int NT>
DSV4CU_DEV void smv_moe_pend_flush(uint8_t *bufs, SmvSmem<NT> &sm, SmvMoeProd &st, const SmvMoeParams &p)
{
    pdl_wait();
    int rows[NT];
    for (int i = 0; i < NT; i++) rows[i] = i < p.nt ? i : 0;
    smv_put_operand(bufs, p.geom.bstride, 0, sm, p.ws.xh, p.ws.xl, p.ws.xs, p.hidden, rows, p.nt);
    st.pend = false;
}

// The activation operand of job jb (bucket bi, slots s0 .. s0 + cnt - 1):
// A jobs read the tokens' x operand, B jobs the slots' SwiGLU operand once
// every A job of the bucket has written it (bounded acquire wait). Returns the
// buffer, or -1 after a timeout. Producer thread.
template <int NT>
DSV4CU_DEV int smv_moe_operand(uint8_t *bufs, SmvSmem<NT> &sm, SmvMoeProd &st, const SmvMoeParams &p,
                               const SmvMoeJob &jb, int bi, bool shared, int s0, int cnt, bool *load)
{
    int rows[NT];
    for (int i = 0; i < NT; i++) rows[i] = 0;
    long long key;
    if (jb.phase == 0) {
        for (int i = 0; i < cnt; i++) rows[i] = shared ? i : p.ws.b_tok[s0 + i];
        key = smv_moe_xkey(rows, cnt);
    } else {
        for (int i = 0; i < cnt; i++) rows[i] = s0 + i;
        key = (1ll << 62) | ((long long)cnt << 40) | (long long)s0;
        const int need = p.inter >> 5, *c = p.ws.ctr + 1 + bi;
        int v;
        asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
        const uint64_t t0 = v < need ? globaltimer_ns() : 0;
        while (v < need) {
            __nanosleep(100);
            asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
            if (v < need && globaltimer_ns() - t0 > MBAR_TIMEOUT_NS) {
                atomicCAS(p.status, 0, SMV_E_DEP);
                atomicExch(&sm.abort_flag, 1);
                return -1;
            }
        }
        // The copy engine reads what the A jobs' generic stores wrote.
        asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    const int b = smv_buf_pick(st.bs, sm, p.geom.nbuf, key, load, p.status);
    if (b >= 0 && *load) {
        if (jb.phase == 0) smv_put_operand(bufs, p.geom.bstride, b, sm, p.ws.xh, p.ws.xl, p.ws.xs, p.hidden, rows, cnt);
        else smv_put_operand(bufs, p.geom.bstride, b, sm, p.ws.hh, p.ws.hl, p.ws.hs, p.inter, rows, cnt);
    }
    return b;
}

// One job: its operand (the first CTAs' first A jobs defer it: st.pend), then
// its stages - A: w1 rows rg * 32 .. + 31, then w3; B: w2 rows rg * 64 ..
// + 31, then + 32 .. + 63; one stage per 1 KB row segment. Returns false
// after a timeout. Producer thread.
template <int NT>
DSV4CU_DEV bool smv_moe_emit(uint8_t *ring, uint8_t *bufs, SmvSmem<NT> &sm, SmvMoeProd &st, const SmvMoeParams &p,
                             int j, int nb, bool pre)
{
    const int ja_per = p.inter >> 5, jb_per = p.hidden >> 6;
    const SmvMoeJob jb = pre ? SmvMoeJob{0, 0, j} : smv_moe_job(j, ja_per, jb_per, nb + p.has_shared);
    const int bi = pre ? -1 : smv_moe_bucket(jb.o, nb, p.has_shared);
    const bool shared = pre || bi == nb;
    const int e = shared ? p.n_experts : p.ws.b_expert[bi];
    int s0 = 0, cnt = p.nt;
    if (!shared) {
        s0 = p.ws.b_off[bi];
        cnt = min(NT, p.ws.b_off[bi + 1] - s0);
    } else if (!pre) {
        s0 = p.ws.b_off[nb];
    }
    bool load = false;
    int b = 0;
    if (!pre) {
        b = smv_moe_operand(bufs, sm, st, p, jb, bi, shared, s0, cnt, &load);
        if (b < 0) return false;
    }
    SmvDesc d;
    d.job = st.jl;
    d.ntok = cnt;
    d.bbuf = b;
    d.bk = jb.phase == 0 ? p.hidden : p.inter;
    d.e0 = jb.phase;
    d.e1 = jb.o;
    d.e2 = jb.rg;
    d.e3 = 2;
    const dsv4cu_expert &ex = p.experts[e];
    bool first = true;
    int issued = 0;
    for (int m = 0; m < 2; m++) {
        const int mi = jb.phase == 0 ? m : 2, row0 = jb.phase == 0 ? jb.rg * 32 : jb.rg * 64 + m * 32;
        const CUtensorMap *mp = p.maps + 2 * (3 * e + mi);
        const SmvMat mat = smv_mat(mi == 0 ? ex.w1 : (mi == 1 ? ex.w3 : ex.w2), mp, mp + 1);
        const int nseg = smv_nseg(mat);
        for (int sg = 0; sg < nseg; sg++) {
            smv_seg_fields(d, mat, row0, sg);
            d.combo = m;
            d.flags = (first ? SMV_F_FIRST : 0) | (first && (load || pre) ? SMV_F_LOAD : 0) |
                      (sg == nseg - 1 ? SMV_F_FLUSH : 0) | (m == 1 && sg == nseg - 1 ? SMV_F_LAST : 0);
            first = false;
            // A deferred operand goes out before the producer could block on a
            // full ring that the consumers cannot drain without it.
            if (st.pend && issued >= p.geom.ns) smv_moe_pend_flush(bufs, sm, st, p);
            if (!smv_slot_free(sm, st.slot, st.ph, p.status)) return false;
            smv_put_stage(ring, sm, st.dr, st.slot, st.ph, d, mat, row0, sg);
            issued++;
            if (++st.slot == p.geom.ns) {
                st.slot = 0;
                st.ph ^= 1u;
            }
        }
    }
    if (st.pend) smv_moe_pend_flush(bufs, sm, st, p);
    st.jl++;
    return true;
}

// Warm the copy engine's descriptor cache with the maps job j will use (its
// expert's w1 and w3, or w2; the FP4 scale map only where rows span stages).
DSV4CU_DEV void smv_moe_prefetch_maps(const SmvMoeParams &p, int j, int nb)
{
    const SmvMoeJob jb = smv_moe_job(j, p.inter >> 5, p.hidden >> 6, nb + p.has_shared);
    const int bi = smv_moe_bucket(jb.o, nb, p.has_shared);
    const int e = bi == nb ? p.n_experts : p.ws.b_expert[bi];
    const dsv4cu_expert &ex = p.experts[e];
    for (int m = jb.phase == 0 ? 0 : 2; m <= (jb.phase == 0 ? 1 : 2); m++) {
        const CUtensorMap *mp = p.maps + 2 * (3 * e + m);
        asm volatile("prefetch.tensormap [%0];" ::"l"(mp) : "memory");
        const dsv4cu_qmat &q = m == 0 ? ex.w1 : (m == 1 ? ex.w3 : ex.w2);
        if (q.wdt == DSV4CU_WFP4 && q.cols / 2 > SMV_SEG) asm volatile("prefetch.tensormap [%0];" ::"l"(mp + 1) : "memory");
    }
}

template <int NT>
DSV4CU_DEV void smv_moe_producer(uint8_t *ring, uint8_t *bufs, SmvSmem<NT> &sm, const SmvMoeParams &p)
{
    SmvMoeProd st;
    st.slot = 0;
    st.ph = 0;
    st.jl = 0;
    st.pend = false;
    st.dr.valid = st.dr.par = 0;
    smv_buf_init(st.bs);
    const int ja_per = p.inter >> 5;
    int j = blockIdx.x;
    bool ok = true, pre = false;
    if (p.has_shared && j < ja_per) {
        // The shared expert's A jobs need nothing from prep: their weights go
        // out at once; the operand (x of tokens 0 .. nt - 1, buffer 0) follows
        // the dependency wait (smv_moe_pend_flush).
        int rows0[NT];
        for (int i = 0; i < NT; i++) rows0[i] = i < p.nt ? i : 0;
        st.bs.key[0] = smv_moe_xkey(rows0, p.nt);
        st.bs.uses[0] = 1;
        st.bs.cur = 0;
        st.pend = true;
        ok = smv_moe_emit<NT>(ring, bufs, sm, st, p, j, 0, true);
        pre = true;
    }
    pdl_wait();
    const int nb = p.ws.meta[0];
    const int njobs = (nb + p.has_shared) * (ja_per + (p.hidden >> 6));
    // The next job's number is fetched one job ahead, so the atomic's round
    // trip overlaps the current job's stages.
    int nj = ok ? atomicAdd(p.ws.ctr, 1) + (int)gridDim.x : njobs;
    if (!pre && j < njobs) smv_moe_prefetch_maps(p, j, nb);
    if (nj < njobs) smv_moe_prefetch_maps(p, nj, nb);
    if (ok && !pre && j < njobs) ok = smv_moe_emit<NT>(ring, bufs, sm, st, p, j, nb, false);
    while (ok && nj < njobs && !smv_aborted(&sm.abort_flag)) {
        const int cur = nj;
        nj = atomicAdd(p.ws.ctr, 1) + (int)gridDim.x;
        if (nj < njobs) smv_moe_prefetch_maps(p, nj, nb);
        ok = smv_moe_emit<NT>(ring, bufs, sm, st, p, cur, nb, false);
    }
    smv_end_marker<NT>(sm, st.dr, st.slot, st.ph, p.status);
    // Lets the next kernel launch; it waits for this grid before it reads.
    pdl_trigger();
}

// SwiGLU with the reference's comparisons (dsv4_ops.c:61-79): up clamped both
// ways, gate from above only, silu(g) = g / (1 + expf(-g)); limit <= 0: none.
DSV4CU_DEV float smv_swiglu(float g, float u, float limit)
{
    if (limit > 0.0f) {
        if (u > limit) u = limit;
        if (u < -limit) u = -limit;
        if (g > limit) g = limit;
    }
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// Epilogue of one finished job (epilogue warp).
template <int NT>
DSV4CU_DEV void smv_moe_epilogue(const SmvMoeParams &p, const SmvSmem<NT> &sm, int eb, const SmvEpi &e)
{
    const int lane = threadIdx.x & 31;
    const int nb = p.ws.meta[0];
    const int bi = smv_moe_bucket(e.e1, nb, p.has_shared);
    const int s0 = p.ws.b_off[bi];
    if (e.e0 == 0) {
        // A job: SwiGLU of row rg * 32 + lane (gate: part 0, up: part 1), then
        // each token's 32 values as one block of the down operand.
        const int row = e.e2 * 32 + lane;
        for (int i = 0; i < e.ntok; i++) {
            const float h = smv_swiglu(smv_job_value(sm, eb, 0, lane, i), smv_job_value(sm, eb, 1, lane, i), p.limit);
            uint16_t hi, lo;
            float fac;
            smv_split32(h, hi, lo, fac);
            const size_t o = (size_t)(s0 + i) * p.inter + row;
            p.ws.hh[o] = hi;
            p.ws.hl[o] = lo;
            if (lane == 0) p.ws.hs[(size_t)(s0 + i) * (p.inter >> 5) + e.e2] = fac;
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.ws.ctr + 1 + bi, 1);
    } else {
        // B job: rows rg * 64 + lane (part 0) and + 32 (part 1).
        const int rb = e.e2 * 64 + lane;
        for (int i = 0; i < e.ntok; i++) {
            p.ws.ypart[(size_t)(s0 + i) * p.hidden + rb] = smv_job_value(sm, eb, 0, lane, i);
            p.ws.ypart[(size_t)(s0 + i) * p.hidden + rb + 32] = smv_job_value(sm, eb, 1, lane, i);
        }
    }
}

// The MoE step as a streamer policy.
struct SmvMoePolicy {
    using Params = SmvMoeParams;
    template <int NT>
    static DSV4CU_DEV bool consumer_prologue(uint8_t *, SmvSmem<NT> &, const Params &)
    {
        return false;    // operands come by bulk copy (smv_moe_operand)
    }
    template <int NT>
    static DSV4CU_DEV void producer(uint8_t *ring, uint8_t *bufs, SmvSmem<NT> &sm, const Params &p)
    {
        smv_moe_producer<NT>(ring, bufs, sm, p);
    }
    template <int NT>
    static DSV4CU_DEV void epilogue(const Params &p, const SmvSmem<NT> &sm, int eb, const SmvEpi &e)
    {
        smv_moe_epilogue<NT>(p, sm, eb, e);
    }
};

// Output rows: per token the routed pairs IN k ORDER with the routing
// weights (dsv4_layer.c:109-113), then the shared expert unweighted (:115).
__global__ void __launch_bounds__(256) smv_moe_combine_kernel(SmvMoeWs ws, int nt, int topk, int hidden,
                                                              int has_shared, float *__restrict__ out)
{
    pdl_wait();
    pdl_trigger();
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    const int h4 = hidden >> 2;
    if (i >= (long)nt * h4) return;
    const int t = (int)(i / h4), row = (int)(i - (long)t * h4) * 4;
    float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
    for (int k = 0; k < topk; k++) {
        const int slot = ws.pos[t * topk + k];
        if (slot < 0) continue;
        const float w = ws.wts[t * topk + k];
        const float4 y = *reinterpret_cast<const float4 *>(ws.ypart + (size_t)slot * hidden + row);
        o0 = __fadd_rn(o0, __fmul_rn(w, y.x));
        o1 = __fadd_rn(o1, __fmul_rn(w, y.y));
        o2 = __fadd_rn(o2, __fmul_rn(w, y.z));
        o3 = __fadd_rn(o3, __fmul_rn(w, y.w));
    }
    if (has_shared) {
        const float4 sh = *reinterpret_cast<const float4 *>(ws.ypart + (size_t)(ws.b_off[ws.meta[0]] + t) * hidden + row);
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

// ------------------------------------------------------------- host side
bool smv_moe_layer_ok(const dsv4cu_expert *hexp, int n_experts, int hidden, int inter)
{
    if (hidden % 64 || inter % 32 || hidden > SMV_MAXK || inter > SMV_MAXK) return false;
    for (int e = 0; e <= n_experts; e++) {
        const dsv4cu_qmat *ms[3] = {&hexp[e].w1, &hexp[e].w3, &hexp[e].w2};
        for (int m = 0; m < 3; m++)
            if (!smv_ok(ms[m]->wdt, ms[m]->w, ms[m]->s, ms[m]->rows, ms[m]->cols, ms[m]->blk_r, ms[m]->blk_c))
                return false;
    }
    return true;
}

// The streamer's tensor maps of every matrix of the layer, in one device
// allocation (the kernel reads them from global memory).
int smv_moe_prepare(dsv4cu_moe *L, const dsv4cu_expert *hexp)
{
    const int nm = 3 * (L->n_experts + 1);
    std::vector<CUtensorMap> maps((size_t)2 * nm);
    for (int e = 0; e <= L->n_experts; e++) {
        const dsv4cu_qmat *ms[3] = {&hexp[e].w1, &hexp[e].w3, &hexp[e].w2};
        for (int m = 0; m < 3; m++) {
            const int r = smv_encode(ms[m], &maps[2 * (3 * e + m)], &maps[2 * (3 * e + m) + 1]);
            if (r) return r;
        }
    }
    void *blk = nullptr;
    cudaError_t ce = cudaMalloc(&blk, maps.size() * sizeof(CUtensorMap));
    if (ce != cudaSuccess) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "moe_create (stream maps): %s", cudaGetErrorString(ce));
    ce = cudaMemcpy(blk, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        cudaFree(blk);
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "moe_create (stream maps): %s", cudaGetErrorString(ce));
    }
    L->smv_block = blk;
    L->smv_maps = (const CUtensorMap *)blk;
    L->smv_ok = 1;
    return DSV4CU_OK;
}

size_t smv_moe_workspace(const dsv4cu_moe *L, int topk, int nt)
{
    return smv_moe_layout(smv_moe_shape(L, topk, nt), nullptr, nullptr);
}

template <int NT>
static int smv_moe_launch(SmvMoeParams p, int sms, cudaStream_t st)
{
    static SmemLimit lim;
    p.geom = smv_geometry<NT>(max(p.hidden, p.inter), 2);
    const int smem = smv_smem_bytes<NT>(p.geom);
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)smv_kernel<NT, SmvMoePolicy>, smem));
    DSV4CU_CUDA_TRY(launch_pdl(smv_kernel<NT, SmvMoePolicy>, dim3(sms), dim3(SMV_THREADS), smem, st, p));
    return DSV4CU_OK;
}

int smv_moe_decode(const dsv4cu_moe *L, float *out, const float *x, const float *logits, const float *bias,
                   const int64_t *tid2eid, const int *token_ids, int topk, float route_scale, float limit, int nt,
                   int *idx_out, float *wts_out, void *wsp, int *status, int sms, cudaStream_t st, cudaEvent_t *ev)
{
    if (nt < 1 || nt > SMV_MAXT || topk > SMV_MOE_MAX_TOPK || L->n_experts > 512)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "moe_decode (stream): nt %d / topk %d", nt, topk);
    const SmvMoeShape s = smv_moe_shape(L, topk, nt);
    SmvMoeWs ws;
    smv_moe_layout(s, (char *)wsp, &ws);
    const float *tab = router_table_get();
    if (!tab) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "moe_decode: router table setup failed");
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
    {
        const int split = (nt * (s.hidden / 32) + 7) / 8;
        const int grid = 1 + min(split, 2 * sms);
        DSV4CU_CUDA_TRY(launch_pdl(smv_moe_prep_kernel, dim3(grid), dim3(256), 0, st, tab, x, logits, bias, tid2eid,
                                   token_ids, s.n_experts, topk, route_scale, s.hidden, nt, s.has_shared, s.nbmax, ws,
                                   idx_out, wts_out));
    }
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));
    SmvMoeParams p;
    p.ws = ws;
    p.experts = L->view.experts;
    p.maps = L->smv_maps;
    p.nt = nt;
    p.hidden = s.hidden;
    p.inter = s.inter;
    p.has_shared = s.has_shared;
    p.n_experts = s.n_experts;
    p.limit = limit;
    p.status = status;
    const int r = nt == 1 ? smv_moe_launch<1>(p, sms, st) : smv_moe_launch<2>(p, sms, st);
    if (r) return r;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[2], st));
    {
        const long n = (long)nt * (s.hidden / 4);
        DSV4CU_CUDA_TRY(launch_pdl(smv_moe_combine_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, ws, nt,
                                   topk, s.hidden, s.has_shared, out));
    }
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[3], st));
    return DSV4CU_OK;
}

}  // namespace dsv4cu
