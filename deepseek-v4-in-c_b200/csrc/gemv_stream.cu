// gemv_stream.cu - the decode GEMV (1 or 2 tokens) of one packed FP8 / FP4
// matrix on the streamed GEMV core (stream_mv.cuh).
//
// Reference: fp8_n / fp4_n (src/10_compute/dsv4_matmul_fp8.c:49-177,
// dsv4_matmul_fp4.c:46-162) behind dsv4_mmq_n (src/10_compute/dsv4_matmul.c:
// 34-73): y[t * rows + o] = sum_c x[t * cols + c] * W[o][c].
//
// Two launches chained by programmatic dependent launch:
//   split   x -> the f16 hi / lo operand (one warp per token and 32-element
//           block); it lets the GEMV launch at its start;
//   stream  the matrix as stages of (32-row group, 1 KB row segment) in row
//           order; CTA c of G takes the contiguous stage range
//           [S c / G, S (c + 1) / G), so every SM streams the same number of
//           bytes. The weights do not depend on the split, so the producer
//           starts at once. A row group inside one CTA's range is finished by
//           its epilogue; a row group split between CTAs leaves one partial
//           per CTA, and the CTA whose partial arrives last (a per-row-group
//           counter) adds them in CTA order.
// Each output is summed in one fixed order that depends on the matrix shape
// and the SM count only: a token's row has the same bits for nt = 1 and 2
// and on every run.
#include <stdio.h>

#include "common.cuh"
#include "ctx.h"
#include "stream_mv.cuh"

namespace dsv4cu {

struct SmvDenseParams {
    SmvGeom geom;
    CUtensorMap wmap, smap;    // streamer maps of the matrix (stream_mv.cuh)
    dsv4cu_qmat q;
    const uint16_t *xh, *xl;   // [nt][K]
    const float *xs;           // [nt][K / 32]
    float *y;                  // [nt][rows]
    float *part;               // [rows / 32][maxparts][32][NT]
    int *cnt;                  // [rows / 32] arrivals (zero between calls)
    int nt, K, nseg, maxparts;
    long long stages;          // (rows / 32) * nseg
    int *status;
    int withhold;              // test fault: CTA 0 skips its stage 2 (dsv4cu_ctx_inject), 0 = none
    const float *x;            // [nt][K] fp32 activations, split by the consumer warps
};

// CTA whose range holds stage q (ranges [S c / G, S (c + 1) / G)).
DSV4CU_DEV int smv_dense_cta(long long q, long long S, int G) { return (int)(((q + 1) * G + S - 1) / S) - 1; }

// The operand built in shared memory by the consumer warps (every token's x,
// buffer 0): after the dependency wait (x may come from the previous kernel)
// each warp splits blocks warp, warp + 16, ... of 32 values into the f16 hi /
// lo pair and the block's power-of-two factor, the layout smv_consume reads.
// The split of all nt tokens into bufs (hi, lo, per-block factor):
template <int NT>
DSV4CU_DEV void smv_dense_split_run(uint8_t *bufs, const SmvDenseParams &p, int bstride)
{
    constexpr int PER = SMV_MAXK / 32 / SMV_CW;     // blocks per warp per token at most
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nblk = p.K >> 5;
    for (int i = 0; i < p.nt; i++) {
        uint8_t *b = bufs + (size_t)i * bstride;
        uint16_t *hi = reinterpret_cast<uint16_t *>(b), *lo = reinterpret_cast<uint16_t *>(b + 2 * (size_t)p.K);
        float *fac = reinterpret_cast<float *>(b + 4 * (size_t)p.K);
        // Every load of this warp's blocks in flight first, then the splits,
        // eight side by side.
        constexpr int G = 8;
        static_assert(PER % G == 0, "split groups");
        float v[PER];
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int k = warp + j * SMV_CW;
            v[j] = k < nblk ? __ldg(p.x + (size_t)i * p.K + k * 32 + lane) : 0.0f;
        }
#pragma unroll
        for (int g0 = 0; g0 < PER; g0 += G) {
            float vg[G], f[G];
            bool live[G];
            uint16_t h[G], l[G];
#pragma unroll
            for (int j = 0; j < G; j++) {
                vg[j] = v[g0 + j];
                live[j] = warp + (g0 + j) * SMV_CW < nblk;
            }
            smv_split32_n<G>(vg, live, h, l, f);
#pragma unroll
            for (int j = 0; j < G; j++) {
                const int k = warp + (g0 + j) * SMV_CW;
                if (!live[j]) continue;
                hi[k * 32 + lane] = h[j];
                lo[k * 32 + lane] = l[j];
                if (lane == 0) fac[k] = f[j];
            }
        }
    }
}

// The consumers' prologue: the dependency wait (x may come from the previous
// kernel), then the split.
template <int NT>
DSV4CU_DEV bool smv_dense_split(uint8_t *bufs, const SmvDenseParams &p, int bstride)
{
    pdl_wait();
    smv_dense_split_run<NT>(bufs, p, bstride);
    return true;
}

// Weights only: no dependency on the previous kernel, so the stages stream
// from the start and the next kernel may launch at once (it waits for this
// one before it reads anything this one writes). Producer thread; stage q =
// (32-row group r, segment sg) with q = r nseg + sg.
template <int NT>
DSV4CU_DEV void smv_dense_producer(uint8_t *ring, uint8_t *bufs, SmvSmem<NT> &sm, const SmvDenseParams &p)
{
    (void)bufs;
    pdl_trigger();
    const long long S = p.stages, G = gridDim.x;
    const long long b0 = S * blockIdx.x / G, b1 = S * (blockIdx.x + 1) / G;
    const SmvMat m = smv_mat(p.q, &p.wmap, &p.smap);
    SmvDrain dr = {0u, 0u};
    int slot = 0;
    uint32_t ph = 0;
    SmvDesc d;
    d.bbuf = 0;
    d.bk = p.K;
    d.ntok = p.nt;
    d.combo = 0;
    d.e3 = 1;
    int job = 0, s0 = 0, r = (int)(b0 / p.nseg), sg = (int)(b0 - (long long)r * p.nseg);
    bool ok = true;
    for (long long q = b0; q < b1 && ok; q++) {
        const bool first = q == b0 || sg == 0, last = q == b1 - 1 || sg == p.nseg - 1;
        if (first) s0 = sg;
        smv_seg_fields(d, m, r * SMV_ROWS, sg);
        d.job = job;
        d.flags = (first ? SMV_F_FIRST : 0) | (last ? SMV_F_FLUSH | SMV_F_LAST : 0);
        d.e0 = r;
        d.e1 = s0;
        d.e2 = last ? sg + 1 : 0;
        ok = smv_slot_free(sm, slot, ph, p.status);
        const bool skip = p.withhold && blockIdx.x == 0 && q - b0 == 2;
        if (ok && !skip) smv_put_stage(ring, sm, dr, slot, ph, d, m, r * SMV_ROWS, sg);
        if (++slot == p.geom.ns) {
            slot = 0;
            ph ^= 1u;
        }
        if (last) job++;
        if (++sg == p.nseg) {
            sg = 0;
            r++;
        }
    }
    smv_end_marker<NT>(sm, dr, slot, ph, p.status);
}

// y value with the reference's NaN bits (ref_row_nan) when the sum is NaN.
DSV4CU_DEV float smv_dense_fix(const SmvDenseParams &p, int row, float v)
{
    if (!isnan(v)) return v;
    const bool fp4 = p.q.wdt == DSV4CU_WFP4;
    const int rb = fp4 ? p.K / 2 : p.K, s_ld = (p.K + p.q.blk_c - 1) / p.q.blk_c;
    const uint8_t *w_row = (const uint8_t *)p.q.w + (size_t)row * rb;
    const uint8_t *s_row = (const uint8_t *)p.q.s + (size_t)(fp4 ? row : row / p.q.blk_r) * s_ld;
    return ref_row_nan(w_row, s_row, p.K, p.q.blk_c, fp4);
}

template <int NT>
DSV4CU_DEV void smv_dense_epilogue(const SmvDenseParams &p, const SmvSmem<NT> &sm, int eb, const SmvEpi &e)
{
    const int lane = threadIdx.x & 31;
    const int r = e.e0, s0 = e.e1, s1 = e.e2, row = r * SMV_ROWS + lane;
    const int rows = p.q.rows;
    if (s0 == 0 && s1 == p.nseg) {
        for (int i = 0; i < e.ntok; i++) p.y[(size_t)i * rows + row] = smv_dense_fix(p, row, smv_job_value(sm, eb, 0, lane, i));
        return;
    }
    // A part of a row group that other CTAs share: store it, count it, and
    // the last arrival sums the parts in CTA order. The parts are the
    // distinct owners of the group's stages (CTAs with empty ranges own none).
    const long long S = p.stages, q0 = (long long)r * p.nseg;
    int nparts = 0, ord = 0, prev = -1;
    for (int k = 0; k < p.nseg; k++) {
        const int c = smv_dense_cta(q0 + k, S, gridDim.x);
        if (c != prev) {
            if (c == (int)blockIdx.x) ord = nparts;
            nparts++;
            prev = c;
        }
    }
    float *base = p.part + (size_t)r * p.maxparts * SMV_ROWS * NT;
    for (int i = 0; i < e.ntok; i++) base[((size_t)ord * SMV_ROWS + lane) * NT + i] = smv_job_value(sm, eb, 0, lane, i);
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(p.cnt + r, 1);
    old = __shfl_sync(0xFFFFFFFFu, old, 0);
    if (old != nparts - 1) return;
    __threadfence();
    for (int i = 0; i < e.ntok; i++) {
        float s = 0.0f;
        for (int k = 0; k < nparts; k++) s += __ldcg(base + ((size_t)k * SMV_ROWS + lane) * NT + i);
        p.y[(size_t)i * rows + row] = smv_dense_fix(p, row, s);
    }
    if (lane == 0) atomicExch(p.cnt + r, 0);    // zero again for the next call
}

struct SmvDensePolicy {
    using Params = SmvDenseParams;
    template <int NT>
    static DSV4CU_DEV bool consumer_prologue(uint8_t *bufs, SmvSmem<NT> &, const Params &p)
    {
        return smv_dense_split<NT>(bufs, p, p.geom.bstride);
    }
    template <int NT>
    static DSV4CU_DEV void producer(uint8_t *ring, uint8_t *bufs, SmvSmem<NT> &sm, const Params &p)
    {
        smv_dense_producer<NT>(ring, bufs, sm, p);
    }
    template <int NT>
    static DSV4CU_DEV void epilogue(const Params &p, const SmvSmem<NT> &sm, int eb, const SmvEpi &e)
    {
        smv_dense_epilogue<NT>(p, sm, eb, e);
    }
};


struct DenseShape {
    int nt, NT, K, nseg, maxparts, groups;
    long long stages;
};

static DenseShape dense_shape(const dsv4cu_qmat *m, int nt)
{
    DenseShape s;
    s.nt = nt;
    s.NT = nt <= 1 ? 1 : 2;
    s.K = m->cols;
    const int rb = m->wdt == DSV4CU_WFP4 ? m->cols / 2 : m->cols;
    s.nseg = (rb + SMV_SEG - 1) / SMV_SEG;
    s.groups = m->rows / SMV_ROWS;
    s.stages = (long long)s.groups * s.nseg;
    s.maxparts = s.nseg;       // each part of a row group owns at least one of its stages
    return s;
}

static size_t dense_layout(const DenseShape &s, char *base, SmvDenseParams *p)
{
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *q = base ? base + off : nullptr;
        off += dsv4cu_align256(bytes);
        return q;
    };
    char *xh = take((size_t)s.nt * s.K * 2), *xl = take((size_t)s.nt * s.K * 2);
    char *xs = take((size_t)s.nt * (s.K / 32) * 4);
    char *part = take((size_t)s.groups * s.maxparts * SMV_ROWS * s.NT * 4);
    if (p) {
        p->xh = (const uint16_t *)xh;
        p->xl = (const uint16_t *)xl;
        p->xs = (const float *)xs;
        p->part = (float *)part;
    }
    return off;
}

static bool dense_ok(const dsv4cu_qmat *m, int nt)
{
    return m && nt >= 1 && nt <= SMV_MAXT && m->rows / SMV_ROWS <= DSV4CU_MAX_COUNTERS &&
           smv_ok(m->wdt, m->w, m->s, m->rows, m->cols, m->blk_r, m->blk_c);
}

template <int NT>
static int dense_launch(SmvDenseParams &p, int sms, cudaStream_t st)
{
    static SmemLimit lim;
    p.geom = smv_geometry<NT>(p.K, 1);
    const int smem = smv_smem_bytes<NT>(p.geom);
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)smv_kernel<NT, SmvDensePolicy>, smem));
    DSV4CU_CUDA_TRY(launch_pdl(smv_kernel<NT, SmvDensePolicy>, dim3(sms), dim3(SMV_THREADS), smem, st, p));
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" size_t dsv4cu_gemv_workspace(const dsv4cu_qmat *m, int nt)
{
    if (!dense_ok(m, nt)) return dsv4cu_mmq_workspace(m, nt);
    return dense_layout(dense_shape(m, nt), nullptr, nullptr);
}

extern "C" int dsv4cu_gemv_ev(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *m, int nt, void *stream,
                              void **events)
{
    if (!ctx || !y || !x || !m) return dsv4cu_set_error(DSV4CU_ERR_ARG, "gemv: NULL argument");
    cudaStream_t st = (cudaStream_t)stream;
    cudaEvent_t *ev = (cudaEvent_t *)events;
    if (!dense_ok(m, nt)) {
        // Shapes the streamer does not read (and nt > 2) take dsv4cu_mmq.
        if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
        if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));
        const int r = dsv4cu_mmq(ctx, y, x, m, nt, stream);
        if (!r && ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[2], st));
        return r;
    }
    const int sms = ctx->sm_count;
    const DenseShape s = dense_shape(m, nt);
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, dense_layout(s, nullptr, nullptr), &ws);
    if (r) return r;
    SmvDenseParams p;
    dense_layout(s, (char *)ws, &p);
    p.q = *m;
    r = smv_encode(m, &p.wmap, &p.smap);
    if (r) return r;
    p.y = y;
    p.cnt = ctx->counters;
    p.nt = nt;
    p.K = s.K;
    p.nseg = s.nseg;
    p.maxparts = s.maxparts;
    p.stages = s.stages;
    p.status = ctx->status;
    p.withhold = ctx->inject == DSV4CU_INJECT_WITHHOLD_STAGE;
    ctx->inject = 0;
    p.x = x;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));
    r = s.NT == 1 ? dense_launch<1>(p, sms, st) : dense_launch<2>(p, sms, st);
    if (r) return r;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[2], st));
    return DSV4CU_OK;
}

extern "C" int dsv4cu_gemv(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *m, int nt, void *stream)
{
    return dsv4cu_gemv_ev(ctx, y, x, m, nt, stream, nullptr);
}
