// gemv.cu - dsv4cu_mmq: the packed matmul on device memory.
//
// Replaces dsv4_mmq_n (src/10_compute/dsv4_matmul.c:63-73) and the per-format
// bodies fp8_n / fp4_n / bf16_n. Two paths:
//   * fast: the tensor-core GEMV tile of gemv_core.cuh, for FP8 (blk_c % 16),
//     FP4 (blk_c % 32) and BF16 weights whose rows are whole 16-byte chunks.
//     Activations are first split into exact hi/lo operands (xprep_kernel).
//   * generic: every other geometry the reference accepts (any blk_r/blk_c,
//     ragged K), one thread per output in the scalar double arithmetic of the
//     reference's own scalar reference (tests/unit/test_matmul.c:54-176).
#include <stdio.h>

#include "common.cuh"
#include "ctx.h"
#include "gemv_core.cuh"
#include "gemv.h"

namespace dsv4cu {

// ------------------------------------------------------------------ xprep
// One warp per (token, 32-element block). F16 mode: P = 14 - floor(log2 amax)
// so the block's magnitudes land in [2^14, 2^15); hi = f16(x 2^P), lo =
// f16(x 2^P - hi), xs = 2^-P. A bf16-valued x (8 significant bits) is exact in
// hi alone. BF16 mode (for BF16 weights): hi = bf16(x), lo = bf16(x - hi), xs = 1.
template <bool BF16MODE>
__global__ void xprep_kernel(const float *__restrict__ x, int cols, int ldx_in, int nt,
                             int ldx, uint16_t *__restrict__ xh, uint16_t *__restrict__ xl,
                             float *__restrict__ xs)
{
    const int nblk = ldx >> 5;
    const int gw = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (gw >= nt * nblk) return;
    const int t = gw / nblk, b = gw - t * nblk, k = b * 32 + lane;
    const float v = k < cols ? x[(size_t)t * ldx_in + k] : 0.0f;
    uint16_t h, l;
    float s = 1.0f;
    if constexpr (BF16MODE) {
        const __nv_bfloat16 hb = __float2bfloat16_rn(v);
        const float hf = __bfloat162float(hb);
        const __nv_bfloat16 lb = isfinite(hf) ? __float2bfloat16_rn(v - hf) : __float2bfloat16_rn(0.0f);
        h = __bfloat16_as_ushort(hb);
        l = __bfloat16_as_ushort(lb);
    } else {
        float a = isfinite(v) ? fabsf(v) : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
        int P = 0;
        if (a > 0.0f) {
            int e;
            frexpf(a, &e);          // a = f 2^e, f in [0.5, 1): floor(log2 a) = e - 1
            P = 15 - e;
            P = P > 125 ? 125 : (P < -125 ? -125 : P);
        }
        const float vs = ldexpf(v, P);
        const __half hh = __float2half_rn(vs);
        const float hf = __half2float(hh);
        const __half lh = isfinite(hf) ? __float2half_rn(vs - hf) : __float2half_rn(0.0f);
        h = __half_as_ushort(hh);
        l = __half_as_ushort(lh);
        s = ldexpf(1.0f, -P);
    }
    xh[(size_t)t * ldx + k] = h;
    xl[(size_t)t * ldx + k] = l;
    if (lane == 0) xs[(size_t)t * nblk + b] = s;
}

// ------------------------------------------------------------- fast GEMV
// grid (row groups of 16, ks K-slices); block NW warps splitting the CTA's
// K-slice. Partial sums are combined in a fixed order, so results are
// deterministic: warps through shared memory, K-slices (ks > 1) by the last
// CTA of a row group, which reads every slice's partial in slice order.
template <int FMT, int NT, int DEPTH>
__global__ void __launch_bounds__(256) gemv_kernel(MatArgs m, XArgs x, int nt, float *__restrict__ y,
                                                   int ks, float *__restrict__ part,
                                                   int *__restrict__ counters)
{
    __shared__ float red[8][NT][16];
    __shared__ int last;
    const int rg = blockIdx.x, kz = blockIdx.y;
    const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ns = (m.row_bytes + 63) >> 6;
    const int cb = (int)((long)kz * ns / ks), ce = (int)((long)(kz + 1) * ns / ks);
    const int wb = cb + (int)((long)warp * (ce - cb) / nw);
    const int we = cb + (int)((long)(warp + 1) * (ce - cb) / nw);

    for (int t0 = 0; t0 < nt; t0 += NT) {
        float acc[NT][2];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.0f;
        XArgs xt = x;
        xt.xh += (size_t)t0 * x.ldx;
        xt.xl += (size_t)t0 * x.ldx;
        xt.xs += (size_t)t0 * (x.ldx >> 5);
        gemv_tile16<FMT, NT, DEPTH>(m, rg * 16, wb, we, xt, nt - t0, acc);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float s0 = quad_sum(acc[t][0]), s1 = quad_sum(acc[t][1]);
            if ((lane & 3) == 0) {
                red[warp][t][lane >> 2] = s0;
                red[warp][t][(lane >> 2) + 8] = s1;
            }
        }
        __syncthreads();
        if (threadIdx.x < NT * 16) {
            const int t = threadIdx.x >> 4, r = threadIdx.x & 15, row = rg * 16 + r;
            float s = 0.0f;
            for (int w = 0; w < nw; w++) s += red[w][t][r];
            if (row < m.rows && t0 + t < nt) {
                if (ks == 1) y[(size_t)(t0 + t) * m.rows + row] = s;
                else part[((size_t)kz * nt + t0 + t) * m.rows + row] = s;
            }
        }
        __syncthreads();
    }
    if (ks == 1) return;

    // Last CTA of this row group sums the ks slices in order.
    __threadfence();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(&counters[rg], 1);
        last = (prev == ks - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = threadIdx.x; i < nt * 16; i += blockDim.x) {
        const int t = i >> 4, row = rg * 16 + (i & 15);
        if (row >= m.rows) continue;
        float s = 0.0f;
        for (int z = 0; z < ks; z++) s += __ldcg(part + ((size_t)z * nt + t) * m.rows + row);
        y[(size_t)t * m.rows + row] = s;
    }
    if (threadIdx.x == 0) counters[rg] = 0;
}

// ----------------------------------------------------------- generic path
// One thread per (token, row): exact decode, block dot in double, one
// multiply by the block scale per block, totals in double, one rounding.
__global__ void gemv_generic_kernel(const uint8_t *__restrict__ W, const uint8_t *__restrict__ S,
                                    int wdt, int rows, int cols, int blk_r, int blk_c,
                                    const float *__restrict__ x, int nt, float *__restrict__ y)
{
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)nt * rows) return;
    const int t = (int)(i / rows), o = (int)(i - (long)t * rows);
    const float *xt = x + (size_t)t * cols;
    if (wdt == DSV4CU_WBF16) {
        const uint16_t *row = reinterpret_cast<const uint16_t *>(W) + (size_t)o * cols;
        double acc = 0.0;
        for (int c = 0; c < cols; c++)
            acc = __dadd_rn(acc, __dmul_rn((double)__uint_as_float((uint32_t)row[c] << 16), (double)xt[c]));
        y[(size_t)t * rows + o] = (float)acc;
        return;
    }
    const int sc = (cols + blk_c - 1) / blk_c;
    const uint8_t *srow = S + (size_t)(o / blk_r) * sc;
    double total = 0.0;
    int bi = 0;
    for (int c0 = 0; c0 < cols; c0 += blk_c, bi++) {
        const int n = min(blk_c, cols - c0);
        double acc = 0.0;
        if (wdt == DSV4CU_WFP8) {
            const uint8_t *rw = W + (size_t)o * cols + c0;
            for (int k = 0; k < n; k++)
                acc = __dadd_rn(acc, __dmul_rn((double)e4m3_to_f32(rw[k]), (double)xt[c0 + k]));
        } else {
            const uint8_t *rw = W + (size_t)o * (cols / 2);
            for (int k = 0; k < n; k++) {
                const int e = c0 + k;
                const uint32_t byte = rw[e >> 1];
                const float wv = e2m1_to_f32((e & 1) ? (byte >> 4) : (byte & 15u));
                acc = __dadd_rn(acc, __dmul_rn((double)wv, (double)xt[e]));
            }
        }
        total = __dadd_rn(total, __dmul_rn(acc, (double)e8m0_to_f32(srow[bi])));
    }
    y[(size_t)t * rows + o] = (float)total;
}

int row_bytes_of(int wdt, int cols)
{
    return wdt == DSV4CU_WFP4 ? cols / 2 : (wdt == DSV4CU_WFP8 ? cols : 2 * cols);
}

MatArgs mat_args(const dsv4cu_qmat *q)
{
    MatArgs m;
    m.w = (const uint8_t *)q->w;
    m.s = (const uint8_t *)q->s;
    m.rows = q->rows;
    m.cols = q->cols;
    m.blk_r = q->wdt == DSV4CU_WBF16 ? 1 : q->blk_r;
    m.blk_c = q->wdt == DSV4CU_WBF16 ? 1 : q->blk_c;
    m.s_cols = q->wdt == DSV4CU_WBF16 ? 0 : (q->cols + q->blk_c - 1) / q->blk_c;
    m.row_bytes = row_bytes_of(q->wdt, q->cols);
    return m;
}

int xprep_launch(const float *x, int cols, int ldx_in, int nt, int ldx, bool bf16mode,
                 uint16_t *xh, uint16_t *xl, float *xs, cudaStream_t st)
{
    const long warps = (long)nt * (ldx >> 5);
    const int threads = 256;
    const unsigned blocks = (unsigned)((warps * 32 + threads - 1) / threads);
    if (bf16mode)
        xprep_kernel<true><<<blocks, threads, 0, st>>>(x, cols, ldx_in, nt, ldx, xh, xl, xs);
    else
        xprep_kernel<false><<<blocks, threads, 0, st>>>(x, cols, ldx_in, nt, ldx, xh, xl, xs);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

template <int FMT>
static int launch_fast(const MatArgs &m, const XArgs &x, int nt, float *y, int ks, float *part,
                       int *counters, cudaStream_t st)
{
    const int rg = (m.rows + 15) / 16;
    dim3 grid(rg, ks), block(256);
    if (nt == 1)
        gemv_kernel<FMT, 1, 2><<<grid, block, 0, st>>>(m, x, nt, y, ks, part, counters);
    else if (nt == 2)
        gemv_kernel<FMT, 2, 2><<<grid, block, 0, st>>>(m, x, nt, y, ks, part, counters);
    else
        gemv_kernel<FMT, 4, 2><<<grid, block, 0, st>>>(m, x, nt, y, ks, part, counters);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

// Split-K factor: enough warps for ~32 per SM, at least 2 segments per warp.
static int choose_ks(const MatArgs &m, int sm_count)
{
    const int rg = (m.rows + 15) / 16, ns = (m.row_bytes + 63) / 64;
    int ks = (sm_count * 32) / (rg * 8);
    const int maxks = ns / 16;   // >= 2 segments per warp of 8
    if (ks > maxks) ks = maxks;
    if (ks < 1) ks = 1;
    if (ks > 64) ks = 64;
    return ks;
}

// The fast path issues 16-byte weight loads: it needs a 16-byte aligned base.
static bool fast_ok(const dsv4cu_qmat *q)
{
    return fast_geometry(q->wdt, q->cols, q->blk_r, q->blk_c) && ((uintptr_t)q->w & 15u) == 0;
}

size_t mmq_workspace(const dsv4cu_qmat *q, int nt, int sm_count)
{
    if (!q || nt <= 0) return 0;
    if (!fast_ok(q)) return 0;
    const size_t ldx = (size_t)((q->cols + 31) / 32) * 32;
    size_t b = dsv4cu_align256(nt * ldx * 2) * 2 + dsv4cu_align256(nt * (ldx / 32) * 4);
    const MatArgs m = mat_args(q);
    const int ks = choose_ks(m, sm_count);
    if (ks > 1) b += dsv4cu_align256((size_t)ks * nt * q->rows * 4);
    return b;
}

int mmq_run(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *q, int nt,
            cudaStream_t st, void *ws, int *counters)
{
    const MatArgs m = mat_args(q);
    if (!fast_ok(q)) {
        const long n = (long)nt * q->rows;
        gemv_generic_kernel<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(
            (const uint8_t *)q->w, (const uint8_t *)q->s, q->wdt, q->rows, q->cols, q->blk_r,
            q->blk_c, x, nt, y);
        DSV4CU_LAUNCH_CHECK();
        return DSV4CU_OK;
    }
    const int ldx = ((q->cols + 31) / 32) * 32;
    char *p = (char *)ws;
    XArgs xa;
    xa.ldx = ldx;
    xa.tok = nullptr;
    xa.xh = (const uint16_t *)p;
    uint16_t *xh = (uint16_t *)p;
    p += dsv4cu_align256((size_t)nt * ldx * 2);
    uint16_t *xl = (uint16_t *)p;
    xa.xl = xl;
    p += dsv4cu_align256((size_t)nt * ldx * 2);
    float *xs = (float *)p;
    xa.xs = xs;
    p += dsv4cu_align256((size_t)nt * (ldx / 32) * 4);
    float *part = (float *)p;
    int r = xprep_launch(x, q->cols, q->cols, nt, ldx, q->wdt == DSV4CU_WBF16, xh, xl, xs, st);
    if (r) return r;
    const int ks = choose_ks(m, ctx ? ctx->sm_count : 148);
    if (ks > 1 && (m.rows + 15) / 16 > DSV4CU_MAX_COUNTERS)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "mmq: too many row groups");
    switch (q->wdt) {
    case DSV4CU_WFP8: return launch_fast<DSV4CU_WFP8>(m, xa, nt, y, ks, part, counters, st);
    case DSV4CU_WFP4: return launch_fast<DSV4CU_WFP4>(m, xa, nt, y, ks, part, counters, st);
    default: return launch_fast<DSV4CU_WBF16>(m, xa, nt, y, ks, part, counters, st);
    }
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" size_t dsv4cu_mmq_workspace(const dsv4cu_qmat *m, int nt)
{
    return mmq_workspace(m, nt, 148);
}

extern "C" int dsv4cu_mmq(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *m,
                          int nt, void *stream)
{
    if (!ctx || !y || !x || !m) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mmq: NULL argument");
    if (nt <= 0) return DSV4CU_OK;   // the reference returns without work (dsv4_matmul.c:65)
    if (m->wdt != DSV4CU_WBF16 && m->wdt != DSV4CU_WFP8 && m->wdt != DSV4CU_WFP4)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "mmq: matrix has unimplemented wdt %d (%dx%d)",
                                m->wdt, m->rows, m->cols);
    if (m->rows <= 0 || m->cols <= 0 || !m->w)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "mmq: bad shape %dx%d", m->rows, m->cols);
    if (m->wdt != DSV4CU_WBF16 && (!m->s || m->blk_r <= 0 || m->blk_c <= 0))
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "mmq: scaled matrix needs s and blk_r/blk_c > 0");
    if (m->wdt == DSV4CU_WFP4 && (m->cols & 1))
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "mmq: FP4 cols must be even");
    void *ws = nullptr;
    const size_t need = mmq_workspace(m, nt, ctx->sm_count);
    if (need) {
        int r = dsv4cu_ws_get(ctx, need, &ws);
        if (r) return r;
    }
    return mmq_run(ctx, y, x, m, nt, (cudaStream_t)stream, ws, ctx->counters);
}
