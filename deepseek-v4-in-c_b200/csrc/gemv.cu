// gemv.cu - dsv4cu_mmq: the packed matmul on device memory.
//
// Replaces dsv4_mmq_n (src/10_compute/dsv4_matmul.c:63-73) and the per-format
// bodies fp8_n / fp4_n / bf16_n. Three paths:
//   * fast: the tensor-core GEMV tile of gemv_core.cuh, for FP8 (blk_c % 16)
//     and FP4 (blk_c % 32) weights whose rows are whole 16-byte chunks.
//     Activations are first split into exact hi/lo operands (xprep_kernel).
//   * generic: every other FP8/FP4 geometry the reference accepts (any
//     blk_r/blk_c, ragged K), one thread per output in the scalar double
//     arithmetic of the reference's own scalar reference
//     (tests/unit/test_matmul.c:54-176).
//   * BF16: gemv_bf16.cu, the reference's double fma tree step for step.
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "ctx.h"
#include "gemv_core.cuh"
#include "gemv.h"
#include "mxgemm.h"
#include "tma_gemv.cuh"
#include "tmap.h"

namespace dsv4cu {

// ------------------------------------------------------------------ xprep
// One warp per (token, 32-element block): P = 14 - floor(log2 amax) so the
// block's magnitudes land in [2^14, 2^15); hi = f16(x 2^P), lo =
// f16(x 2^P - hi), xs = 2^-P. A bf16-valued x (8 significant bits) is exact in
// hi alone.
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
    const uint16_t h = __half_as_ushort(hh), l = __half_as_ushort(lh);
    const float s = ldexpf(1.0f, -P);
    xh[(size_t)t * ldx + k] = h;
    xl[(size_t)t * ldx + k] = l;
    if (lane == 0) xs[(size_t)t * nblk + b] = s;
}

// ------------------------------------------------------------- fast GEMV
// TMA-staged (tma_gemv.cuh): a CTA of 8 consumer warps + 1 producer covers R
// rows x the full K as 8 streams of 16 rows x one of P = 8 / (R/16) K-parts;
// the K-parts meet in shared memory in a fixed order, so results are
// deterministic and no cross-CTA reduction is needed. R is chosen so the grid
// fills about three CTAs per SM in a single wave.
constexpr int GEMV_STAGES = 2, GEMV_THREADS = 288;
using GemvSmem = TmaSmem<GEMV_STAGES>;

template <int FMT, int NT>
__global__ void __launch_bounds__(GEMV_THREADS, 3) gemv_tma_kernel(MatArgs m, const __grid_constant__ CUtensorMap tw,
                                                                  const __grid_constant__ CUtensorMap ts, int staged,
                                                                  XArgs x, int nt, int R, float *__restrict__ y,
                                                                  int *__restrict__ err)
{
    extern __shared__ __align__(128) unsigned char dsmem[];
    __shared__ Stream streams[8];
    __shared__ float red[8][NT][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int P = 8 / (R >> 4);
    const int row0 = blockIdx.x * R;
    // K-part length: whole 256-byte stages (stage-aligned part starts)
    const int L = (((m.row_bytes + P - 1) / P + TMA_SB - 1) / TMA_SB) * TMA_SB;
    if (threadIdx.x < 8) {
        Stream st;
        st.m = m;
        st.tw = &tw;
        st.ts = staged ? &ts : nullptr;
        st.row0 = row0 + (threadIdx.x / P) * 16;
        st.kb0 = (threadIdx.x % P) * L;
        streams[threadIdx.x] = st;
    }
    __syncthreads();
    for (int t0 = 0; t0 < nt; t0 += NT) {
        XArgs xt = x;
        xt.xh += (size_t)t0 * x.ldx;
        xt.xl += (size_t)t0 * x.ldx;
        xt.xs += (size_t)t0 * (x.ldx >> 5);
        float acc[NT][2];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.0f;
        tma_gemv_streams<FMT, NT, GEMV_STAGES>(dsmem, streams, L, xt, nt - t0, acc, err);
        if (warp < 8) {
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float s0 = quad_sum(acc[t][0]), s1 = quad_sum(acc[t][1]);
                if ((lane & 3) == 0) {
                    red[warp][t][lane >> 2] = s0;
                    red[warp][t][(lane >> 2) + 8] = s1;
                }
            }
        }
        __syncthreads();
        // rows of stream group w / P, K-parts summed in order
        for (int i = threadIdx.x; i < NT * R; i += blockDim.x) {
            const int t = i / R, r = i - t * R, grp = r >> 4, rr = r & 15, row = row0 + r;
            float v = 0.0f;
            for (int p = 0; p < P; p++) v += red[grp * P + p][t][rr];
            if (row < m.rows && t0 + t < nt) {
                if (isnan(v))
                    v = ref_row_nan(m.w + (size_t)row * m.row_bytes, m.s + (size_t)(row / m.blk_r) * m.s_cols,
                                    m.cols, m.blk_c, FMT == DSV4CU_WFP4);
                y[(size_t)(t0 + t) * m.rows + row] = v;
            }
        }
        __syncthreads();
    }
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
    float v = (float)total;
    if (isnan(v))
        v = ref_row_nan(W + (size_t)o * (wdt == DSV4CU_WFP4 ? cols / 2 : cols), srow, cols, blk_c,
                        wdt == DSV4CU_WFP4);
    y[(size_t)t * rows + o] = v;
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

int xprep_launch(const float *x, int cols, int ldx_in, int nt, int ldx, uint16_t *xh, uint16_t *xl, float *xs,
                 cudaStream_t st)
{
    const long warps = (long)nt * (ldx >> 5);
    const int threads = 256;
    const unsigned blocks = (unsigned)((warps * 32 + threads - 1) / threads);
    xprep_kernel<<<blocks, threads, 0, st>>>(x, cols, ldx_in, nt, ldx, xh, xl, xs);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

// Rows per CTA: the smallest of 16/32/64/128 whose grid still fits in one
// wave of three CTAs per SM (a second partial wave would double the tail).
static int choose_rows(const MatArgs &m, int sm_count)
{
    const int slots = 3 * sm_count;
    for (int R = 16; R <= 128; R <<= 1)
        if ((m.rows + R - 1) / R <= slots) return R;
    return 128;
}

template <int FMT>
static int launch_fast(const dsv4cu_qmat *q, const MatArgs &m, const XArgs &x, int nt, float *y, int sm_count,
                       int *err, cudaStream_t st)
{
    CUtensorMap tw, ts;
    memset(&ts, 0, sizeof ts);
    int staged = 0;
    int r = tmap_encode(q, &tw, &ts, &staged);
    if (r) return r;
    const int R = choose_rows(m, sm_count);
    const int grid = (m.rows + R - 1) / R;
    const int smem = GemvSmem::BYTES;
    if (nt == 1) {
        DSV4CU_CUDA_TRY(cudaFuncSetAttribute(gemv_tma_kernel<FMT, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        gemv_tma_kernel<FMT, 1><<<grid, GEMV_THREADS, smem, st>>>(m, tw, ts, staged, x, nt, R, y, err);
    } else {
        DSV4CU_CUDA_TRY(cudaFuncSetAttribute(gemv_tma_kernel<FMT, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        gemv_tma_kernel<FMT, 4><<<grid, GEMV_THREADS, smem, st>>>(m, tw, ts, staged, x, nt, R, y, err);
    }
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

// The fast path issues 16-byte weight loads: it needs a 16-byte aligned base.
static bool fast_ok(const dsv4cu_qmat *q)
{
    return fast_geometry(q->wdt, q->cols, q->blk_r, q->blk_c) && tmap_weights_ok(q);
}

size_t mmq_workspace(const dsv4cu_qmat *q, int nt, int sm_count)
{
    if (!q || nt <= 0) return 0;
    if (q->wdt == DSV4CU_WBF16) return bf16_chain_workspace(q->cols, nt);
    if (!fast_ok(q)) return 0;
    const size_t ldx = (size_t)((q->cols + 31) / 32) * 32;
    size_t b = dsv4cu_align256(nt * ldx * 2) * 2 + dsv4cu_align256(nt * (ldx / 32) * 4);
    return b;
}

int mmq_run(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *q, int nt,
            cudaStream_t st, void *ws, int *counters)
{
    if (q->wdt == DSV4CU_WBF16)
        return bf16_chain_run(y, x, q, nt, ws, ctx->status, st);
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
    (void)counters;
    int *err = ctx->status;
    int r = xprep_launch(x, q->cols, q->cols, nt, ldx, xh, xl, xs, st);
    if (r) return r;
    const int sms = ctx ? ctx->sm_count : 148;
    if (q->wdt == DSV4CU_WFP8) return launch_fast<DSV4CU_WFP8>(q, m, xa, nt, y, sms, err, st);
    return launch_fast<DSV4CU_WFP4>(q, m, xa, nt, y, sms, err, st);
}

}  // namespace dsv4cu

using namespace dsv4cu;

// Products of many tokens go to the tcgen05 GEMM; its per-matrix preparation
// (tensor map, scale blocks) is made in the workspace for this one call.
static bool mmq_use_mx(const dsv4cu_qmat *m, int nt) { return nt >= MX_MMQ_MIN_TOKENS && mx_supported(m); }

static size_t mmq_mx_workspace(const dsv4cu_qmat *m, int nt, int sms)
{
    MxMat tm;
    memset(&tm, 0, sizeof(tm));
    tm.q = *m;
    tm.kc = m->cols / 128;
    tm.tiles_m = (m->rows + 127) / 128;
    return dsv4cu_align256(mx_sfa_bytes(m)) + mx_workspace(&tm, nt, MX_MMQ_TERMS, sms);
}

extern "C" size_t dsv4cu_mmq_workspace(const dsv4cu_qmat *m, int nt)
{
    if (m && nt > 0 && mmq_use_mx(m, nt)) return mmq_mx_workspace(m, nt, mx_device_sms());
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
    if (mmq_use_mx(m, nt)) {
        int r = dsv4cu_ws_get(ctx, mmq_mx_workspace(m, nt, ctx->sm_count), &ws);
        if (r) return r;
        MxMat tm;
        r = mx_prepare(&tm, m, (uint8_t *)ws, (cudaStream_t)stream);
        if (r) return r;
        return mx_gemm(&tm, y, x, nt, MX_MMQ_TERMS, 0, 0, (char *)ws + dsv4cu_align256(mx_sfa_bytes(m)),
                       ctx->sm_count, ctx->status, (cudaStream_t)stream);
    }
    const size_t need = mmq_workspace(m, nt, ctx->sm_count);
    if (need) {
        int r = dsv4cu_ws_get(ctx, need, &ws);
        if (r) return r;
    }
    return mmq_run(ctx, y, x, m, nt, (cudaStream_t)stream, ws, ctx->counters);
}
