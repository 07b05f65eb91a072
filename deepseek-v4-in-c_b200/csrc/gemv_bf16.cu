// gemv_bf16.cu - the BF16 matmul in the reference's own double arithmetic.
//
// Reference: bf16_n (src/10_compute/dsv4_matmul.c:88-113) with BLOCK_DOT_V
// (src/10_compute/dsv4_dec_common.h:45-61). Its scalar twin BLOCK_DOT_S
// (tests/unit/test_matmul.c:54-67) is held to the same bits by the reference's
// own gate. Per (token, row), with w and x widened exactly to double and
// n16 = 16 * floor(n / 16):
//   a[c] = fma chain over i = c, c + 16, c + 32, ... < n16, from +0   (c = 0..15)
//   b[j] = (a[j] + a[j + 4]) + (a[j + 8] + a[j + 12])                (j = 0..3)
//   acc  = (b[0] + b[1]) + (b[2] + b[3]); acc = fma(w[i], x[i], acc) for i >= n16
//   y    = (float)acc
// Every step here is the same IEEE double operation in the same order, so y
// carries the reference's bits (a NaN's payload aside: the GPU returns its
// canonical NaN). A bf16 x fp32 product has at most 32 significant bits, so each
// fma is the exact product plus one rounded add, as on the host.
//
// Work split (both kernels): lanes 2r and 2r + 1 of a warp own chains 0-7 and
// 8-15 of row r, 16 rows per row group. x is widened once per call into a
// double copy (xd, rows of ldxd doubles, zero-padded). Weights are widened with
// integer ops: a normal bf16 becomes the double whose high word is
// sign | (exponent + 896) << 20 | mantissa << 13; a 16-byte word that holds a
// zero, subnormal, inf or NaN takes the float conversion instead, which is exact
// for every bf16.
//
// bf16_chain_tma_kernel (rows of 16-byte multiples, at least 128 bytes, aligned
// base): one producer warp streams each consumer warp's rows through a ring of
// shared-memory stages with tensor-map TMA (16-row x 128-byte boxes, 128-byte
// swizzle, 256 bytes of every row per stage) and the stage's 128 activation
// columns as doubles with a bulk copy; the consumers read both from shared
// memory. Every wait is bounded and records an error code instead of hanging.
// bf16_chain_kernel (any other geometry): each lane loads its row's 16-byte
// words directly, the next 64-column group in flight, and reads xd through L1.
#include "common.cuh"
#include "ctx.h"
#include "gemv.h"
#include "tma_gemv.cuh"
#include "tmap.h"

namespace dsv4cu {

constexpr int BFC_WARPS = 8;            // 128 rows per CTA
constexpr int BFC_THREADS = 32 * BFC_WARPS;

// x rows widened to double, zero-padded to ldxd columns.
__global__ void bf16_xwiden_kernel(const float *__restrict__ x, int cols, int nt, int ldxd,
                                   double *__restrict__ xd)
{
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)nt * ldxd) return;
    const int t = (int)(i / ldxd), k = (int)(i - (long)t * ldxd);
    xd[i] = k < cols ? (double)x[(size_t)t * cols + k] : 0.0;
}

// All 8 bf16 of the word have an exponent field in 1..254. Per halfword with
// exponent field E: ((E + 1) >> 1) & 0x7F is zero exactly for E = 0 and 255;
// adding 0x7F00 then sets the halfword's top bit exactly when it is not.
DSV4CU_DEV bool bf16x8_normal(uint4 u)
{
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t ok = 0xFFFFFFFFu;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t g = ((w[i] & 0x7F807F80u) + 0x00800080u) & 0x7F007F00u;
        ok &= g + 0x7F007F00u;
    }
    return (ok & 0x80008000u) == 0x80008000u;
}

// The normal bf16 held in bits 31..16 of u, as a double.
DSV4CU_DEV double bf16_top_to_f64(uint32_t u)
{
    const uint32_t hi = ((uint32_t)((int32_t)u >> 3) & 0x8FFFE000u) + 0x38000000u;
    return __hiloint2double((int)hi, 0);
}

DSV4CU_DEV void bf16x8_to_f64(uint4 u, bool normal, double (&w)[8])
{
    const uint32_t q[4] = {u.x, u.y, u.z, u.w};
    if (normal) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = bf16_top_to_f64(q[i] << 16);
            w[2 * i + 1] = bf16_top_to_f64(q[i]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = (double)__uint_as_float(q[i] << 16);
            w[2 * i + 1] = (double)__uint_as_float(q[i] & 0xFFFF0000u);
        }
    }
}

// The 8 bf16 of row `row` at column c (c % 8 == 0). VEC: the row's bytes are
// 16-byte aligned, one vector load; otherwise 8 halfword loads.
template <bool VEC>
DSV4CU_DEV uint4 bf16x8_load(const uint16_t *__restrict__ row, int c)
{
    if constexpr (VEC) {
        return __ldg(reinterpret_cast<const uint4 *>(row + c));
    } else {
        uint32_t q[4];
#pragma unroll
        for (int i = 0; i < 4; i++)
            q[i] = (uint32_t)__ldg(row + c + 2 * i) | ((uint32_t)__ldg(row + c + 2 * i + 1) << 16);
        return make_uint4(q[0], q[1], q[2], q[3]);
    }
}

// One 16-column step for the lane's 8 chains and every token of the tile.
template <int NT>
DSV4CU_DEV void bf16_step(uint4 u, const double *__restrict__ xs, int ldxd, int ntile, double (&a)[NT][8])
{
    double w[8];
    bf16x8_to_f64(u, bf16x8_normal(u), w);
#pragma unroll
    for (int t = 0; t < NT; t++) {
        if (t >= ntile) break;
        const double2 *xp = reinterpret_cast<const double2 *>(xs + (size_t)t * ldxd);
        double2 xv[4];
#pragma unroll
        for (int i = 0; i < 4; i++) xv[i] = __ldg(xp + i);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            a[t][2 * i] = __fma_rn(w[2 * i], xv[i].x, a[t][2 * i]);
            a[t][2 * i + 1] = __fma_rn(w[2 * i + 1], xv[i].y, a[t][2 * i + 1]);
        }
    }
}

template <int NT, bool VEC>
__global__ void __launch_bounds__(BFC_THREADS) bf16_chain_kernel(const uint16_t *__restrict__ W, int rows, int cols,
                                                                  const double *__restrict__ xd, int ldxd, int nt,
                                                                  float *__restrict__ y)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = (blockIdx.x * BFC_WARPS + warp) * 16 + (lane >> 1), h = lane & 1;
    const int t0 = blockIdx.y * NT, ntile = min(NT, nt - t0);
    if ((blockIdx.x * BFC_WARPS + warp) * 16 >= rows) return;       // whole warp past the end
    const uint16_t *wrow = W + (size_t)min(row, rows - 1) * cols;  // rows past the end load row rows - 1
    const double *xt = xd + (size_t)t0 * ldxd;
    double a[NT][8];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int q = 0; q < 8; q++) a[t][q] = 0.0;

    const int M = cols >> 4;         // whole 16-column steps
    const int G = M >> 2;            // whole 64-column groups
    uint4 nxt[4];
    if (G > 0) {
#pragma unroll
        for (int s = 0; s < 4; s++) nxt[s] = bf16x8_load<VEC>(wrow, 16 * s + 8 * h);
    }
    for (int g = 0; g < G; g++) {
        uint4 cur[4];
#pragma unroll
        for (int s = 0; s < 4; s++) cur[s] = nxt[s];
        if (g + 1 < G) {
#pragma unroll
            for (int s = 0; s < 4; s++) nxt[s] = bf16x8_load<VEC>(wrow, 64 * (g + 1) + 16 * s + 8 * h);
        }
#pragma unroll
        for (int s = 0; s < 4; s++) bf16_step<NT>(cur[s], xt + 64 * g + 16 * s + 8 * h, ldxd, ntile, a);
    }
    for (int m = 4 * G; m < M; m++) bf16_step<NT>(bf16x8_load<VEC>(wrow, 16 * m + 8 * h), xt + 16 * m + 8 * h,
                                                  ldxd, ntile, a);

    // Fold: lane h = 0 holds chains 0-7, h = 1 chains 8-15. Each forms
    // a[j] + a[j + 4] on its half; the pair then adds the halves.
#pragma unroll
    for (int t = 0; t < NT; t++) {
        double b[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const double mine = a[t][j] + a[t][j + 4];
            const double other = __shfl_xor_sync(0xFFFFFFFFu, mine, 1);
            b[j] = h ? other + mine : mine + other;
        }
        if (t >= ntile || h) continue;
        double acc = (b[0] + b[1]) + (b[2] + b[3]);
        const double *xr = xt + (size_t)t * ldxd;
        for (int i = 16 * M; i < cols; i++)
            acc = __fma_rn((double)__uint_as_float((uint32_t)__ldg(wrow + i) << 16), xr[i], acc);
        if (row < rows) y[(size_t)(t0 + t) * rows + row] = __double2float_rn(acc);
    }
}

// ------------------------------------------------------- TMA-staged variant
// Stage layout: [CW consumer warps][R row groups][2 boxes of 16 rows x 128 B]
// of weights, then [NT][128] activation doubles. Stage sizes are multiples of
// 1 KB, so every box stays on the 1024-byte boundary of the 128-byte swizzle.
// One CTA per SM: the stages fill about 220 KB. The kernel is latency-bound
// (dependent widening -> fma chains per lane), so CW = 16 consumer warps with
// one row group each keep twice the warps in flight of 8 warps with two (the
// four-token tiles hold 4x the chains per lane and use 12 warps to stay in
// registers).
template <int R, int NT, int CW>
struct BfcCfg {
    static constexpr int STREAM = 16 * R * TMA_SB;     // weight bytes per warp per stage
    static constexpr int WBYTES = CW * STREAM;
    static constexpr int XBYTES = NT * 128 * 8;
    static constexpr int STAGE = WBYTES + XBYTES;
    static constexpr int STAGES = (220 * 1024) / STAGE < 6 ? (220 * 1024) / STAGE : 6;
    static constexpr int SMEM = 1024 + STAGES * STAGE + 2 * STAGES * 8;
    static constexpr int THREADS = 32 * (CW + 1);      // CW consumer warps + 1 producer warp
    static_assert(STAGES >= 2 && CW <= 32, "stage ring");
};

DSV4CU_DEV void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

template <int R, int NT, int CW>
__global__ void __launch_bounds__(BfcCfg<R, NT, CW>::THREADS, 1) bf16_chain_tma_kernel(
    const __grid_constant__ CUtensorMap tw, const uint16_t *__restrict__ W, int rows, int cols,
    const double *__restrict__ xd, int ldxd, int nt, float *__restrict__ y, int *__restrict__ err)
{
    using C = BfcCfg<R, NT, CW>;
    extern __shared__ __align__(128) unsigned char dsmem[];
    unsigned char *base = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(base + C::STAGES * C::STAGE);
    uint64_t *empty = full + C::STAGES;
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row_cta = blockIdx.x * 16 * R * CW;
    const int t0 = blockIdx.y * NT, ntile = min(NT, nt - t0);
    const int M = cols >> 4;                       // chain steps; stage k holds steps 8k .. 8k + 7
    const int nst = (M + 7) >> 3;
    const int rb = 2 * cols;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, CW);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == CW) {
        // ---------------- producer: lane w < CW loads warp w's boxes, lane t < ntile token t's columns
        const int row_w = row_cta + 16 * R * lane;
        for (int k = 0; k < nst; k++) {
            const int s = k % C::STAGES;
            if (k >= C::STAGES) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(empty + s, ((k / C::STAGES) - 1) & 1, err, 0x201);
                ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
                if (!ok) {
                    if (lane == 0) abort_flag = 1;
                    break;
                }
            }
            const int x0 = k * TMA_SB;
            uint32_t bytes = lane < ntile ? 1024u : 0u;
            if (lane < CW) {
#pragma unroll
                for (int g = 0; g < R; g++) {
                    const bool in = row_w + 16 * g < rows;
                    bytes += (in && x0 < rb ? 2048u : 0u) + (in && x0 + TMA_BOX_HALF < rb ? 2048u : 0u);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) bytes += __shfl_xor_sync(0xFFFFFFFFu, bytes, o);
            if (lane == 0) mbar_arrive_expect_tx(full + s, bytes);
            __syncwarp();
            unsigned char *st = base + s * C::STAGE;
            if (lane < CW) {
#pragma unroll
                for (int g = 0; g < R; g++) {
                    const int r0 = row_w + 16 * g;
                    unsigned char *dst = st + lane * C::STREAM + g * 4096;
                    if (r0 < rows && x0 < rb) tma_load_2d(dst, &tw, x0, r0, full + s);
                    if (r0 < rows && x0 + TMA_BOX_HALF < rb) tma_load_2d(dst + 2048, &tw, x0 + TMA_BOX_HALF, r0, full + s);
                }
            }
            if (lane < ntile)
                bulk_copy_g2s(st + C::WBYTES + lane * 1024, xd + (size_t)(t0 + lane) * ldxd + (size_t)k * 128, 1024u,
                              full + s);
        }
        return;
    }

    // ---------------- consumers: lane (r, h), rows row_cta + 16 R warp + 16 g + r
    const int r = lane >> 1, h = lane & 1;
    double a[NT][R][8];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int g = 0; g < R; g++)
#pragma unroll
            for (int q = 0; q < 8; q++) a[t][g][q] = 0.0;
    for (int k = 0; k < nst; k++) {
        const int s = k % C::STAGES;
        const bool ok = mbar_wait(full + s, (k / C::STAGES) & 1, err, 0x202);
        if (!__all_sync(0xFFFFFFFFu, ok) || abort_flag) break;
        const unsigned char *sw = base + s * C::STAGE + warp * C::STREAM;
        const double *sx = reinterpret_cast<const double *>(base + s * C::STAGE + C::WBYTES);
        const int nsteps = min(8, M - 8 * k);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            if (i >= nsteps) break;
            const int lb = i * 32 + 16 * h, box = lb >> 7, j = (lb & 127) >> 4;
            double w[R][8];
#pragma unroll
            for (int g = 0; g < R; g++) {
                const uint4 u = *reinterpret_cast<const uint4 *>(sw + g * 4096 + box * 2048 + r * 128 +
                                                                 ((j ^ (r & 7)) << 4));
                bf16x8_to_f64(u, bf16x8_normal(u), w[g]);
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t >= ntile) break;
                const double2 *xp = reinterpret_cast<const double2 *>(sx + t * 128 + i * 16 + 8 * h);
                double2 xv[4];
#pragma unroll
                for (int q = 0; q < 4; q++) xv[q] = xp[q];
#pragma unroll
                for (int g = 0; g < R; g++)
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        a[t][g][2 * q] = __fma_rn(w[g][2 * q], xv[q].x, a[t][g][2 * q]);
                        a[t][g][2 * q + 1] = __fma_rn(w[g][2 * q + 1], xv[q].y, a[t][g][2 * q + 1]);
                    }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + s);
    }

    // Fold as in bf16_chain_kernel, then the ragged tail from global memory.
#pragma unroll
    for (int g = 0; g < R; g++) {
        const int row = row_cta + 16 * R * warp + 16 * g + r;
        const uint16_t *wrow = W + (size_t)min(row, rows - 1) * cols;
#pragma unroll
        for (int t = 0; t < NT; t++) {
            double b[4];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const double mine = a[t][g][jj] + a[t][g][jj + 4];
                const double other = __shfl_xor_sync(0xFFFFFFFFu, mine, 1);
                b[jj] = h ? other + mine : mine + other;
            }
            if (t >= ntile || h || row >= rows) continue;
            double acc = (b[0] + b[1]) + (b[2] + b[3]);
            const double *xr = xd + (size_t)(t0 + t) * ldxd;
            for (int i = 16 * M; i < cols; i++)
                acc = __fma_rn((double)__uint_as_float((uint32_t)__ldg(wrow + i) << 16), xr[i], acc);
            y[(size_t)(t0 + t) * rows + row] = __double2float_rn(acc);
        }
    }
}

// One token, a matrix of few rows (the router, the compressor and indexer
// projections): a half-warp per row, lane c of it runs chain c over columns
// c, c + 16, ... in order, then the same fold (((c0 + c4) + (c8 + c12)) for
// each of c = 0..3, paired (b0 + b1) + (b2 + b3)) and the ragged tail in
// order - the BLOCK_DOT_V operations - spread over 8x more CTAs than the
// 256-row stages of the streaming kernel give such a matrix.
__global__ void __launch_bounds__(256) bf16_chain_small_kernel(const uint16_t *__restrict__ W, int rows, int cols,
                                                               const double *__restrict__ xd, float *__restrict__ y)
{
    const int lane = threadIdx.x & 31, c = lane & 15, half = lane >> 4;
    const int row = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 2 + half;
    const int M = cols >> 4;
    const uint16_t *wrow = W + (size_t)min(row, rows - 1) * cols;
    double acc = 0.0;
#pragma unroll 32
    for (int i = 0; i < M; i++) {
        const int k = 16 * i + c;
        acc = __fma_rn((double)__uint_as_float((uint32_t)__ldg(wrow + k) << 16), __ldg(xd + k), acc);
    }
    double v = acc + __shfl_down_sync(0xFFFFFFFFu, acc, 4);   // c in 0..3, 8..11: c_j + c_j+4, c_8+j + c_12+j
    v = v + __shfl_down_sync(0xFFFFFFFFu, v, 8);              // c in 0..3: b_c
    v = v + __shfl_down_sync(0xFFFFFFFFu, v, 1);              // c = 0: b0 + b1, c = 2: b2 + b3
    v = v + __shfl_down_sync(0xFFFFFFFFu, v, 2);              // c = 0: (b0 + b1) + (b2 + b3)
    if (c != 0 || row >= rows) return;
    for (int i = 16 * M; i < cols; i++)
        v = __fma_rn((double)__uint_as_float((uint32_t)__ldg(wrow + i) << 16), xd[i], v);
    y[row] = __double2float_rn(v);
}

// The activation copy: rows of ldxd doubles, ldxd a multiple of 128 columns so
// every TMA stage's 128 columns lie inside the row.
static int bf16_ldxd(int cols) { return ((cols + 127) / 128) * 128; }

size_t bf16_chain_workspace(int cols, int nt)
{
    return dsv4cu_align256((size_t)nt * bf16_ldxd(cols) * sizeof(double));
}

template <int R, int NT, int CW>
static int bf16_tma_launch(const CUtensorMap &tw, const dsv4cu_qmat *q, const double *xd, int ldxd, int nt, float *y,
                           int *err, cudaStream_t st)
{
    using C = BfcCfg<R, NT, CW>;
    static SmemLimit lim;
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)bf16_chain_tma_kernel<R, NT, CW>, C::SMEM));
    constexpr int ROWS = 16 * R * CW;
    const dim3 grid((unsigned)((q->rows + ROWS - 1) / ROWS), (unsigned)((nt + NT - 1) / NT));
    bf16_chain_tma_kernel<R, NT, CW><<<grid, C::THREADS, C::SMEM, st>>>(tw, (const uint16_t *)q->w, q->rows, q->cols,
                                                                       xd, ldxd, nt, y, err);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

int bf16_chain_run(float *y, const float *x, const dsv4cu_qmat *q, int nt, void *ws, int *err, cudaStream_t st)
{
    const int rows = q->rows, cols = q->cols;
    const uint16_t *W = (const uint16_t *)q->w;
    const int ldxd = bf16_ldxd(cols);
    double *xd = (double *)ws;
    const long n = (long)nt * ldxd;
    bf16_xwiden_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, cols, nt, ldxd, xd);
    DSV4CU_LAUNCH_CHECK();
    if (nt == 1 && rows <= 8192) {
        const unsigned grid = (unsigned)((rows + 15) / 16);     // 8 warps x 2 rows per CTA
        bf16_chain_small_kernel<<<grid, 256, 0, st>>>(W, rows, cols, xd, y);
        DSV4CU_LAUNCH_CHECK();
        return DSV4CU_OK;
    }
    if (tmap_weights_ok(q) && cols >= 16) {
        CUtensorMap tw;
        int staged = 0;
        int r = tmap_encode(q, &tw, nullptr, &staged);
        if (r) return r;
        return nt == 1 ? bf16_tma_launch<1, 1, 16>(tw, q, xd, ldxd, nt, y, err, st)
                       : bf16_tma_launch<1, 4, 12>(tw, q, xd, ldxd, nt, y, err, st);   // 4-token chains: registers
    }
    const bool vec = cols % 8 == 0 && ((uintptr_t)W & 15u) == 0;
    const unsigned gx = (unsigned)((rows + 16 * BFC_WARPS - 1) / (16 * BFC_WARPS));
    if (nt == 1) {
        if (vec)
            bf16_chain_kernel<1, true><<<dim3(gx, 1), BFC_THREADS, 0, st>>>(W, rows, cols, xd, ldxd, nt, y);
        else
            bf16_chain_kernel<1, false><<<dim3(gx, 1), BFC_THREADS, 0, st>>>(W, rows, cols, xd, ldxd, nt, y);
    } else {
        const unsigned gy = (unsigned)((nt + 3) / 4);
        if (vec)
            bf16_chain_kernel<4, true><<<dim3(gx, gy), BFC_THREADS, 0, st>>>(W, rows, cols, xd, ldxd, nt, y);
        else
            bf16_chain_kernel<4, false><<<dim3(gx, gy), BFC_THREADS, 0, st>>>(W, rows, cols, xd, ldxd, nt, y);
    }
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

}  // namespace dsv4cu
