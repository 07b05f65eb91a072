// mxgemm.cu - packed-weight GEMM on the sm_100a tensor cores.
//
// y[t][o] = sum_k x[t][k] * W[o][k] for W in the reference pack layouts (FP4
// e2m1 with 1x32 E8M0 scales, FP8 e4m3 with 128x128 E8M0 scales), computed by
// tcgen05.mma.kind::mxf8f6f4.block_scale: the tensor core reads the e2m1 /
// e4m3 weight bytes straight from shared memory and applies the E8M0 scales
// itself, so no CUDA-core instruction touches a weight element.
//
// Activations. The MMA's B operand is e4m3 with one E8M0 scale per 32 values
// and per column. An fp32 activation x is written as a sum of T e4m3 terms:
// term j = RNE_e4m3(r_j / s_j) * s_j with r_0 = x, r_{j+1} = r_j - term j
// (each subtraction is exact) and s_j the smallest power of two with
// max|r_j| / s_j <= 448 over the 32-block. Every term is its own B column
// with its own scales; the epilogue sums the T columns of a token. The
// remaining error per element is below 2^(-4T) of its block's magnitude:
// T = 3 keeps matmul results within the 1e-3 bar with margin, T = 4 is close
// to fp32.
//
// Kernel structure (one CTA per SM, persistent over 128-row x NB-column
// tiles, 192 threads):
//   warp 0      TMA producer: per 128-wide K chunk one A box (128 rows x 128
//               elements, 128-byte swizzle), one B box (NB columns x 128),
//               and two 1-D bulk copies of prepared scale-factor blocks,
//               into a STAGES-deep ring (mbarrier full / empty);
//   warp 1      TMEM owner and MMA issuer: copies the stage's scale blocks
//               into TMEM (tcgen05.cp) and issues 4 MMAs (K = 32 each), then
//               commits the stage back to the producer; after a tile's last
//               chunk it commits the accumulator to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (one TMEM lane =
//               one output row), sum of the T term columns, coalesced stores.
// Two accumulator buffers in TMEM let the epilogue of tile i overlap the
// MMAs of tile i + 1. Every wait is bounded (2 s of %globaltimer); a timeout
// records an error code and the CTA drains its own copies and MMAs, frees its
// TMEM and exits.
//
// Scale factors reach TMEM in the layout the MMA reads (umma.cuh): weights'
// scales are rearranged once per matrix into 512-byte blocks (one per 128
// rows x 128 K), activation scales are written in that layout by the
// activation-split kernel.
#include <cuda.h>
#include <stdlib.h>
#include <string.h>

#include "ctx.h"
#include "gemv.h"
#include "mxgemm.h"
#include "tma_gemv.cuh"
#include "umma.cuh"

namespace dsv4cu {

// ------------------------------------------------------------ device code
DSV4CU_DEV void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

template <int NB>
struct MxCfg {
    static constexpr int NBB = (NB + 127) / 128;          // 128-column scale blocks of B
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = NB * 128;
    static constexpr int SFA_BYTES = 512;
    static constexpr int SFB_BYTES = NBB * 512;
    static constexpr int STAGE = ((A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES + 1023) / 1024) * 1024;
    static constexpr int SF_SLOTS = 4;
    static constexpr int SFB_COLS = 4 * NBB;
    static constexpr int SF_COLS = SF_SLOTS * (4 + SFB_COLS);
    static constexpr int ACC_BUFS = (2 * NB + SF_COLS <= 512) ? 2 : 1;
    static constexpr int SFA_COL = ACC_BUFS * NB;
    static constexpr int SFB_COL = SFA_COL + 4 * SF_SLOTS;
    static constexpr int USED = SFB_COL + SFB_COLS * SF_SLOTS;
    static constexpr int TMEM_COLS = USED <= 32 ? 32 : USED <= 64 ? 64 : USED <= 128 ? 128 : USED <= 256 ? 256 : 512;
    static_assert(NB % 32 == 0 && NB >= 32 && NB <= 256, "NB: 32..256, multiple of 32");
    static_assert(USED <= 512, "TMEM budget");
};

constexpr int MX_THREADS = 192;

enum { MXE_EMPTY = 21, MXE_FULL = 22, MXE_ACC_EMPTY = 23, MXE_ACC_FULL = 24, MXE_DRAIN = 25 };

template <int NB, int STAGES>
__global__ void __launch_bounds__(MX_THREADS, 1)
    mxgemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, MxArgs g)
{
    using C = MxCfg<NB>;
    extern __shared__ uint8_t mx_smem_raw[];
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], accf[2], acce[2], drain;
    __shared__ uint32_t tmem_holder;
    __shared__ volatile int abort_flag;

    uint8_t *smem = (uint8_t *)(((uintptr_t)mx_smem_raw + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = g.tiles_m * g.tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], 4);
        }
        mbar_init(&drain, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        umma::tmem_alloc(&tmem_holder, C::TMEM_COLS);
        umma::tmem_relinquish();
    }
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    const uint32_t tmem = tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int it = 0;
            const uint32_t tx = g.a_tx + C::B_BYTES + C::SFA_BYTES + C::SFB_BYTES;
            for (int t = blockIdx.x; t < ntiles && !abort_flag; t += gridDim.x) {
                const int tm = t % g.tiles_m, tn = t / g.tiles_m;
                for (int c = 0; c < g.kc; c++, it++) {
                    const int s = it % STAGES, r = it / STAGES;
                    if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, g.err, MXE_EMPTY)) {
                        abort_flag = 1;
                        break;
                    }
                    uint8_t *st = smem + s * C::STAGE;
                    mbar_arrive_expect_tx(&full[s], tx);
                    tma_load_2d(st, &ta, c * 128, tm * 128, &full[s]);
                    tma_load_2d(st + C::A_BYTES, &tb, c * 128, tn * NB, &full[s]);
                    bulk_load(st + C::A_BYTES + C::B_BYTES, g.sfa + ((size_t)tm * g.kc + c) * 512, C::SFA_BYTES,
                              &full[s]);
                    bulk_load(st + C::A_BYTES + C::B_BYTES + C::SFA_BYTES,
                              g.sfb + ((size_t)tn * g.kc + c) * C::SFB_BYTES, C::SFB_BYTES, &full[s]);
                }
            }
            // Every issued copy must land before the CTA can exit.
            for (int j = max(0, it - STAGES); j < it; j++)
                mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int it = 0, tcount = 0;
            for (int t = blockIdx.x; t < ntiles && !abort_flag; t += gridDim.x, tcount++) {
                const int ab = tcount % C::ACC_BUFS, use = tcount / C::ACC_BUFS;
                if (use > 0 && !mbar_wait(&acce[ab], (use - 1) & 1, g.err, MXE_ACC_EMPTY)) {
                    abort_flag = 1;
                    break;
                }
                umma::fence_after();
                const uint32_t dacc = tmem + ab * NB;
                bool ok = true;
                for (int c = 0; c < g.kc; c++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&full[s], (it / STAGES) & 1, g.err, MXE_FULL)) {
                        ok = false;
                        break;
                    }
                    umma::fence_after();
                    const uint8_t *st = smem + s * C::STAGE;
                    const int slot = it % C::SF_SLOTS;
                    const uint32_t tsfa = tmem + C::SFA_COL + 4 * slot;
                    const uint32_t tsfb = tmem + C::SFB_COL + C::SFB_COLS * slot;
                    umma::cp_sf(tsfa, umma::desc_sf(st + C::A_BYTES + C::B_BYTES));
#pragma unroll
                    for (int b = 0; b < C::NBB; b++)
                        umma::cp_sf(tsfb + 4 * b, umma::desc_sf(st + C::A_BYTES + C::B_BYTES + C::SFA_BYTES + 512 * b));
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint32_t id = g.idesc | ((uint32_t)k << 4) | ((uint32_t)k << 29);
                        umma::mma_mx(dacc, umma::desc_sw128(st + 32 * k), umma::desc_sw128(st + C::A_BYTES + 32 * k),
                                     id, (c | k) ? 1u : 0u, tsfa | ((uint32_t)k << 30), tsfb | ((uint32_t)k << 30));
                    }
                    umma::commit(&empty[s]);
                }
                if (!ok) {
                    abort_flag = 1;
                    break;
                }
                umma::commit(&accf[ab]);
            }
            // Drain: every MMA / copy this thread issued completes before TMEM is freed.
            umma::commit(&drain);
            mbar_wait(&drain, 0, g.err, MXE_DRAIN);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue
        const int q = warp & 3;             // the TMEM lane quarter this warp may read
        const int row_l = q * 32 + lane;
        int tcount = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, tcount++) {
            const int ab = tcount % C::ACC_BUFS, use = tcount / C::ACC_BUFS;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&accf[ab], use & 1, g.err, MXE_ACC_FULL);
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok || abort_flag) {
                abort_flag = 1;
                break;
            }
            umma::fence_after();
            const int tm = t % g.tiles_m, tn = t / g.tiles_m;
            const int row = tm * 128 + row_l;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * NB;
            for (int tb = 0; tb < g.tpt; tb += 8) {
                float acc[8];
                umma::ld_x8(tbase + tb, acc);
                for (int j = 1; j < g.terms; j++) {
                    float v[8];
                    umma::ld_x8(tbase + j * g.tpt + tb, v);
#pragma unroll
                    for (int i = 0; i < 8; i++) acc[i] += v[i];
                }
                if (row < g.rows) {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int tok = tn * g.tpt + tb + i;
                        if (tok < g.nt) g.y[(size_t)tok * g.ldy + row] = acc[i];
                    }
                }
            }
            umma::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[ab]);
        }
    }

    umma::fence_before();
    __syncthreads();
    if (warp == 1) {
        umma::fence_after();
        umma::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// Weight scale factors -> 512-byte blocks (128 rows x 4 K-blocks of 32):
// byte (m % 32) * 16 + (m / 32) * 4 + kb of block (row tile, K chunk).
__global__ void sfa_atoms_kernel(uint8_t *__restrict__ out, const uint8_t *__restrict__ s, int rows, int cols,
                                 int blk_r, int blk_c, int kc, int tiles_m)
{
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;   // one 32-bit word each
    if (i >= (long)tiles_m * kc * 128) return;
    const int atom = (int)(i >> 7), w = (int)(i & 127);
    const int rt = atom / kc, c = atom - rt * kc;
    const int m0 = w >> 2, m1 = w & 3;
    const int row = rt * 128 + m1 * 32 + m0;
    const int sc = (cols + blk_c - 1) / blk_c;
    uint32_t v = 0;
    if (row < rows) {
        for (int kb = 0; kb < 4; kb++) {
            const int k = (c * 4 + kb) * 32;
            v |= (uint32_t)s[(size_t)(row / blk_r) * sc + k / blk_c] << (8 * kb);
        }
    }
    ((uint32_t *)out)[(size_t)atom * 128 + m0 * 4 + m1] = v;
}

// Activation split: one warp per (B column, 32-wide K block), lane = element.
// Column n of N-tile tn holds term (n % NB) / tpt of token tn * tpt + n % tpt.
__global__ void xsplit_kernel(const float *__restrict__ x, int nt, int K, int ldx, int terms, int tpt, int NB,
                              int tiles_n, uint8_t *__restrict__ xq, uint8_t *__restrict__ sfb)
{
    const long gw = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31, nblk = K >> 5;
    if (gw >= (long)tiles_n * NB * nblk) return;
    const int n = (int)(gw / nblk), blk = (int)(gw - (long)n * nblk);
    const int tn = n / NB, nl = n - tn * NB, term = nl / tpt, tl = nl - term * tpt, tok = tn * tpt + tl;
    uint8_t q = 0, sbyte = 0;
    if (term < terms && tok < nt) {
        // Non-finite inputs stay out of the block maximum and reach the MMA as
        // e4m3 NaN (NaN) or +-448 (infinities saturate).
        float r = x[(size_t)tok * ldx + blk * 32 + lane];
        for (int j = 0;; j++) {
            float a = isfinite(r) ? fabsf(r) : 0.0f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
            int e = 0;
            if (a > 0.0f) {
                int E;
                const float f = frexpf(a, &E);
                e = max(-127, min(127, E - 9 + (f > 0.875f ? 1 : 0)));
            }
            const float v = ldexpf(r, -e);
            uint16_t two;
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(two) : "f"(0.0f), "f"(v));
            const uint8_t qb = (uint8_t)(two & 0xFF);
            if (j == term) {
                q = qb;
                sbyte = (uint8_t)(127 + e);
                break;
            }
            r = r - ldexpf(e4m3_to_f32(qb), e);
        }
    }
    xq[(size_t)n * K + blk * 32 + lane] = q;
    if (lane == 0) {
        const int c = blk >> 2, kb = blk & 3, nbb = (NB + 127) / 128;
        const int b = nl >> 7, w = nl & 127;
        sfb[(((size_t)tn * (K >> 7) + c) * nbb + b) * 512 + (w & 31) * 16 + (w >> 5) * 4 + kb] = sbyte;
    }
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn mx_encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// 2-D K-major operand map: `inner` elements per row (K), `outer` rows, box
// 128 elements x box_rows, 128-byte swizzle.
static int encode_kmajor(CUtensorMap *map, const void *base, bool fp4, uint64_t inner, uint64_t outer,
                         uint64_t row_bytes, uint32_t box_rows)
{
    EncodeTiledFn enc = mx_encode_fn();
    if (!enc) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                     const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled: %d", (int)r);
    return DSV4CU_OK;
}

bool mx_supported(const dsv4cu_qmat *q)
{
    if (!q || !q->w || !q->s || q->rows <= 0 || q->cols <= 0 || q->cols % 128) return false;
    if (q->blk_r <= 0 || q->blk_c <= 0 || q->blk_c % 32) return false;
    if (q->wdt == DSV4CU_WFP4) return ((uintptr_t)q->w & 31u) == 0 && (q->cols / 2) % 32 == 0;
    if (q->wdt == DSV4CU_WFP8) return ((uintptr_t)q->w & 15u) == 0;
    return false;
}

int mx_prepare(MxMat *m, const dsv4cu_qmat *q, cudaStream_t st)
{
    memset(m, 0, sizeof(*m));
    if (!mx_supported(q))
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED,
                                "mx matrix: needs FP4/FP8, cols %% 128 == 0, blk_c %% 32 == 0, aligned weights");
    m->q = *q;
    m->fp4 = q->wdt == DSV4CU_WFP4;
    m->kc = q->cols / 128;
    m->tiles_m = (q->rows + 127) / 128;
    const size_t rb = m->fp4 ? (size_t)q->cols / 2 : (size_t)q->cols;
    int r = encode_kmajor(&m->ta, q->w, m->fp4, (uint64_t)q->cols, (uint64_t)q->rows, rb, 128);
    if (r) return r;
    const size_t bytes = (size_t)m->tiles_m * m->kc * 512;
    DSV4CU_CUDA_TRY(cudaMalloc((void **)&m->sfa, bytes));
    const long words = (long)m->tiles_m * m->kc * 128;
    sfa_atoms_kernel<<<(unsigned)((words + 255) / 256), 256, 0, st>>>(m->sfa, (const uint8_t *)q->s, q->rows,
                                                                      q->cols, q->blk_r, q->blk_c, m->kc, m->tiles_m);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

void mx_release(MxMat *m)
{
    if (m && m->sfa) cudaFree(m->sfa);
    if (m) m->sfa = nullptr;
}

// Column tiling for nt tokens and T terms.
struct MxTiling {
    int NB, tpt, tiles_n;
};

static MxTiling mx_tiling(int nt, int terms)
{
    MxTiling t;
    // Small batches: 32 columns (decode); large: 192 (3 terms x 64 tokens) or 256.
    if (nt * terms <= 32 && (32 / terms) / 8 * 8 >= nt) t.NB = 32;
    else if (nt * terms <= 64 && (64 / terms) / 8 * 8 >= nt) t.NB = 64;
    else t.NB = (terms == 3) ? 192 : 256;
    t.tpt = (t.NB / terms) / 8 * 8;
    t.tiles_n = (nt + t.tpt - 1) / t.tpt;
    return t;
}

size_t mx_workspace(const MxMat *m, int nt, int terms)
{
    const MxTiling t = mx_tiling(nt, terms);
    const size_t cols = (size_t)t.tiles_n * t.NB;
    return dsv4cu_align256(cols * m->q.cols) + dsv4cu_align256((size_t)t.tiles_n * m->kc * ((t.NB + 127) / 128) * 512);
}

template <int NB, int STAGES>
static int mx_launch(const MxMat *m, const CUtensorMap &tb, const MxArgs &a, int sms, cudaStream_t st)
{
    const size_t smem = (size_t)STAGES * MxCfg<NB>::STAGE + 1024;
    DSV4CU_CUDA_TRY(cudaFuncSetAttribute(mxgemm_kernel<NB, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
    const int tiles = a.tiles_m * a.tiles_n;
    mxgemm_kernel<NB, STAGES><<<tiles < sms ? tiles : sms, MX_THREADS, smem, st>>>(m->ta, tb, a);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

int mx_gemm(const MxMat *m, float *y, const float *x, int nt, int terms, void *ws, int sms, int *err,
            cudaStream_t st)
{
    if (terms < 1 || terms > 4) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mx gemm: terms must be 1..4");
    if (nt <= 0) return DSV4CU_OK;
    const MxTiling t = mx_tiling(nt, terms);
    const int K = m->q.cols;
    uint8_t *xq = (uint8_t *)ws;
    uint8_t *sfb = xq + dsv4cu_align256((size_t)t.tiles_n * t.NB * K);
    {
        const long warps = (long)t.tiles_n * t.NB * (K / 32);
        xsplit_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(x, nt, K, K, terms, t.tpt, t.NB,
                                                                           t.tiles_n, xq, sfb);
        DSV4CU_LAUNCH_CHECK();
    }
    CUtensorMap tb;
    int r = encode_kmajor(&tb, xq, false, (uint64_t)K, (uint64_t)t.tiles_n * t.NB, (uint64_t)K, (uint32_t)t.NB);
    if (r) return r;
    MxArgs a;
    a.sfa = m->sfa;
    a.sfb = sfb;
    a.kc = m->kc;
    a.tiles_m = m->tiles_m;
    a.tiles_n = t.tiles_n;
    a.rows = m->q.rows;
    a.nt = nt;
    a.tpt = t.tpt;
    a.terms = terms;
    a.y = y;
    a.ldy = m->q.rows;
    a.idesc = umma::idesc_mx(m->fp4 ? umma::FMT_E2M1 : umma::FMT_E4M3, umma::FMT_E4M3, 128, t.NB);
    a.a_tx = m->fp4 ? 128 * 64 : 128 * 128;
    a.err = err;
    switch (t.NB) {
    case 32: return mx_launch<32, 8>(m, tb, a, sms, st);
    case 64: return mx_launch<64, 8>(m, tb, a, sms, st);
    case 192: return mx_launch<192, 4>(m, tb, a, sms, st);
    default: return mx_launch<256, 4>(m, tb, a, sms, st);
    }
}

}  // namespace dsv4cu

// ------------------------------------------------------------ C ABI
using namespace dsv4cu;

struct dsv4cu_mat {
    MxMat m;
    int device;
};

extern "C" int dsv4cu_mat_create(dsv4cu_mat **out, const dsv4cu_qmat *q, void *stream)
{
    if (!out || !q) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mat_create: NULL argument");
    *out = nullptr;
    dsv4cu_mat *h = (dsv4cu_mat *)calloc(1, sizeof(dsv4cu_mat));
    if (!h) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "mat_create: host allocation failed");
    DSV4CU_CUDA_TRY(cudaGetDevice(&h->device));
    int r = mx_prepare(&h->m, q, (cudaStream_t)stream);
    if (r) {
        mx_release(&h->m);
        free(h);
        return r;
    }
    *out = h;
    return DSV4CU_OK;
}

extern "C" void dsv4cu_mat_destroy(dsv4cu_mat *h)
{
    if (!h) return;
    mx_release(&h->m);
    free(h);
}

extern "C" size_t dsv4cu_mat_workspace(const dsv4cu_mat *h, int nt, int terms)
{
    return h ? mx_workspace(&h->m, nt, terms) : 0;
}

extern "C" int dsv4cu_mat_gemm(dsv4cu_ctx *ctx, const dsv4cu_mat *h, float *y, const float *x, int nt, int terms,
                               void *stream)
{
    if (!ctx || !h || !y || !x) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mat_gemm: NULL argument");
    if (nt < 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mat_gemm: nt < 0");
    if (nt == 0) return DSV4CU_OK;
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, mx_workspace(&h->m, nt, terms), &ws);
    if (r) return r;
    return mx_gemm(&h->m, y, x, nt, terms, ws, ctx->sm_count, ctx->status, (cudaStream_t)stream);
}
