// f16w_gemm.cu - exact-weight GEMM on the bf16 tensor cores (tcgen05 kind::f16).
//
// y[t][o] = sum_c x[t][c] * W[o][c] for a packed FP8 (e4m3) or FP4 (e2m1)
// matrix with E8M0 block scales, the prefill GEMM of the reference's Vulkan
// seam (src/80_prefill/dsv4_prefill_vk_gemm.c:63-137, shaders gemm_fp8.comp /
// gemm_fp4.comp) in its exact-weight form: every weight w * 2^e is a bf16
// value exactly (e4m3 and e2m1 carry at most 4 significant bits and the scale
// is a power of two), so the tensor core multiplies the reference's own
// dequantized weights. The activations enter as one bf16 term (x rounded to
// nearest: each activation off by up to 2^-9 of itself, so the max-rel error
// against fp32 activations sits near 2^-9 / sqrt(3) ~ 1.1e-3 on Gaussian data)
// or as two (hi + lo, 16 significand bits, ~1e-5 - inside the 1e-3 matmul
// bar; each token then takes two B rows). Apart from that rounding the result
// is fp32 accumulation.
//
// Tile: 128 weight rows (MMA M) x 256 tokens (N), K in 64-element chunks (one
// 128-byte bf16 row per operand row, 128-byte swizzle). Roles, 704 threads,
// one CTA per SM, persistent over tiles (tile t = row tile t % tiles_m, token
// tile t / tiles_m):
//   warp 0       TMA of the stage's bf16 activation chunk (256 rows x 128
//                bytes) and of its packed weights (128 rows x 64 or 32 bytes),
//                both counted on one barrier;
//   warp 1       TMEM (two 256-column fp32 accumulators) and the single MMA
//                thread: four K = 16 MMAs per chunk, tcgen05.commit frees the
//                stage, the tile's last commit hands the accumulator over;
//   warps 2-17   converters: each warp dequantizes 8 weight rows of the chunk
//                from the packed box in shared memory (4 lanes per row, 16
//                elements each; the E8M0 scales two steps ahead from L2),
//                cvt to f16, times the block scale, to bf16 (all exact), and
//                writes them swizzled into the stage; fence.proxy.async, arrive;
//   warps 18-21  epilogue: tcgen05.ld of the accumulator (TMEM lane = weight
//                row), y stored token by token (32 consecutive rows per store).
// Every wait is bounded (2 s): a role that times out records an error code in
// the context status word and leaves its loop; the others run into their own
// bounded waits; TMEM is freed after the MMAs in flight have drained.
#include <cuda.h>

#include "common.cuh"
#include "ctx.h"
#include "tma_gemv.cuh"
#include "tmap.h"
#include "umma.cuh"

namespace dsv4cu {

constexpr int FW_M = 128;                 // weight rows per tile
constexpr int FW_N = 256;                 // tokens per tile
constexpr int FW_KC = 64;                 // K elements per stage
constexpr int FW_STAGES = 4;
constexpr int FW_CONV_WARPS = 16;
constexpr int FW_RPW = FW_M / FW_CONV_WARPS;   // weight rows per converter warp
constexpr int FW_LPR = 32 / FW_RPW;            // lanes per row
constexpr int FW_EPL = FW_KC / FW_LPR;         // elements per lane and chunk (16 or 32: inside one scale block)
constexpr int FW_CPL = FW_EPL / 8;             // 16-byte bf16 pieces per lane
static_assert(FW_EPL == 16 || FW_EPL == 32, "converter lane layout");
constexpr int FW_EPI_WARPS = 4;
constexpr int FW_THREADS = 32 * (2 + FW_CONV_WARPS + FW_EPI_WARPS);
constexpr int FW_A_BYTES = FW_M * 128;
constexpr int FW_B_BYTES = FW_N * 128;
constexpr int FW_STAGE = FW_A_BYTES + FW_B_BYTES;
constexpr int FW_RAW = FW_M * 64;          // packed weight box of a stage (FP8: 64 B rows, FP4: 32 B rows)
constexpr int FW_SMEM = FW_STAGES * (FW_STAGE + FW_RAW) + 1024;

enum { FWE_EMPTY = 41, FWE_AFULL = 42, FWE_BFULL = 43, FWE_ACCF = 44, FWE_ACCE = 45, FWE_DRAIN = 46 };

struct FwParams {
    const uint8_t *w;        // packed weights [rows][row_bytes]
    const uint8_t *s;        // E8M0 scales [ceil(rows / blk_r)][s_cols]; blk_r, blk_c powers of two
    int rows, cols, fp4, blk_r_log2, blk_c_log2, s_cols, row_bytes;
    int tiles_m, tiles_n, nt, terms;   // terms: bf16 activation terms per token (1 or 2), B rows per token
    int pre;                 // 1: the weights were dequantized to bf16 beforehand; tw maps them, no converters
    float *y;                // [nt][rows]
    int *err;
};

// Instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), A and
// B bf16 (bits 7-9 and 10-12 = 1), both K-major, N >> 3 in bits 17-22, M >> 4
// in bits 24-28.
__host__ __device__ constexpr uint32_t fw_idesc(int M, int N)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

DSV4CU_DEV void fw_mma(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 ::"r"(d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Bounded wait without the suspend hint, for the single-thread roles (the MMA
// issuer, the copy issuer): they poll, so a completed phase is seen at once.
DSV4CU_DEV bool fw_spin(uint64_t *bar, uint32_t parity, int *err, int code)
{
    const uint32_t a = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t i = 0;; i++) {
        uint32_t ok;
        asm volatile("{\n\t.reg .pred p;\n\t"
                     "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(ok) : "r"(a), "r"(parity) : "memory");
        if (ok) return true;
        if ((i & 255u) == 0u) {
            const uint64_t now = globaltimer_ns();
            if (i == 0) t0 = now;
            else if (now - t0 > MBAR_TIMEOUT_NS) break;
        }
    }
    if (err) atomicCAS(err, 0, code);
    return false;
}

// Two fp32 -> one bf16x2 word (round to nearest; exact for these values).
DSV4CU_DEV uint32_t fw_bf2(float a, float b)
{
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// f16x2 word times a power of two -> bf16x2 word.
DSV4CU_DEV uint32_t fw_scale_bf2(uint32_t h2, float sc)
{
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h2));
    return fw_bf2(f.x * sc, f.y * sc);
}

// Activation rows as bf16 terms. terms = 1: xb[t][c] = RN_bf16(x[t][c]);
// terms = 2: rows 2t and 2t + 1 hold hi = RN_bf16(x) and lo = RN_bf16(x - hi)
// (x - hi is exact in fp32; hi + lo carries 16 significand bits).
// Blocks blk = 0 .. nblk - 1 of a grid-stride pass.
DSV4CU_DEV void fw_xbf16_part(const float *__restrict__ x, __nv_bfloat16 *__restrict__ xb, int cols, long n4,
                              int terms, int blk, int nblk)
{
    const int c4 = cols / 4;
    for (long i = blk * (long)blockDim.x + threadIdx.x; i < n4; i += (long)nblk * blockDim.x) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
        uint2 hi;
        hi.x = fw_bf2(v.x, v.y);
        hi.y = fw_bf2(v.z, v.w);
        if (terms == 1) {
            reinterpret_cast<uint2 *>(xb)[i] = hi;
            continue;
        }
        const long t = i / c4, c = i - t * c4;
        const float2 h01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&hi.x));
        const float2 h23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&hi.y));
        uint2 lo;
        lo.x = fw_bf2(v.x - h01.x, v.y - h01.y);
        lo.y = fw_bf2(v.z - h23.x, v.w - h23.y);
        reinterpret_cast<uint2 *>(xb)[(2 * t) * c4 + c] = hi;
        reinterpret_cast<uint2 *>(xb)[(2 * t + 1) * c4 + c] = lo;
    }
}

// Whole matrix to bf16 once (pre-dequantized mode): the same exact
// conversion as the converter warps, 16 elements of one row per thread
// (inside one scale block, blk_c >= 32).
DSV4CU_DEV void fw_dequant_part(const FwParams &p, uint4 *__restrict__ wb, int blk)
{
    const long i = blk * (long)blockDim.x + threadIdx.x, per_row = p.cols / 16;
    if (i >= (long)p.rows * per_row) return;
    const int row = (int)(i / per_row), c0 = (int)(i - (long)row * per_row) * 16;
    const float sc = e8m0_to_f32(__ldg(p.s + (size_t)(row >> p.blk_r_log2) * p.s_cols + (c0 >> p.blk_c_log2)));
    uint32_t o[8];
    if (p.fp4) {
        const uint2 v = __ldg(reinterpret_cast<const uint2 *>(p.w + (size_t)row * p.row_bytes + c0 / 2));
        const uint32_t wv[2] = {v.x, v.y};
#pragma unroll
        for (int j = 0; j < 2; j++) {
            uint32_t h0, h1, h2, h3;
            cvt_e2m1x8(wv[j], h0, h1, h2, h3);
            o[4 * j] = fw_scale_bf2(h0, sc);
            o[4 * j + 1] = fw_scale_bf2(h1, sc);
            o[4 * j + 2] = fw_scale_bf2(h2, sc);
            o[4 * j + 3] = fw_scale_bf2(h3, sc);
        }
    } else {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p.w + (size_t)row * p.row_bytes + c0));
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t lo, hi;
            cvt_e4m3x4(wv[j], lo, hi);
            o[2 * j] = fw_scale_bf2(lo, sc);
            o[2 * j + 1] = fw_scale_bf2(hi, sc);
        }
    }
    uint4 *dst = wb + (size_t)row * (p.cols / 8) + c0 / 8;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// The GEMM's operands in one launch: blocks [0, xblocks) write the activation
// terms, the rest (pre-dequantized mode) the bf16 weights. The GEMM is
// launched programmatically behind it and sets up while this runs.
__global__ void __launch_bounds__(256) fw_prep_kernel(const float *__restrict__ x, __nv_bfloat16 *__restrict__ xb,
                                                      int cols, long n4, int terms, int xblocks, const FwParams p,
                                                      uint4 *__restrict__ wb)
{
    pdl_trigger();
    if ((int)blockIdx.x < xblocks)
        fw_xbf16_part(x, xb, cols, n4, terms, blockIdx.x, xblocks);
    else
        fw_dequant_part(p, wb, blockIdx.x - xblocks);
}

__global__ void __launch_bounds__(FW_THREADS, 1) fw_kernel(const __grid_constant__ CUtensorMap tb,
                                                           const __grid_constant__ CUtensorMap tw, const FwParams p)
{
    extern __shared__ uint8_t fw_raw[];
    __shared__ __align__(8) uint64_t a_full[FW_STAGES], b_full[FW_STAGES], empty[FW_STAGES], accf[2], acce[2],
        drain;
    __shared__ uint32_t tmem_holder;
    uint8_t *smem = (uint8_t *)(((uintptr_t)fw_raw + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kch = p.cols / FW_KC, ntiles = p.tiles_m * p.tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < FW_STAGES; s++) {
            mbar_init(&a_full[s], FW_CONV_WARPS);
            mbar_init(&b_full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], FW_EPI_WARPS);
        }
        mbar_init(&drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        umma::tmem_alloc(&tmem_holder, 512);
        umma::tmem_relinquish();
    }
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    const uint32_t tmem = tmem_holder;
    // Set-up above overlaps the operand pass; its outputs are read below.
    pdl_wait();

    if (warp == 0) {
        // ------------------------------------------------ activation chunks
        if (lane == 0) {
            int g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int tn = t / p.tiles_m, tm = t - tn * p.tiles_m;
                const int wbox = p.fp4 ? FW_KC / 2 : FW_KC;    // packed bytes of a chunk row
                for (int kc = 0; kc < kch; kc++, g++) {
                    const int s = g % FW_STAGES, u = g / FW_STAGES;
                    if (u > 0 && !fw_spin(&empty[s], (u - 1) & 1, p.err, FWE_EMPTY)) {
                        ok = false;
                        break;
                    }
                    // one barrier for both boxes: the converters wait on it for
                    // the packed weights, the MMA for the activations (and, in
                    // the pre-dequantized mode, for the bf16 weight box too)
                    if (p.pre) {
                        mbar_arrive_expect_tx(&b_full[s], FW_B_BYTES + FW_A_BYTES);
                        tma_load_2d(smem + s * FW_STAGE, &tw, kc * FW_KC, tm * FW_M, &b_full[s]);
                    } else {
                        mbar_arrive_expect_tx(&b_full[s], FW_B_BYTES + FW_M * wbox);
                        tma_load_2d(smem + FW_STAGES * FW_STAGE + s * FW_RAW, &tw, kc * wbox, tm * FW_M, &b_full[s]);
                    }
                    tma_load_2d(smem + s * FW_STAGE + FW_A_BYTES, &tb, kc * FW_KC, tn * FW_N, &b_full[s]);
                }
            }
            // every issued copy lands before the CTA can exit
            for (int j = max(0, g - FW_STAGES); j < g; j++)
                mbar_wait(&b_full[j % FW_STAGES], (j / FW_STAGES) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = fw_idesc(FW_M, FW_N);
            int g = 0, tc = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, tc++) {
                const int ab = tc & 1, use = tc >> 1;
                if (use > 0 && !fw_spin(&acce[ab], (use - 1) & 1, p.err, FWE_ACCE)) break;
                umma::fence_after();
                const uint32_t d = tmem + ab * FW_N;
                for (int kc = 0; kc < kch; kc++, g++) {
                    const int s = g % FW_STAGES, u = g / FW_STAGES;
                    if ((!p.pre && !fw_spin(&a_full[s], u & 1, p.err, FWE_AFULL)) ||
                        !fw_spin(&b_full[s], u & 1, p.err, FWE_BFULL)) {
                        ok = false;
                        break;
                    }
                    umma::fence_after();
                    const uint8_t *st = smem + s * FW_STAGE;
#pragma unroll
                    for (int k = 0; k < FW_KC / 16; k++)
                        fw_mma(d, umma::desc_sw128(st + 32 * k), umma::desc_sw128(st + FW_A_BYTES + 32 * k), idesc,
                               (kc > 0 || k > 0) ? 1u : 0u);
                    umma::commit(&empty[s]);
                }
                if (ok) umma::commit(&accf[ab]);
            }
            // the MMAs in flight complete before TMEM is released
            umma::commit(&drain);
            mbar_wait(&drain, 0, p.err, FWE_DRAIN);
        }
    } else if (warp < 2 + FW_CONV_WARPS) {
        // ------------------------------------------------ weight converters
        // The CTA's (tile, chunk) steps in order; the packed bytes and the
        // scale of the next two steps are in flight while this step waits for
        // its stage and converts, so the L2 round trip overlaps the work.
        // Positions advance incrementally (one division per tile).
        const int cw = warp - 2, r = FW_RPW * cw + lane / FW_LPR, h = lane % FW_LPR;
        struct Pos {
            int t, kc;
            const uint8_t *wrow, *srow;
        };
        auto set_tile = [&](Pos &q) {
            q.wrow = nullptr;
            if (q.t >= ntiles) return;
            const int row = (q.t % p.tiles_m) * FW_M + r;
            if (row >= p.rows) return;
            q.wrow = p.w + (size_t)row * p.row_bytes;
            q.srow = p.s + (size_t)(row >> p.blk_r_log2) * p.s_cols;
        };
        auto advance = [&](Pos &q) {
            if (++q.kc == kch) {
                q.kc = 0;
                q.t += gridDim.x;
                set_tile(q);
            }
        };
        auto fetch = [&](const Pos &q, float &sc) {
            sc = 0.0f;
            if (!q.wrow) return;
            const int c0 = q.kc * FW_KC + FW_EPL * h;      // this lane's elements (one scale block)
            sc = e8m0_to_f32(__ldg(q.srow + (c0 >> p.blk_c_log2)));
        };
        const int wbox = p.fp4 ? FW_KC / 2 : FW_KC;
        const int total = p.pre ? 0 : (blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0) * kch;
        Pos pf{(int)blockIdx.x, 0, nullptr, nullptr};
        set_tile(pf);
        float as, bs;
        fetch(pf, as);                                      // step 0
        advance(pf);
        fetch(pf, bs);                                      // step 1
        advance(pf);
        for (int g = 0; g < total; g++) {
            const int s = g % FW_STAGES, u = g / FW_STAGES;
            const float sc = as;
            as = bs;
            fetch(pf, bs);                                  // step g + 2
            advance(pf);
            // the packed box of this stage has landed (so the MMAs of the
            // stage's previous use are done: the copy waited for them)
            bool full_ok = true;
            if (lane == 0) full_ok = mbar_wait(&b_full[s], u & 1, p.err, FWE_BFULL);
            if (!__shfl_sync(0xFFFFFFFFu, full_ok, 0)) break;
            const uint8_t *rb = smem + FW_STAGES * FW_STAGE + s * FW_RAW + r * wbox;
            uint4 raw0 = make_uint4(0u, 0u, 0u, 0u), raw1 = raw0;
            if (p.fp4) {
                if constexpr (FW_EPL == 32) {
                    raw0 = *reinterpret_cast<const uint4 *>(rb + FW_EPL / 2 * h);
                } else {
                    const uint2 v = *reinterpret_cast<const uint2 *>(rb + FW_EPL / 2 * h);
                    raw0.x = v.x;
                    raw0.y = v.y;
                }
            } else {
                raw0 = *reinterpret_cast<const uint4 *>(rb + FW_EPL * h);
                if constexpr (FW_EPL == 32) raw1 = *reinterpret_cast<const uint4 *>(rb + FW_EPL * h + 16);
            }
            uint32_t o[FW_EPL / 2];                             // FW_EPL bf16 values
            if (p.fp4) {
                const uint32_t wv[4] = {raw0.x, raw0.y, raw0.z, raw0.w};
#pragma unroll
                for (int i = 0; i < FW_EPL / 8; i++) {
                    uint32_t h0, h1, h2, h3;
                    cvt_e2m1x8(wv[i], h0, h1, h2, h3);
                    o[4 * i] = fw_scale_bf2(h0, sc);
                    o[4 * i + 1] = fw_scale_bf2(h1, sc);
                    o[4 * i + 2] = fw_scale_bf2(h2, sc);
                    o[4 * i + 3] = fw_scale_bf2(h3, sc);
                }
            } else {
                const uint32_t wv[8] = {raw0.x, raw0.y, raw0.z, raw0.w, raw1.x, raw1.y, raw1.z, raw1.w};
#pragma unroll
                for (int i = 0; i < FW_EPL / 4; i++) {
                    uint32_t lo, hi;
                    cvt_e4m3x4(wv[i], lo, hi);
                    o[2 * i] = fw_scale_bf2(lo, sc);
                    o[2 * i + 1] = fw_scale_bf2(hi, sc);
                }
            }
            // 16-byte pieces FW_CPL h .. FW_CPL (h + 1) - 1 of row r, 128-byte swizzle
            uint8_t *arow = smem + s * FW_STAGE + r * 128;
#pragma unroll
            for (int j = 0; j < FW_CPL; j++) {
                const int cchunk = (FW_CPL * h + j) ^ (r & 7);
                *reinterpret_cast<uint4 *>(arow + 16 * cchunk) =
                    make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[s]);
        }
    } else {
        // ------------------------------------------------ epilogue
        const int q = warp & 3;
        int tc = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, tc++) {
            const int ab = tc & 1, use = tc >> 1;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&accf[ab], use & 1, p.err, FWE_ACCF);
            if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) break;
            umma::fence_after();
            const int tm = t % p.tiles_m, tn = t / p.tiles_m;
            const int row = tm * FW_M + q * 32 + lane;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * FW_N;
            for (int c8 = 0; c8 < FW_N; c8 += 8) {
                float v[8];
                umma::ld_x8(tbase + c8, v);
                if (row >= p.rows) continue;
                if (p.terms == 1) {
                    const int t0 = tn * FW_N + c8;
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        if (t0 + i < p.nt) p.y[(size_t)(t0 + i) * p.rows + row] = v[i];
                } else {                            // columns 2j, 2j + 1: hi and lo term of one token
                    const int t0 = (tn * FW_N + c8) / 2;
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        if (t0 + i < p.nt) p.y[(size_t)(t0 + i) * p.rows + row] = v[2 * i] + v[2 * i + 1];
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
        umma::tmem_dealloc(tmem, 512);
    }
}

}  // namespace dsv4cu

using namespace dsv4cu;

// Weight conversion: in the converter warps (every 256-token tile converts
// the weights again) or once per call into a bf16 copy in the workspace.
static int g_fw_path = DSV4CU_BF16W_AUTO;

extern "C" int dsv4cu_gemm_bf16w_set_path(int path)
{
    if (path != DSV4CU_BF16W_AUTO && path != DSV4CU_BF16W_CONVERT && path != DSV4CU_BF16W_PREDEQUANT)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "gemm_bf16w_set_path: unknown path %d", path);
    g_fw_path = path;
    return DSV4CU_OK;
}

// Pre-dequantized when the call has more than one token tile (the weights
// would otherwise be converted once per tile).
static bool fw_use_pre(int nt, int terms)
{
    if (g_fw_path != DSV4CU_BF16W_AUTO) return g_fw_path == DSV4CU_BF16W_PREDEQUANT;
    return (long)nt * terms > FW_N;
}

extern "C" size_t dsv4cu_gemm_bf16w_workspace(const dsv4cu_qmat *m, int nt, int terms)
{
    if (!m || nt <= 0 || terms < 1 || terms > 2) return 0;
    size_t b = dsv4cu_align256((size_t)nt * terms * m->cols * 2);
    if (fw_use_pre(nt, terms)) b += dsv4cu_align256((size_t)m->rows * m->cols * 2);
    return b;
}

extern "C" int dsv4cu_gemm_bf16w(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *m, int nt, int terms,
                                 void *stream)
{
    if (terms < 1 || terms > 2) return dsv4cu_set_error(DSV4CU_ERR_ARG, "gemm_bf16w: terms %d (1 or 2)", terms);
    if (!ctx || !y || !x || !m || !m->w || !m->s) return dsv4cu_set_error(DSV4CU_ERR_ARG, "gemm_bf16w: NULL argument");
    if (nt <= 0) return DSV4CU_OK;
    const bool fp4 = m->wdt == DSV4CU_WFP4;
    if (!fp4 && m->wdt != DSV4CU_WFP8)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "gemm_bf16w: FP8 or FP4 weights only");
    const int row_bytes = fp4 ? m->cols / 2 : m->cols;
    const auto pow2 = [](int v) { return v > 0 && (v & (v - 1)) == 0; };
    if (m->rows <= 0 || m->cols <= 0 || m->cols % FW_KC || !pow2(m->blk_r) || !pow2(m->blk_c) || m->blk_c < 32 ||
        ((uintptr_t)m->w & 15u) || row_bytes % 16 || ((uintptr_t)x & 15u))
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED,
                                "gemm_bf16w: needs cols %% 64 == 0, power-of-two blocks with blk_c >= 32, 16-byte "
                                "aligned weights and x (rows %d cols %d blk %dx%d)", m->rows, m->cols, m->blk_r,
                                m->blk_c);
    cudaStream_t st = (cudaStream_t)stream;
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, dsv4cu_gemm_bf16w_workspace(m, nt, terms), &ws);
    if (r) return r;
    __nv_bfloat16 *xb = (__nv_bfloat16 *)ws;
    const long n4 = (long)nt * m->cols / 4;
    CUtensorMap tb;
    if ((r = tmap_encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xb, (uint64_t)m->cols, (uint64_t)nt * terms,
                            (uint64_t)m->cols * 2, FW_KC, FW_N, CU_TENSOR_MAP_SWIZZLE_128B)))
        return r;
    FwParams p;
    p.w = (const uint8_t *)m->w;
    p.s = (const uint8_t *)m->s;
    p.rows = m->rows;
    p.cols = m->cols;
    p.fp4 = fp4;
    p.blk_r_log2 = __builtin_ctz((unsigned)m->blk_r);
    p.blk_c_log2 = __builtin_ctz((unsigned)m->blk_c);
    p.s_cols = (m->cols + m->blk_c - 1) / m->blk_c;
    p.row_bytes = row_bytes;
    p.tiles_m = (m->rows + FW_M - 1) / FW_M;
    p.tiles_n = (nt * terms + FW_N - 1) / FW_N;
    p.nt = nt;
    p.terms = terms;
    p.y = y;
    p.err = ctx->status;
    p.pre = fw_use_pre(nt, terms);
    CUtensorMap tw;
    // bf16 copy of the weights (pre-dequantized mode) after the activation
    // rows; 128 rows x one chunk per box with the 128-byte swizzle (the
    // converters' layout)
    uint4 *wb = (uint4 *)((char *)ws + dsv4cu_align256((size_t)nt * terms * m->cols * 2));
    {
        const int xblocks = (int)min(4096L, (n4 + 255) / 256);
        const long wblocks = p.pre ? ((long)m->rows * (m->cols / 16) + 255) / 256 : 0;
        fw_prep_kernel<<<(unsigned)(xblocks + wblocks), 256, 0, st>>>(x, xb, m->cols, n4, terms, xblocks, p, wb);
        DSV4CU_LAUNCH_CHECK();
    }
    if (p.pre) {
        if ((r = tmap_encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, wb, (uint64_t)m->cols, (uint64_t)m->rows,
                                (uint64_t)m->cols * 2, FW_KC, FW_M, CU_TENSOR_MAP_SWIZZLE_128B)))
            return r;
    } else if ((r = tmap_encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, m->w, (uint64_t)row_bytes, (uint64_t)m->rows,
                                   (uint64_t)row_bytes, fp4 ? FW_KC / 2 : FW_KC, FW_M, CU_TENSOR_MAP_SWIZZLE_NONE))) {
        // packed weights: 128 rows x one chunk (64 elements) per box, rows past the end read as 0
        return r;
    }
    static SmemLimit lim;
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)fw_kernel, FW_SMEM));
    const int grid = min(ctx->sm_count, p.tiles_m * p.tiles_n);
    DSV4CU_CUDA_TRY(launch_pdl(fw_kernel, dim3(grid), dim3(FW_THREADS), FW_SMEM, st, tb, tw, p));
    return DSV4CU_OK;
}
