// indexer.cu - CSA lightning-indexer score, bit-identical to the reference.
//
// Reference: dsv4_indexer_score (src/10_compute/dsv4_indexer.c:66-90) with the
// dot product dsv4_dot_f32d (src/10_compute/dsv4_dot.h:20-42):
//   dot(q_h, k_t) = 16 fma chains in double, chain l taking elements 16j + l,
//                   folded as ((p_l + p_{l+4}) + (p_{l+8} + p_{l+12})) for
//                   l = 0..3, then (b0 + b1) + (b2 + b3); a d % 16 tail
//                   continues with fma on the folded value.
//   total_t       = sum over heads IN ORDER of dot * (double)w_h, dot > 0 only
//   out[t]        = (float)total_t * ((1/sqrtf(d)) * (1/sqrtf(h)))  [float]
// The GPU replays exactly these IEEE operations (DFMA, DADD, DMUL, one
// double->float rounding and one float multiply), so every score is the same
// bit pattern as the reference and the top-k indices match exactly.
//
// Layout: a persistent grid; each CTA stages q as double in shared memory once
// and its warps walk positions. One warp computes two heads at a time: lanes
// 0-15 run the 16 chains of head h, lanes 16-31 those of head h+1.
#include "common.cuh"
#include "ctx.h"

namespace dsv4cu {

constexpr int IDX_MAX_D = 256;       // head_dim bound (chains of <= 16 elements)
constexpr int IDX_WARPS = 16;

// load(t, i) = key element i of position t as a double; raw / rscale / val
// split it into the global loads and the conversion, so loads can run ahead.
struct KeysF32 {
    using Raw = float;
    const float *kv;
    int ld;
    DSV4CU_DEV double load(int t, int i) const { return (double)__ldg(kv + (size_t)t * ld + i); }
    DSV4CU_DEV Raw raw(int t, int i) const { return __ldg(kv + (size_t)t * ld + i); }
    DSV4CU_DEV float rscale(int) const { return 1.0f; }
    DSV4CU_DEV double val(Raw r, float) const { return (double)r; }
};
struct KeysFP8 {
    using Raw = uint32_t;
    const uint8_t *k8;
    const float *ks;
    int ld;
    DSV4CU_DEV double load(int t, int i) const
    {
        const float v = __fmul_rn(e4m3_to_f32(__ldg(k8 + (size_t)t * ld + i)), __ldg(ks + t));
        return (double)v;
    }
    DSV4CU_DEV Raw raw(int t, int i) const { return __ldg(k8 + (size_t)t * ld + i); }
    DSV4CU_DEV float rscale(int t) const { return __ldg(ks + t); }
    DSV4CU_DEV double val(Raw r, float sc) const { return (double)__fmul_rn(e4m3_to_f32((uint8_t)r), sc); }
};

template <class K>
__global__ void __launch_bounds__(IDX_WARPS * 32) indexer_score_kernel(
    float *__restrict__ out, const double *__restrict__ qd_g, const float *__restrict__ w, int H, int D,
    int n_pos, float scale, K keys)
{
    extern __shared__ double qs[];   // [H][D]
    for (int i = threadIdx.x; i < H * D; i += blockDim.x) qs[i] = qd_g[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, l = lane & 15, half = lane >> 4;
    const int nfull = D >> 4, tail0 = nfull << 4;

    for (int t = blockIdx.x * IDX_WARPS + warp; t < n_pos; t += gridDim.x * IDX_WARPS) {
        double kr[IDX_MAX_D / 16];
#pragma unroll
        for (int j = 0; j < IDX_MAX_D / 16; j++) kr[j] = (j < nfull) ? keys.load(t, 16 * j + l) : 0.0;
        double total = 0.0;
        for (int h0 = 0; h0 < H; h0 += 2) {
            const int h = h0 + half;
            const double *qh = qs + (size_t)(h < H ? h : 0) * D;
            double p = 0.0;
#pragma unroll
            for (int j = 0; j < IDX_MAX_D / 16; j++)
                if (j < nfull) p = __fma_rn(qh[16 * j + l], kr[j], p);
            // (p_l + p_{l+4}) then + (p_{l+8} + p_{l+12}) for l < 4, then the pair tree.
            p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 4));
            p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 8));
            p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 1));
            p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 2));
            // lanes 0 and 16 hold the folded dot of heads h0 and h0 + 1.
            if (l == 0) {
                for (int i = tail0; i < D; i++) p = __fma_rn(qh[i], keys.load(t, i), p);
            }
            const double d1 = __shfl_sync(0xFFFFFFFFu, p, 16);
            if (lane == 0) {
                if (p > 0.0) total = __dadd_rn(total, __dmul_rn(p, (double)__ldg(w + h0)));
                if (h0 + 1 < H && d1 > 0.0) total = __dadd_rn(total, __dmul_rn(d1, (double)__ldg(w + h0 + 1)));
            }
        }
        if (lane == 0) out[t] = __fmul_rn((float)total, scale);
    }
}

// The same IEEE operations, arranged for throughput when head_dim = 16 J and
// n_heads % 16 == 0. A warp covers 4 positions: half h (lanes 16h .. 16h+15)
// takes positions 2h and 2h + 1, lane l of a half runs chain l of both, so
// every q element read from shared memory (a broadcast to both halves) feeds
// two fma. Heads go 16 at a time; the 16 chain values of the 16 heads are
// folded by recursive halving over lane bits 2, 3, 0, 1: partners xor 4 and
// xor 8 give (p_l + p_{l+4}) + (p_{l+8} + p_{l+12}) = b_{l mod 4}, partners
// xor 1 and xor 2 give (b0 + b1) + (b2 + b3) - the reference's tree, with
// each addition's two operands the same (IEEE addition is commutative) - and
// each lane keeps the dot of head 8 b2 + 4 b3 + 2 b0 + b1 (b_i = bit i of l).
// The dots go to shared memory and four lanes add the heads in order.
constexpr int IDXF_WARPS = 12;

template <int J, class K>
__global__ void __launch_bounds__(IDXF_WARPS * 32, 1) indexer_fast_kernel(
    float *__restrict__ out, const double *__restrict__ qd_g, const float *__restrict__ w, int H, int n_pos,
    float scale, K keys)
{
    constexpr int D = 16 * J;
    extern __shared__ double ism[];          // q [H][D], then dots [IDXF_WARPS][4][H]
    double *qs = ism;
    for (int i = threadIdx.x; i < H * D; i += blockDim.x) qs[i] = qd_g[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, l = lane & 15, half = lane >> 4;
    const bool b0 = l & 1, b1 = l & 2, b2 = l & 4, b3 = l & 8;
    const int hoff = 8 * b2 + 4 * b3 + 2 * b0 + b1;
    double *dw = ism + H * D + warp * 4 * H;

    // The next positions' key bytes are requested before this position's math.
    typename K::Raw raw[2][J];
    float rsc[2];
    auto fetch = [&](int tb) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int t = tb + 2 * half + r;
            const bool ok = t < n_pos;
            rsc[r] = ok ? keys.rscale(t) : 0.0f;
#pragma unroll
            for (int j = 0; j < J; j++) raw[r][j] = ok ? keys.raw(t, 16 * j + l) : (typename K::Raw)0;
        }
    };
    const int tstride = gridDim.x * IDXF_WARPS * 4;
    fetch((blockIdx.x * IDXF_WARPS + warp) * 4);
    for (int t0 = (blockIdx.x * IDXF_WARPS + warp) * 4; t0 < n_pos; t0 += tstride) {
        double k[2][J];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const bool ok = t0 + 2 * half + r < n_pos;
#pragma unroll
            for (int j = 0; j < J; j++) k[r][j] = ok ? keys.val(raw[r][j], rsc[r]) : 0.0;
        }
        fetch(t0 + tstride);
        for (int hg = 0; hg < H; hg += 16) {
            double v[2][16];
#pragma unroll
            for (int hh = 0; hh < 16; hh++) {
                const double *qh = qs + (size_t)(hg + hh) * D + l;
                double p0 = 0.0, p1 = 0.0;
#pragma unroll
                for (int j = 0; j < J; j++) {
                    const double qv = qh[16 * j];
                    p0 = __fma_rn(qv, k[0][j], p0);
                    p1 = __fma_rn(qv, k[1][j], p1);
                }
                v[0][hh] = p0;
                v[1][hh] = p1;
            }
#pragma unroll
            for (int r = 0; r < 2; r++) {
                double a8[8], a4[4], a2[2];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const double send = b2 ? v[r][i] : v[r][8 + i];
                    a8[i] = __dadd_rn(b2 ? v[r][8 + i] : v[r][i], __shfl_xor_sync(0xFFFFFFFFu, send, 4));
                }
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const double send = b3 ? a8[i] : a8[4 + i];
                    a4[i] = __dadd_rn(b3 ? a8[4 + i] : a8[i], __shfl_xor_sync(0xFFFFFFFFu, send, 8));
                }
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const double send = b0 ? a4[i] : a4[2 + i];
                    a2[i] = __dadd_rn(b0 ? a4[2 + i] : a4[i], __shfl_xor_sync(0xFFFFFFFFu, send, 1));
                }
                const double send = b1 ? a2[0] : a2[1];
                dw[(2 * half + r) * H + hg + hoff] =
                    __dadd_rn(b1 ? a2[1] : a2[0], __shfl_xor_sync(0xFFFFFFFFu, send, 2));
            }
        }
        __syncwarp();
        if (lane < 4 && t0 + lane < n_pos) {
            const double *dd = dw + lane * H;
            double total = 0.0;
            for (int h = 0; h < H; h++) {
                const double d = dd[h];
                if (d > 0.0) total = __dadd_rn(total, __dmul_rn(d, (double)__ldg(w + h)));
            }
            out[t0 + lane] = __fmul_rn((float)total, scale);
        }
        __syncwarp();
    }
}


// ------------------------------------------------------------ FP8 keys, FP64 tensor cores
// For the FP8 cache (64 heads x 128) the dots can run on the FP64 tensor
// core (mma.m8n8k4.f64) without changing a bit, when every scale involved
// is a power of two 2^e with -117 <= e <= 118 (or zero): then each q and k
// value is fl32(e4m3 x scale) = an integer below 2^18 times a quantum of
// 2^-9 x scale, exactly, each product is an integer below 2^36 times the
// product of the quanta, and all 128 products of a dot and every partial sum
// are integers below 2^43 in those units - exact in double. The reference's
// fma chains and pairwise fold therefore never round, and neither does any
// other order: the dot is the exact value either way. The head sum
// total = sum_h relu(dot_h) w_h stays in the reference's order, per position.
// A warp task (16 positions) whose key scales (or the q scales) fail the
// test is computed by the exact replay instead.
constexpr int IDXM_WARPS = 8, IDXM_POS = 16, IDXM_H = 64, IDXM_D = 128;
constexpr int IDXM_DSTRIDE = IDXM_H + 1;   // dot rows padded against bank conflicts

DSV4CU_DEV bool idx_pow2_scale(float s)
{
    const uint32_t u = __float_as_uint(s) & 0x7FFFFFFFu;
    if (u == 0u) return true;
    const int e = (int)(u >> 23) - 127;
    return (u & 0x7FFFFFu) == 0u && e >= -117 && e <= 118;
}

// D[8x8] += A[8x4] B[4x8] in FP64; lane: a = A[lane / 4][lane % 4],
// b = B[lane % 4][lane / 4], d = D[lane / 4][2 (lane % 4) + {0, 1}].
DSV4CU_DEV void dmma_884(double (&d)[2], double a, double b)
{
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

// q element (h, k) in the fragment order [k / 4][h / 8][(h % 8) * 4 + k % 4].
DSV4CU_DEV double idxm_q(const double *qf, int h, int k)
{
    return qf[((k >> 2) * 8 + (h >> 3)) * 32 + (h & 7) * 4 + (k & 3)];
}

// The exact replay of one position (16 fma chains, the reference's fold),
// two heads at a time; writes dot[h] for every head.
DSV4CU_DEV void idxm_replay(const double *qf, const KeysFP8 &keys, int t, double *dot)
{
    const int lane = threadIdx.x & 31, l = lane & 15, half = lane >> 4;
    double kr[IDXM_D / 16];
#pragma unroll
    for (int j = 0; j < IDXM_D / 16; j++) kr[j] = keys.load(t, 16 * j + l);
    for (int h0 = 0; h0 < IDXM_H; h0 += 2) {
        const int h = h0 + half;
        double p = 0.0;
#pragma unroll
        for (int j = 0; j < IDXM_D / 16; j++) p = __fma_rn(idxm_q(qf, h, 16 * j + l), kr[j], p);
        p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 4));
        p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 8));
        p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 1));
        p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 2));
        if (l == 0) dot[h] = p;
    }
}


__global__ void __launch_bounds__(IDXM_WARPS * 32, 1) indexer_dmma_kernel(
    float *__restrict__ out, const double *__restrict__ qd_g, const float *__restrict__ qscale,
    const float *__restrict__ w, int n_pos, float scale, KeysFP8 keys)
{
    extern __shared__ double idxm_sm[];
    double *qf = idxm_sm;                                  // [32][8][32] fragment order
    double *dots = qf + IDXM_D / 4 * 8 * 32;               // [IDXM_WARPS][IDXM_POS][IDXM_DSTRIDE]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < IDXM_H * IDXM_D; i += blockDim.x) {
        const int ks = i >> 8, mt = (i >> 5) & 7, L = i & 31;
        qf[i] = qd_g[(mt * 8 + (L >> 2)) * IDXM_D + 4 * ks + (L & 3)];
    }
    const int q_ok = __syncthreads_and(tid < IDXM_H ? idx_pow2_scale(__ldg(qscale + tid)) : 1);
    double *dw = dots + warp * IDXM_POS * IDXM_DSTRIDE;
    const int g = lane >> 2, c = lane & 3;

    for (int task = blockIdx.x * IDXM_WARPS + warp; task * IDXM_POS < n_pos; task += gridDim.x * IDXM_WARPS) {
        const int t0 = task * IDXM_POS;
        const int tl = t0 + (lane & 15);
        const bool ok = __all_sync(0xFFFFFFFFu, tl >= n_pos || idx_pow2_scale(__ldg(keys.ks + tl))) && q_ok;
        if (ok) {
            double acc[2][8][2];
#pragma unroll
            for (int nt = 0; nt < 2; nt++)
#pragma unroll
                for (int mt = 0; mt < 8; mt++) acc[nt][mt][0] = acc[nt][mt][1] = 0.0;
            // B: position t0 + 8 nt + g, element 4 ks + c.
            const uint8_t *row[2];
            float ksc[2];
            bool live[2];
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                const int t = t0 + 8 * nt + g;
                live[nt] = t < n_pos;
                row[nt] = keys.k8 + (size_t)(live[nt] ? t : 0) * keys.ld;
                ksc[nt] = live[nt] ? __ldg(keys.ks + t) : 0.0f;
            }
#pragma unroll 4
            for (int ks = 0; ks < IDXM_D / 4; ks++) {
                double b[2];
#pragma unroll
                for (int nt = 0; nt < 2; nt++)
                    b[nt] = live[nt] ? (double)__fmul_rn(e4m3_to_f32(__ldg(row[nt] + 4 * ks + c)), ksc[nt]) : 0.0;
                const double *qa = qf + ks * 256 + lane;
#pragma unroll
                for (int mt = 0; mt < 8; mt++) {
                    const double a = qa[mt * 32];
                    dmma_884(acc[0][mt], a, b[0]);
                    dmma_884(acc[1][mt], a, b[1]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 2; nt++)
#pragma unroll
                for (int mt = 0; mt < 8; mt++)
#pragma unroll
                    for (int j = 0; j < 2; j++) dw[(8 * nt + 2 * c + j) * IDXM_DSTRIDE + mt * 8 + g] = acc[nt][mt][j];
        } else {
            for (int p = 0; p < IDXM_POS && t0 + p < n_pos; p++) idxm_replay(qf, keys, t0 + p, dw + p * IDXM_DSTRIDE);
        }
        __syncwarp();
        if (lane < IDXM_POS && t0 + lane < n_pos) {
            const double *dd = dw + lane * IDXM_DSTRIDE;
            double total = 0.0;
            for (int h = 0; h < IDXM_H; h++) {
                const double d = dd[h];
                if (d > 0.0) total = __dadd_rn(total, __dmul_rn(d, (double)__ldg(w + h)));
            }
            out[t0 + lane] = __fmul_rn((float)total, scale);
        }
        __syncwarp();
    }
}

static float indexer_scale(int H, int D);

static int indexer_dmma_launch(float *out, const double *qd, const float *qscale, const float *w, int n_pos,
                               KeysFP8 keys, cudaStream_t st)
{
    const size_t smem = ((size_t)IDXM_H * IDXM_D + (size_t)IDXM_WARPS * IDXM_POS * IDXM_DSTRIDE) * sizeof(double);
    static SmemLimit lim;
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)indexer_dmma_kernel, (int)smem));
    int blocks = device_sms();
    const int need = (n_pos + IDXM_WARPS * IDXM_POS - 1) / (IDXM_WARPS * IDXM_POS);
    if (blocks > need) blocks = need;
    indexer_dmma_kernel<<<blocks, IDXM_WARPS * 32, smem, st>>>(out, qd, qscale, w, n_pos,
                                                               indexer_scale(IDXM_H, IDXM_D), keys);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

// ------------------------------------------------------------ FP8 keys, int8 tensor cores
// The same exact dots (every scale a power of two), computed in integers on
// the int8 tensor cores (mma.sync m16n8k32 s8 -> s32). With q = e4m3 x 2^eq
// and k = e4m3 x 2^ek, each element is an integer I below 2^18 in units of
// 2^-9 times its scale; written as three signed base-128 digits
// I = d0 + 128 d1 + 16384 d2 (|d0|, |d1| <= 127, |d2| <= 14, all with the
// sign of I), the dot is
//   sum_k Iq Ik = sum over digit pairs (a, b) of 128^(a+b) D_ab,
//   D_ab = sum_k dq_a dk_b           (one int8 GEMM per digit pair).
// The five weights 128^L are folded in two int32 accumulators by Horner's
// rule: hi = D_(L=2) + 128 (D_(L=3) + 128 D_(L=4)) and lo = D_(L=0) + 128
// D_(L=1); with 128 elements |hi| < 4.8e8 and |lo| < 2^30, and the dot
// 16384 hi + lo < 2^43 is an exact double, scaled by 2^(eq + ek - 18).
// Integer sums do not depend on the order of the terms, so the k order
// inside a fragment is free: lane c of a quad takes the 32 contiguous
// elements [32c, 32c + 32) of each row, two 16-byte loads. The head sum per
// position, the NaN handling (a NaN byte in q or in a 16-position task sends
// it to the exact replay, whose NaN dots fail "dot > 0" as in the reference)
// and the output rounding are those of the other kernels.
constexpr int IDXL_WARPS = 16;
constexpr int IDXL_ZERO = -100000;   // exponent marker of a zero scale
static int g_idx_limbs = 1;          // 0: the FP64 tensor-core kernel (dsv4cu_indexer_set_path)

// The e4m3 byte b as digits (bytes 0-2 of the word, int8 each).
DSV4CU_DEV uint32_t idxl_digits(uint32_t b)
{
    const uint32_t E = (b >> 3) & 15u, m = b & 7u;
    uint32_t I = E ? (8u + m) << (E - 1u) : m;
    if ((b & 0x7Fu) == 0x7Fu) I = 0u;   // NaN: never used (the task is replayed)
    int d0 = (int)(I & 127u), d1 = (int)((I >> 7) & 127u), d2 = (int)(I >> 14);
    if (b & 0x80u) {
        d0 = -d0;
        d1 = -d1;
        d2 = -d2;
    }
    return ((uint32_t)d0 & 0xFFu) | (((uint32_t)d1 & 0xFFu) << 8) | (((uint32_t)d2 & 0xFFu) << 16);
}

DSV4CU_DEV bool idxl_has_nan(uint32_t w) { return __vcmpeq4(w & 0x7F7F7F7Fu, 0x7F7F7F7Fu) != 0u; }

// Four e4m3 bytes -> digit words l0, l1, l2 (byte i of l_a = digit a of byte i).
DSV4CU_DEV void idxl_split(const uint32_t *tbl, uint32_t w, uint32_t &l0, uint32_t &l1, uint32_t &l2)
{
    const uint32_t t0 = tbl[w & 0xFFu], t1 = tbl[(w >> 8) & 0xFFu], t2 = tbl[(w >> 16) & 0xFFu], t3 = tbl[w >> 24];
    const uint32_t x = __byte_perm(t0, t1, 0x5140), y = __byte_perm(t2, t3, 0x5140);
    l0 = __byte_perm(x, y, 0x5410);
    l1 = __byte_perm(x, y, 0x7632);
    l2 = __byte_perm(__byte_perm(t0, t1, 0x0062), __byte_perm(t2, t3, 0x0062), 0x5410);
}

// D[16x8] += A[16x32] B[32x8] in int8 -> int32; lane (g = lane / 4, c = lane % 4):
// a = rows g, g + 8 x k {4c..4c+3, 16+4c..16+4c+3}, b = k {4c.., 16+4c..} x column g,
// d = rows g, g + 8 x columns 2c, 2c + 1.
DSV4CU_DEV void imma_16832(int (&d)[4], const uint32_t (&a)[4], uint2 b)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}

DSV4CU_DEV int idxl_exp(float s)
{
    const uint32_t u = __float_as_uint(s) & 0x7FFFFFFFu;
    return u ? (int)(u >> 23) - 127 : IDXL_ZERO;
}

// The exact replay of one position with q read from its e4m3 bytes.
DSV4CU_DEV void idxl_replay(const uint8_t *q8, const float *qscale, const KeysFP8 &keys, int t, double *dot)
{
    const int lane = threadIdx.x & 31, l = lane & 15, half = lane >> 4;
    double kr[IDXM_D / 16];
#pragma unroll
    for (int j = 0; j < IDXM_D / 16; j++) kr[j] = keys.load(t, 16 * j + l);
    for (int h0 = 0; h0 < IDXM_H; h0 += 2) {
        const int h = h0 + half;
        const float qs = __ldg(qscale + h);
        double p = 0.0;
#pragma unroll
        for (int j = 0; j < IDXM_D / 16; j++)
            p = __fma_rn((double)__fmul_rn(e4m3_to_f32(__ldg(q8 + h * IDXM_D + 16 * j + l)), qs), kr[j], p);
        p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 4));
        p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 8));
        p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 1));
        p = __dadd_rn(p, __shfl_down_sync(0xFFFFFFFFu, p, 2));
        if (l == 0) dot[h] = p;
    }
}

__global__ void __launch_bounds__(IDXL_WARPS * 32, 1) indexer_limb_kernel(
    float *__restrict__ out, const uint8_t *__restrict__ q8, const float *__restrict__ qscale,
    const float *__restrict__ w, int n_pos, float scale, KeysFP8 keys)
{
    extern __shared__ __align__(16) unsigned char idxl_sm[];
    // q digits in fragment order: entry ((a * 4 + s) * 8 + nt) * 32 + L holds
    // digit a of head 8 nt + L / 4, elements 32 (L % 4) + 8 s + {0..3 | 4..7}.
    uint2 *qfrag = reinterpret_cast<uint2 *>(idxl_sm);
    double *dots = reinterpret_cast<double *>(idxl_sm + 3 * 4 * 8 * 32 * sizeof(uint2));
    __shared__ uint32_t tbl[256];
    __shared__ int qexp[IDXM_H];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < 256; i += blockDim.x) tbl[i] = idxl_digits((uint32_t)i);
    int okq = 1;
    if (tid < IDXM_H) {
        const float s = __ldg(qscale + tid);
        okq = idx_pow2_scale(s);
        qexp[tid] = idxl_exp(s);
    }
    __syncthreads();
    for (int i = tid; i < 4 * 8 * 32; i += blockDim.x) {
        const int L = i & 31, nt = (i >> 5) & 7, s = i >> 8;
        const uint8_t *src = q8 + (8 * nt + (L >> 2)) * IDXM_D + 32 * (L & 3) + 8 * s;
        uint32_t v[2];
#pragma unroll
        for (int hw = 0; hw < 2; hw++)
            v[hw] = (uint32_t)__ldg(src + 4 * hw) | ((uint32_t)__ldg(src + 4 * hw + 1) << 8) |
                    ((uint32_t)__ldg(src + 4 * hw + 2) << 16) | ((uint32_t)__ldg(src + 4 * hw + 3) << 24);
        okq &= !idxl_has_nan(v[0]) && !idxl_has_nan(v[1]);
        uint32_t a[3], b[3];
        idxl_split(tbl, v[0], a[0], a[1], a[2]);
        idxl_split(tbl, v[1], b[0], b[1], b[2]);
#pragma unroll
        for (int d = 0; d < 3; d++) qfrag[(d * 4 + s) * 256 + nt * 32 + L] = make_uint2(a[d], b[d]);
    }
    const int q_ok = __syncthreads_and(okq);
    double *dw = dots + warp * IDXM_POS * IDXM_DSTRIDE;
    const int g = lane >> 2, c = lane & 3;

    for (int task = blockIdx.x * IDXL_WARPS + warp; task * IDXM_POS < n_pos; task += gridDim.x * IDXL_WARPS) {
        const int t0 = task * IDXM_POS;
        const int tl = t0 + (lane & 15);
        // rows g and g + 8 of the task, elements [32c, 32c + 32)
        uint4 kw[2][2];
        bool bad = false;
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int t = t0 + g + 8 * r;
            if (t < n_pos) {
                const uint4 *p = reinterpret_cast<const uint4 *>(keys.k8 + (size_t)t * keys.ld + 32 * c);
                kw[r][0] = __ldg(p);
                kw[r][1] = __ldg(p + 1);
            } else {
                kw[r][0] = kw[r][1] = make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int hh = 0; hh < 2; hh++)
                bad |= idxl_has_nan(kw[r][hh].x) | idxl_has_nan(kw[r][hh].y) | idxl_has_nan(kw[r][hh].z) |
                       idxl_has_nan(kw[r][hh].w);
        }
        const bool ok = q_ok && !__any_sync(0xFFFFFFFFu, bad) &&
                        __all_sync(0xFFFFFFFFu, tl >= n_pos || idx_pow2_scale(__ldg(keys.ks + tl)));
        if (ok) {
            // A[digit][k step][register]: k step s takes words 2s (registers 0, 1)
            // and 2s + 1 (registers 2, 3) of rows g (0, 2) and g + 8 (1, 3).
            uint32_t A[3][4][4];
#pragma unroll
            for (int r = 0; r < 2; r++)
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const uint4 v = kw[r][q >> 2];
                    const uint32_t word = (q & 3) == 0 ? v.x : (q & 3) == 1 ? v.y : (q & 3) == 2 ? v.z : v.w;
                    const int s = q >> 1, reg = r + 2 * (q & 1);
                    idxl_split(tbl, word, A[0][s][reg], A[1][s][reg], A[2][s][reg]);
                }
            int ek[2];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int t = t0 + g + 8 * r;
                ek[r] = t < n_pos ? idxl_exp(__ldg(keys.ks + t)) : IDXL_ZERO;
            }
            // Heads in two halves of 32 (n tiles 4 hb .. 4 hb + 3): 16 accumulators.
#pragma unroll 1
            for (int hb = 0; hb < 2; hb++) {
                const uint2 *qb = qfrag + hb * 4 * 32 + lane;
                int acc[4][4];
                auto zero = [&]() {
#pragma unroll
                    for (int nt = 0; nt < 4; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) acc[nt][i] = 0;
                };
                auto times128 = [&]() {
#pragma unroll
                    for (int nt = 0; nt < 4; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) acc[nt][i] *= 128;
                };
                auto mac = [&](int ka, int qa) {   // acc += (key digit ka) x (q digit qa), all 128 elements
#pragma unroll
                    for (int s = 0; s < 4; s++)
#pragma unroll
                        for (int nt = 0; nt < 4; nt++) imma_16832(acc[nt], A[ka][s], qb[(qa * 4 + s) * 256 + nt * 32]);
                };
                zero();
                mac(2, 2);
                times128();
                mac(1, 2);
                mac(2, 1);
                times128();
                mac(0, 2);
                mac(1, 1);
                mac(2, 0);
#pragma unroll
                for (int nt = 0; nt < 4; nt++)
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        dw[(g + 8 * (i >> 1)) * IDXM_DSTRIDE + 32 * hb + 8 * nt + 2 * c + (i & 1)] =
                            (double)acc[nt][i] * 16384.0;
                zero();
                mac(0, 1);
                mac(1, 0);
                times128();
                mac(0, 0);
#pragma unroll
                for (int nt = 0; nt < 4; nt++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int h = 32 * hb + 8 * nt + 2 * c + (i & 1);
                        double *slot = dw + (g + 8 * (i >> 1)) * IDXM_DSTRIDE + h;
                        const int eq = qexp[h], e = ek[i >> 1];
                        const double v = __dadd_rn(*slot, (double)acc[nt][i]);   // 16384 hi + lo, exact
                        *slot = (eq == IDXL_ZERO || e == IDXL_ZERO)
                                    ? 0.0
                                    : v * __hiloint2double((eq + e - 18 + 1023) << 20, 0);
                    }
            }
        } else {
            for (int p = 0; p < IDXM_POS && t0 + p < n_pos; p++)
                idxl_replay(q8, qscale, keys, t0 + p, dw + p * IDXM_DSTRIDE);
        }
        __syncwarp();
        if (lane < IDXM_POS && t0 + lane < n_pos) {
            const double *dd = dw + lane * IDXM_DSTRIDE;
            double total = 0.0;
            for (int h = 0; h < IDXM_H; h++) {
                const double d = dd[h];
                if (d > 0.0) total = __dadd_rn(total, __dmul_rn(d, (double)__ldg(w + h)));
            }
            out[t0 + lane] = __fmul_rn((float)total, scale);
        }
        __syncwarp();
    }
}

static int indexer_limb_launch(float *out, const uint8_t *q8, const float *qscale, const float *w, int n_pos,
                               KeysFP8 keys, cudaStream_t st)
{
    const size_t smem = (size_t)3 * 4 * 8 * 32 * sizeof(uint2) +
                        (size_t)IDXL_WARPS * IDXM_POS * IDXM_DSTRIDE * sizeof(double);
    static SmemLimit lim;
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)indexer_limb_kernel, (int)smem));
    int blocks = device_sms();
    const int need = (n_pos + IDXL_WARPS * IDXM_POS - 1) / (IDXL_WARPS * IDXM_POS);
    if (blocks > need) blocks = need;
    indexer_limb_kernel<<<blocks, IDXL_WARPS * 32, smem, st>>>(out, q8, qscale, w, n_pos,
                                                               indexer_scale(IDXM_H, IDXM_D), keys);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

// q (fp32, or e4m3 * per-head scale in float) -> double, once per call.
__global__ void indexer_q_kernel(double *qd, const float *q, const uint8_t *q8, const float *qscale, int H, int D)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= H * D) return;
    qd[i] = q ? (double)q[i] : (double)__fmul_rn(e4m3_to_f32(q8[i]), qscale[i / D]);
}

// Scale computed as the reference does, in float: (1/sqrtf(d)) * (1/sqrtf(h)).
static float indexer_scale(int H, int D)
{
    const float a = 1.0f / sqrtf((float)D), b = 1.0f / sqrtf((float)H);
    volatile float r = a * b;
    return r;
}

template <int J, class K>
static int indexer_fast_launch(float *out, double *qd, const float *w, int H, int n_pos, K keys, cudaStream_t st)
{
    const size_t smem = ((size_t)H * 16 * J + (size_t)IDXF_WARPS * 4 * H) * sizeof(double);
    auto kern = indexer_fast_kernel<J, K>;
    static SmemLimit lim;
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)kern, (int)smem));
    int blocks = device_sms();      // one CTA per SM (its registers fill the SM)
    const int need = (n_pos + IDXF_WARPS * 4 - 1) / (IDXF_WARPS * 4);
    if (blocks > need) blocks = need;
    kern<<<blocks, IDXF_WARPS * 32, smem, st>>>(out, qd, w, H, n_pos, indexer_scale(H, 16 * J), keys);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

template <class K>
static int indexer_launch(float *out, double *qd, const float *w, int H, int D, int n_pos, K keys,
                          cudaStream_t st)
{
    // Fast arrangement: whole 16-element chains, heads in groups of 16, q +
    // dot scratch within 200 KB of shared memory.
    if (H % 16 == 0 && ((size_t)H * D + (size_t)IDXF_WARPS * 4 * H) * sizeof(double) <= 200 * 1024) {
        if (D == 64) return indexer_fast_launch<4>(out, qd, w, H, n_pos, keys, st);
        if (D == 128) return indexer_fast_launch<8>(out, qd, w, H, n_pos, keys, st);
    }
    const size_t smem = (size_t)H * D * sizeof(double);
    if (smem > 200 * 1024)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "indexer: n_heads*head_dim too large");
    auto kern = indexer_score_kernel<K>;
    static SmemLimit lim;
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)kern, (int)smem));
    const int sms = device_sms();
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, IDX_WARPS * 32, smem);
    if (per_sm < 1) per_sm = 1;
    int blocks = sms * per_sm;
    const int need = (n_pos + IDX_WARPS - 1) / IDX_WARPS;
    if (blocks > need) blocks = need;
    kern<<<blocks, IDX_WARPS * 32, smem, st>>>(out, qd, w, H, D, n_pos, indexer_scale(H, D), keys);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

// The q staging buffer lives in a small per-thread cache so these calls need
// no context; it is sized for IDX_MAX_D * 512 heads.
static double *idx_qbuf(size_t n)
{
    static thread_local double *buf = nullptr;
    static thread_local size_t cap = 0;
    static thread_local int dev = -1;
    int cur = 0;
    cudaGetDevice(&cur);
    if (buf && (cap < n || dev != cur)) {
        cudaDeviceSynchronize();
        cudaFree(buf);
        buf = nullptr;
        cap = 0;
    }
    if (!buf) {
        if (cudaMalloc(&buf, n * sizeof(double)) != cudaSuccess) { buf = nullptr; return nullptr; }
        cap = n;
        dev = cur;
    }
    return buf;
}

static int idx_check(int H, int D, int n_pos)
{
    if (H <= 0 || D <= 0 || n_pos < 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "indexer: bad shape");
    if (D > IDX_MAX_D) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "indexer: head_dim %d > %d", D, IDX_MAX_D);
    return DSV4CU_OK;
}

extern "C" int dsv4cu_indexer_score(float *out, const float *q, const float *kv, const float *weights,
                                    int n_heads, int head_dim, int n_pos, void *stream)
{
    int r = idx_check(n_heads, head_dim, n_pos);
    if (r) return r;
    if (n_pos == 0) return DSV4CU_OK;
    double *qd = idx_qbuf((size_t)n_heads * head_dim);
    if (!qd) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "indexer: q buffer");
    cudaStream_t st = (cudaStream_t)stream;
    const int n = n_heads * head_dim;
    indexer_q_kernel<<<(n + 255) / 256, 256, 0, st>>>(qd, q, nullptr, nullptr, n_heads, head_dim);
    DSV4CU_LAUNCH_CHECK();
    KeysF32 k{kv, head_dim};
    return indexer_launch(out, qd, weights, n_heads, head_dim, n_pos, k, st);
}

extern "C" int dsv4cu_indexer_set_path(int path)
{
    if (path != DSV4CU_INDEXER_AUTO && path != DSV4CU_INDEXER_FP64)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "indexer_set_path: unknown path %d", path);
    g_idx_limbs = path == DSV4CU_INDEXER_AUTO;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_indexer_score_fp8(float *out, const uint8_t *q8, const float *q_scale, const uint8_t *k8,
                                        const float *k_scale, const float *weights, int n_heads, int head_dim,
                                        int n_pos, int k_stride, void *stream)
{
    int r = idx_check(n_heads, head_dim, n_pos);
    if (r) return r;
    if (k_stride < head_dim) return dsv4cu_set_error(DSV4CU_ERR_ARG, "indexer_fp8: k_stride < head_dim");
    if (n_pos == 0) return DSV4CU_OK;
    cudaStream_t st = (cudaStream_t)stream;
    KeysFP8 k{k8, k_scale, k_stride};
    // int8 tensor-core dots where the key rows allow 16-byte loads.
    if (n_heads == IDXM_H && head_dim == IDXM_D && k_stride % 16 == 0 && ((uintptr_t)k8 & 15u) == 0u &&
        g_idx_limbs)
        return indexer_limb_launch(out, q8, q_scale, weights, n_pos, k, st);
    double *qd = idx_qbuf((size_t)n_heads * head_dim);
    if (!qd) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "indexer: q buffer");
    const int n = n_heads * head_dim;
    indexer_q_kernel<<<(n + 255) / 256, 256, 0, st>>>(qd, nullptr, q8, q_scale, n_heads, head_dim);
    DSV4CU_LAUNCH_CHECK();
    if (n_heads == IDXM_H && head_dim == IDXM_D)
        return indexer_dmma_launch(out, qd, q_scale, weights, n_pos, k, st);
    return indexer_launch(out, qd, weights, n_heads, head_dim, n_pos, k, st);
}
