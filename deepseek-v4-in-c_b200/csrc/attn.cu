// attn.cu - sparse attention with sinks over index-gathered KV rows.
//
// Reference: dsv4_sparse_attn (src/10_compute/dsv4_attn.c:60-107). One KV head
// shared by all query heads; idxs[j] = -1 masks slot j; per head
//   s_j   = dot(q, kv[idxs[j]]) * scale         (valid slots only)
//   m     = max_j s_j                             (the sink is NOT in the max)
//   denom = sum_j exp(s_j - m) + exp(sink - m)    (the sink is ONLY here)
//   o     = sum_j exp(s_j - m) kv[idxs[j]] / denom
// A slot list with no valid entry gives o = 0, as in the reference.
//
// Split over the selected rows (flash-decoding): CTA (row chunk, head group)
// gathers its CH rows into shared memory once for HG heads and emits the
// chunk's max, exp-sum and unnormalised output; a second kernel rescales the
// chunks to the global max and applies the sink. fp32 arithmetic throughout;
// the reference accumulates the dot in double and the output in float, so the
// contract is a relative-error tolerance, not bit identity.
#include <math.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "ctx.h"

namespace dsv4cu {
namespace cg = cooperative_groups;

constexpr int ATT_CH = 32;    // selected rows per CTA
constexpr int ATT_HG = 16;    // heads per CTA
constexpr int ATT_THREADS = 256;

// VEC: D % 4 == 0 and q / kv aligned for 16-byte (f32) or 8-byte (bf16)
// loads. Otherwise rows are gathered element by element into shared rows of
// DA = D rounded up to 4 columns whose tail is zero, so the 4-column loops
// below add exact zeros there, and the output is stored element by element.
template <bool BF16, bool VEC>
__global__ void __launch_bounds__(ATT_THREADS) attn_chunk_kernel(
    const float *__restrict__ q, const void *__restrict__ kvp, const int *__restrict__ idxs, int H, int D,
    int topk, float scale, float *__restrict__ pm, float *__restrict__ pl, float *__restrict__ po)
{
    extern __shared__ float smem[];
    const int DA = VEC ? D : ((D + 3) & ~3);
    const int DP = DA + 8;                     // padded row stride (floats): rows 4 lanes apart miss each other's banks
    float *kvs = smem;                         // [CH][DP]
    float *qs = kvs + ATT_CH * DP;             // [HG][DA]
    float *ss = qs + ATT_HG * DA;              // [HG][CH] scores, then weights
    __shared__ int rows[ATT_CH];

    const int chunk = blockIdx.x, h0 = blockIdx.y * ATT_HG, tid = threadIdx.x;
    const int nh = min(ATT_HG, H - h0);
    if (tid < ATT_CH) {
        const int j = chunk * ATT_CH + tid;
        rows[tid] = (j < topk) ? idxs[j] : -1;
    }
    __syncthreads();
    // Gather rows and the head group's q.
    if constexpr (!VEC) {
        for (int i = tid; i < ATT_CH * DA; i += ATT_THREADS) {
            const int r = i / DA, c = i - r * DA, src = rows[r];
            float v = 0.0f;
            if (src >= 0 && c < D) {
                if constexpr (BF16)
                    v = __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short *>(kvp) +
                                                        (size_t)src * D + c) << 16);
                else
                    v = __ldg(reinterpret_cast<const float *>(kvp) + (size_t)src * D + c);
            }
            kvs[r * DP + c] = v;
        }
        for (int i = tid; i < nh * DA; i += ATT_THREADS) {
            const int hh = i / DA, c = i - hh * DA;
            qs[hh * DA + c] = (c < D) ? __ldg(q + (size_t)(h0 + hh) * D + c) : 0.0f;
        }
    }
    if constexpr (VEC) {
        const int d4 = D >> 2;
        for (int i = tid; i < ATT_CH * d4; i += ATT_THREADS) {
            const int r = i / d4, c = (i - r * d4) * 4, src = rows[r];
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (src >= 0) {
                if constexpr (BF16) {
                    const uint2 u = __ldg(reinterpret_cast<const uint2 *>(
                        reinterpret_cast<const uint16_t *>(kvp) + (size_t)src * D + c));
                    v = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                    __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
                } else {
                    v = __ldg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(kvp) + (size_t)src * D + c));
                }
            }
            *reinterpret_cast<float4 *>(kvs + r * DP + c) = v;
        }
        for (int i = tid; i < nh * d4; i += ATT_THREADS) {
            const int hh = i / d4, c = (i - hh * d4) * 4;
            *reinterpret_cast<float4 *>(qs + hh * D + c) =
                __ldg(reinterpret_cast<const float4 *>(q + (size_t)(h0 + hh) * D + c));
        }
    }
    __syncthreads();

    // Scores: warp w -> heads 2w, 2w + 1; lane -> rows rp, rp + 16 (rp = lane / 2)
    // over the 4-column groups of parity lane & 1; lane pairs add their halves.
    {
        const int hp = tid >> 5, lane = tid & 31, rp = lane >> 1, ds = lane & 1;
        const int ha = 2 * hp, hb = 2 * hp + 1;
        if (ha < nh) {
            const float *qa = qs + ha * DA, *qb = qs + (hb < nh ? hb : ha) * DA;
            const float *k0 = kvs + rp * DP, *k1 = kvs + (rp + 16) * DP;
            float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
            for (int c = 4 * ds; c < DA; c += 8) {
                const float4 x = *reinterpret_cast<const float4 *>(qa + c);
                const float4 y = *reinterpret_cast<const float4 *>(qb + c);
                const float4 v0 = *reinterpret_cast<const float4 *>(k0 + c);
                const float4 v1 = *reinterpret_cast<const float4 *>(k1 + c);
                a00 = fmaf(x.x, v0.x, fmaf(x.y, v0.y, fmaf(x.z, v0.z, fmaf(x.w, v0.w, a00))));
                a01 = fmaf(x.x, v1.x, fmaf(x.y, v1.y, fmaf(x.z, v1.z, fmaf(x.w, v1.w, a01))));
                a10 = fmaf(y.x, v0.x, fmaf(y.y, v0.y, fmaf(y.z, v0.z, fmaf(y.w, v0.w, a10))));
                a11 = fmaf(y.x, v1.x, fmaf(y.y, v1.y, fmaf(y.z, v1.z, fmaf(y.w, v1.w, a11))));
            }
            a00 += __shfl_xor_sync(0xFFFFFFFFu, a00, 1);
            a01 += __shfl_xor_sync(0xFFFFFFFFu, a01, 1);
            a10 += __shfl_xor_sync(0xFFFFFFFFu, a10, 1);
            a11 += __shfl_xor_sync(0xFFFFFFFFu, a11, 1);
            if (ds == 0) {
                ss[ha * ATT_CH + rp] = a00 * scale;
                ss[ha * ATT_CH + rp + 16] = a01 * scale;
                if (hb < nh) {
                    ss[hb * ATT_CH + rp] = a10 * scale;
                    ss[hb * ATT_CH + rp + 16] = a11 * scale;
                }
            }
        }
    }
    __syncthreads();
    // Chunk max / exp-sum per head: warp w handles heads w and w + 8, lane = row.
    {
        const int warp = tid >> 5, lane = tid & 31;
        for (int hh = warp; hh < nh; hh += ATT_THREADS / 32) {
            const bool valid = rows[lane] >= 0;
            const float s = valid ? ss[hh * ATT_CH + lane] : -INFINITY;
            float m = s;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
            const float e = (valid && m != -INFINITY) ? expf(s - m) : 0.0f;
            const float l = warp_sum(e);
            ss[hh * ATT_CH + lane] = e;
            if (lane == 0) {
                pm[(size_t)chunk * H + h0 + hh] = m;
                pl[(size_t)chunk * H + h0 + hh] = l;
            }
        }
    }
    __syncthreads();
    // Unnormalised chunk output: warp w -> heads 2w, 2w + 1; lane -> 4-column
    // groups lane, lane + 32, ...
    {
        const int hp = tid >> 5, lane = tid & 31;
        const int ha = 2 * hp, hb = 2 * hp + 1;
        if (ha < nh) {
            const float *wa = ss + ha * ATT_CH, *wb = ss + (hb < nh ? hb : ha) * ATT_CH;
            float *da = po + ((size_t)chunk * H + h0 + ha) * D, *db = po + ((size_t)chunk * H + h0 + hb) * D;
            for (int c = 4 * lane; c < DA; c += 128) {
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f), y = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
                for (int j = 0; j < ATT_CH; j++) {
                    const float u = wa[j], w = wb[j];
                    const float4 v = *reinterpret_cast<const float4 *>(kvs + j * DP + c);
                    x.x = fmaf(u, v.x, x.x);
                    x.y = fmaf(u, v.y, x.y);
                    x.z = fmaf(u, v.z, x.z);
                    x.w = fmaf(u, v.w, x.w);
                    y.x = fmaf(w, v.x, y.x);
                    y.y = fmaf(w, v.y, y.y);
                    y.z = fmaf(w, v.z, y.z);
                    y.w = fmaf(w, v.w, y.w);
                }
                if constexpr (VEC) {
                    *reinterpret_cast<float4 *>(da + c) = x;
                    if (hb < nh) *reinterpret_cast<float4 *>(db + c) = y;
                } else {
                    const int nk = D - c;        // >= 1
                    da[c] = x.x;
                    if (nk > 1) da[c + 1] = x.y;
                    if (nk > 2) da[c + 2] = x.z;
                    if (nk > 3) da[c + 3] = x.w;
                    if (hb < nh) {
                        db[c] = y.x;
                        if (nk > 1) db[c + 1] = y.y;
                        if (nk > 2) db[c + 2] = y.z;
                        if (nk > 3) db[c + 3] = y.w;
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------- tensor-core chunks
// bf16 KV, head_dim 512 or 576, n_heads % 16 == 0: the whole attention on the
// bf16 tensor cores (mma.sync m16n8k16, fp32 accumulation), one thread-block
// cluster of CL CTAs per group of 16 heads, 8 warps per CTA:
//   gather   CTA r of the cluster takes the 64-row sub-chunks r, r + CL, ...
//            of the selected rows; each is copied into shared memory with
//            cp.async (16-byte pieces), the next one while the current one is
//            used; masked or missing slots are zero rows.
//   scores   S[16 heads x 64 rows] = Q K^T split over k: warp w takes the
//            k steps w, w + 8, ... for all 64 rows, its slice of Q held in
//            registers as mma fragments for the whole kernel; the 8 partial
//            tiles are added in warp order through shared memory. Q is fp32:
//            it enters as three bf16 terms q = hi + mid + lo, which carry all
//            24 significand bits, and KV is bf16 already, so the products are
//            those of fp32 and only the fp32 accumulation rounds, as in the
//            fp32 kernel.
//   softmax  online over the CTA's sub-chunks, 16 threads per head: running
//            max and exp-sum, the running output rescaled by exp(m_old -
//            m_new); the weights P = exp(S - m) as three bf16 terms again.
//   output   O[16 x D] += P V, warp w taking columns [D/8 w, ..); V is the same
//            shared rows read transposed (ldmatrix.trans).
//   combine  every CTA stores its partial output columns and (max, exp-sum)
//            straight into the shared memory of the CTA that owns those
//            columns (CTA r owns [D/CL r, D/CL (r + 1))); after one cluster
//            barrier each CTA forms the global max, the denominator with the
//            sink (in double) and writes its columns - no remote loads, no
//            partials in global memory.
constexpr int ATM_ROWS = 64;
constexpr int ATM_HEADS = 16;
constexpr int ATM_THREADS = 256;
static int g_attn_mma = 1;        // 0: fp32 kernel always, 2: 8-CTA clusters (dsv4cu_sparse_attn_set_path)

DSV4CU_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

DSV4CU_DEV void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
DSV4CU_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
DSV4CU_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

DSV4CU_DEV void ldsm_x4(uint32_t (&r)[4], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
DSV4CU_DEV void ldsm_x2(uint32_t (&r)[2], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
DSV4CU_DEV void ldsm_x4_t(uint32_t (&r)[4], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
DSV4CU_DEV void ldsm_x2_t(uint32_t (&r)[2], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(smem_u32(p)));
}

// D[16x8] += A[16x16] B[16x8], bf16 inputs, fp32 accumulators.
DSV4CU_DEV void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Three bf16 terms of an fp32 value, x = t0 + t1 + t2: each term takes the
// next 8 significand bits of the remainder (the subtractions are exact).
constexpr int ATM_TERMS = 3;
DSV4CU_DEV void split3_bf16(float x, uint16_t (&t)[ATM_TERMS])
{
    float r = x;
#pragma unroll
    for (int i = 0; i < ATM_TERMS; i++) {
        const __nv_bfloat16 b = __float2bfloat16_rn(r);
        t[i] = __bfloat16_as_ushort(b);
        r -= __bfloat162float(b);
    }
}
// Term i of two values as one bf16x2 word.
DSV4CU_DEV void split3_bf16x2(float x, float y, uint32_t (&w)[ATM_TERMS])
{
    uint16_t a[ATM_TERMS], b[ATM_TERMS];
    split3_bf16(x, a);
    split3_bf16(y, b);
#pragma unroll
    for (int i = 0; i < ATM_TERMS; i++) w[i] = (uint32_t)a[i] | ((uint32_t)b[i] << 16);
}

template <int D, int CL>
__global__ void __launch_bounds__(ATM_THREADS, 1) attn_mma_kernel(
    const float *__restrict__ q, const uint16_t *__restrict__ kv, const int *__restrict__ idxs,
    const float *__restrict__ sink, int H, int topk, float scale, float *__restrict__ o)
{
    constexpr int KS = D + 8;                 // shared row stride in bf16 (odd multiple of 16 bytes)
    constexpr int PS = ATM_ROWS + 8;
    constexpr int NW = ATM_THREADS / 32;
    constexpr int KST = D / 16;               // k steps
    constexpr int KPW = (KST + NW - 1) / NW;  // k steps per warp (the last ones may be missing)
    constexpr int ON = D / 8 / NW;            // output n tiles per warp
    constexpr int P16 = D / 8;                // 16-byte pieces per row
    constexpr int OC = D / CL;                // output columns owned by each rank
    static_assert(D % 64 == 0 && ATM_ROWS == 64 && ON >= 1 && OC % 2 == 0, "shape");
    extern __shared__ __align__(16) uint16_t atm_sm[];
    uint16_t *kb = atm_sm;                                              // [2][ROWS][KS] row buffers
    float *spart = reinterpret_cast<float *>(kb + 2 * ATM_ROWS * KS);   // [NW][16][ROWS] partial scores
    uint16_t *pt = reinterpret_cast<uint16_t *>(spart);                // [TERMS][16][PS] weights (after the sum)
    float *stage = spart + NW * ATM_HEADS * ATM_ROWS;                   // [CL][16][OC] pushed partial outputs
    __shared__ int rows[2][ATM_ROWS];
    __shared__ float run_m[ATM_HEADS], run_l[ATM_HEADS], s_alpha[ATM_HEADS];
    __shared__ float st_m[CL][ATM_HEADS], st_l[CL][ATM_HEADS], fac[CL][ATM_HEADS], s_inv[ATM_HEADS];

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int h0 = blockIdx.y * ATM_HEADS, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, c = lane & 3;
    const int nsub = (topk + ATM_ROWS - 1) / ATM_ROWS;
    const int nmine = rank < nsub ? (nsub - 1 - rank) / CL + 1 : 0;

    auto load_rows = [&](int it) {            // row indices of sub-chunk `it` into rows[it & 1]
        if (tid < ATM_ROWS) {
            const int jj = (rank + CL * it) * ATM_ROWS + tid;
            rows[it & 1][tid] = jj < topk ? __ldg(idxs + jj) : -1;
        }
    };
    auto gather = [&](int it) {               // needs rows[it & 1] behind a barrier
        const int buf = it & 1;
        uint16_t *dstb = kb + buf * ATM_ROWS * KS;
        for (int i = tid; i < ATM_ROWS * P16; i += ATM_THREADS) {
            const int r = i / P16, p = i - r * P16, src = rows[buf][r];
            uint16_t *dst = dstb + r * KS + 8 * p;
            if (src >= 0)
                cp_async16(dst, kv + (size_t)src * D + 8 * p);
            else
                *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
        }
        cp_async_commit();
    };
    if (nmine > 0) load_rows(0);
    if (nmine > 1) load_rows(1);
    if (tid < ATM_HEADS) {
        run_m[tid] = -INFINITY;
        run_l[tid] = 0.0f;
    }
    __syncthreads();
    if (nmine > 0) gather(0);                 // the first rows arrive while Q is split
    // this warp's Q slice as A fragments, three bf16 terms: k step w + 8j,
    // registers (row g, k 2c), (row g + 8, k 2c), (row g, k 2c + 8), (row g + 8, k 2c + 8)
    uint32_t qa[KPW][ATM_TERMS][4];
    {
        float2 v[KPW][4];
#pragma unroll
        for (int j = 0; j < KPW; j++) {
            const int kk = warp + NW * j;
#pragma unroll
            for (int rr = 0; rr < 4; rr++) {
                const int hh = g + 8 * (rr & 1), col = 16 * kk + 2 * c + 8 * (rr >> 1);
                v[j][rr] = kk < KST ? __ldg(reinterpret_cast<const float2 *>(q + (size_t)(h0 + hh) * D + col))
                                    : make_float2(0.f, 0.f);
            }
        }
#pragma unroll
        for (int j = 0; j < KPW; j++)
#pragma unroll
            for (int rr = 0; rr < 4; rr++) {
                uint32_t w[ATM_TERMS];
                split3_bf16x2(v[j][rr].x, v[j][rr].y, w);
#pragma unroll
                for (int t = 0; t < ATM_TERMS; t++) qa[j][t][rr] = w[t];
            }
    }

    float oacc[ON][4];
#pragma unroll
    for (int n = 0; n < ON; n++) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.0f;
    const int arow = (lane & 7) + 8 * ((lane >> 3) & 1), acol = 8 * (lane >> 4);   // A (x4) / V (x4.trans)
    const int brow = (lane & 7) + 8 * (lane >> 4), bcol = 8 * ((lane >> 3) & 1);   // B (x4, two n tiles)
    const int c0 = warp * ON * 8;
    const int rh = tid >> 4, rr0 = (tid & 15) * 4;                                 // softmax: head, 4 rows

    for (int it = 0; it < nmine; it++) {
        const int buf = it & 1;
        const uint16_t *kbuf = kb + buf * ATM_ROWS * KS;
        if (it + 1 < nmine) {
            gather(it + 1);                   // into the buffer the previous sub-chunk used
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        // ---- partial scores over this warp's k steps, all 64 rows
        {
            float sacc[8][4];
#pragma unroll
            for (int n = 0; n < 8; n++) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.0f;
#pragma unroll
            for (int j = 0; j < KPW; j++) {
                const int kk = warp + NW * j;
                if (kk < KST) {
#pragma unroll
                    for (int np = 0; np < 4; np++) {
                        uint32_t b[4];
                        ldsm_x4(b, kbuf + (16 * np + brow) * KS + 16 * kk + bcol);
#pragma unroll
                        for (int t = ATM_TERMS - 1; t >= 0; t--) {
                            mma_bf16_16816(sacc[2 * np], qa[j][t], b[0], b[1]);
                            mma_bf16_16816(sacc[2 * np + 1], qa[j][t], b[2], b[3]);
                        }
                    }
                }
            }
            float *sw = spart + warp * ATM_HEADS * ATM_ROWS;
#pragma unroll
            for (int n = 0; n < 8; n++) {
                *reinterpret_cast<float2 *>(sw + g * ATM_ROWS + 8 * n + 2 * c) = make_float2(sacc[n][0], sacc[n][1]);
                *reinterpret_cast<float2 *>(sw + (g + 8) * ATM_ROWS + 8 * n + 2 * c) =
                    make_float2(sacc[n][2], sacc[n][3]);
            }
        }
        __syncthreads();
        // ---- scores (warp order), online softmax: thread -> head rh, rows rr0 .. rr0 + 3
        float sv[4];
        {
            float4 acc4 = *reinterpret_cast<const float4 *>(spart + rh * ATM_ROWS + rr0);
#pragma unroll
            for (int w = 1; w < NW; w++) {
                const float4 x = *reinterpret_cast<const float4 *>(spart + (w * ATM_HEADS + rh) * ATM_ROWS + rr0);
                acc4.x += x.x;
                acc4.y += x.y;
                acc4.z += x.z;
                acc4.w += x.w;
            }
            sv[0] = acc4.x;
            sv[1] = acc4.y;
            sv[2] = acc4.z;
            sv[3] = acc4.w;
        }
        float cm = -INFINITY;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            sv[i] = rows[buf][rr0 + i] >= 0 ? sv[i] * scale : -INFINITY;
            cm = fmaxf(cm, sv[i]);
        }
#pragma unroll
        for (int o2 = 1; o2 < 16; o2 <<= 1) cm = fmaxf(cm, __shfl_xor_sync(0xFFFFFFFFu, cm, o2));
        const float old = run_m[rh], nm = fmaxf(old, cm);
        const float alpha = old == -INFINITY ? 0.0f : expf(old - nm);
        float e[4], ls = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            e[i] = sv[i] != -INFINITY ? expf(sv[i] - nm) : 0.0f;
            ls += e[i];
        }
#pragma unroll
        for (int o2 = 1; o2 < 16; o2 <<= 1) ls += __shfl_xor_sync(0xFFFFFFFFu, ls, o2);
        if (it + 2 < nmine) load_rows(it + 2);   // rows[buf]'s masks are read
        __syncthreads();                      // partial scores and run_m read: the weights overwrite them
        if ((tid & 15) == 0) {
            run_m[rh] = nm;
            run_l[rh] = run_l[rh] * alpha + ls;
            s_alpha[rh] = alpha;
        }
        {
            uint32_t w0[ATM_TERMS], w1[ATM_TERMS];
            split3_bf16x2(e[0], e[1], w0);
            split3_bf16x2(e[2], e[3], w1);
#pragma unroll
            for (int t = 0; t < ATM_TERMS; t++)
                *reinterpret_cast<uint2 *>(pt + (t * ATM_HEADS + rh) * PS + rr0) = make_uint2(w0[t], w1[t]);
        }
        __syncthreads();
        // ---- output: rescale, then += P V over the 64 rows
        const float al0 = s_alpha[g], al1 = s_alpha[g + 8];
#pragma unroll
        for (int n = 0; n < ON; n++) {
            oacc[n][0] *= al0;
            oacc[n][1] *= al0;
            oacc[n][2] *= al1;
            oacc[n][3] *= al1;
        }
#pragma unroll
        for (int kk = 0; kk < ATM_ROWS / 16; kk++) {
            uint32_t a[ATM_TERMS][4];
#pragma unroll
            for (int t = 0; t < ATM_TERMS; t++) ldsm_x4(a[t], pt + (t * ATM_HEADS + arow) * PS + 16 * kk + acol);
#pragma unroll
            for (int n = 0; n + 1 < ON; n += 2) {
                uint32_t b[4];
                ldsm_x4_t(b, kbuf + (16 * kk + arow) * KS + c0 + 8 * n + acol);
#pragma unroll
                for (int t = ATM_TERMS - 1; t >= 0; t--) {
                    mma_bf16_16816(oacc[n], a[t], b[0], b[1]);
                    mma_bf16_16816(oacc[n + 1], a[t], b[2], b[3]);
                }
            }
            if (ON & 1) {
                uint32_t b[2];
                ldsm_x2_t(b, kbuf + (16 * kk + arow) * KS + c0 + 8 * (ON - 1));
#pragma unroll
                for (int t = ATM_TERMS - 1; t >= 0; t--) mma_bf16_16816(oacc[ON - 1], a[t], b[0], b[1]);
            }
        }
        __syncthreads();                      // this buffer and the weights are free again
    }

    // ---- combine: push the partial columns and statistics to their owners
#pragma unroll
    for (int n = 0; n < ON; n++) {
        const int col = c0 + 8 * n + 2 * c, d = col / OC, lc = col - d * OC;
        float *dst = cluster.map_shared_rank(stage, d) + (rank * ATM_HEADS + g) * OC + lc;
        *reinterpret_cast<float2 *>(dst) = make_float2(oacc[n][0], oacc[n][1]);
        *reinterpret_cast<float2 *>(dst + 8 * OC) = make_float2(oacc[n][2], oacc[n][3]);
    }
    if (tid < CL * ATM_HEADS) {
        const int d = tid / ATM_HEADS, hh = tid % ATM_HEADS;
        cluster.map_shared_rank(&st_m[0][0], d)[rank * ATM_HEADS + hh] = run_m[hh];
        cluster.map_shared_rank(&st_l[0][0], d)[rank * ATM_HEADS + hh] = run_l[hh];
    }
    cluster.sync();                           // every rank's pushes have landed
    // thread (head hh, rank r) for r < CL: the global max and the rank's factor
    // by shuffles over the CL lanes of a head, the denominator in double in a
    // fixed tree order
    static_assert(ATM_HEADS * CL <= ATM_THREADS && 32 % CL == 0, "combine layout");
    if (tid < ATM_HEADS * CL) {
        const int hh = tid / CL, r = tid % CL;
        const float mr = st_m[r][hh];
        float m = mr;
#pragma unroll
        for (int o2 = 1; o2 < CL; o2 <<= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o2));
        const float f = mr != -INFINITY ? expf(mr - m) : 0.0f;   // no valid row there: nothing
        fac[r][hh] = f;
        double dsum = (double)st_l[r][hh] * (double)f;
#pragma unroll
        for (int o2 = 1; o2 < CL; o2 <<= 1) dsum += __shfl_xor_sync(0xFFFFFFFFu, dsum, o2);
        if (r == 0)   // m = -inf (no valid row at all): the sink term is inf and o = 0
            s_inv[hh] = (float)(1.0 / (dsum + (double)expf(__ldg(sink + h0 + hh) - m)));
    }
    __syncthreads();
    for (int i = tid; i < ATM_HEADS * OC; i += ATM_THREADS) {
        const int hh = i / OC, lc = i - hh * OC;
        float acc = 0.0f;
#pragma unroll
        for (int r = 0; r < CL; r++) acc = fmaf(stage[(r * ATM_HEADS + hh) * OC + lc], fac[r][hh], acc);
        o[(size_t)(h0 + hh) * D + rank * OC + lc] = acc * s_inv[hh];
    }
}

// Block (h, column slice): the head's chunk factors f_c = exp(m_c - m) and the
// denominator are formed once in shared memory (denominator summed in chunk
// order, in double), then each thread combines its columns in chunk order.
constexpr int ATT_COMB_COLS = 128;
constexpr int ATT_MAX_CHUNKS = 1024;

__global__ void __launch_bounds__(ATT_COMB_COLS) attn_combine_kernel(
    const float *__restrict__ pm, const float *__restrict__ pl, const float *__restrict__ po,
    const float *__restrict__ sink, int H, int D, int nchunks, float *__restrict__ o)
{
    __shared__ float fac[ATT_MAX_CHUNKS], lsum[ATT_MAX_CHUNKS];
    __shared__ float s_m, s_inv;
    __shared__ float red[ATT_COMB_COLS / 32];
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float m = -INFINITY;
    for (int c = tid; c < nchunks; c += blockDim.x) {
        const float mc = pm[(size_t)c * H + h];
        fac[c] = mc;
        lsum[c] = pl[(size_t)c * H + h];
        m = fmaxf(m, mc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) mm = fmaxf(mm, red[w]);
        s_m = mm;
    }
    __syncthreads();
    m = s_m;
    // f_c = 0 marks a chunk without a valid row (its max is -inf).
    for (int c = tid; c < nchunks; c += blockDim.x) {
        const float mc = fac[c];
        fac[c] = (mc != -INFINITY) ? expf(mc - m) : 0.0f;
    }
    __syncthreads();
    // A chunk without a valid row has l = 0 and an all-zero output, so it
    // adds exactly nothing below.
    if (tid == 0) {
        double denom = 0.0;
        for (int c = 0; c < nchunks; c++) denom += (double)lsum[c] * (double)fac[c];
        denom += (double)expf(sink[h] - m);
        s_inv = (float)(1.0 / denom);
    }
    __syncthreads();
    const float inv = s_inv;
    const int col = blockIdx.y * ATT_COMB_COLS + tid;
    if (col >= D) return;
    float acc = 0.0f;
    const float *src = po + (size_t)h * D + col;
    const size_t cstride = (size_t)H * D;
    int c = 0;
    for (; c + 16 <= nchunks; c += 16) {       // 16 loads in flight, then the fma in chunk order
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; u++) v[u] = __ldg(src + (size_t)(c + u) * cstride);
#pragma unroll
        for (int u = 0; u < 16; u++) acc = fmaf(v[u], fac[c + u], acc);
    }
    for (; c < nchunks; c++) acc = fmaf(__ldg(src + (size_t)c * cstride), fac[c], acc);
    o[(size_t)h * D + col] = acc * inv;
}

// Cluster of 16 CTAs (one per SM: ~208 KB of shared memory each) where the
// device can co-schedule one per head group, else 8.
template <int D, int CL>
static int attn_mma_launch(float *o, const float *q, const void *kv, const float *sink, const int *idxs, int H,
                           int topk, float scale, cudaStream_t st, bool probe, int *fits)
{
    const size_t smem = (size_t)2 * ATM_ROWS * (D + 8) * 2 + (size_t)(ATM_THREADS / 32) * ATM_HEADS * ATM_ROWS * 4 +
                        (size_t)ATM_HEADS * D * 4;
    auto kern = attn_mma_kernel<D, CL>;
    static SmemLimit lim;
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)kern, (int)smem));
    if (CL > 8) DSV4CU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL, H / ATM_HEADS);
    cfg.blockDim = dim3(ATM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (probe) {
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, (const void *)kern, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        *fits = n;
        return DSV4CU_OK;
    }
    DSV4CU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, q, (const uint16_t *)kv, idxs, sink, H, topk, scale, o));
    return DSV4CU_OK;
}

template <int D>
static int attn_mma_run(float *o, const float *q, const void *kv, const float *sink, const int *idxs, int H,
                        int topk, float scale, cudaStream_t st)
{
    static int clusters16 = -1;   // how many 16-CTA clusters the device co-schedules
    if (clusters16 < 0) {
        int n = 0;
        int r = attn_mma_launch<D, 16>(o, q, kv, sink, idxs, H, topk, scale, st, true, &n);
        clusters16 = r ? 0 : n;
    }
    if (clusters16 >= H / ATM_HEADS && g_attn_mma != 2)
        return attn_mma_launch<D, 16>(o, q, kv, sink, idxs, H, topk, scale, st, false, nullptr);
    return attn_mma_launch<D, 8>(o, q, kv, sink, idxs, H, topk, scale, st, false, nullptr);
}

size_t attn_workspace(int H, int D, int topk)
{
    const size_t nch = (size_t)(topk + ATT_CH - 1) / ATT_CH;
    return dsv4cu_align256(nch * H * 4) * 2 + dsv4cu_align256(nch * H * (size_t)D * 4);
}

int attn_run(float *o, const float *q, const void *kv, int kv_bf16, const float *sink, const int *idxs, int H,
             int D, int topk, float scale, void *ws, cudaStream_t st)
{
    const int nch = (topk + ATT_CH - 1) / ATT_CH;
    char *p = (char *)ws;
    float *pm = (float *)p;
    p += dsv4cu_align256((size_t)nch * H * 4);
    float *pl = (float *)p;
    p += dsv4cu_align256((size_t)nch * H * 4);
    float *po = (float *)p;
    // One cluster per 16 heads on the tensor cores for the bf16 cache at the
    // model's head widths.
    if (kv_bf16 && (D == 576 || D == 512) && H % ATM_HEADS == 0 && ((uintptr_t)q & 15) == 0 &&
        ((uintptr_t)kv & 15) == 0 && g_attn_mma)
        return D == 576 ? attn_mma_run<576>(o, q, kv, sink, idxs, H, topk, scale, st)
                        : attn_mma_run<512>(o, q, kv, sink, idxs, H, topk, scale, st);
    const bool vec = D % 4 == 0 && ((uintptr_t)q & 15) == 0 && ((uintptr_t)kv & (kv_bf16 ? 7 : 15)) == 0;
    const size_t DA = (size_t)((D + 3) & ~3);
    const size_t smem = ((size_t)ATT_CH * (DA + 8) + (size_t)ATT_HG * DA + ATT_HG * ATT_CH) * sizeof(float);
    if (smem > 220 * 1024) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "sparse_attn: head dim %d too large", D);
    if (nch > ATT_MAX_CHUNKS)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "sparse_attn: topk %d > %d", topk, ATT_MAX_CHUNKS * ATT_CH);
    dim3 grid(nch, (H + ATT_HG - 1) / ATT_HG);
    static SmemLimit lim[4];
    void (*kern)(const float *, const void *, const int *, int, int, int, float, float *, float *, float *) =
        kv_bf16 ? (vec ? attn_chunk_kernel<true, true> : attn_chunk_kernel<true, false>)
                : (vec ? attn_chunk_kernel<false, true> : attn_chunk_kernel<false, false>);
    DSV4CU_CUDA_TRY(smem_limit(lim[(kv_bf16 ? 2 : 0) + (vec ? 1 : 0)], (const void *)kern, (int)smem));
    kern<<<grid, ATT_THREADS, smem, st>>>(q, kv, idxs, H, D, topk, scale, pm, pl, po);
    DSV4CU_LAUNCH_CHECK();
    attn_combine_kernel<<<dim3(H, (D + ATT_COMB_COLS - 1) / ATT_COMB_COLS), ATT_COMB_COLS, 0, st>>>(
        pm, pl, po, sink, H, D, nch, o);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_sparse_attn_set_path(int path)
{
    if (path != DSV4CU_ATTN_AUTO && path != DSV4CU_ATTN_FP32 && path != DSV4CU_ATTN_CLUSTER8)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn_set_path: unknown path %d", path);
    g_attn_mma = path == DSV4CU_ATTN_AUTO ? 1 : path == DSV4CU_ATTN_CLUSTER8 ? 2 : 0;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_sparse_attn(dsv4cu_ctx *ctx, float *o, const float *q, const void *kv, int kv_bf16,
                                  const float *sink, const int *idxs, int h, int d, int topk, float scale,
                                  void *stream)
{
    if (!ctx || !o || !q || !kv || !sink) return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn: NULL argument");
    if (h <= 0 || d <= 0 || topk < 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn: bad shape");
    cudaStream_t st = (cudaStream_t)stream;
    if (topk == 0) {
        // No slot at all: the reference output is zero (denominator = sink only).
        DSV4CU_CUDA_TRY(cudaMemsetAsync(o, 0, (size_t)h * d * sizeof(float), st));
        return DSV4CU_OK;
    }
    if (!idxs) return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn: NULL idxs");
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, attn_workspace(h, d, topk), &ws);
    if (r) return r;
    return attn_run(o, q, kv, kv_bf16, sink, idxs, h, d, topk, scale, ws, st);
}
