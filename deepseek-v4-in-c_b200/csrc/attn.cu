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

#include "common.cuh"
#include "ctx.h"

namespace dsv4cu {

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
// bf16 KV, head_dim % 64 == 0, n_heads % 16 == 0: the same chunk outputs from
// the bf16 tensor cores (mma.sync m16n8k16, fp32 accumulation). CTA (chunk of
// ATM_ROWS selected rows, 16 heads), 8 warps:
//   gather   the chunk's KV rows into shared memory with cp.async (16-byte
//            pieces, three commit groups over the columns so the score loop
//            starts on the first third while the rest arrives); masked or
//            missing slots are zero rows.
//   scores   S[16 heads x ROWS] = Q K^T, warp w taking rows [ROWS/8 w, ..).
//            Q is fp32: it enters as three bf16 terms q = hi + mid + lo, which
//            carry all 24 significand bits, and KV is bf16 already, so the
//            products are those of fp32 and only the fp32 accumulation
//            rounds, as in the fp32 kernel.
//   softmax  chunk max and exp-sum per head (warp partials through shared
//            memory); P = exp(S - m) as three bf16 terms again.
//   output   O[16 x D] = P V, warp w taking columns [D/8 w, ..); V is the same
//            shared rows read transposed (ldmatrix.trans).
constexpr int ATM_ROWS = 64;
static int g_attn_mma = 1;        // 0: the fp32 chunk kernel for every shape (dsv4cu_sparse_attn_set_path)
constexpr int ATM_HEADS = 16;
constexpr int ATM_THREADS = 256;

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

template <int D>
__global__ void __launch_bounds__(ATM_THREADS, 1) attn_mma_kernel(
    const float *__restrict__ q, const uint16_t *__restrict__ kv, const int *__restrict__ idxs, int H, int topk,
    float scale, float *__restrict__ pm, float *__restrict__ pl, float *__restrict__ po)
{
    constexpr int KS = D + 8;                 // shared row stride in bf16 (odd multiple of 16 bytes)
    constexpr int PS = ATM_ROWS + 8;
    constexpr int NW = ATM_THREADS / 32;
    constexpr int SN = ATM_ROWS / 8 / NW;     // score n tiles per warp
    constexpr int ON = D / 8 / NW;            // output n tiles per warp
    static_assert(D % 64 == 0 && SN >= 1 && ON >= 1, "shape");
    extern __shared__ __align__(16) uint16_t atm_sm[];
    uint16_t *ks = atm_sm;                            // [ROWS][KS]
    uint16_t *qt = ks + ATM_ROWS * KS;                // [TERMS][16][KS]
    uint16_t *pt = qt + ATM_TERMS * ATM_HEADS * KS;   // [TERMS][16][PS]
    __shared__ int rows[ATM_ROWS];
    __shared__ float red[NW][ATM_HEADS];
    __shared__ float s_m[ATM_HEADS];

    const int chunk = blockIdx.x, h0 = blockIdx.y * ATM_HEADS, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, c = lane & 3;
    if (tid < ATM_ROWS) {
        const int j = chunk * ATM_ROWS + tid;
        rows[tid] = j < topk ? __ldg(idxs + j) : -1;
    }
    __syncthreads();
    // gather: three column groups, each one commit group
    constexpr int P16 = D / 8;                // 16-byte pieces per row
#pragma unroll
    for (int grp = 0; grp < 3; grp++) {
        const int p0 = grp * P16 / 3, p1 = (grp + 1) * P16 / 3, np = p1 - p0;
        for (int i = tid; i < ATM_ROWS * np; i += ATM_THREADS) {
            const int r = i / np, p = p0 + (i - r * np), src = rows[r];
            uint16_t *dst = ks + r * KS + 8 * p;
            if (src >= 0)
                cp_async16(dst, kv + (size_t)src * D + 8 * p);
            else
                *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
        }
        cp_async_commit();
    }
    // q (fp32) -> three bf16 terms
    for (int i = tid; i < ATM_HEADS * D / 2; i += ATM_THREADS) {
        const int hh = i / (D / 2), cc = 2 * (i - hh * (D / 2));
        const float2 v = __ldg(reinterpret_cast<const float2 *>(q + (size_t)(h0 + hh) * D + cc));
        uint32_t w[ATM_TERMS];
        split3_bf16x2(v.x, v.y, w);
#pragma unroll
        for (int t = 0; t < ATM_TERMS; t++)
            *reinterpret_cast<uint32_t *>(qt + (t * ATM_HEADS + hh) * KS + cc) = w[t];
    }

    // ---- scores
    float sacc[SN][4];
#pragma unroll
    for (int n = 0; n < SN; n++) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.0f;
    const int arow = (lane & 7) + 8 * ((lane >> 3) & 1), acol = 8 * (lane >> 4);   // A (x4) lane address
    const int brow = lane & 7, bcol = 8 * ((lane >> 3) & 1);                       // B (x2) lane address
    const int r0 = warp * SN * 8;
    auto score_steps = [&](int k0, int k1) {
        for (int kk = k0; kk < k1; kk++) {
            uint32_t a[ATM_TERMS][4];
#pragma unroll
            for (int t = 0; t < ATM_TERMS; t++) ldsm_x4(a[t], qt + (t * ATM_HEADS + arow) * KS + 16 * kk + acol);
#pragma unroll
            for (int n = 0; n < SN; n++) {
                uint32_t b[2];
                ldsm_x2(b, ks + (r0 + 8 * n + brow) * KS + 16 * kk + bcol);
#pragma unroll
                for (int t = ATM_TERMS - 1; t >= 0; t--) mma_bf16_16816(sacc[n], a[t], b[0], b[1]);
            }
        }
    };
    // k steps whose 16 columns lie inside the groups that have arrived
    constexpr int KST = D / 16;
    cp_async_wait<2>();
    __syncthreads();
    score_steps(0, (P16 / 3) / 2);
    cp_async_wait<1>();
    __syncthreads();
    score_steps((P16 / 3) / 2, (2 * P16 / 3) / 2);
    cp_async_wait<0>();
    __syncthreads();
    score_steps((2 * P16 / 3) / 2, KST);

    // ---- softmax over the chunk: lane holds heads g, g + 8 x rows r0 + 8n + 2c + {0, 1}
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < SN; n++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = r0 + 8 * n + 2 * c + (i & 1);
            const float s = rows[r] >= 0 ? sacc[n][i] * scale : -INFINITY;
            sacc[n][i] = s;
            mx[i >> 1] = fmaxf(mx[i >> 1], s);
        }
#pragma unroll
    for (int j = 0; j < 2; j++) {
        mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xFFFFFFFFu, mx[j], 1));
        mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xFFFFFFFFu, mx[j], 2));
    }
    if (c == 0) {
        red[warp][g] = mx[0];
        red[warp][g + 8] = mx[1];
    }
    __syncthreads();
    if (tid < ATM_HEADS) {
        float m = red[0][tid];
#pragma unroll
        for (int w = 1; w < NW; w++) m = fmaxf(m, red[w][tid]);
        s_m[tid] = m;
    }
    __syncthreads();
    const float m0 = s_m[g], m1 = s_m[g + 8];
    float sum[2] = {0.0f, 0.0f};
#pragma unroll
    for (int n = 0; n < SN; n++) {
        float e[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float m = (i >> 1) ? m1 : m0;
            e[i] = (sacc[n][i] != -INFINITY) ? expf(sacc[n][i] - m) : 0.0f;
            sum[i >> 1] += e[i];
        }
        const int col = r0 + 8 * n + 2 * c;
        uint32_t w0[ATM_TERMS], w1[ATM_TERMS];
        split3_bf16x2(e[0], e[1], w0);
        split3_bf16x2(e[2], e[3], w1);
#pragma unroll
        for (int t = 0; t < ATM_TERMS; t++) {
            *reinterpret_cast<uint32_t *>(pt + (t * ATM_HEADS + g) * PS + col) = w0[t];
            *reinterpret_cast<uint32_t *>(pt + (t * ATM_HEADS + g + 8) * PS + col) = w1[t];
        }
    }
#pragma unroll
    for (int j = 0; j < 2; j++) {
        sum[j] += __shfl_xor_sync(0xFFFFFFFFu, sum[j], 1);
        sum[j] += __shfl_xor_sync(0xFFFFFFFFu, sum[j], 2);
    }
    if (c == 0) {
        red[warp][g] = sum[0];
        red[warp][g + 8] = sum[1];
    }
    __syncthreads();
    if (tid < ATM_HEADS) {
        float l = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) l += red[w][tid];
        pm[(size_t)chunk * H + h0 + tid] = s_m[tid];
        pl[(size_t)chunk * H + h0 + tid] = l;
    }

    // ---- output: warp w -> columns [8 ON w, 8 ON (w + 1))
    float oacc[ON][4];
#pragma unroll
    for (int n = 0; n < ON; n++) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.0f;
    const int c0 = warp * ON * 8;
    const int vrow = (lane & 7) + 8 * ((lane >> 3) & 1), vcol = 8 * (lane >> 4);   // V (x4.trans) lane address
#pragma unroll
    for (int kk = 0; kk < ATM_ROWS / 16; kk++) {
        uint32_t a[ATM_TERMS][4];
#pragma unroll
        for (int t = 0; t < ATM_TERMS; t++) ldsm_x4(a[t], pt + (t * ATM_HEADS + arow) * PS + 16 * kk + acol);
#pragma unroll
        for (int n = 0; n + 1 < ON; n += 2) {
            uint32_t b[4];
            ldsm_x4_t(b, ks + (16 * kk + vrow) * KS + c0 + 8 * n + vcol);
#pragma unroll
            for (int t = ATM_TERMS - 1; t >= 0; t--) {
                mma_bf16_16816(oacc[n], a[t], b[0], b[1]);
                mma_bf16_16816(oacc[n + 1], a[t], b[2], b[3]);
            }
        }
        if (ON & 1) {
            uint32_t b[2];
            ldsm_x2_t(b, ks + (16 * kk + vrow) * KS + c0 + 8 * (ON - 1));
#pragma unroll
            for (int t = ATM_TERMS - 1; t >= 0; t--) mma_bf16_16816(oacc[ON - 1], a[t], b[0], b[1]);
        }
    }
#pragma unroll
    for (int n = 0; n < ON; n++) {
        const int col = c0 + 8 * n + 2 * c;
        *reinterpret_cast<float2 *>(po + ((size_t)chunk * H + h0 + g) * D + col) = make_float2(oacc[n][0], oacc[n][1]);
        *reinterpret_cast<float2 *>(po + ((size_t)chunk * H + h0 + g + 8) * D + col) =
            make_float2(oacc[n][2], oacc[n][3]);
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
    // Tensor-core chunks for the bf16 cache at the model's head widths.
    if (kv_bf16 && (D == 576 || D == 512) && H % ATM_HEADS == 0 && ((uintptr_t)q & 15) == 0 &&
        ((uintptr_t)kv & 15) == 0 && g_attn_mma) {
        const int nc = (topk + ATM_ROWS - 1) / ATM_ROWS;
        const size_t smem =
            ((size_t)ATM_ROWS * (D + 8) + (size_t)ATM_TERMS * ATM_HEADS * (D + 8 + ATM_ROWS + 8)) * 2;
        auto kern = D == 576 ? attn_mma_kernel<576> : attn_mma_kernel<512>;
        static SmemLimit lim_m[2];
        DSV4CU_CUDA_TRY(smem_limit(lim_m[D == 576], (const void *)kern, (int)smem));
        kern<<<dim3(nc, H / ATM_HEADS), ATM_THREADS, smem, st>>>(q, (const uint16_t *)kv, idxs, H, topk, scale, pm,
                                                                   pl, po);
        DSV4CU_LAUNCH_CHECK();
        attn_combine_kernel<<<dim3(H, (D + ATT_COMB_COLS - 1) / ATT_COMB_COLS), ATT_COMB_COLS, 0, st>>>(
            pm, pl, po, sink, H, D, nc, o);
        DSV4CU_LAUNCH_CHECK();
        return DSV4CU_OK;
    }
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
    if (path != DSV4CU_ATTN_AUTO && path != DSV4CU_ATTN_FP32)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn_set_path: unknown path %d", path);
    g_attn_mma = path == DSV4CU_ATTN_AUTO;
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
