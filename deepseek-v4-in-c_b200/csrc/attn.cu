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

template <bool BF16>
__global__ void __launch_bounds__(ATT_THREADS) attn_chunk_kernel(
    const float *__restrict__ q, const void *__restrict__ kvp, const int *__restrict__ idxs, int H, int D,
    int topk, float scale, float *__restrict__ pm, float *__restrict__ pl, float *__restrict__ po)
{
    extern __shared__ float smem[];
    const int DP = D + 4;                      // padded row stride (floats)
    float *kvs = smem;                         // [CH][DP]
    float *qs = kvs + ATT_CH * DP;             // [HG][D]
    float *ss = qs + ATT_HG * D;               // [HG][CH] scores, then weights
    __shared__ int rows[ATT_CH];

    const int chunk = blockIdx.x, h0 = blockIdx.y * ATT_HG, tid = threadIdx.x;
    const int nh = min(ATT_HG, H - h0);
    if (tid < ATT_CH) {
        const int j = chunk * ATT_CH + tid;
        rows[tid] = (j < topk) ? idxs[j] : -1;
    }
    __syncthreads();
    // Gather rows (D % 4 == 0) and the head group's q.
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
    __syncthreads();

    // Scores: thread (hh, jj) -> rows jj and jj + 16 of head hh.
    {
        const int hh = tid >> 4, jj = tid & 15;
        if (hh < nh) {
            const float *qh = qs + hh * D, *k0 = kvs + jj * DP, *k1 = kvs + (jj + 16) * DP;
            float a0 = 0.f, a1 = 0.f;
            for (int c = 0; c < D; c += 4) {
                const float4 qv = *reinterpret_cast<const float4 *>(qh + c);
                const float4 v0 = *reinterpret_cast<const float4 *>(k0 + c);
                const float4 v1 = *reinterpret_cast<const float4 *>(k1 + c);
                a0 = fmaf(qv.x, v0.x, fmaf(qv.y, v0.y, fmaf(qv.z, v0.z, fmaf(qv.w, v0.w, a0))));
                a1 = fmaf(qv.x, v1.x, fmaf(qv.y, v1.y, fmaf(qv.z, v1.z, fmaf(qv.w, v1.w, a1))));
            }
            ss[hh * ATT_CH + jj] = a0 * scale;
            ss[hh * ATT_CH + jj + 16] = a1 * scale;
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
    // Unnormalised chunk output: thread -> head tid/16, columns 4*(tid%16) + 64*i.
    {
        const int hh = tid >> 4, cg = (tid & 15) * 4;
        if (hh < nh) {
            float *dst = po + ((size_t)chunk * H + h0 + hh) * D;
            for (int c = cg; c < D; c += 64) {
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
                for (int j = 0; j < ATT_CH; j++) {
                    const float w = ss[hh * ATT_CH + j];
                    const float4 v = *reinterpret_cast<const float4 *>(kvs + j * DP + c);
                    acc.x = fmaf(w, v.x, acc.x);
                    acc.y = fmaf(w, v.y, acc.y);
                    acc.z = fmaf(w, v.z, acc.z);
                    acc.w = fmaf(w, v.w, acc.w);
                }
                *reinterpret_cast<float4 *>(dst + c) = acc;
            }
        }
    }
}

__global__ void attn_combine_kernel(const float *__restrict__ pm, const float *__restrict__ pl,
                                    const float *__restrict__ po, const float *__restrict__ sink, int H, int D,
                                    int nchunks, float *__restrict__ o)
{
    const int h = blockIdx.x;
    float m = -INFINITY;
    for (int c = 0; c < nchunks; c++) m = fmaxf(m, pm[(size_t)c * H + h]);
    double denom = 0.0;
    for (int c = 0; c < nchunks; c++) {
        const float mc = pm[(size_t)c * H + h];
        if (mc != -INFINITY) denom += (double)pl[(size_t)c * H + h] * (double)expf(mc - m);
    }
    denom += (double)expf(sink[h] - m);
    const float inv = (float)(1.0 / denom);
    for (int col = threadIdx.x; col < D; col += blockDim.x) {
        float acc = 0.0f;
        for (int c = 0; c < nchunks; c++) {
            const float mc = pm[(size_t)c * H + h];
            if (mc == -INFINITY) continue;
            acc = fmaf(po[((size_t)c * H + h) * D + col], expf(mc - m), acc);
        }
        o[(size_t)h * D + col] = acc * inv;
    }
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
    const size_t smem = ((size_t)ATT_CH * (D + 4) + (size_t)ATT_HG * D + ATT_HG * ATT_CH) * sizeof(float);
    if (smem > 220 * 1024) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "sparse_attn: head dim %d too large", D);
    dim3 grid(nch, (H + ATT_HG - 1) / ATT_HG);
    if (kv_bf16) {
        DSV4CU_CUDA_TRY(cudaFuncSetAttribute(attn_chunk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attn_chunk_kernel<true><<<grid, ATT_THREADS, smem, st>>>(q, kv, idxs, H, D, topk, scale, pm, pl, po);
    } else {
        DSV4CU_CUDA_TRY(cudaFuncSetAttribute(attn_chunk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attn_chunk_kernel<false><<<grid, ATT_THREADS, smem, st>>>(q, kv, idxs, H, D, topk, scale, pm, pl, po);
    }
    DSV4CU_LAUNCH_CHECK();
    attn_combine_kernel<<<H, 256, 0, st>>>(pm, pl, po, sink, H, D, nch, o);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_sparse_attn(dsv4cu_ctx *ctx, float *o, const float *q, const void *kv, int kv_bf16,
                                  const float *sink, const int *idxs, int h, int d, int topk, float scale,
                                  void *stream)
{
    if (!ctx || !o || !q || !kv || !sink) return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn: NULL argument");
    if (h <= 0 || d <= 0 || topk < 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn: bad shape");
    if (d % 4) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "sparse_attn: head dim must be a multiple of 4");
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
