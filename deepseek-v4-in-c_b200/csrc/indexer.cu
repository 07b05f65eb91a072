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

struct KeysF32 {
    const float *kv;
    int ld;
    DSV4CU_DEV double load(int t, int i) const { return (double)__ldg(kv + (size_t)t * ld + i); }
};
struct KeysFP8 {
    const uint8_t *k8;
    const float *ks;
    int ld;
    DSV4CU_DEV double load(int t, int i) const
    {
        const float v = __fmul_rn(e4m3_to_f32(__ldg(k8 + (size_t)t * ld + i)), __ldg(ks + t));
        return (double)v;
    }
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

template <class K>
static int indexer_launch(float *out, double *qd, const float *w, int H, int D, int n_pos, K keys,
                          cudaStream_t st)
{
    const size_t smem = (size_t)H * D * sizeof(double);
    if (smem > 200 * 1024)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "indexer: n_heads*head_dim too large");
    auto kern = indexer_score_kernel<K>;
    DSV4CU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
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

extern "C" int dsv4cu_indexer_score_fp8(float *out, const uint8_t *q8, const float *q_scale, const uint8_t *k8,
                                        const float *k_scale, const float *weights, int n_heads, int head_dim,
                                        int n_pos, int k_stride, void *stream)
{
    int r = idx_check(n_heads, head_dim, n_pos);
    if (r) return r;
    if (k_stride < head_dim) return dsv4cu_set_error(DSV4CU_ERR_ARG, "indexer_fp8: k_stride < head_dim");
    if (n_pos == 0) return DSV4CU_OK;
    double *qd = idx_qbuf((size_t)n_heads * head_dim);
    if (!qd) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "indexer: q buffer");
    cudaStream_t st = (cudaStream_t)stream;
    const int n = n_heads * head_dim;
    indexer_q_kernel<<<(n + 255) / 256, 256, 0, st>>>(qd, nullptr, q8, q_scale, n_heads, head_dim);
    DSV4CU_LAUNCH_CHECK();
    KeysFP8 k{k8, k_scale, k_stride};
    return indexer_launch(out, qd, weights, n_heads, head_dim, n_pos, k, st);
}
