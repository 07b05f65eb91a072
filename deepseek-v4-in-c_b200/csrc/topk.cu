// topk.cu - top-k indices, descending, ties to the LOWER index.
//
// Reference: dsv4_topk (src/10_compute/dsv4_topk.c:76-112), whose definition is
// the scan topk_ref in tests/unit/test_indexer.c:20-34. Scores compare as
// floats, so -0.0 and +0.0 tie; k is clamped to n. The reference aborts above
// k = 1024 (dsv4_topk.c:80-84); this kernel has no such bound below its
// shared-memory sort limit (TOPK_MAX_SORT).
//
// One CTA of 1024 threads:
//   1. key(i) = order-preserving uint32 of score i (larger score -> larger key).
//   2. Radix select, 4 passes of 8 bits from the top: the k-th largest key T
//      and how many of the keys equal to T belong in the result (need_eq).
//   3. Ordered compaction over i ascending: every key > T, and the first need_eq
//      indices whose key == T (the lower indices win the tie).
//   4. Bitonic sort of (key, ~index) descending: score descending, then index
//      ascending - exactly the reference output order.
#include "common.cuh"
#include "ctx.h"

namespace dsv4cu {

constexpr int TOPK_THREADS = 1024;
constexpr int TOPK_MAX_SORT = 8192;

__device__ __forceinline__ uint32_t score_key(const float *s, int i) { return float_order_key(__ldg(s + i)); }

// Block-wide exclusive scan of one int per thread; returns the total.
__device__ int block_exscan(int v, int *out_prefix, int *sh_warp)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < (int)(blockDim.x >> 5) ? sh_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        sh_warp[lane] = w;   // inclusive warp totals
    }
    __syncthreads();
    const int total = sh_warp[(blockDim.x >> 5) - 1];
    *out_prefix = x - v + (warp ? sh_warp[warp - 1] : 0);
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(TOPK_THREADS) topk_kernel(const float *__restrict__ scores, int n, int k,
                                                            int *__restrict__ out, int sort_n)
{
    __shared__ int hist[256];
    __shared__ int sh_warp[32];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_need;
    extern __shared__ unsigned long long sel[];   // [sort_n]

    const int tid = threadIdx.x;
    if (tid == 0) { s_prefix = 0u; s_mask = 0u; s_need = k; }
    __syncthreads();

    // --- radix select: find T, the k-th largest key, 8 bits at a time
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int i = tid; i < n; i += blockDim.x) {
            const uint32_t key = score_key(scores, i);
            const bool act = (key & mask) == prefix;
            const unsigned d = (key >> shift) & 255u;
            // Warp-aggregated histogram update: scores cluster in a few top
            // digits, and per-lane shared atomics on one bin would serialise.
            const unsigned am = __activemask();
            const unsigned peers = __match_any_sync(am, act ? d : 256u + (threadIdx.x & 31));
            if (act && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[d], __popc(peers));
        }
        __syncthreads();
        if (tid == 0) {
            int need = s_need, d = 255;
            for (; d > 0; d--) {
                if (hist[d] >= need) break;
                need -= hist[d];
            }
            s_need = need;   // keys with this digit still needed
            s_prefix = prefix | ((uint32_t)d << shift);
            s_mask = mask | (255u << shift);
        }
        __syncthreads();
    }
    const uint32_t T = s_prefix;
    const int need_eq = s_need;          // how many keys == T are taken

    // --- ordered compaction: thread tid owns a contiguous index range
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
    int cgt = 0, ceq = 0;
    for (int i = i0; i < i1; i++) {
        const uint32_t key = score_key(scores, i);
        cgt += key > T;
        ceq += key == T;
    }
    int pgt, peq;
    const int ngt = block_exscan(cgt, &pgt, sh_warp);
    block_exscan(ceq, &peq, sh_warp);
    int wgt = pgt, weq = peq;
    for (int i = i0; i < i1; i++) {
        const uint32_t key = score_key(scores, i);
        const unsigned long long v = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)i);
        if (key > T) sel[wgt++] = v;
        else if (key == T) {
            if (weq < need_eq) sel[ngt + weq] = v;
            weq++;
        }
    }
    for (int i = k + tid; i < sort_n; i += blockDim.x) sel[i] = 0ull;   // padding sorts last
    __syncthreads();

    // --- bitonic sort, descending
    for (int size = 2; size <= sort_n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < (sort_n >> 1); i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const unsigned long long a = sel[lo], b = sel[hi];
                if ((a < b) == desc) { sel[lo] = b; sel[hi] = a; }
            }
            __syncthreads();
        }
    }
    for (int i = tid; i < k; i += blockDim.x) out[i] = (int)(0xFFFFFFFFu - (uint32_t)(sel[i] & 0xFFFFFFFFull));
}

int topk_run(int *idx, const float *scores, int n, int k, cudaStream_t st)
{
    int sort_n = 1;
    while (sort_n < k) sort_n <<= 1;
    if (sort_n < 2) sort_n = 2;
    const size_t smem = (size_t)sort_n * sizeof(unsigned long long);
    DSV4CU_CUDA_TRY(cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    topk_kernel<<<1, TOPK_THREADS, smem, st>>>(scores, n, k, idx, sort_n);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_topk(dsv4cu_ctx *ctx, int *idx, const float *scores, int n, int k, void *stream)
{
    (void)ctx;
    if (k > n) k = n;
    if (k <= 0 || n <= 0) return DSV4CU_OK;
    if (!idx || !scores) return dsv4cu_set_error(DSV4CU_ERR_ARG, "topk: NULL argument");
    if (k > TOPK_MAX_SORT) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "topk: k=%d exceeds %d", k, TOPK_MAX_SORT);
    return topk_run(idx, scores, n, k, (cudaStream_t)stream);
}
