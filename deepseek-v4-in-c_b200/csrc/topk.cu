// topk.cu - top-k indices, descending, ties to the LOWER index.
//
// Reference: dsv4_topk (src/10_compute/dsv4_topk.c:76-112), whose definition is
// the scan topk_ref in tests/unit/test_indexer.c:20-34. Scores compare as
// floats, so -0.0 and +0.0 tie; k is clamped to n. The reference aborts above
// k = 1024 (dsv4_topk.c:80-84); these kernels have no such bound below
// TOPK_MAX_SORT.
//
// Small n (below TOPK_CL x 1024 keys), one CTA of 1024 threads:
//   1. key(i) = order-preserving uint32 of score i (larger score -> larger key),
//      staged in shared memory when the keys fit (n <= ~47K for k <= 2048).
//   2. Radix select, 3 passes of 11, 11 and 10 bits from the top: the k-th
//      largest key T and how many of the keys equal to T belong in the result
//      (need_eq); each pass finds its digit with one block scan.
//   3. Ordered compaction over i ascending (ballots per 32 indices): every
//      key > T, and the first need_eq indices whose key == T (the lower
//      indices win the tie).
//   4. Bitonic sort of (key, ~index) descending: score descending, then index
//      ascending - exactly the reference output order.
// Large n: the cluster select and the rank kernel further down.
#include <cooperative_groups.h>

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

// Bitonic sort of sel[0 .. sort_n) into descending order, all 1024 threads.
// For 64 <= sort_n <= 2048, warp w holds elements 64 w + l and 64 w + 32 + l
// in registers: stages of stride 32 compare a lane's pair, strides below 32
// exchange with lane l ^ stride, and only strides of 64 and more go through
// shared memory (15 barrier stages for 2048 instead of 66).
__device__ void bitonic_desc(unsigned long long *sel, int sort_n)
{
    const int tid = threadIdx.x;
    auto smem_stage = [&](int size, int stride) {
        for (int i = tid; i < (sort_n >> 1); i += blockDim.x) {
            const int lo = 2 * i - (i & (stride - 1));
            const int hi = lo + stride;
            const bool desc = ((lo & size) == 0);
            const unsigned long long a = sel[lo], b = sel[hi];
            if ((a < b) == desc) { sel[lo] = b; sel[hi] = a; }
        }
        __syncthreads();
    };
    if (sort_n < 64 || sort_n > 2048) {
        for (int size = 2; size <= sort_n; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) smem_stage(size, stride);
        return;
    }
    const int lane = tid & 31, warp = tid >> 5;
    const bool live = warp * 64 < sort_n;
    const int i0 = warp * 64 + lane, i1 = i0 + 32;
    unsigned long long v0 = 0ull, v1 = 0ull;
    if (live) {
        v0 = sel[i0];
        v1 = sel[i1];
    }
    for (int size = 2; size <= sort_n; size <<= 1) {
        int stride = size >> 1;
        if (stride >= 64) {
            if (live) {
                sel[i0] = v0;
                sel[i1] = v1;
            }
            __syncthreads();
            for (; stride >= 64; stride >>= 1) smem_stage(size, stride);
            if (live) {
                v0 = sel[i0];
                v1 = sel[i1];
            }
        }
        if (!live) continue;
        for (; stride > 0; stride >>= 1) {
            if (stride == 32) {
                const bool desc = (i0 & size) == 0;
                const unsigned long long hi = v0 > v1 ? v0 : v1, lo = v0 > v1 ? v1 : v0;
                v0 = desc ? hi : lo;
                v1 = desc ? lo : hi;
            } else {
                const bool lower = (lane & stride) == 0;
                const unsigned long long o0 = __shfl_xor_sync(0xFFFFFFFFu, v0, stride);
                const unsigned long long o1 = __shfl_xor_sync(0xFFFFFFFFu, v1, stride);
                const bool d0 = (i0 & size) == 0, d1 = (i1 & size) == 0;
                // the lower index of a descending pair keeps the larger value
                v0 = (lower == d0) ? (v0 > o0 ? v0 : o0) : (v0 < o0 ? v0 : o0);
                v1 = (lower == d1) ? (v1 > o1 ? v1 : o1) : (v1 < o1 ? v1 : o1);
            }
        }
    }
    if (live) {
        sel[i0] = v0;
        sel[i1] = v1;
    }
    __syncthreads();
}

// Radix digits, most significant first: 11 + 11 + 10 bits.
constexpr int TOPK_BINS = 2048;
__device__ __constant__ int topk_shift[3] = {21, 10, 0};
__device__ __constant__ int topk_width[3] = {11, 11, 10};

template <bool SMEM_KEYS>
__global__ void __launch_bounds__(TOPK_THREADS) topk_kernel(const float *__restrict__ scores, int n, int k,
                                                            int *__restrict__ out, int sort_n)
{
    __shared__ int hist[TOPK_BINS];
    __shared__ int sh_warp[32];
    __shared__ int warp_gt[32], warp_eq[32];
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_need;
    extern __shared__ unsigned long long sel[];   // [sort_n], then (SMEM_KEYS) keys [n]
    uint32_t *skeys = (uint32_t *)(sel + sort_n);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (SMEM_KEYS) {
        // Several independent loads in flight per thread.
        constexpr int U = 8;
        for (int b = 0; b < n; b += U * TOPK_THREADS) {
            float v[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = b + u * TOPK_THREADS + tid;
                v[u] = i < n ? __ldg(scores + i) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = b + u * TOPK_THREADS + tid;
                if (i < n) skeys[i] = float_order_key(v[u]);
            }
        }
    }
    auto key_at = [&](int i) -> uint32_t { return SMEM_KEYS ? skeys[i] : score_key(scores, i); };
    if (tid == 0) { s_prefix = 0u; s_mask = 0u; s_need = k; }

    // --- radix select: T = the k-th largest key, need = how many keys == T are taken
    for (int pass = 0; pass < 3; pass++) {
        const int shift = topk_shift[pass], width = topk_width[pass], nb = 1 << width;
        for (int i = tid; i < TOPK_BINS; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int i = tid; i < n; i += blockDim.x) {
            const uint32_t key = key_at(i);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & (nb - 1)], 1);
        }
        __syncthreads();
        // Digits in descending order, two per thread; the thread whose range
        // holds the need-th key (counting from the top) picks the digit.
        const int dA = nb - 1 - 2 * tid, dB = dA - 1;
        const int cA = dA >= 0 ? hist[dA] : 0, cB = dB >= 0 ? hist[dB] : 0;
        const int need = s_need;          // read before the scan's barriers; written after them
        int above;
        block_exscan(cA + cB, &above, sh_warp);
        if (above < need && need <= above + cA + cB) {
            const bool inA = need <= above + cA;
            const int d = inA ? dA : dB;
            s_need = need - above - (inA ? 0 : cA);
            s_prefix = prefix | ((uint32_t)d << shift);
            s_mask = mask | ((uint32_t)(nb - 1) << shift);
        }
        __syncthreads();
    }
    const uint32_t T = s_prefix;
    const int need_eq = s_need;

    // --- ordered compaction: warp w owns indices [w * span, (w + 1) * span),
    // walked 32 at a time; ballots keep index order inside the warp.
    const int nw = blockDim.x >> 5;
    const int span = ((n + nw - 1) / nw + 31) & ~31;
    const int w0 = min(n, warp * span), w1 = min(n, w0 + span);
    int cgt = 0, ceq = 0;
    for (int b = w0; b < w1; b += 32) {
        const int i = b + lane;
        const uint32_t key = i < w1 ? key_at(i) : 0u;
        cgt += __popc(__ballot_sync(0xFFFFFFFFu, i < w1 && key > T));
        ceq += __popc(__ballot_sync(0xFFFFFFFFu, i < w1 && key == T));
    }
    if (lane == 0) {
        warp_gt[warp] = cgt;
        warp_eq[warp] = ceq;
    }
    __syncthreads();
    if (warp == 0) {
        int g = lane < nw ? warp_gt[lane] : 0, e = lane < nw ? warp_eq[lane] : 0;
        int gi = g, ei = e;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xFFFFFFFFu, gi, o), c = __shfl_up_sync(0xFFFFFFFFu, ei, o);
            if (lane >= o) {
                gi += a;
                ei += c;
            }
        }
        if (lane < nw) {
            warp_gt[lane] = gi - g;   // exclusive
            warp_eq[lane] = ei - e;
        }
        if (lane == nw - 1) s_need = gi;   // keys > T in all
    }
    __syncthreads();
    const int ngt = s_need;
    int wgt = warp_gt[warp], weq = warp_eq[warp];
    const unsigned lt = (1u << lane) - 1u;
    for (int b = w0; b < w1; b += 32) {
        const int i = b + lane;
        const uint32_t key = i < w1 ? key_at(i) : 0u;
        const bool gt = i < w1 && key > T, eq = i < w1 && key == T;
        const unsigned mg = __ballot_sync(0xFFFFFFFFu, gt), me = __ballot_sync(0xFFFFFFFFu, eq);
        const unsigned long long v = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)i);
        if (gt) sel[wgt + __popc(mg & lt)] = v;
        if (eq) {
            const int r = weq + __popc(me & lt);
            if (r < need_eq) sel[ngt + r] = v;
        }
        wgt += __popc(mg);
        weq += __popc(me);
    }
    for (int i = k + tid; i < sort_n; i += blockDim.x) sel[i] = 0ull;   // padding sorts last
    __syncthreads();

    // --- bitonic sort, descending
    bitonic_desc(sel, sort_n);
    for (int i = tid; i < k; i += blockDim.x) out[i] = (int)(0xFFFFFFFFu - (uint32_t)(sel[i] & 0xFFFFFFFFull));
}


// Cluster form for large n (TOPK_CL CTAs, n up to TOPK_CL x ~50K keys), two
// launches:
//  select  CTA c of the cluster stages keys [c * span, (c + 1) * span) in its
//          shared memory. Radix select over 8-bit digits from the top: each
//          pass builds per-CTA histograms (the first one with one shared
//          atomic per distinct digit and warp), and after a cluster barrier every CTA sums the
//          TOPK_CL histograms through distributed shared memory and picks the
//          same digit (identical inputs, identical arithmetic). The passes
//          stop early once the digit's whole bucket is taken. Every key whose
//          selected prefix is above the threshold is picked, and of those
//          equal to it the first `need` in index order (the reference's tie
//          rule); the k picks (key, ~index) go to a workspace in any order.
//  rank    k / 32 CTAs: pick p's output position is the number of picks
//          whose (key, ~index) is larger - score descending, then index
//          ascending, exactly the reference order. Each CTA ranks 32 picks,
//          its 32 warps each counting over k / 32 of the others, so the
//          ordering runs on most of the GPU instead of on one cluster.
constexpr int TOPK_CL = 8;
constexpr int TOPK_RANK_PICKS = 32;
namespace cg = cooperative_groups;

DSV4CU_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
DSV4CU_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(TOPK_THREADS) topk_select_kernel(const float *__restrict__ scores, int n, int k,
                                                                   unsigned long long *__restrict__ picks, int span)
{
    __shared__ int hist[2][256];
    __shared__ int sh_warp[32];
    __shared__ int warp_gt[32], warp_eq[32];
    __shared__ int cta_cnt[2];                    // this CTA's keys above / equal to the threshold
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_need, s_done;
    extern __shared__ uint32_t skeys[];           // [span]
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g0 = min(n, rank * span), g1 = min(n, g0 + span), cnt = g1 - g0;

    constexpr int U = 8;
    for (int b = 0; b < cnt; b += U * TOPK_THREADS) {
        float v[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = b + u * TOPK_THREADS + tid;
            v[u] = i < cnt ? __ldg(scores + g0 + i) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = b + u * TOPK_THREADS + tid;
            if (i < cnt) skeys[i] = float_order_key(v[u]);
        }
    }
    if (tid == 0) { s_prefix = 0u; s_mask = 0u; s_need = k; s_done = 0; }

    for (int pass = 0; pass < 4; pass++) {
        const int shift = 24 - 8 * pass;
        int *hb = hist[pass & 1];
        if (tid < 256) hb[tid] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int b = 0; b < cnt; b += TOPK_THREADS) {
            const int i = b + tid;
            int bin = -1;
            if (i < cnt) {
                const uint32_t key = skeys[i];
                if ((key & mask) == prefix) bin = (int)((key >> shift) & 255u);
            }
            if (pass == 0) {                      // few distinct top digits: one atomic per digit and warp
                const unsigned grp = __match_any_sync(0xFFFFFFFFu, bin);
                if (bin >= 0 && lane == __ffs(grp) - 1) atomicAdd(&hb[bin], __popc(grp));
            } else if (bin >= 0) {                // inside one bucket the digits spread out
                atomicAdd(&hb[bin], 1);
            }
        }
        cluster.sync();                           // every CTA's histogram is complete
        // thread t < 256 holds digit 255 - t: the scan runs from the top digit down
        int cd = 0;
        if (tid < 256) {
            int rv[TOPK_CL];
#pragma unroll
            for (int r = 0; r < TOPK_CL; r++) rv[r] = cluster.map_shared_rank(hb, r)[255 - tid];
#pragma unroll
            for (int r = 0; r < TOPK_CL; r++) cd += rv[r];
        }
        const int need = s_need;                  // read before the scan's barriers; written after them
        int above;
        block_exscan(cd, &above, sh_warp);
        if (cd > 0 && above < need && need <= above + cd) {
            s_need = need - above;
            s_prefix = prefix | ((uint32_t)(255 - tid) << shift);
            s_mask = mask | (0xFFu << shift);
            s_done = need - above == cd;          // the whole bucket is taken
        }
        __syncthreads();
        if (s_done) break;                        // same decision in every CTA of the cluster
    }
    const uint32_t T = s_prefix, M = s_mask;
    const int need_eq = s_need;

    // counts of this CTA's slice, per warp in index order
    const int nw = blockDim.x >> 5;
    const int wspan = ((cnt + nw - 1) / nw + 31) & ~31;
    const int w0 = min(cnt, warp * wspan), w1 = min(cnt, w0 + wspan);
    int cgt = 0, ceq = 0;
    for (int b = w0; b < w1; b += 32) {
        const int i = b + lane;
        const uint32_t key = i < w1 ? (skeys[i] & M) : 0u;
        cgt += __popc(__ballot_sync(0xFFFFFFFFu, i < w1 && key > T));
        ceq += __popc(__ballot_sync(0xFFFFFFFFu, i < w1 && key == T));
    }
    if (lane == 0) {
        warp_gt[warp] = cgt;
        warp_eq[warp] = ceq;
    }
    __syncthreads();
    if (warp == 0) {
        int g = lane < nw ? warp_gt[lane] : 0, e = lane < nw ? warp_eq[lane] : 0;
        int gi = g, ei = e;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xFFFFFFFFu, gi, o), c = __shfl_up_sync(0xFFFFFFFFu, ei, o);
            if (lane >= o) {
                gi += a;
                ei += c;
            }
        }
        if (lane < nw) {
            warp_gt[lane] = gi - g;
            warp_eq[lane] = ei - e;
        }
        if (lane == nw - 1) {
            cta_cnt[0] = gi;
            cta_cnt[1] = ei;
        }
    }
    cluster.sync();                               // every CTA's counts are complete
    int gbase = 0, ebase = 0;
    {
        int rg[TOPK_CL], re[TOPK_CL];             // all remote loads in flight, then the sums
#pragma unroll
        for (int r = 0; r < TOPK_CL; r++) {
            const int *rc = cluster.map_shared_rank(cta_cnt, r);
            rg[r] = rc[0];
            re[r] = rc[1];
        }
#pragma unroll
        for (int r = 0; r < TOPK_CL; r++)
            if (r < rank) {
                gbase += rg[r];
                ebase += re[r];
            }
    }
    cluster_arrive();                             // remote reads done; the wait comes before exit
    // Picks above the threshold fill [0, k - need_eq) in index order; the
    // first need_eq equal ones fill [k - need_eq, k).
    int wgt = gbase + warp_gt[warp], weq = ebase + warp_eq[warp];
    const unsigned lt = (1u << lane) - 1u;
    for (int b = w0; b < w1; b += 32) {
        const int i = b + lane;
        const uint32_t full = i < w1 ? skeys[i] : 0u, key = full & M;
        const bool gt = i < w1 && key > T, eq = i < w1 && key == T;
        const unsigned mg = __ballot_sync(0xFFFFFFFFu, gt), me = __ballot_sync(0xFFFFFFFFu, eq);
        const unsigned long long v = ((unsigned long long)full << 32) | (0xFFFFFFFFu - (uint32_t)(g0 + i));
        if (gt) picks[wgt + __popc(mg & lt)] = v;
        if (eq) {
            const int r = weq + __popc(me & lt);
            if (r < need_eq) picks[k - need_eq + r] = v;
        }
        wgt += __popc(mg);
        weq += __popc(me);
    }
    pdl_trigger();
    cluster_wait();
}

__global__ void __launch_bounds__(TOPK_THREADS) topk_rank_kernel(const unsigned long long *__restrict__ picks, int k,
                                                                 int *__restrict__ out)
{
    extern __shared__ unsigned long long pv[];   // [k]
    __shared__ int part[32][33];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait();
    for (int i = tid; i < k; i += blockDim.x) pv[i] = picks[i];
    __syncthreads();
    const int p = blockIdx.x * TOPK_RANK_PICKS + lane;
    const unsigned long long v = p < k ? pv[p] : ~0ull;
    const int qs = (k + 31) / 32, q0 = min(k, warp * qs), q1 = min(k, q0 + qs);
    int c0 = 0, c1 = 0, c2 = 0, c3 = 0;
    int q = q0;
    for (; q + 4 <= q1; q += 4) {
        c0 += pv[q] > v;
        c1 += pv[q + 1] > v;
        c2 += pv[q + 2] > v;
        c3 += pv[q + 3] > v;
    }
    for (; q < q1; q++) c0 += pv[q] > v;
    part[warp][lane] = (c0 + c1) + (c2 + c3);
    __syncthreads();
    if (warp == 0 && p < k) {
        int r = 0;
#pragma unroll 8
        for (int w = 0; w < 32; w++) r += part[w][lane];
        out[r] = (int)(0xFFFFFFFFu - (uint32_t)(v & 0xFFFFFFFFull));
    }
}

// Shared memory above the static arrays: the sort buffer and, when they fit,
// the n keys.
constexpr size_t TOPK_DYN_SMEM = 200 * 1024;

int topk_run(dsv4cu_ctx *ctx, int *idx, const float *scores, int n, int k, cudaStream_t st)
{
    int sort_n = 1;
    while (sort_n < k) sort_n <<= 1;
    if (sort_n < 2) sort_n = 2;
    const size_t sort_b = (size_t)sort_n * sizeof(unsigned long long);
    // Cluster form when each CTA's slice fits in shared memory.
    const int span = ((n + TOPK_CL - 1) / TOPK_CL + 31) & ~31;
    if (ctx && n >= TOPK_CL * 1024 && (size_t)span * 4 <= TOPK_DYN_SMEM) {
        void *ws = nullptr;
        int r = dsv4cu_ws_get(ctx, (size_t)k * sizeof(unsigned long long), &ws);
        if (r) return r;
        unsigned long long *picks = (unsigned long long *)ws;
        const size_t smem = (size_t)span * 4;
        static SmemLimit lim_sel, lim_rank;
        DSV4CU_CUDA_TRY(smem_limit(lim_sel, (const void *)topk_select_kernel, (int)smem));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(TOPK_CL);
        cfg.blockDim = dim3(TOPK_THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = TOPK_CL;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        DSV4CU_CUDA_TRY(cudaLaunchKernelEx(&cfg, topk_select_kernel, scores, n, k, picks, span));
        const size_t rsmem = (size_t)k * sizeof(unsigned long long);
        DSV4CU_CUDA_TRY(smem_limit(lim_rank, (const void *)topk_rank_kernel, (int)rsmem));
        cudaLaunchConfig_t rc = {};
        rc.gridDim = dim3((k + TOPK_RANK_PICKS - 1) / TOPK_RANK_PICKS);
        rc.blockDim = dim3(TOPK_THREADS);
        rc.dynamicSmemBytes = rsmem;
        rc.stream = st;
        cudaLaunchAttribute ra[1];
        ra[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        ra[0].val.programmaticStreamSerializationAllowed = 1;
        rc.attrs = ra;
        rc.numAttrs = 1;
        DSV4CU_CUDA_TRY(cudaLaunchKernelEx(&rc, topk_rank_kernel, (const unsigned long long *)picks, k, idx));
        return DSV4CU_OK;
    }
    const bool in_smem = sort_b + (size_t)n * 4 <= TOPK_DYN_SMEM;
    const size_t smem = in_smem ? sort_b + (size_t)n * 4 : sort_b;
    auto kern = in_smem ? topk_kernel<true> : topk_kernel<false>;
    static SmemLimit lim_a, lim_b;
    DSV4CU_CUDA_TRY(smem_limit(in_smem ? lim_a : lim_b, (const void *)kern, (int)smem));
    kern<<<1, TOPK_THREADS, smem, st>>>(scores, n, k, idx, sort_n);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_topk(dsv4cu_ctx *ctx, int *idx, const float *scores, int n, int k, void *stream)
{
    if (k > n) k = n;
    if (k <= 0 || n <= 0) return DSV4CU_OK;
    if (!idx || !scores) return dsv4cu_set_error(DSV4CU_ERR_ARG, "topk: NULL argument");
    if (k > TOPK_MAX_SORT) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "topk: k=%d exceeds %d", k, TOPK_MAX_SORT);
    return topk_run(ctx, idx, scores, n, k, (cudaStream_t)stream);
}
