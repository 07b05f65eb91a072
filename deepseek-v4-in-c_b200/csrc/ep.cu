// ep.cu - device side of the expert-parallel MoE layer.
//
// Experts e live on rank e / epr (epr = n_experts / n_ranks experts per rank).
// A rank routes its own tokens (dsv4cu_route), then:
//   pack    : every (token t, slot k) pair becomes one send row, grouped by
//             the owning rank and, inside a rank, ordered by p = t * topk + k;
//             the row holds x[t] followed by the owner-local expert id (as a
//             float) and padding to hidden + 4 floats (16-byte rows).
//   (host)  : counts all-to-all, then the rows all-to-all (NCCL).
//   tail    : the received rows get the rank's own tokens appended with the
//             shared-expert id, and the ids are unpacked to int.
//   (dsv4cu_moe_rows computes every row's expert output on the tensor cores.)
//   (host)  : the rows go back with the reverse all-to-all.
//   combine : out[t] = sum over k IN ORDER of w[t][k] * y(t, k), then + the
//             shared expert's y[t] - the reference's per-token order
//             (src/70_decode/dsv4_layer.c:109-116) and the same float
//             operations as the single-device layer, so the result is the
//             same bits on any number of ranks.
#include "common.cuh"
#include "ctx.h"

namespace dsv4cu {

constexpr int EP_MAX_RANKS = 16;
constexpr int EP_PLAN_THREADS = 1024;
constexpr int EP_ERR_EXPERT = 31;    // status: an expert id outside 0 .. epr * n_ranks - 1

// Block-wide exclusive scan of one int per thread (1024 threads); returns the total.
DSV4CU_DEV int ep_block_exscan(int v, int *prefix, int *sh)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = sh[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        sh[lane] = w;
    }
    __syncthreads();
    const int total = sh[31];
    *prefix = x - v + (warp ? sh[warp - 1] : 0);
    __syncthreads();
    return total;
}

// One block: thread i owns pairs [i * per, (i + 1) * per). Per rank, the
// threads' counts are scanned, so the rows of a rank keep the pair order.
__global__ void __launch_bounds__(EP_PLAN_THREADS) ep_plan_kernel(const int *__restrict__ idx, int npairs, int epr,
                                                                  int n_ranks, int *__restrict__ pair_slot,
                                                                  int *__restrict__ row_pair, int *__restrict__ counts,
                                                                  int *status)
{
    __shared__ int sh[32];
    __shared__ int base[EP_MAX_RANKS + 1];
    const int tid = threadIdx.x;
    const int per = (npairs + EP_PLAN_THREADS - 1) / EP_PLAN_THREADS;
    const int p0 = min(npairs, tid * per), p1 = min(npairs, p0 + per);
    int off[EP_MAX_RANKS];
    for (int d = 0; d < EP_MAX_RANKS; d++) off[d] = 0;
    for (int p = p0; p < p1; p++) {
        const int e = idx[p];
        const int d = (e >= 0 && e < epr * n_ranks) ? e / epr : -1;
        if (d < 0) {
            atomicCAS(status, 0, EP_ERR_EXPERT);
            continue;
        }
        for (int j = 0; j < EP_MAX_RANKS; j++)
            if (j == d) off[j]++;
    }
    int tot[EP_MAX_RANKS];
    for (int d = 0; d < EP_MAX_RANKS; d++) {
        if (d < n_ranks) {
            int pre;
            tot[d] = ep_block_exscan(off[d], &pre, sh);
            off[d] = pre;
        } else {
            tot[d] = 0;
        }
    }
    if (tid == 0) {
        int run = 0;
        for (int d = 0; d < n_ranks; d++) {
            base[d] = run;
            counts[d] = tot[d];
            run += tot[d];
        }
        base[n_ranks] = run;
    }
    __syncthreads();
    for (int p = p0; p < p1; p++) {
        const int e = idx[p];
        const int d = (e >= 0 && e < epr * n_ranks) ? e / epr : -1;
        if (d < 0) {
            pair_slot[p] = -1;
            continue;
        }
        int r = 0;
        for (int j = 0; j < EP_MAX_RANKS; j++)
            if (j == d) r = off[j]++;
        const int slot = base[d] + r;
        pair_slot[p] = slot;
        row_pair[slot] = p;
    }
}

// Send rows: [hidden floats of x[t]][local expert id][0][0][0].
__global__ void __launch_bounds__(256) ep_gather_kernel(const float *__restrict__ x, const int *__restrict__ idx,
                                                        const int *__restrict__ row_pair, const int *__restrict__ counts,
                                                        int n_ranks, int topk, int hidden, int epr,
                                                        float *__restrict__ send, long max_rows)
{
    const int w4 = (hidden + 4) >> 2;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= max_rows * w4) return;
    int nrows = 0;
    for (int d = 0; d < n_ranks; d++) nrows += counts[d];
    const int r = (int)(i / w4), c = (int)(i - (long)r * w4) * 4;
    if (r >= nrows) return;
    const int p = row_pair[r], t = p / topk;
    float4 v;
    if (c < hidden) v = *reinterpret_cast<const float4 *>(x + (size_t)t * hidden + c);
    else v = make_float4((float)(idx[p] % epr), 0.f, 0.f, 0.f);
    *reinterpret_cast<float4 *>(send + (size_t)r * (hidden + 4) + c) = v;
}

// ids[r] from the received rows; rows nrecv .. nrecv + nt - 1 = own tokens
// for the shared expert.
__global__ void __launch_bounds__(256) ep_tail_kernel(float *__restrict__ recv, int nrecv, const float *__restrict__ x,
                                                      int nt, int hidden, int shared_id, int *__restrict__ ids)
{
    const int w4 = (hidden + 4) >> 2;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)(nrecv + nt) * w4) return;
    const int r = (int)(i / w4), c = (int)(i - (long)r * w4) * 4;
    float *row = recv + (size_t)r * (hidden + 4);
    if (r < nrecv) {
        if (c == hidden) ids[r] = (int)row[hidden];
        return;
    }
    if (c < hidden) *reinterpret_cast<float4 *>(row + c) = *reinterpret_cast<const float4 *>(x + (size_t)(r - nrecv) * hidden + c);
    else ids[r] = shared_id;
}

// out[t] = ((0 + w0 y0) + w1 y1) + ... + shared[t], float operations in k order.
__global__ void __launch_bounds__(256) ep_combine_kernel(const float *__restrict__ back, const int *__restrict__ pair_slot,
                                                         const float *__restrict__ wts, const float *__restrict__ shared,
                                                         int nt, int topk, int hidden, float *__restrict__ out)
{
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    const int h4 = hidden >> 2;
    if (i >= (long)nt * h4) return;
    const int t = (int)(i / h4), c = (int)(i - (long)t * h4) * 4;
    float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
    for (int k = 0; k < topk; k++) {
        const int slot = pair_slot[(size_t)t * topk + k];
        if (slot < 0) continue;
        const float w = wts[(size_t)t * topk + k];
        const float4 y = *reinterpret_cast<const float4 *>(back + (size_t)slot * hidden + c);
        o0 = __fadd_rn(o0, __fmul_rn(w, y.x));
        o1 = __fadd_rn(o1, __fmul_rn(w, y.y));
        o2 = __fadd_rn(o2, __fmul_rn(w, y.z));
        o3 = __fadd_rn(o3, __fmul_rn(w, y.w));
    }
    if (shared) {
        const float4 s = *reinterpret_cast<const float4 *>(shared + (size_t)t * hidden + c);
        o0 = __fadd_rn(o0, s.x);
        o1 = __fadd_rn(o1, s.y);
        o2 = __fadd_rn(o2, s.z);
        o3 = __fadd_rn(o3, s.w);
    }
    *reinterpret_cast<float4 *>(out + (size_t)t * hidden + c) = make_float4(o0, o1, o2, o3);
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_ep_pack(dsv4cu_ctx *ctx, float *send, int *counts, int *pair_slot, const float *x,
                              const int *idx, int nt, int topk, int hidden, int experts_per_rank, int n_ranks,
                              void *stream)
{
    if (!ctx || !send || !counts || !pair_slot || !x || !idx) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_pack: NULL argument");
    if (nt < 0 || topk < 1 || hidden <= 0 || hidden % 4 || experts_per_rank < 1 || n_ranks < 1)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_pack: bad shape");
    if (n_ranks > EP_MAX_RANKS) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "ep_pack: more than %d ranks", EP_MAX_RANKS);
    cudaStream_t st = (cudaStream_t)stream;
    const long npairs = (long)nt * topk;
    if (npairs == 0) {
        DSV4CU_CUDA_TRY(cudaMemsetAsync(counts, 0, (size_t)n_ranks * sizeof(int), st));
        return DSV4CU_OK;
    }
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, (size_t)npairs * sizeof(int), &ws);
    if (r) return r;
    int *row_pair = (int *)ws;
    ep_plan_kernel<<<1, EP_PLAN_THREADS, 0, st>>>(idx, (int)npairs, experts_per_rank, n_ranks, pair_slot, row_pair,
                                                  counts, ctx->status);
    DSV4CU_LAUNCH_CHECK();
    const long items = npairs * ((hidden + 4) / 4);
    ep_gather_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(x, idx, row_pair, counts, n_ranks, topk, hidden,
                                                                      experts_per_rank, send, npairs);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_ep_tail(float *recv, int nrecv, const float *x, int nt, int hidden, int shared_id, int *ids,
                              void *stream)
{
    if (!recv || !ids || (nt > 0 && !x)) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_tail: NULL argument");
    if (nrecv < 0 || nt < 0 || hidden <= 0 || hidden % 4) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_tail: bad shape");
    const long items = (long)(nrecv + nt) * ((hidden + 4) / 4);
    if (items == 0) return DSV4CU_OK;
    ep_tail_kernel<<<(unsigned)((items + 255) / 256), 256, 0, (cudaStream_t)stream>>>(recv, nrecv, x, nt, hidden,
                                                                                      shared_id, ids);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_ep_combine(float *out, const float *back, const int *pair_slot, const float *wts,
                                 const float *shared, int nt, int topk, int hidden, void *stream)
{
    if (!out || !pair_slot || !wts || (nt > 0 && !back && topk > 0)) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_combine: NULL argument");
    if (nt < 0 || topk < 0 || hidden <= 0 || hidden % 4) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_combine: bad shape");
    const long items = (long)nt * (hidden / 4);
    if (items == 0) return DSV4CU_OK;
    ep_combine_kernel<<<(unsigned)((items + 255) / 256), 256, 0, (cudaStream_t)stream>>>(back, pair_slot, wts, shared, nt,
                                                                                         topk, hidden, out);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}
