// ep_p2p.cu - one expert-parallel MoE layer step on device, the ranks joined
// by NVLink peer memory.
//
// The reference reaches every expert of a layer from one process through its
// disk-streamed expert cache (src/60_cache) and runs dsv4_layer_moe
// (src/70_decode/dsv4_layer.c:48-117) per token. Here the routed experts live
// in HBM, partitioned over the ranks of one box (expert e on rank e / epr),
// and every rank is the home of its own tokens. One call, all on the stream,
// nothing synchronised with the host (the step can be captured in a graph):
//
//   route     (grid)   one warp per home token (route_token_warp = dsv4_route).
//   plan      (1 CTA)  give every (token t, slot k) pair its owner d = e / epr
//                      and a row pos in the owner's inbox slab for this rank,
//                      in pair order (warp match + per-warp count scan).
//   dispatch  (grid)   each pair's x[t] row is stored straight into the
//                      owner's inbox (peer stores over NVLink) with the
//                      owner-local expert id; the own tokens go to the local
//                      shared-expert slab. The last CTA to finish publishes
//                      the per-owner row counts, then the step's epoch as the
//                      dispatch flag (release, system scope).
//   gather    (1 CTA)  wait (bounded) until every rank's dispatch flag shows
//                      the epoch, then one expert id per inbox row: the sent
//                      rows carry their expert, empty capacity -1 (skipped).
//   experts            dsv4cu_moe_rows over the inbox: every received row
//                      through its expert, the own tokens through the shared
//                      expert, on the tensor cores.
//   return    (grid)   each received row's result goes back into its home
//                      rank's outbox at the pair's row; last CTA: return flag.
//   combine   (grid)   wait (bounded) for every rank's return flag, then
//                      out[t] = sum over k IN ORDER of w[t][k] * y(t, k), then
//                      + the shared expert's row - the float operations of the
//                      single-device layer, so the output bits do not depend
//                      on the number of ranks.
//
// Buffers have fixed capacity (nt_max * topk rows per source rank), so no
// count crosses to the host. One buffer set suffices across steps: a rank
// stores into an owner's inbox for step s + 1 only after its own combine of
// step s saw every owner's return flag, which each owner raises after its
// expert GEMMs of step s finished reading the inbox; likewise for the outbox.
// Flags carry a per-rank epoch counter that every rank advances once per call
// (the ranks call in lockstep). Every wait gives up after 2 s, records a
// status code and lets the step finish (dsv4cu_ctx_status reports it). Peer
// memory is only ever written, with plain stores.
#include <string.h>

#include "common.cuh"
#include "ctx.h"
#include "moe.h"
#include "router.cuh"
#include "tma_gemv.cuh"

namespace dsv4cu {

constexpr int EPP_MAX_RANKS = 16;
constexpr int EPP_MAX_NT = 64;
constexpr int EPP_MAX_PAIRS = 512;        // nt_max * topk: one plan thread per pair
constexpr int EPP_MAGIC = 0x45505032;
// Device status codes (dsv4cu_ctx_status).
constexpr int EPP_E_DISPATCH = 61;        // a rank's dispatch flag did not arrive in time
constexpr int EPP_E_RETURN = 62;          // a rank's return flag did not arrive in time
constexpr int EPP_E_EXPERT = 63;          // a routed id outside 0 .. epr * world - 1, or a bad inbox id

// Byte offsets inside each rank's exported allocation (the same on every rank).
struct EppLayout {
    size_t inbox, meta, dcount, dflag, outbox, rflag, total;
};

static EppLayout epp_layout(int world, int cap, int hidden)
{
    EppLayout l;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += dsv4cu_align256(b);
        return o;
    };
    l.inbox = take((size_t)(world + 1) * cap * (hidden + 4) * 4);   // slab s < world: rows from rank s; slab world: own tokens
    l.meta = take((size_t)world * cap * 4);                         // owner-local expert id of each inbox row
    l.dcount = take((size_t)world * 4);                             // rows rank s stored this step
    l.dflag = take((size_t)world * 4);                              // epoch of rank s's finished dispatch
    l.outbox = take((size_t)world * cap * hidden * 4);              // slab d: results of the pairs sent to rank d
    l.rflag = take((size_t)world * 4);                              // epoch of rank d's finished return
    l.total = off;
    return l;
}

struct EppPeers {
    char *box[EPP_MAX_RANKS];
};

// Rank-local state (not exported).
struct EppLocal {
    unsigned *epoch;      // [1]
    int *done;            // [2]: last-CTA tickets of dispatch and return
    int *pair_slot;       // [cap]: owner * cap + row, -1 = dropped pair
    int *idx;             // [cap]: routed expert of each pair
    float *wts;           // [cap]
    int *send_count;      // [world]
    int *recv_count;      // [world]: rows received from each source this step
    int *ids;             // [(world + 1) * cap]
    float *y;             // [(world + 1) * cap][hidden]
};

struct EppShape {
    int rank, world, cap, hidden, topk, epr;
    EppLayout lay;
};

DSV4CU_DEV unsigned epp_ld_acquire(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

DSV4CU_DEV void epp_st_release(unsigned *p, unsigned v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *flag equals epoch; false after 2 s.
DSV4CU_DEV bool epp_wait_flag(const unsigned *flag, unsigned epoch)
{
    if (epp_ld_acquire(flag) == epoch) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        __nanosleep(64);
        if (epp_ld_acquire(flag) == epoch) return true;
        if (globaltimer_ns() - t0 > MBAR_TIMEOUT_NS) return false;
    }
}

// ----------------------------------------------------------------- route
__global__ void __launch_bounds__(256) epp_route_kernel(const float *__restrict__ tab, const float *__restrict__ logits,
                                                        int nt, int n_total, int topk, float route_scale, EppLocal loc)
{
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= nt) return;
    route_token_warp(tab, logits + (size_t)t * n_total, nullptr, nullptr, 0, n_total, topk, route_scale,
                     loc.idx + t * topk, loc.wts + t * topk, nullptr, nullptr);
}

// ------------------------------------------------------------------ plan
__global__ void __launch_bounds__(EPP_MAX_PAIRS) epp_plan_kernel(int nt, EppShape sh, EppLocal loc, int *status,
                                                                 int *__restrict__ idx_out,
                                                                 float *__restrict__ wts_out)
{
    constexpr int NW = EPP_MAX_PAIRS / 32;
    __shared__ int s_wc[NW][EPP_MAX_RANKS];
    const int tid = threadIdx.x, warp = tid >> 5;
    const int npairs = nt * sh.topk;
    if (tid == 0) loc.epoch[0] = loc.epoch[0] + 1u;
    for (int i = tid; i < NW * EPP_MAX_RANKS; i += blockDim.x) (&s_wc[0][0])[i] = 0;
    __syncthreads();
    const int p = tid;
    int e = -1, d = -2;
    if (p < npairs) {
        e = loc.idx[p];
        d = (e >= 0 && e < sh.epr * sh.world) ? e / sh.epr : -1;
        if (d < 0) atomicCAS(status, 0, EPP_E_EXPERT);
        if (idx_out) {
            idx_out[p] = e;
            wts_out[p] = loc.wts[p];
        }
    }
    // Rows of one owner keep the pair order: rank inside the warp, then the
    // owner's count over the lower warps.
    const unsigned same = __match_any_sync(0xFFFFFFFFu, d);
    unsigned lt;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
    const int wrank = __popc(same & lt);
    if (d >= 0 && wrank == 0) s_wc[warp][d] = __popc(same);
    __syncthreads();
    if (tid < sh.world) {
        int run = 0;
        for (int w = 0; w < NW; w++) {
            const int c = s_wc[w][tid];
            s_wc[w][tid] = run;
            run += c;
        }
        loc.send_count[tid] = run;
    }
    __syncthreads();
    if (p < npairs) loc.pair_slot[p] = d >= 0 ? d * sh.cap + s_wc[warp][d] + wrank : -1;
}

// Last CTA of the grid to finish (after every CTA's system fence) returns true.
DSV4CU_DEV bool epp_last_cta(int *ticket)
{
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(ticket, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    return last;
}

// Row copies spread over every thread of the grid, 16 bytes an item and
// EPP_UNROLL independent loads in flight per thread before the stores.
constexpr int EPP_UNROLL = 4;

// -------------------------------------------------------------- dispatch
// Rows 0 .. npairs - 1: pair r's x[t] to its owner's inbox; rows npairs ..
// + nt - 1: the home tokens to the local shared-expert slab.
DSV4CU_DEV float4 *epp_dispatch_dst(const EppShape &sh, const EppLocal &loc, const EppPeers &peers, int npairs, int r,
                                    const float *x, const float4 **src)
{
    const size_t row_b = (size_t)(sh.hidden + 4) * 4;
    if (r < npairs) {
        const int slot = loc.pair_slot[r];
        if (slot < 0) return nullptr;
        const int d = slot / sh.cap, pos = slot - d * sh.cap;
        *src = reinterpret_cast<const float4 *>(x + (size_t)(r / sh.topk) * sh.hidden);
        return reinterpret_cast<float4 *>(peers.box[d] + sh.lay.inbox + ((size_t)sh.rank * sh.cap + pos) * row_b);
    }
    const int t = r - npairs;
    *src = reinterpret_cast<const float4 *>(x + (size_t)t * sh.hidden);
    return reinterpret_cast<float4 *>(peers.box[sh.rank] + sh.lay.inbox + ((size_t)sh.world * sh.cap + t) * row_b);
}

__global__ void __launch_bounds__(256) epp_dispatch_kernel(const float *__restrict__ x, int nt, EppShape sh,
                                                           EppLocal loc, EppPeers peers)
{
    const int npairs = nt * sh.topk, h4 = sh.hidden >> 2;
    const long items = (long)(npairs + nt) * h4, stride = (long)gridDim.x * blockDim.x;
    for (long i0 = blockIdx.x * (long)blockDim.x + threadIdx.x; i0 < items; i0 += stride * EPP_UNROLL) {
        float4 v[EPP_UNROLL];
        float4 *dst[EPP_UNROLL];
#pragma unroll
        for (int u = 0; u < EPP_UNROLL; u++) {
            const long i = i0 + u * stride;
            dst[u] = nullptr;
            if (i >= items) continue;
            const int r = (int)(i / h4), c = (int)(i - (long)r * h4);
            const float4 *src;
            float4 *d = epp_dispatch_dst(sh, loc, peers, npairs, r, x, &src);
            if (!d) continue;
            v[u] = src[c];
            dst[u] = d + c;
            if (c == 0 && r < npairs) {
                const int slot = loc.pair_slot[r], o = slot / sh.cap;
                reinterpret_cast<int *>(peers.box[o] + sh.lay.meta)[(size_t)sh.rank * sh.cap + slot - o * sh.cap] =
                    loc.idx[r] % sh.epr;
            }
        }
#pragma unroll
        for (int u = 0; u < EPP_UNROLL; u++)
            if (dst[u]) *dst[u] = v[u];
    }
    if (epp_last_cta(loc.done) && threadIdx.x == 0) {
        const unsigned epoch = loc.epoch[0];
        for (int d = 0; d < sh.world; d++)
            reinterpret_cast<int *>(peers.box[d] + sh.lay.dcount)[sh.rank] = loc.send_count[d];
        __threadfence_system();
        for (int d = 0; d < sh.world; d++)
            epp_st_release(reinterpret_cast<unsigned *>(peers.box[d] + sh.lay.dflag) + sh.rank, epoch);
        loc.done[0] = 0;
    }
}

// ---------------------------------------------------------------- gather
__global__ void __launch_bounds__(1024) epp_gather_kernel(int nt, EppShape sh, EppLocal loc, char *box, int *status)
{
    __shared__ int s_n[EPP_MAX_RANKS];
    const int tid = threadIdx.x;
    const unsigned epoch = loc.epoch[0];
    if (tid < sh.world) {
        const bool ok = epp_wait_flag(reinterpret_cast<const unsigned *>(box + sh.lay.dflag) + tid, epoch);
        if (!ok) atomicCAS(status, 0, EPP_E_DISPATCH);
        const int n = reinterpret_cast<const volatile int *>(box + sh.lay.dcount)[tid];
        s_n[tid] = ok ? min(max(n, 0), sh.cap) : 0;
        loc.recv_count[tid] = s_n[tid];
    }
    __syncthreads();
    const int *meta = reinterpret_cast<const int *>(box + sh.lay.meta);
    for (int j = tid; j < (sh.world + 1) * sh.cap; j += blockDim.x) {
        const int s = j / sh.cap, i = j - s * sh.cap;
        int id = -1;
        if (s < sh.world) {
            if (i < s_n[s]) {
                id = meta[j];
                if (id < 0 || id >= sh.epr) {
                    atomicCAS(status, 0, EPP_E_EXPERT);
                    id = -1;
                }
            }
        } else if (i < nt) {
            id = sh.epr;                      // the shared expert
        }
        loc.ids[j] = id;
    }
}

// ---------------------------------------------------------------- return
// The received rows are the first recv_count[s] rows of each source slab s:
// item j walks them in order (a prefix over the <= 16 sources finds the slab).
__global__ void __launch_bounds__(256) epp_return_kernel(EppShape sh, EppLocal loc, EppPeers peers)
{
    __shared__ int s_pre[EPP_MAX_RANKS + 1];
    if (threadIdx.x == 0) {
        int run = 0;
        for (int q = 0; q < sh.world; q++) {
            s_pre[q] = run;
            run += loc.recv_count[q];
        }
        s_pre[sh.world] = run;
    }
    __syncthreads();
    const int h4 = sh.hidden >> 2;
    const long items = (long)s_pre[sh.world] * h4, stride = (long)gridDim.x * blockDim.x;
    for (long i0 = blockIdx.x * (long)blockDim.x + threadIdx.x; i0 < items; i0 += stride * EPP_UNROLL) {
        float4 v[EPP_UNROLL];
        float4 *dst[EPP_UNROLL];
#pragma unroll
        for (int u = 0; u < EPP_UNROLL; u++) {
            const long i = i0 + u * stride;
            dst[u] = nullptr;
            if (i >= items) continue;
            const int j = (int)(i / h4), c = (int)(i - (long)j * h4);
            int q = 0;
            while (q + 1 < sh.world && j >= s_pre[q + 1]) q++;
            const int row = j - s_pre[q];
            v[u] = reinterpret_cast<const float4 *>(loc.y + ((size_t)q * sh.cap + row) * sh.hidden)[c];
            dst[u] = reinterpret_cast<float4 *>(peers.box[q] + sh.lay.outbox) +
                     ((size_t)sh.rank * sh.cap + row) * h4 + c;
        }
#pragma unroll
        for (int u = 0; u < EPP_UNROLL; u++)
            if (dst[u]) *dst[u] = v[u];
    }
    if (epp_last_cta(loc.done + 1) && threadIdx.x == 0) {
        const unsigned epoch = loc.epoch[0];
        for (int d = 0; d < sh.world; d++)
            epp_st_release(reinterpret_cast<unsigned *>(peers.box[d] + sh.lay.rflag) + sh.rank, epoch);
        loc.done[1] = 0;
    }
}

// --------------------------------------------------------------- combine
__global__ void __launch_bounds__(256) epp_combine_kernel(int nt, EppShape sh, EppLocal loc, const char *box,
                                                          float *__restrict__ out, int *status)
{
    __shared__ int s_ok;
    const unsigned epoch = loc.epoch[0];
    if (threadIdx.x == 0) s_ok = 1;
    __syncthreads();
    if (threadIdx.x < sh.world &&
        !epp_wait_flag(reinterpret_cast<const unsigned *>(box + sh.lay.rflag) + threadIdx.x, epoch)) {
        atomicCAS(status, 0, EPP_E_RETURN);
        s_ok = 0;
    }
    __syncthreads();
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    const int h4 = sh.hidden >> 2, topk = sh.topk;
    if (i >= (long)nt * h4) return;
    const int t = (int)(i / h4), c = (int)(i - (long)t * h4) * 4;
    const float *back = reinterpret_cast<const float *>(box + sh.lay.outbox);
    float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
    for (int k = 0; k < topk; k++) {
        const int slot = loc.pair_slot[(size_t)t * topk + k];
        if (slot < 0 || !s_ok) continue;
        const float w = loc.wts[(size_t)t * topk + k];
        const float4 y = *reinterpret_cast<const float4 *>(back + (size_t)slot * sh.hidden + c);
        o0 = __fadd_rn(o0, __fmul_rn(w, y.x));
        o1 = __fadd_rn(o1, __fmul_rn(w, y.y));
        o2 = __fadd_rn(o2, __fmul_rn(w, y.z));
        o3 = __fadd_rn(o3, __fmul_rn(w, y.w));
    }
    const float4 s = *reinterpret_cast<const float4 *>(loc.y + ((size_t)sh.world * sh.cap + t) * sh.hidden + c);
    o0 = __fadd_rn(o0, s.x);
    o1 = __fadd_rn(o1, s.y);
    o2 = __fadd_rn(o2, s.z);
    o3 = __fadd_rn(o3, s.w);
    *reinterpret_cast<float4 *>(out + (size_t)t * sh.hidden + c) = make_float4(o0, o1, o2, o3);
}

}  // namespace dsv4cu

using namespace dsv4cu;

struct dsv4cu_ep {
    int rank, world, nt_max, hidden, topk, epr, cap, device, connected;
    EppLayout lay;
    char *box;                       // this rank's exported allocation
    void *local_block;
    EppLocal loc;
    EppPeers peers;
    char *opened[EPP_MAX_RANKS];     // IPC mappings of the peers' boxes
};

// The exported handle: the IPC handle, then the geometry every rank must share.
struct EppBlob {
    cudaIpcMemHandle_t h;
    int magic, rank, world, nt_max, hidden, topk, epr, pad;
    unsigned long long total;
};
static_assert(sizeof(EppBlob) <= DSV4CU_EP_HANDLE_BYTES, "EP handle blob too large");

extern "C" int dsv4cu_ep_create(dsv4cu_ep **out, int rank, int world, int nt_max, int hidden, int topk,
                                int experts_per_rank)
{
    if (!out) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_create: out is NULL");
    *out = nullptr;
    if (world < 1 || world > EPP_MAX_RANKS || rank < 0 || rank >= world)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_create: rank %d of world %d (world <= %d)", rank, world,
                                EPP_MAX_RANKS);
    if (nt_max < 1 || nt_max > EPP_MAX_NT || topk < 1 || nt_max * topk > EPP_MAX_PAIRS || topk > 16)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_create: nt_max %d x topk %d (nt_max <= %d, pairs <= %d)", nt_max,
                                topk, EPP_MAX_NT, EPP_MAX_PAIRS);
    if (hidden < 4 || hidden % 4 || experts_per_rank < 1 || experts_per_rank * world > 512)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_create: hidden %d, experts_per_rank %d", hidden,
                                experts_per_rank);
    dsv4cu_ep *ep = new dsv4cu_ep();
    ep->rank = rank;
    ep->world = world;
    ep->nt_max = nt_max;
    ep->hidden = hidden;
    ep->topk = topk;
    ep->epr = experts_per_rank;
    ep->cap = nt_max * topk;
    cudaGetDevice(&ep->device);
    ep->lay = epp_layout(world, ep->cap, hidden);
    auto fail = [&](int code, const char *what) {
        if (ep->box) cudaFree(ep->box);
        if (ep->local_block) cudaFree(ep->local_block);
        delete ep;
        return dsv4cu_set_error(code, "ep_create: %s", what);
    };
    if (cudaMalloc((void **)&ep->box, ep->lay.total) != cudaSuccess) return fail(DSV4CU_ERR_NOMEM, "box");
    // Flags and counts start at zero; epoch 0 is never a step's epoch.
    if (cudaMemset(ep->box + ep->lay.meta, 0, ep->lay.outbox - ep->lay.meta) != cudaSuccess ||
        cudaMemset(ep->box + ep->lay.rflag, 0, world * 4) != cudaSuccess)
        return fail(DSV4CU_ERR_CUDA, "memset");
    const int cap = ep->cap, rows = (world + 1) * cap;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += dsv4cu_align256(b);
        return o;
    };
    const size_t o_epoch = take(64), o_pair = take((size_t)cap * 4), o_idx = take((size_t)cap * 4),
                 o_wts = take((size_t)cap * 4), o_cnt = take((size_t)world * 8), o_ids = take((size_t)rows * 4),
                 o_y = take((size_t)rows * hidden * 4);
    if (cudaMalloc(&ep->local_block, off) != cudaSuccess) return fail(DSV4CU_ERR_NOMEM, "local state");
    char *b = (char *)ep->local_block;
    if (cudaMemset(b, 0, o_pair) != cudaSuccess) return fail(DSV4CU_ERR_CUDA, "memset");
    ep->loc.epoch = (unsigned *)(b + o_epoch);
    ep->loc.done = (int *)(b + o_epoch + 16);
    ep->loc.pair_slot = (int *)(b + o_pair);
    ep->loc.idx = (int *)(b + o_idx);
    ep->loc.wts = (float *)(b + o_wts);
    ep->loc.send_count = (int *)(b + o_cnt);
    ep->loc.recv_count = (int *)(b + o_cnt) + world;
    ep->loc.ids = (int *)(b + o_ids);
    ep->loc.y = (float *)(b + o_y);
    for (int r = 0; r < EPP_MAX_RANKS; r++) ep->peers.box[r] = nullptr;
    ep->peers.box[rank] = ep->box;
    *out = ep;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_ep_handle(const dsv4cu_ep *ep, void *blob)
{
    if (!ep || !blob) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_handle: NULL argument");
    EppBlob bl;
    memset(&bl, 0, sizeof bl);
    if (cudaIpcGetMemHandle(&bl.h, ep->box) != cudaSuccess) {
        cudaGetLastError();
        return dsv4cu_set_error(DSV4CU_ERR_COMM, "ep_handle: cudaIpcGetMemHandle failed");
    }
    bl.magic = EPP_MAGIC;
    bl.rank = ep->rank;
    bl.world = ep->world;
    bl.nt_max = ep->nt_max;
    bl.hidden = ep->hidden;
    bl.topk = ep->topk;
    bl.epr = ep->epr;
    bl.total = ep->lay.total;
    memset(blob, 0, DSV4CU_EP_HANDLE_BYTES);
    memcpy(blob, &bl, sizeof bl);
    return DSV4CU_OK;
}

extern "C" int dsv4cu_ep_connect(dsv4cu_ep *ep, const void *blobs)
{
    if (!ep || !blobs) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_connect: NULL argument");
    if (ep->connected) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_connect: already connected");
    for (int r = 0; r < ep->world; r++) {
        EppBlob bl;
        memcpy(&bl, (const char *)blobs + (size_t)r * DSV4CU_EP_HANDLE_BYTES, sizeof bl);
        if (bl.magic != EPP_MAGIC || bl.rank != r || bl.world != ep->world || bl.nt_max != ep->nt_max ||
            bl.hidden != ep->hidden || bl.topk != ep->topk || bl.epr != ep->epr || bl.total != ep->lay.total)
            return dsv4cu_set_error(DSV4CU_ERR_COMM, "ep_connect: handle %d does not match this rank's geometry", r);
    }
    for (int r = 0; r < ep->world; r++) {
        if (r == ep->rank) continue;
        EppBlob bl;
        memcpy(&bl, (const char *)blobs + (size_t)r * DSV4CU_EP_HANDLE_BYTES, sizeof bl);
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, bl.h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            for (int q = 0; q < r; q++)
                if (ep->opened[q]) {
                    cudaIpcCloseMemHandle(ep->opened[q]);
                    ep->opened[q] = nullptr;
                    ep->peers.box[q] = nullptr;
                }
            return dsv4cu_set_error(DSV4CU_ERR_COMM, "ep_connect: cannot map rank %d's buffers (peer access)", r);
        }
        ep->opened[r] = (char *)p;
        ep->peers.box[r] = (char *)p;
    }
    ep->connected = 1;
    return DSV4CU_OK;
}

extern "C" size_t dsv4cu_ep_workspace(const dsv4cu_ep *ep, const dsv4cu_moe *layer, int nt)
{
    if (!ep || !layer || !layer->mx_ok) return 0;
    return moe_mx_rows_workspace(layer, ep->world * ep->cap + nt, nt * (ep->topk + 1));
}

extern "C" int dsv4cu_ep_forward(dsv4cu_ctx *ctx, dsv4cu_ep *ep, const dsv4cu_moe *layer, float *out, const float *x,
                                 const float *logits, int nt, float route_scale, float limit, int *idx_out,
                                 float *wts_out, void *stream, void **events)
{
    if (!ctx || !ep || !layer || !out || !x || !logits)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_forward: NULL argument");
    if (!ep->connected) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_forward: dsv4cu_ep_connect first");
    if ((idx_out == nullptr) != (wts_out == nullptr))
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_forward: idx_out and wts_out go together");
    if (nt < 1 || nt > ep->nt_max) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_forward: nt %d (nt_max %d)", nt, ep->nt_max);
    if (layer->hidden != ep->hidden || layer->n_experts != ep->epr || !layer->has_shared)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ep_forward: layer (hidden %d, %d experts, shared %d) is not this "
                                "rank's %d experts + shared of hidden %d", layer->hidden, layer->n_experts,
                                layer->has_shared, ep->epr, ep->hidden);
    if (!layer->mx_ok)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "ep_forward: the layer has no tensor-core path");
    const float *tab = router_table_get();
    if (!tab) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "ep_forward: router table setup failed");
    cudaStream_t st = (cudaStream_t)stream;
    cudaEvent_t *ev = (cudaEvent_t *)events;
    EppShape sh;
    sh.rank = ep->rank;
    sh.world = ep->world;
    sh.cap = ep->cap;
    sh.hidden = ep->hidden;
    sh.topk = ep->topk;
    sh.epr = ep->epr;
    sh.lay = ep->lay;
    const int nrows = ep->world * ep->cap + nt;
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, moe_mx_rows_workspace(layer, nrows, nt * (ep->topk + 1)), &ws);
    if (r) return r;
    const int grid = ctx->sm_count * 2;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
    epp_route_kernel<<<(nt + 7) / 8, 256, 0, st>>>(tab, logits, nt, ep->epr * ep->world, ep->topk, route_scale,
                                                   ep->loc);
    DSV4CU_LAUNCH_CHECK();
    epp_plan_kernel<<<1, EPP_MAX_PAIRS, 0, st>>>(nt, sh, ep->loc, ctx->status, idx_out, wts_out);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));
    epp_dispatch_kernel<<<grid, 256, 0, st>>>(x, nt, sh, ep->loc, ep->peers);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[2], st));
    epp_gather_kernel<<<1, 1024, 0, st>>>(nt, sh, ep->loc, ep->box, ctx->status);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[3], st));
    r = moe_mx_rows(layer, ep->loc.y, (const float *)(ep->box + ep->lay.inbox), ep->hidden + 4, ep->loc.ids, nrows,
                    nt * (ep->topk + 1), limit, ws, ctx->status, ctx->sm_count, st);
    if (r) return r;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[4], st));
    epp_return_kernel<<<grid, 256, 0, st>>>(sh, ep->loc, ep->peers);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[5], st));
    const long items = (long)nt * (ep->hidden / 4);
    epp_combine_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(nt, sh, ep->loc, ep->box, out, ctx->status);
    DSV4CU_LAUNCH_CHECK();
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[6], st));
    return DSV4CU_OK;
}

extern "C" void dsv4cu_ep_destroy(dsv4cu_ep *ep)
{
    if (!ep) return;
    for (int r = 0; r < EPP_MAX_RANKS; r++)
        if (ep->opened[r]) cudaIpcCloseMemHandle(ep->opened[r]);
    cudaFree(ep->box);
    cudaFree(ep->local_block);
    delete ep;
}
