// router.cuh - the MoE router (dsv4_route) for one token in one warp.
//
// Semantics of src/10_compute/dsv4_ops.c:117-156 and :43-46:
//   orig[e]   = sqrtf(softplus(logit[e])), softplus(x) = x > 20 ? x : log1p(exp(x))
//   scores[e] = orig[e] + bias[e]   (bias steers SELECTION only)
//   idx       = tid2eid[token] (hash layers) or top-k of scores by repeated
//               argmax: strict '>' over e in increasing order, so ties go to
//               the lower index and a NaN wins only as the first untaken entry
//   wts[k]    = orig[idx[k]] * (float)(1 / double sum) * route_scale
// The score of a bf16-valued logit (every logit the configs feed: the router
// input is bf16) is read from a 65536-entry table built once per device by
// the host side of this library with the host C library's expf / log1pf /
// sqrtf - the calls the reference makes - so it is the reference's value bit
// for bit. glibc's log1pf is not correctly rounded (it differs from the
// correctly rounded result on ~0.6% of bf16 inputs), so no device evaluation
// can promise that. Any other fp32 logit is evaluated in double and rounded
// once per function, which is the correctly rounded value and differs from
// glibc by at most one ulp on those rare inputs.
#pragma once
#include "common.cuh"

namespace dsv4cu {

// Device address of the bf16 score table on the current device, building it
// on first use (host computation + one copy). Returns nullptr on failure.
const float *router_table_get();

// sqrtf(softplus(x)) evaluated in double and rounded once per function; kept
// out of line so the common table path stays a few instructions long.
static __device__ __noinline__ float router_score_slow(float x)
{
    float sp;
    if (x > 20.0f) {
        sp = x;
    } else {
        const float e = (float)exp((double)x);
        sp = (float)log1p((double)e);
    }
    return __fsqrt_rn(sp);
}

DSV4CU_DEV float router_score(float x, const float *__restrict__ tab)
{
    const uint32_t u = __float_as_uint(x);
    if (tab && (u & 0xFFFFu) == 0u) return __ldg(tab + (u >> 16));
    return router_score_slow(x);
}

// One warp routes one token; n_experts <= 32 * RMAX_PER_LANE. Expert
// lane + 32 j is held by lane `lane` in slot j. All logit and table loads are
// issued before any use (the router runs right after the previous layer's
// weight streams have cycled the L2, so each load is a DRAM round trip).
//
// Selection. Without NaN scores the reference's repeated argmax (strict '>'
// in increasing expert order) takes the experts in descending score order,
// ties to the lower index. Each lane sorts its own slots in that order once
// (a sorting network on registers); a round is then one warp argmax over the
// lanes' heads (two redux.sync: the largest key, then the lowest expert with
// it) and the winner pops its head. A NaN score can win only as the first
// untaken expert, an order no static sort expresses: any NaN (ballot) and
// hash routing take the round-by-round scan of the reference instead.
constexpr int RMAX_PER_LANE = 16;

DSV4CU_DEV uint32_t route_key(float v)
{
    const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);   // -0 ties with +0, as '>' does
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Slot i of a lane's sorted list: key (0 = none: route_key never gives 0 for
// a non-NaN score), expert, unbiased score.
struct RouteItem {
    uint32_t key, e;
    float o;
};

DSV4CU_DEV void route_cx(RouteItem &a, RouteItem &b)
{
    const bool swap = b.key > a.key || (b.key == a.key && b.e < a.e);
    if (swap) {
        const RouteItem t = a;
        a = b;
        b = t;
    }
}

// Bitonic sort of R (power of two) items, best first.
template <int R>
DSV4CU_DEV void route_sort(RouteItem (&it)[R])
{
#pragma unroll
    for (int k = 2; k <= R; k <<= 1)
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
            for (int i = 0; i < R; i++) {
                const int l = i ^ j;
                if (l > i) {
                    if ((i & k) == 0) route_cx(it[i], it[l]);
                    else route_cx(it[l], it[i]);
                }
            }
}

template <int R>
DSV4CU_DEV void route_token_warp_r(const float *__restrict__ tab, const float *__restrict__ logits,
                                   const float *__restrict__ bias, const int64_t *__restrict__ tid2eid, int token_id,
                                   int n_experts, int topk, float route_scale, int *__restrict__ idx_out,
                                   float *__restrict__ wts_out, float *__restrict__ scores_out,
                                   float *__restrict__ orig_out)
{
    const int lane = threadIdx.x & 31;
    float ov[R], sv[R];
#pragma unroll
    for (int j = 0; j < R; j++) {
        const int e = lane + 32 * j;
        ov[j] = e < n_experts ? logits[e] : 0.0f;
        sv[j] = (bias && e < n_experts) ? bias[e] : 0.0f;
    }
    bool fast[R];
#pragma unroll
    for (int j = 0; j < R; j++) {
        const uint32_t u = __float_as_uint(ov[j]);
        fast[j] = tab && (u & 0xFFFFu) == 0u;
        if (lane + 32 * j < n_experts && fast[j]) ov[j] = __ldg(tab + (u >> 16));
    }
    bool nan = false;
#pragma unroll
    for (int j = 0; j < R; j++) {
        const int e = lane + 32 * j;
        if (e >= n_experts) continue;
        if (!fast[j]) ov[j] = router_score_slow(ov[j]);
        sv[j] = bias ? __fadd_rn(ov[j], sv[j]) : ov[j];
        nan |= isnan(sv[j]);
        if (orig_out) orig_out[e] = ov[j];
        if (scores_out) scores_out[e] = sv[j];
    }
    int my_sel = 0;         // lane k < topk keeps selection k
    float my_w = 0.0f;
    double sum = 0.0;
    if (!tid2eid && !__any_sync(0xFFFFFFFFu, nan)) {
        RouteItem it[R];
#pragma unroll
        for (int j = 0; j < R; j++) {
            const int e = lane + 32 * j;
            it[j].key = e < n_experts ? route_key(sv[j]) : 0u;
            it[j].e = (uint32_t)e;
            it[j].o = ov[j];
        }
        route_sort<R>(it);
#pragma unroll 1
        for (int k = 0; k < topk; k++) {
            const uint32_t kmax = __reduce_max_sync(0xFFFFFFFFu, it[0].key);
            const uint32_t best = __reduce_min_sync(0xFFFFFFFFu, it[0].key == kmax ? it[0].e : 0xFFFFFFFFu);
            const float o = __shfl_sync(0xFFFFFFFFu, it[0].o, best & 31);
            if ((best & 31) == (uint32_t)lane) {
#pragma unroll
                for (int j = 0; j + 1 < R; j++) it[j] = it[j + 1];
                it[R - 1].key = 0u;
                it[R - 1].e = 0xFFFFFFFFu;
            }
            sum = __dadd_rn(sum, (double)o);     // double sum in k order
            if (lane == k) {
                my_sel = (int)best;
                my_w = o;
            }
        }
    } else {
        unsigned taken = 0u;    // bit j: expert lane + 32 j already selected
#pragma unroll 1
        for (int k = 0; k < topk; k++) {
            int best;
            if (tid2eid) {
                best = (int)tid2eid[(int64_t)token_id * topk + k];
            } else {
                // The reference scan: best = first untaken expert, then strict
                // '>' over the untaken ones in increasing order. So ties go to
                // the lower index, a NaN score is skipped, and a NaN first
                // candidate stays.
                uint32_t bkey = 0u, first = 0xFFFFFFFFu, bi = 0xFFFFFFFFu;
#pragma unroll
                for (int j = 0; j < R; j++) {
                    const int e = lane + 32 * j;
                    if (e >= n_experts || ((taken >> j) & 1u)) continue;
                    first = min(first, (uint32_t)e);
                    if (isnan(sv[j])) continue;
                    const uint32_t kv = route_key(sv[j]);
                    if (bi == 0xFFFFFFFFu || kv > bkey) {
                        bkey = kv;
                        bi = (uint32_t)e;
                    }
                }
                const uint32_t kmax = __reduce_max_sync(0xFFFFFFFFu, bi != 0xFFFFFFFFu ? bkey : 0u);
                const uint32_t any = __ballot_sync(0xFFFFFFFFu, bi != 0xFFFFFFFFu);
                const uint32_t wbi =
                    __reduce_min_sync(0xFFFFFFFFu, (bi != 0xFFFFFFFFu && bkey == kmax) ? bi : 0xFFFFFFFFu);
                const uint32_t wfirst = __reduce_min_sync(0xFFFFFFFFu, first);
                // NaN at the first untaken expert: read from its owner lane.
                float fsv = 0.0f;
#pragma unroll
                for (int j = 0; j < R; j++)
                    if ((uint32_t)j == (wfirst >> 5)) fsv = sv[j];
                fsv = __shfl_sync(0xFFFFFFFFu, fsv, wfirst & 31);
                best = (wfirst != 0xFFFFFFFFu && (isnan(fsv) || !any)) ? (int)wfirst : (int)wbi;
            }
            // Weight: the unbiased score of the selection, from its owner lane.
            float o = 0.0f;
            const bool in_range = best >= 0 && best < n_experts;
#pragma unroll
            for (int j = 0; j < R; j++)
                if (in_range && j == (best >> 5)) o = ov[j];
            o = __shfl_sync(0xFFFFFFFFu, o, in_range ? (best & 31) : 0);
            if (!in_range) o = 0.0f;
            sum = __dadd_rn(sum, (double)o);     // double sum in k order
            if (in_range && (best & 31) == lane) taken |= 1u << (best >> 5);
            if (lane == k) {
                my_sel = best;
                my_w = o;
            }
        }
    }
    const float inv = (sum != 0.0) ? (float)__drcp_rn(sum) : 0.0f;
    if (lane < topk) {
        idx_out[lane] = my_sel;
        wts_out[lane] = __fmul_rn(__fmul_rn(my_w, inv), route_scale);
    }
}

DSV4CU_DEV void route_token_warp(const float *__restrict__ tab, const float *__restrict__ logits,
                                 const float *__restrict__ bias, const int64_t *__restrict__ tid2eid, int token_id,
                                 int n_experts, int topk, float route_scale, int *__restrict__ idx_out,
                                 float *__restrict__ wts_out, float *__restrict__ scores_out,
                                 float *__restrict__ orig_out)
{
    if (n_experts <= 256)
        route_token_warp_r<8>(tab, logits, bias, tid2eid, token_id, n_experts, topk, route_scale, idx_out, wts_out,
                              scores_out, orig_out);
    else
        route_token_warp_r<RMAX_PER_LANE>(tab, logits, bias, tid2eid, token_id, n_experts, topk, route_scale,
                                          idx_out, wts_out, scores_out, orig_out);
}

}  // namespace dsv4cu
