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

DSV4CU_DEV float router_score(float x, const float *__restrict__ tab)
{
    const uint32_t u = __float_as_uint(x);
    if (tab && (u & 0xFFFFu) == 0u) return __ldg(tab + (u >> 16));
    float sp;
    if (x > 20.0f) {
        sp = x;
    } else {
        const float e = (float)exp((double)x);
        sp = (float)log1p((double)e);
    }
    return __fsqrt_rn(sp);
}

// One warp routes one token. n_experts <= 32 * RMAX_PER_LANE.
constexpr int RMAX_PER_LANE = 16;

DSV4CU_DEV void route_token_warp(const float *__restrict__ tab, const float *__restrict__ logits,
                                 const float *__restrict__ bias, const int64_t *__restrict__ tid2eid, int token_id,
                                 int n_experts, int topk, float route_scale,
                                 int *__restrict__ idx_out, float *__restrict__ wts_out,
                                 float *__restrict__ scores_out, float *__restrict__ orig_out)
{
    const int lane = threadIdx.x & 31;
    float sv[RMAX_PER_LANE], ov[RMAX_PER_LANE];
    unsigned taken = 0u;   // bit j: expert lane + 32 j already selected
#pragma unroll
    for (int j = 0; j < RMAX_PER_LANE; j++) {
        const int e = lane + 32 * j;
        float o = 0.0f, s = 0.0f;
        if (e < n_experts) {
            o = router_score(logits[e], tab);
            s = bias ? __fadd_rn(o, bias[e]) : o;
            if (orig_out) orig_out[e] = o;
            if (scores_out) scores_out[e] = s;
        }
        ov[j] = o;
        sv[j] = s;
    }
    int sel[16];
    for (int k = 0; k < topk; k++) {
        if (tid2eid) {
            sel[k] = (int)tid2eid[(int64_t)token_id * topk + k];
            continue;
        }
        // First untaken index (its NaN score, if any, sticks like the scan's).
        int first = 0x7FFFFFFF;
        float bv = 0.0f;
        int bi = 0x7FFFFFFF;
#pragma unroll
        for (int j = 0; j < RMAX_PER_LANE; j++) {
            const int e = lane + 32 * j;
            if (e >= n_experts || (taken >> j) & 1u) continue;
            if (e < first) first = e;
            const float v = sv[j];
            if (isnan(v)) continue;
            if (bi == 0x7FFFFFFF || v > bv) { bv = v; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
            const int i2 = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            const int f2 = __shfl_xor_sync(0xFFFFFFFFu, first, o);
            first = min(first, f2);
            if (i2 != 0x7FFFFFFF && (bi == 0x7FFFFFFF || v2 > bv || (v2 == bv && i2 < bi))) {
                bv = v2;
                bi = i2;
            }
        }
        // The scan starts from the first untaken expert: a NaN there is kept.
        const int fl = first & 31, fj = first >> 5;
        float fsv = 0.0f;
#pragma unroll
        for (int j = 0; j < RMAX_PER_LANE; j++) if (j == fj) fsv = sv[j];
        fsv = __shfl_sync(0xFFFFFFFFu, fsv, fl);
        const int best = (first != 0x7FFFFFFF && (isnan(fsv) || bi == 0x7FFFFFFF)) ? first : bi;
        sel[k] = best;
        if ((best & 31) == lane) taken |= 1u << (best >> 5);
    }
    // Weights from the unbiased scores; double sum in k order.
    double sum = 0.0;
    float w[16];
    for (int k = 0; k < topk; k++) {
        const int e = sel[k];
        float o = 0.0f;
#pragma unroll
        for (int j = 0; j < RMAX_PER_LANE; j++) if (j == (e >> 5)) o = ov[j];
        o = __shfl_sync(0xFFFFFFFFu, o, e & 31);
        w[k] = o;
        sum = __dadd_rn(sum, (double)o);
    }
    const float inv = (sum != 0.0) ? (float)__drcp_rn(sum) : 0.0f;
    if (lane == 0) {
        for (int k = 0; k < topk; k++) {
            idx_out[k] = sel[k];
            wts_out[k] = __fmul_rn(__fmul_rn(w[k], inv), route_scale);
        }
    }
}

}  // namespace dsv4cu
