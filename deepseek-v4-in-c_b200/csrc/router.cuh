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

// One warp routes one token. n_experts <= 32 * RMAX_PER_LANE. sv / ov: this
// warp's scratch of n_experts floats each (shared or global memory) for the
// biased and unbiased scores. The loops stay rolled: the router runs once per
// token right after the weight streams of the previous layer have cycled the
// L2, so its code is fetched cold and its length is its cost.
constexpr int RMAX_PER_LANE = 16;

DSV4CU_DEV void route_token_warp(const float *__restrict__ tab, const float *__restrict__ logits,
                                 const float *__restrict__ bias, const int64_t *__restrict__ tid2eid, int token_id,
                                 int n_experts, int topk, float route_scale,
                                 int *__restrict__ idx_out, float *__restrict__ wts_out,
                                 float *__restrict__ scores_out, float *__restrict__ orig_out,
                                 float *sv, float *ov)
{
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int e = lane; e < n_experts; e += 32) {
        const float o = router_score(logits[e], tab);
        const float s = bias ? __fadd_rn(o, bias[e]) : o;
        ov[e] = o;
        sv[e] = s;
        if (orig_out) orig_out[e] = o;
        if (scores_out) scores_out[e] = s;
    }
    __syncwarp();
    unsigned taken = 0u;    // bit j: expert lane + 32 j already selected
    int my_sel = 0;         // lane k < topk keeps selection k
#pragma unroll 1
    for (int k = 0; k < topk; k++) {
        int best;
        if (tid2eid) {
            best = (int)tid2eid[(int64_t)token_id * topk + k];
        } else {
            // The reference scan: best = first untaken expert, then strict '>'
            // over the untaken ones in increasing order. So ties go to the lower
            // index, a NaN score is skipped, and a NaN first candidate stays.
            int first = 0x7FFFFFFF, bi = 0x7FFFFFFF;
            float bv = 0.0f;
#pragma unroll 1
            for (int j = 0; j < RMAX_PER_LANE; j++) {
                const int e = lane + 32 * j;
                if (e >= n_experts) break;
                if ((taken >> j) & 1u) continue;
                first = min(first, e);
                const float v = sv[e];
                if (isnan(v)) continue;
                if (bi == 0x7FFFFFFF || v > bv) {
                    bv = v;
                    bi = e;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float v2 = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                const int i2 = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
                first = min(first, __shfl_xor_sync(0xFFFFFFFFu, first, o));
                if (i2 != 0x7FFFFFFF && (bi == 0x7FFFFFFF || v2 > bv || (v2 == bv && i2 < bi))) {
                    bv = v2;
                    bi = i2;
                }
            }
            const bool first_nan = first != 0x7FFFFFFF && isnan(sv[first]);
            best = (first != 0x7FFFFFFF && (first_nan || bi == 0x7FFFFFFF)) ? first : bi;
        }
        if ((best & 31) == lane && best >= 0 && best < 32 * RMAX_PER_LANE) taken |= 1u << (best >> 5);
        if (lane == k) my_sel = best;
    }
    // Weights from the unbiased scores; double sum in k order.
    const bool in_range = my_sel >= 0 && my_sel < n_experts;
    const float my_w = (lane < topk && in_range) ? ov[my_sel] : 0.0f;
    double sum = 0.0;
#pragma unroll 1
    for (int k = 0; k < topk; k++) sum = __dadd_rn(sum, (double)__shfl_sync(0xFFFFFFFFu, my_w, k));
    const float inv = (sum != 0.0) ? (float)__drcp_rn(sum) : 0.0f;
    if (lane < topk) {
        idx_out[lane] = my_sel;
        wts_out[lane] = __fmul_rn(__fmul_rn(my_w, inv), route_scale);
    }
}

}  // namespace dsv4cu
