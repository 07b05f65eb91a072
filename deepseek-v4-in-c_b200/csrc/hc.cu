// hc.cu - mHC pre-mix (dsv4_hc_pre with dsv4_hc_split_sinkhorn, and the
// output head's hc_head) and the KV compressor step on the device.
//
// Reference: src/10_compute/dsv4_hc.c. Per token, over the hc residual copies
// x [hc][hidden] (hcdim = hc * hidden):
//   sq       = dot(x, x)                     the 16-chain double tree of
//   mixes[m] = (float)dot(fn[m], x) * rsqrt  dsv4_dot_f32d (dsv4_dot.h:20-42),
//   rsqrt    = (float)(1 / sqrt(sq / hcdim + norm_eps))
//   pre / post / comb = the Sinkhorn split of mixes (sigmoids, a row softmax,
//              then iters - 1 rounds of row and column normalising, sums in
//              double, divisors (float)sum + eps)
//   y[d]     = (float)(sum over j in order of fma(pre[j], x[j][d]))
// Every dot, sum, division and product is the reference's IEEE operation in
// its order, uncontracted. The one operation that is not is expf: the
// reference calls glibc's, which no device formula reproduces bit for bit;
// here it is exp in double rounded once to float - the correctly rounded
// value, which glibc's expf (accurate to about half an ulp) also returns
// except when the exact value lies very close to a float rounding midpoint.
//
// One CTA per token: thread (dot m, chain c) runs chain c of dot m (m = 0 is
// sq), 16 consecutive lanes read 16 consecutive floats; one thread folds each
// dot; thread 0 runs the Sinkhorn split (a few hundred dependent float ops);
// all threads then form y.
#include "common.cuh"
#include "ctx.h"

namespace dsv4cu {

constexpr int HC_MAX = 6;

DSV4CU_DEV float hc_expf(float v) { return __double2float_rn(exp((double)v)); }
DSV4CU_DEV float hc_sigmoid(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, hc_expf(-v))); }

// The dots of dsv4_hc_pre: dot 0 = x.x, dot m = fn[m - 1].x (m = 1 .. mix), each
// the reference's 16-chain tree (dsv4_dot_f32d): chain c sums elements c, c +
// 16, ... in order, one double fma each, then the fixed fold. One CTA per
// (dot, token): its row and x are staged in shared memory by the whole CTA
// (every load in flight at once), then 16 threads run the chains from there.
// The reference uses dot 0 in double and rounds the others to float before
// anything else, so the float dots go to mixes (scaled in place by the second
// kernel) and dot 0's two 32-bit halves to post[t][0] and comb[t][0]; the
// second kernel reads them before it writes those outputs.
__global__ void __launch_bounds__(256) hc_pre_dots_kernel(float *__restrict__ post, float *__restrict__ comb,
                                                          float *__restrict__ mixes, const float *__restrict__ x,
                                                          const float *__restrict__ fn, int hc, int hidden)
{
    extern __shared__ float hc_stage[];
    const int m = blockIdx.x, t = blockIdx.y, hcdim = hc * hidden, n16 = hcdim & ~15;
    const float *xt = x + (size_t)t * hcdim;
    const float *a = m == 0 ? xt : fn + (size_t)(m - 1) * hcdim;
    float *sx = hc_stage, *sa = hc_stage + hcdim;
    if ((hcdim & 3) == 0 && ((uintptr_t)xt & 15) == 0 && ((uintptr_t)a & 15) == 0) {
        const int n4 = hcdim >> 2;
        const float4 *x4 = reinterpret_cast<const float4 *>(xt), *a4 = reinterpret_cast<const float4 *>(a);
        float4 *sx4 = reinterpret_cast<float4 *>(sx), *sa4 = reinterpret_cast<float4 *>(sa);
#pragma unroll 4
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            sx4[i] = __ldg(x4 + i);
            sa4[i] = __ldg(a4 + i);
        }
    } else {
        for (int i = threadIdx.x; i < hcdim; i += blockDim.x) {
            sx[i] = __ldg(xt + i);
            sa[i] = __ldg(a + i);
        }
    }
    __syncthreads();
    __shared__ double chains[16];
    if (threadIdx.x < 16) {
        const int c = threadIdx.x;
        double acc = 0.0;
#pragma unroll 8
        for (int i = c; i < n16; i += 16) acc = __fma_rn((double)sa[i], (double)sx[i], acc);
        chains[c] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double bb[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
            bb[j] = __dadd_rn(__dadd_rn(chains[j], chains[j + 4]), __dadd_rn(chains[j + 8], chains[j + 12]));
        double acc = __dadd_rn(__dadd_rn(bb[0], bb[1]), __dadd_rn(bb[2], bb[3]));
        for (int i = n16; i < hcdim; i++) acc = __fma_rn((double)sa[i], (double)sx[i], acc);
        if (m == 0) {
            const unsigned long long b = (unsigned long long)__double_as_longlong(acc);
            post[(size_t)t * hc] = __uint_as_float((unsigned)b);
            comb[(size_t)t * hc * hc] = __uint_as_float((unsigned)(b >> 32));
        } else {
            mixes[(size_t)t * (2 + hc) * hc + m - 1] = __double2float_rn(acc);
        }
    }
}

// dsv4_hc_pre's tail for hc = 4 (the model's value) in one warp: lane e < 16
// owns comb[e / 4][e % 4]; each row or column sum gathers its four values by
// shuffles and adds them in the reference's order (0, 1, 2, 3), so every lane
// computes the same rounding the sequential loop does; the 20 Sinkhorn
// passes then cost a few shuffles and one division per lane each.
__global__ void __launch_bounds__(256) hc_pre4_kernel(float *__restrict__ y, float *__restrict__ post,
                                                      float *__restrict__ comb_out, float *__restrict__ mixes_out,
                                                      const float *__restrict__ x, const float *__restrict__ base,
                                                      const float *__restrict__ scale, int hidden, int iters,
                                                      float norm_eps, float hc_eps)
{
    constexpr int HC = 4, MIX = (2 + HC) * HC;
    __shared__ float s_pre[HC];
    const int t = blockIdx.x, hcdim = HC * hidden;
    const float *xt = x + (size_t)t * hcdim;
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x, k = lane & 3;
        const double dot0 = __longlong_as_double(
            (long long)(((unsigned long long)__float_as_uint(comb_out[(size_t)t * HC * HC]) << 32) |
                        __float_as_uint(post[(size_t)t * HC])));
        const float rsq = __double2float_rn(
            __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(dot0, (double)hcdim), (double)norm_eps))));
        __syncwarp();
        static_assert(MIX <= 32, "one mixing value per lane");
        const float mix_a = __fmul_rn(mixes_out[(size_t)t * MIX + lane % MIX], rsq);    // lane < MIX: mixes[lane]
        __syncwarp();
        if (lane < MIX) mixes_out[(size_t)t * MIX + lane] = mix_a;
        // pre[j] from mixes[j], post[j] from mixes[4 + j], comb from mixes[8 + e]
        const float m_pre = __shfl_sync(0xFFFFFFFFu, mix_a, lane & 3);
        const float m_post = __shfl_sync(0xFFFFFFFFu, mix_a, 4 + (lane & 3));
        const float m_comb = __shfl_sync(0xFFFFFFFFu, mix_a, 8 + (lane & 15));
        if (lane < HC) {
            s_pre[lane] = __fadd_rn(hc_sigmoid(__fadd_rn(__fmul_rn(m_pre, scale[0]), base[lane])), hc_eps);
            post[(size_t)t * HC + lane] =
                __fmul_rn(2.0f, hc_sigmoid(__fadd_rn(__fmul_rn(m_post, scale[1]), base[lane + HC])));
        }
        const int e = lane & 15;
        float c = __fadd_rn(__fmul_rn(m_comb, scale[2]), base[2 * HC + e]);
        auto row_val = [&](float v, int kk) { return __shfl_sync(0xFFFFFFFFu, v, (lane & ~3) + kk); };
        auto col_val = [&](float v, int jj) { return __shfl_sync(0xFFFFFFFFu, v, (lane & 16) + 4 * jj + k); };
        // First pass: row softmax (max over k with '>' in order), + eps, then a column normalise.
        {
            float mx = row_val(c, 0);
            for (int kk = 1; kk < HC; kk++) {
                const float v = row_val(c, kk);
                if (v > mx) mx = v;
            }
            const float ex = hc_expf(__fsub_rn(c, mx));
            double sum = 0.0;
            for (int kk = 0; kk < HC; kk++) sum = __dadd_rn(sum, (double)row_val(ex, kk));
            const float inv = __double2float_rn(__ddiv_rn(1.0, sum));
            c = __fadd_rn(__fmul_rn(ex, inv), hc_eps);
        }
        {
            double cs = 0.0;
            for (int jj = 0; jj < HC; jj++) cs = __dadd_rn(cs, (double)col_val(c, jj));
            c = __fdiv_rn(c, __fadd_rn(__double2float_rn(cs), hc_eps));
        }
        for (int it = 0; it < iters - 1; it++) {
            double rs = 0.0;
            for (int kk = 0; kk < HC; kk++) rs = __dadd_rn(rs, (double)row_val(c, kk));
            c = __fdiv_rn(c, __fadd_rn(__double2float_rn(rs), hc_eps));
            double cs = 0.0;
            for (int jj = 0; jj < HC; jj++) cs = __dadd_rn(cs, (double)col_val(c, jj));
            c = __fdiv_rn(c, __fadd_rn(__double2float_rn(cs), hc_eps));
        }
        if (lane < HC * HC) comb_out[(size_t)t * HC * HC + lane] = c;
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) {
        double acc = 0.0;
#pragma unroll
        for (int jj = 0; jj < HC; jj++)
            acc = __fma_rn((double)s_pre[jj], (double)__ldg(xt + (size_t)jj * hidden + d), acc);
        y[(size_t)t * hidden + d] = __double2float_rn(acc);
    }
}

// The rest of dsv4_hc_pre for token blockIdx.x, from the dots hc_pre_dots_kernel
// left in its outputs.
__global__ void __launch_bounds__(256) hc_pre_kernel(float *__restrict__ y, float *__restrict__ post,
                                                     float *__restrict__ comb_out, float *__restrict__ mixes_out,
                                                     const float *__restrict__ x, const float *__restrict__ base,
                                                     const float *__restrict__ scale, int hc, int hidden, int iters,
                                                     float norm_eps, float hc_eps)
{
    __shared__ double dot0;
    __shared__ float s_pre[HC_MAX];
    const int t = blockIdx.x, hcdim = hc * hidden, mix = (2 + hc) * hc;
    const float *xt = x + (size_t)t * hcdim;
    if (threadIdx.x == 0)
        dot0 = __longlong_as_double((long long)(((unsigned long long)__float_as_uint(comb_out[(size_t)t * hc * hc]) << 32) |
                                                __float_as_uint(post[(size_t)t * hc])));
    __syncthreads();

    if (threadIdx.x == 0) {
        const float rsq = __double2float_rn(
            __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(dot0, (double)hcdim), (double)norm_eps))));
        float mixes[(2 + HC_MAX) * HC_MAX], pre[HC_MAX], po[HC_MAX], comb[HC_MAX * HC_MAX];
        for (int m = 0; m < mix; m++) {
            mixes[m] = __fmul_rn(mixes_out[(size_t)t * mix + m], rsq);
            mixes_out[(size_t)t * mix + m] = mixes[m];
        }
        for (int j = 0; j < hc; j++)
            pre[j] = __fadd_rn(hc_sigmoid(__fadd_rn(__fmul_rn(mixes[j], scale[0]), base[j])), hc_eps);
        for (int j = 0; j < hc; j++)
            po[j] = __fmul_rn(2.0f, hc_sigmoid(__fadd_rn(__fmul_rn(mixes[j + hc], scale[1]), base[j + hc])));
        for (int j = 0; j < hc; j++)
            for (int k = 0; k < hc; k++) {
                const int o = j * hc + k + 2 * hc;
                comb[j * hc + k] = __fadd_rn(__fmul_rn(mixes[o], scale[2]), base[o]);
            }
        // First pass: row softmax, + eps, then a column normalise.
        for (int j = 0; j < hc; j++) {
            float mx = comb[j * hc];
            for (int k = 1; k < hc; k++)
                if (comb[j * hc + k] > mx) mx = comb[j * hc + k];
            double sum = 0.0;
            for (int k = 0; k < hc; k++) {
                const float e = hc_expf(__fsub_rn(comb[j * hc + k], mx));
                comb[j * hc + k] = e;
                sum = __dadd_rn(sum, (double)e);
            }
            const float inv = __double2float_rn(__ddiv_rn(1.0, sum));
            for (int k = 0; k < hc; k++) comb[j * hc + k] = __fadd_rn(__fmul_rn(comb[j * hc + k], inv), hc_eps);
        }
        for (int k = 0; k < hc; k++) {
            double cs = 0.0;
            for (int j = 0; j < hc; j++) cs = __dadd_rn(cs, (double)comb[j * hc + k]);
            const float d = __fadd_rn(__double2float_rn(cs), hc_eps);
            for (int j = 0; j < hc; j++) comb[j * hc + k] = __fdiv_rn(comb[j * hc + k], d);
        }
        // The remaining iters - 1 passes: rows, then columns.
        for (int it = 0; it < iters - 1; it++) {
            for (int j = 0; j < hc; j++) {
                double rs = 0.0;
                for (int k = 0; k < hc; k++) rs = __dadd_rn(rs, (double)comb[j * hc + k]);
                const float d = __fadd_rn(__double2float_rn(rs), hc_eps);
                for (int k = 0; k < hc; k++) comb[j * hc + k] = __fdiv_rn(comb[j * hc + k], d);
            }
            for (int k = 0; k < hc; k++) {
                double cs = 0.0;
                for (int j = 0; j < hc; j++) cs = __dadd_rn(cs, (double)comb[j * hc + k]);
                const float d = __fadd_rn(__double2float_rn(cs), hc_eps);
                for (int j = 0; j < hc; j++) comb[j * hc + k] = __fdiv_rn(comb[j * hc + k], d);
            }
        }
        for (int j = 0; j < hc; j++) {
            s_pre[j] = pre[j];
            post[(size_t)t * hc + j] = po[j];
        }
        for (int i = 0; i < hc * hc; i++) comb_out[(size_t)t * hc * hc + i] = comb[i];
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc = __fma_rn((double)s_pre[j], (double)__ldg(xt + (size_t)j * hidden + d), acc);
        y[(size_t)t * hidden + d] = __double2float_rn(acc);
    }
}

// The output head's mHC (hc_head, src/90_cli/dsv4_decode.c:102-125): sq and
// each copy's mixing dot are single sequential chains in the reference (no
// tree), so one thread runs each, in separate warps so they run side by side;
// then pre[j] = sigmoid(m * scale[0] + base[j]) + hc_eps and y as above (the
// sum over copies as products then adds, which equals fma: each product is
// exact in double).
__global__ void __launch_bounds__(256) hc_head_kernel(float *__restrict__ y, const float *__restrict__ x,
                                                      const float *__restrict__ fn, const float *__restrict__ base,
                                                      const float *__restrict__ scale, int hc, int hidden,
                                                      float norm_eps, float hc_eps)
{
    __shared__ double dots[HC_MAX + 1];
    __shared__ float s_pre[HC_MAX];
    const int t = blockIdx.x, hcdim = hc * hidden, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *xt = x + (size_t)t * hcdim;
    if (lane == 0 && warp <= hc) {
        double acc = 0.0;
        if (warp == 0) {
            for (int i = 0; i < hcdim; i++) {
                const double v = (double)__ldg(xt + i);
                acc = __dadd_rn(acc, __dmul_rn(v, v));
            }
        } else {
            const float *row = fn + (size_t)(warp - 1) * hcdim;
            for (int i = 0; i < hcdim; i++) acc = __fma_rn((double)__ldg(row + i), (double)__ldg(xt + i), acc);
        }
        dots[warp] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float rs = __double2float_rn(
            __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(dots[0], (double)hcdim), (double)norm_eps))));
        for (int j = 0; j < hc; j++) {
            const float m = __fmul_rn(__double2float_rn(dots[j + 1]), rs);
            s_pre[j] = __fadd_rn(hc_sigmoid(__fadd_rn(__fmul_rn(m, scale[0]), base[j])), hc_eps);
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) {
        double acc = 0.0;
        for (int j = 0; j < hc; j++) acc = __fma_rn((double)s_pre[j], (double)__ldg(xt + (size_t)j * hidden + d), acc);
        y[(size_t)t * hidden + d] = __double2float_rn(acc);
    }
}

// ------------------------------------------------------------ compressor
// dsv4_compress_step (src/10_compute/dsv4_compress.c): the token's kv and
// score (+ ape[pos % ratio]) go into its slot; when the window closes each
// channel pools its slots with a softmax over the slot axis (max, then
// e = expf(v - max) over finite slots, denominator and weighted sum in double
// in slot order, (float)(acc / denom)). Ratio 4 overlaps the previous window:
// slots 0..3 read the first half of each slot's channels, slots 4..7 the
// second half, and the state then slides by one window. expf as above.
__global__ void compress_place_kernel(float *__restrict__ kv_state, float *__restrict__ score_state,
                                      const float *__restrict__ kv_in, const float *__restrict__ score_in,
                                      const float *__restrict__ apr, int slot, int width)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= width) return;
    kv_state[(size_t)slot * width + c] = kv_in[c];
    score_state[(size_t)slot * width + c] = __fadd_rn(score_in[c], apr[c]);
}

__global__ void compress_pool_kernel(float *__restrict__ out, const float *__restrict__ kv_state,
                                     const float *__restrict__ score_state, int ratio, int head_dim, int overlap)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= head_dim) return;
    const int width = (1 + overlap) * head_dim, nslot = overlap ? 2 * ratio : ratio;
    auto at = [&](int s) -> size_t { return (size_t)s * width + ((overlap && s >= ratio) ? head_dim : 0) + c; };
    float mx = -INFINITY;
    for (int s = 0; s < nslot; s++) {
        const float v = score_state[at(s)];
        if (v > mx) mx = v;
    }
    if (mx == -INFINITY) {
        out[c] = 0.0f;
        return;
    }
    double denom = 0.0, acc = 0.0;
    for (int s = 0; s < nslot; s++) {
        const float v = score_state[at(s)];
        if (v == -INFINITY) continue;
        const double e = (double)hc_expf(__fsub_rn(v, mx));
        denom = __dadd_rn(denom, e);
        acc = __dadd_rn(acc, __dmul_rn(e, (double)kv_state[at(s)]));
    }
    out[c] = __double2float_rn(__ddiv_rn(acc, denom));
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_compress_step(float *out, const float *kv_in, const float *score_in, const float *ape,
                                    float *kv_state, float *score_state, int pos, int ratio, int head_dim,
                                    void *stream)
{
    if (!out || !kv_in || !score_in || !ape || !kv_state || !score_state || pos < 0 || ratio <= 0 || head_dim <= 0)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "compress_step: bad args");
    cudaStream_t st = (cudaStream_t)stream;
    const int overlap = ratio == 4, width = (1 + overlap) * head_dim, phase = pos % ratio;
    const int slot = overlap ? ratio + phase : phase;
    compress_place_kernel<<<(unsigned)((width + 255) / 256), 256, 0, st>>>(kv_state, score_state, kv_in, score_in,
                                                                          ape + (size_t)phase * width, slot, width);
    DSV4CU_LAUNCH_CHECK();
    if ((pos + 1) % ratio != 0) return 0;
    compress_pool_kernel<<<(unsigned)((head_dim + 127) / 128), 128, 0, st>>>(out, kv_state, score_state, ratio,
                                                                            head_dim, overlap);
    DSV4CU_LAUNCH_CHECK();
    if (overlap) {
        const size_t b = (size_t)ratio * width * sizeof(float);
        DSV4CU_CUDA_TRY(cudaMemcpyAsync(kv_state, kv_state + (size_t)ratio * width, b, cudaMemcpyDeviceToDevice, st));
        DSV4CU_CUDA_TRY(
            cudaMemcpyAsync(score_state, score_state + (size_t)ratio * width, b, cudaMemcpyDeviceToDevice, st));
    }
    return 1;
}

extern "C" int dsv4cu_hc_head(float *y, const float *x, const float *fn, const float *base, const float *scale,
                              int nt, int hc, int hidden, float norm_eps, float hc_eps, void *stream)
{
    if (!y || !x || !fn || !base || !scale || nt <= 0 || hidden <= 0)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "hc_head: bad args");
    if (hc < 1 || hc > HC_MAX) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "hc_head: hc %d (1..%d)", hc, HC_MAX);
    hc_head_kernel<<<(unsigned)nt, 256, 0, (cudaStream_t)stream>>>(y, x, fn, base, scale, hc, hidden, norm_eps,
                                                                   hc_eps);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_hc_pre(float *y, float *post, float *comb, float *mixes, const float *x, const float *fn,
                             const float *base, const float *scale, int nt, int hc, int hidden, int iters,
                             float norm_eps, float hc_eps, void *stream)
{
    if (!y || !post || !comb || !mixes || !x || !fn || !base || !scale || nt <= 0 || hidden <= 0 || iters < 1)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "hc_pre: bad args");
    if (hc < 1 || hc > HC_MAX) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "hc_pre: hc %d (1..%d)", hc, HC_MAX);
    const int ndots = (2 + hc) * hc + 1;
    const size_t smem = (size_t)2 * hc * hidden * sizeof(float);
    static SmemLimit lim;
    DSV4CU_CUDA_TRY(smem_limit(lim, (const void *)hc_pre_dots_kernel, (int)smem));
    hc_pre_dots_kernel<<<dim3((unsigned)ndots, (unsigned)nt), 256, smem, (cudaStream_t)stream>>>(post, comb, mixes, x,
                                                                                               fn, hc, hidden);
    DSV4CU_LAUNCH_CHECK();
    if (hc == 4)
        hc_pre4_kernel<<<(unsigned)nt, 256, 0, (cudaStream_t)stream>>>(y, post, comb, mixes, x, base, scale, hidden,
                                                                       iters, norm_eps, hc_eps);
    else
        hc_pre_kernel<<<(unsigned)nt, 256, 0, (cudaStream_t)stream>>>(y, post, comb, mixes, x, base, scale, hc,
                                                                      hidden, iters, norm_eps, hc_eps);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}
