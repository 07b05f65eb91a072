// misc.cu - router, SwiGLU, index offset, weight quantizers, synthetic fill.
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "ctx.h"
#include "router.cuh"
#include <string.h>

namespace dsv4cu {

// sqrtf(softplus(x)) for every bf16 bit pattern x (src/10_compute/dsv4_ops.c:43-46,
// :123), filled from the host C library once per device.
__device__ float g_router_bf16[65536];

const float *router_table_get()
{
    static std::mutex mu;
    static bool ready[256];
    static float host[65536];
    static bool host_ready = false;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!host_ready) {
        for (uint32_t u = 0; u < 65536u; u++) {
            const uint32_t b = u << 16;
            float x;
            memcpy(&x, &b, 4);
            const float sp = (x > 20.0f) ? x : log1pf(expf(x));
            host[u] = sqrtf(sp);
        }
        host_ready = true;
    }
    if (!ready[dev]) {
        if (cudaMemcpyToSymbol(g_router_bf16, host, sizeof host) != cudaSuccess) return nullptr;
        ready[dev] = true;
    }
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_router_bf16) != cudaSuccess) return nullptr;
    return (const float *)p;
}

__global__ void route_kernel(const float *tab, int *idx, float *wts, float *scores, float *orig, const float *logits,
                             const float *bias, const int64_t *tid2eid, const int *token_ids, int n_experts,
                             int topk, float route_scale, int nt)
{
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= nt) return;
    route_token_warp(tab, logits + (size_t)t * n_experts, bias, tid2eid, token_ids ? token_ids[t] : 0, n_experts,
                     topk, route_scale, idx + (size_t)t * topk, wts + (size_t)t * topk,
                     scores ? scores + (size_t)t * n_experts : nullptr,
                     orig ? orig + (size_t)t * n_experts : nullptr);
}

// SwiGLU exactly as dsv4_swiglu (src/10_compute/dsv4_ops.c:61-79).
__global__ void swiglu_kernel(float *y, const float *gate, const float *up, int n, float limit)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float u = up[i], g = gate[i];
    if (limit > 0.0f) {
        if (u > limit) u = limit;
        if (u < -limit) u = -limit;
        if (g > limit) g = limit;
    }
    y[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

__global__ void offset_kernel(int *idxs, int n, int offset)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && idxs[i] >= 0) idxs[i] += offset;
}

// E8M0 exponent of the smallest power of two s with amax / s <= qmax, where
// qmax = qf * 2^qe (448 = 0.875 * 2^9, 6 = 0.75 * 2^3). With amax = f 2^E,
// f in [0.5, 1): e = E - qe + (f > qf). Exact; no division is rounded.
__device__ __forceinline__ int e8m0_exponent(float amax, float qf, int qe)
{
    if (!(amax > 0.0f) || !isfinite(amax)) return 0;
    int E;
    const float f = frexpf(amax, &E);
    int e = E - qe + (f > qf ? 1 : 0);
    return max(-127, min(127, e));
}

// FP8: one CTA per 128x128 block.
__global__ void __launch_bounds__(256) quant_fp8_kernel(uint8_t *w, uint8_t *s, const float *src, int rows,
                                                        int cols)
{
    const int br = blockIdx.y, bc = blockIdx.x, s_cols = (cols + 127) / 128;
    const int r0 = br * 128, c0 = bc * 128;
    __shared__ float red[8];
    float a = 0.0f;
    for (int i = threadIdx.x; i < 128 * 128; i += 256) {
        const int r = r0 + (i >> 7), c = c0 + (i & 127);
        if (r < rows && c < cols) {
            const float v = fabsf(src[(size_t)r * cols + c]);
            if (isfinite(v)) a = fmaxf(a, v);
        }
    }
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 16));
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 8));
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 4));
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 2));
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 1));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
    __syncthreads();
    float amax = 0.0f;
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, red[i]);
    const int e = e8m0_exponent(amax, 0.875f, 9);
    if (threadIdx.x == 0) s[(size_t)br * s_cols + bc] = (uint8_t)(127 + e);
    for (int i = threadIdx.x; i < 128 * 64; i += 256) {
        const int r = r0 + (i >> 6), c = c0 + 2 * (i & 63);
        if (r >= rows || c >= cols) continue;
        const float v0 = ldexpf(src[(size_t)r * cols + c], -e);
        const float v1 = (c + 1 < cols) ? ldexpf(src[(size_t)r * cols + c + 1], -e) : 0.0f;
        uint16_t two;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(two) : "f"(v1), "f"(v0));
        w[(size_t)r * cols + c] = (uint8_t)(two & 0xFF);
        if (c + 1 < cols) w[(size_t)r * cols + c + 1] = (uint8_t)(two >> 8);
    }
}

// FP4: one warp per 1x32 block; lane = element.
__global__ void quant_fp4_kernel(uint8_t *w, uint8_t *s, const float *src, int rows, int cols)
{
    const long gw = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31, nb = cols / 32;
    if (gw >= (long)rows * nb) return;
    const int r = (int)(gw / nb), b = (int)(gw - (long)r * nb), c = b * 32 + lane;
    const float v = src[(size_t)r * cols + c];
    float a = isfinite(v) ? fabsf(v) : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
    const int e = e8m0_exponent(a, 0.75f, 3);
    if (lane == 0) s[(size_t)r * nb + b] = (uint8_t)(127 + e);
    const float vs = ldexpf(v, -e);
    const float other = __shfl_down_sync(0xFFFFFFFFu, vs, 1);
    if ((lane & 1) == 0) {
        uint16_t packed;
        // first operand -> high nibble: the odd element; second -> low nibble.
        asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}"
            : "=h"(packed) : "f"(other), "f"(vs));
        w[(size_t)r * (cols / 2) + (c >> 1)] = (uint8_t)packed;
    }
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Box-Muller on two 24-bit uniforms drawn from (seed, pair index).
__global__ void fill_normal_kernel(float *dst, size_t n, uint64_t seed, float mean, float stdv)
{
    const size_t pair = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (2 * pair >= n) return;
    const uint64_t h = splitmix64(seed * 0x9E3779B97F4A7C15ull ^ splitmix64(pair));
    const float u1 = ((float)(uint32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = ((float)(uint32_t)((h >> 16) & 0xFFFFFFu) + 0.5f) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    dst[2 * pair] = mean + stdv * r * cs;
    if (2 * pair + 1 < n) dst[2 * pair + 1] = mean + stdv * r * sn;
}

__global__ void round_bf16_kernel(float *x, size_t n)
{
    const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (i < n) x[i] = __bfloat162float(__float2bfloat16_rn(x[i]));
}

// ------------------------------------------------------------- mHC post
// dsv4_hc_post (src/10_compute/dsv4_hc.c) per token t: for copy k and dim d,
// acc = post[k] * x[d] in double (exact), then fma(comb[j][k], residual[j][d],
// acc) for j in order (each product exact, one rounded add, as the reference's
// vector body and scalar tail both do), y = (float)acc. One thread per output.
__global__ void hc_post_kernel(float *__restrict__ y, const float *__restrict__ x,
                               const float *__restrict__ residual, const float *__restrict__ post,
                               const float *__restrict__ comb, int nt, int hc, int hidden)
{
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)nt * hc * hidden) return;
    const int d = (int)(i % hidden);
    const long tk = i / hidden;
    const int k = (int)(tk % hc), t = (int)(tk / hc);
    const float *res = residual + (size_t)t * hc * hidden;
    const float *cm = comb + (size_t)t * hc * hc;
    double acc = __dmul_rn((double)__ldg(post + (size_t)t * hc + k), (double)__ldg(x + (size_t)t * hidden + d));
    for (int j = 0; j < hc; j++)
        acc = __fma_rn((double)__ldg(cm + j * hc + k), (double)__ldg(res + (size_t)j * hidden + d), acc);
    y[i] = __double2float_rn(acc);
}

// ------------------------------------------------------------- rope
// dsv4_rope_apply (src/10_compute/dsv4_rope.c) over v [nt][nh][head_dim]:
// the last rd dims of every head are (re, im) pairs rotated by table entry
// (pos[t], i), -sin when inverse. One thread per pair, the reference's float
// multiplies and one subtract / add, uncontracted, so the bits match.
__global__ void rope_kernel(float *__restrict__ v, int nt, int nh, int head_dim, int rd,
                            const float *__restrict__ cs, const float *__restrict__ sn,
                            const int *__restrict__ pos, int table_half, int n_pos, int inverse,
                            int *__restrict__ err)
{
    const int half = rd >> 1;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)nt * nh * half) return;
    const int j = (int)(i % half);
    const long vh = i / half;
    const int t = (int)(vh / nh);
    const int p = __ldg(pos + t);
    if (p < 0 || p >= n_pos) {
        if (err) atomicCAS(err, 0, 41);
        return;
    }
    float *tail = v + vh * head_dim + (head_dim - rd);
    const float ci = __ldg(cs + (size_t)p * table_half + j);
    const float s0 = __ldg(sn + (size_t)p * table_half + j);
    const float si = inverse ? __fmul_rn(-1.0f, s0) : s0;
    const float re = tail[2 * j], im = tail[2 * j + 1];
    tail[2 * j] = __fsub_rn(__fmul_rn(re, ci), __fmul_rn(im, si));
    tail[2 * j + 1] = __fadd_rn(__fmul_rn(re, si), __fmul_rn(im, ci));
}

// ------------------------------------------------------------- rmsnorm
// dsv4_rmsnorm (src/10_compute/dsv4_ops.c:26-33): sum of x^2 in double in
// index order, inv = (float)(1 / sqrt(sum / n + eps)), y = w * (x * inv).
// The only rounding-order-dependent step is the sequential sum; everything
// after it is monotone in the sum. So the CTA sums in parallel (S', within
// (n / threads + log2 threads) ulps of the exact sum, as the sequential sum T
// is within (n - 1) ulps), evaluates the reference's inv at both ends of an
// interval that must hold T, and uses that inv when the two agree - then it
// is the reference's inv whatever T's exact rounding was. When they differ
// (a sum within about n ulps of a float rounding boundary of inv, or a
// non-finite or tiny sum) one thread replays the reference's sequential sum.
// Each square of a float is exact in double, so S' and T differ only by
// the sums' roundings.
constexpr int NORM_THREADS = 256;

DSV4CU_DEV float norm_inv(double sum, int n, float eps)
{
    return __double2float_rn(1.0 / sqrt(__dadd_rn(__ddiv_rn(sum, (double)n), (double)eps)));
}

__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(float *__restrict__ y, const float *__restrict__ x,
                                                               const float *__restrict__ w, int n, float eps)
{
    __shared__ double red[NORM_THREADS / 32];
    __shared__ float s_inv;
    const float *xr = x + (size_t)blockIdx.x * n;
    float *yr = y + (size_t)blockIdx.x * n;
    double acc = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double v = (double)xr[i];
        acc = __dadd_rn(acc, __dmul_rn(v, v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) s = __dadd_rn(s, red[i]);
        // Relative bound on |T - S'|: (n - 1) + n / threads + log2(threads) + 5 unit
        // roundoffs, doubled, plus the two roundings of the interval ends.
        const double g = (2.0 * n + 64.0) * 0x1.0p-53;
        bool done = false;
        if (isfinite(s) && s > 0x1.0p-900) {
            const float lo = norm_inv(s * (1.0 + g) * (1.0 + 0x1.0p-50), n, eps);
            const float hi = norm_inv(s * (1.0 - g) * (1.0 - 0x1.0p-50), n, eps);
            if (lo == hi) {
                s_inv = lo;
                done = true;
            }
        }
        if (!done) {
            double t = 0.0;
            for (int i = 0; i < n; i++) {
                const double v = (double)xr[i];
                t = __dadd_rn(t, __dmul_rn(v, v));
            }
            s_inv = norm_inv(t, n, eps);
        }
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = __fmul_rn(w[i], __fmul_rn(xr[i], inv));
}

// ------------------------------------------------------------- argmax
// Greedy pick over a row of logits, as the reference's argmax
// (src/90_cli/dsv4_decode.c:128-133): best starts at 0 and moves to v only
// when lg[v] > lg[best]. So a NaN at index 0 keeps 0; other NaNs are never
// picked; -0.0 and +0.0 tie; ties go to the lower index. One CTA per row:
// each thread keeps (order key, index) over a strided range, then the CTA
// reduces with larger key first, lower index on a tie.
constexpr int ARGMAX_THREADS = 1024;

DSV4CU_DEV void argmax_take(uint32_t &bk, int &bi, uint32_t k, int i)
{
    if (k > bk || (k == bk && i < bi)) {
        bk = k;
        bi = i;
    }
}

__global__ void __launch_bounds__(ARGMAX_THREADS) argmax_kernel(const float *__restrict__ logits, int n,
                                                                 int *__restrict__ best)
{
    __shared__ uint32_t s_k[ARGMAX_THREADS / 32];
    __shared__ int s_i[ARGMAX_THREADS / 32];
    const float *lg = logits + (size_t)blockIdx.x * n;
    uint32_t bk = 0;            // below every non-NaN key (float_order_key(-inf) = 0x007FFFFF)
    int bi = 0x7FFFFFFF;
    for (int v = threadIdx.x; v < n; v += blockDim.x) {
        const float f = __ldg(lg + v);
        if (!isnan(f)) argmax_take(bk, bi, float_order_key(f), v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint32_t k = __shfl_xor_sync(0xFFFFFFFFu, bk, o);
        const int i = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        argmax_take(bk, bi, k, i);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        s_k[warp] = bk;
        s_i[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) argmax_take(bk, bi, s_k[w], s_i[w]);
        best[blockIdx.x] = (n <= 0 || isnan(__ldg(lg)) || bi == 0x7FFFFFFF) ? 0 : bi;
    }
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_route(int *idx, float *wts, float *scores, float *orig, const float *logits,
                            const float *bias, const int64_t *tid2eid, const int *token_ids, int n_experts,
                            int topk, float route_scale, int nt, void *stream)
{
    if (!idx || !wts || !logits) return dsv4cu_set_error(DSV4CU_ERR_ARG, "route: NULL argument");
    if (topk < 1 || topk > 16 || n_experts < 1 || n_experts > 32 * RMAX_PER_LANE)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "route: topk %d / n_experts %d out of range", topk, n_experts);
    if (!tid2eid && topk > n_experts) return dsv4cu_set_error(DSV4CU_ERR_ARG, "route: topk > n_experts");
    if (tid2eid && !token_ids) return dsv4cu_set_error(DSV4CU_ERR_ARG, "route: hash routing needs token_ids");
    if (nt <= 0) return DSV4CU_OK;
    const float *tab = router_table_get();
    if (!tab) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "route: router table setup failed");
    route_kernel<<<(nt + 3) / 4, 128, 0, (cudaStream_t)stream>>>(tab, idx, wts, scores, orig, logits, bias, tid2eid,
                                                                  token_ids, n_experts, topk, route_scale, nt);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_swiglu(float *y, const float *gate, const float *up, int n, float limit, void *stream)
{
    if (n <= 0) return DSV4CU_OK;
    if (!y || !gate || !up) return dsv4cu_set_error(DSV4CU_ERR_ARG, "swiglu: NULL argument");
    swiglu_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(y, gate, up, n, limit);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_indexer_offset(int *idxs, int n, int offset, void *stream)
{
    if (n <= 0) return DSV4CU_OK;
    offset_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(idxs, n, offset);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_quantize_fp8(uint8_t *w, uint8_t *s, const float *src, int rows, int cols, void *stream)
{
    if (!w || !s || !src || rows <= 0 || cols <= 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "quantize_fp8: bad args");
    dim3 grid((cols + 127) / 128, (rows + 127) / 128);
    quant_fp8_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(w, s, src, rows, cols);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_quantize_fp4(uint8_t *w, uint8_t *s, const float *src, int rows, int cols, void *stream)
{
    if (!w || !s || !src || rows <= 0 || cols <= 0 || cols % 32)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "quantize_fp4: bad args (cols must be a multiple of 32)");
    const long warps = (long)rows * (cols / 32);
    quant_fp4_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(w, s, src, rows, cols);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_fill_normal(float *dst, size_t n, uint64_t seed, float mean, float stdv, void *stream)
{
    if (!dst) return dsv4cu_set_error(DSV4CU_ERR_ARG, "fill_normal: NULL");
    if (!n) return DSV4CU_OK;
    const size_t pairs = (n + 1) / 2;
    fill_normal_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, (cudaStream_t)stream>>>(dst, n, seed, mean, stdv);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_round_bf16(float *x, size_t n, void *stream)
{
    if (!x) return dsv4cu_set_error(DSV4CU_ERR_ARG, "round_bf16: NULL");
    if (!n) return DSV4CU_OK;
    round_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, n);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_argmax(int *best, const float *logits, int n, int nt, void *stream)
{
    if (!best || !logits || n <= 0 || nt <= 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "argmax: bad args");
    argmax_kernel<<<(unsigned)nt, ARGMAX_THREADS, 0, (cudaStream_t)stream>>>(logits, n, best);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_head(dsv4cu_ctx *ctx, float *logits, int *best, const float *x, const dsv4cu_qmat *head, int nt,
                           void *stream)
{
    if (!ctx || !logits || !best || !x || !head) return dsv4cu_set_error(DSV4CU_ERR_ARG, "head: NULL argument");
    int r = dsv4cu_mmq(ctx, logits, x, head, nt, stream);
    if (r) return r;
    return dsv4cu_argmax(best, logits, head->rows, nt, stream);
}

extern "C" int dsv4cu_rmsnorm(float *y, const float *x, const float *w, int n, int nt, float eps, void *stream)
{
    if (!y || !x || !w || n <= 0 || nt <= 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "rmsnorm: bad args");
    rmsnorm_kernel<<<(unsigned)nt, NORM_THREADS, 0, (cudaStream_t)stream>>>(y, x, w, n, eps);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_rope_apply(dsv4cu_ctx *ctx, float *v, int nt, int nh, int head_dim, int rd, const float *cs,
                                 const float *sn, const int *pos, int table_half, int n_pos, int inverse,
                                 void *stream)
{
    if (!v || !cs || !sn || !pos || nt <= 0 || nh <= 0 || rd <= 0 || rd % 2 || rd > head_dim ||
        rd / 2 > table_half || n_pos <= 0)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "rope_apply: bad args");
    const long n = (long)nt * nh * (rd / 2);
    rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        v, nt, nh, head_dim, rd, cs, sn, pos, table_half, n_pos, inverse, ctx ? ctx->status : nullptr);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int dsv4cu_hc_post(float *y, const float *x, const float *residual, const float *post, const float *comb,
                              int nt, int hc, int hidden, void *stream)
{
    if (!y || !x || !residual || !post || !comb || nt <= 0 || hc <= 0 || hidden <= 0)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "hc_post: bad args");
    const long n = (long)nt * hc * hidden;
    hc_post_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(y, x, residual, post, comb, nt, hc,
                                                                                 hidden);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}
