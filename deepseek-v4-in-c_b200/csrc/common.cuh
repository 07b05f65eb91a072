// common.cuh - shared device helpers for the dsv4cu library (sm_100a only).
//
// Numeric formats follow the reference's definitions exactly
// (src/10_compute/dsv4_quant.h:72-172):
//   E8M0  byte b -> 2^(b-127); b == 0 is the f32 subnormal 2^-127, b == 255 NaN.
//   E4M3  float8_e4m3fn: bias 7, no infinities, 0x7F/0xFF NaN, max 448.
//   E2M1  float4_e2m1fn: {0,.5,1,1.5,2,3,4,6} and negatives; the LOW nibble of a
//         byte is the even-indexed element.
// The hardware converters used below (cvt.rn.f16x2.e4m3x2, cvt.rn.f16x2.e2m1x2)
// widen these formats exactly: every e4m3 and e2m1 value is representable in f16.
#pragma once

#include <cuda_runtime.h>
#include <utility>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/dsv4cu.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "dsv4cu is written for sm_100a (B200) only"
#endif

#define DSV4CU_DEV __device__ __forceinline__

// ---------------------------------------------------------------- decoders
DSV4CU_DEV float e8m0_to_f32(uint32_t b)
{
    const uint32_t u = (b == 0xFFu) ? 0x7FC00000u : (b == 0u ? 0x00400000u : (b << 23));
    return __uint_as_float(u);
}

// Exact scalar E4M3 decode (used by the generic path and tests).
DSV4CU_DEV float e4m3_to_f32(uint32_t b)
{
    const uint32_t sign = (b & 0x80u) << 24, e = (b >> 3) & 15u, m = b & 7u;
    if (e == 15u && m == 7u) return __uint_as_float(sign | 0x7FC00000u);
    float v = (e == 0u) ? (float)m * 0.001953125f /* 2^-9 */
                        : __uint_as_float(((e + 120u) << 23) | (m << 20));
    return __uint_as_float(__float_as_uint(v) | sign);
}

DSV4CU_DEV float e2m1_to_f32(uint32_t nib)
{
    const uint32_t mag = nib & 7u;
    // 2*|v| is the integer {0,1,2,3,4,6,8,12}[mag], one byte per entry.
    const uint32_t twice = (uint32_t)((0x0C08060403020100ull >> (mag * 8)) & 0xFFu);
    const float v = (float)twice * 0.5f;
    return (nib & 8u) ? -v : v;
}

// Two e4m3 codes (low byte = first element) -> f16x2 (first element low).
// The float the reference's scalar FP8/FP4 matmul returns for a row whose
// result is NaN. Its double arithmetic carries the first NaN operand it meets,
// sign included, and its decoders give quiet NaNs: E4M3 0x7F -> 0x7FC00000,
// E4M3 0xFF -> 0xFFC00000, E8M0 0xFF -> 0x7FC00000 (src/10_compute/
// dsv4_quant.h:72-83 and the E4M3 table after it). The row's scale blocks are
// scanned in order: the first NaN weight code of the first block holding one
// gives its sign, else that block's NaN scale gives +NaN. A row with neither
// got its NaN from the activations (inf - inf, 0 x inf), for which x86 gives
// its default NaN 0xFFC00000; a NaN activation's own payload is not kept.
DSV4CU_DEV float ref_row_nan(const uint8_t *w_row, const uint8_t *s_row, int cols, int blk_c, bool fp4)
{
    for (int c0 = 0, b = 0; c0 < cols; c0 += blk_c, b++) {
        if (!fp4) {
            const int n = min(blk_c, cols - c0);
            for (int k = 0; k < n; k++) {
                const uint32_t code = w_row[c0 + k];
                if ((code & 0x7Fu) == 0x7Fu) return __uint_as_float(0x7FC00000u | ((code & 0x80u) << 24));
            }
        }
        if (s_row[b] == 0xFFu) return __uint_as_float(0x7FC00000u);
    }
    return __uint_as_float(0xFFC00000u);
}

DSV4CU_DEV uint32_t cvt_e4m3x2_f16x2(uint16_t two)
{
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(two));
    return r;
}

// Four e4m3 bytes -> two f16x2 (elements 0,1 and 2,3).
DSV4CU_DEV void cvt_e4m3x4(uint32_t w, uint32_t &lo, uint32_t &hi)
{
    lo = cvt_e4m3x2_f16x2((uint16_t)(w & 0xFFFFu));
    hi = cvt_e4m3x2_f16x2((uint16_t)(w >> 16));
}

// One byte of two e2m1 codes -> f16x2; the low nibble (even element) lands in
// the low half, matching the reference nibble order.
DSV4CU_DEV void cvt_e2m1x8(uint32_t w, uint32_t &h0, uint32_t &h1, uint32_t &h2, uint32_t &h3)
{
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3) : "r"(w));
}

// ------------------------------------------------------------ tensor core
// mma.sync m16n8k16, f16 x f16 -> f32. Fragment layout (PTX ISA):
//   A: a0 (row g, k 2c..2c+1) a1 (row g+8, k 2c..) a2 (row g, k 2c+8..) a3 (row g+8, k 2c+8..)
//   B: b0 (k 2c..2c+1, col g) b1 (k 2c+8..2c+9, col g)
//   C: c0,c1 (row g, col 2c, 2c+1) c2,c3 (row g+8, col 2c, 2c+1)
// with g = lane / 4 and c = lane % 4.
DSV4CU_DEV void mma_f16_16816(float &d0, float &d1, float &d2, float &d3,
                              uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                              uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
DSV4CU_DEV uint4 ld_stream16(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

DSV4CU_DEV float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Monotone uint32 key of a float for "larger float -> larger key"; -0.0 is
// canonicalised to +0.0 because the reference compares with < and >, under
// which the two zeros tie (src/10_compute/dsv4_topk.c:39-51).
DSV4CU_DEV uint32_t float_order_key(float f)
{
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------- host side
#define DSV4CU_CUDA_TRY(expr)                                                   \
    do {                                                                        \
        cudaError_t _e = (expr);                                                \
        if (_e != cudaSuccess) {                                                \
            dsv4cu_set_error(DSV4CU_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__,\
                             #expr, cudaGetErrorString(_e));                    \
            return DSV4CU_ERR_CUDA;                                             \
        }                                                                       \
    } while (0)

#define DSV4CU_LAUNCH_CHECK()                                                   \
    do {                                                                        \
        cudaError_t _e = cudaGetLastError();                                    \
        if (_e != cudaSuccess) {                                                \
            dsv4cu_set_error(DSV4CU_ERR_CUDA, "%s:%d launch: %s", __FILE__,     \
                             __LINE__, cudaGetErrorString(_e));                 \
            return DSV4CU_ERR_CUDA;                                             \
        }                                                                       \
    } while (0)

extern "C" int dsv4cu_set_error(int code, const char *fmt, ...);

namespace dsv4cu {

// Programmatic dependent launch (sm_90+): a kernel launched with
// launch_pdl may start while the previous kernel on the stream is still
// running; it must call pdl_wait() before it reads anything that kernel
// writes. pdl_trigger() lets the next kernel start launching once every CTA
// of this grid has executed it (or exited).
DSV4CU_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DSV4CU_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host-side per-device caches, so a call costs no attribute queries after
// the first: SmemLimit (one per call site) remembers the largest dynamic
// shared-memory limit set for a kernel on each device; device_sms() the SM
// count of the current device.
struct SmemLimit {
    int set[64];
};
static inline cudaError_t smem_limit(SmemLimit &c, const void *kernel, int bytes)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool cache = dev >= 0 && dev < 64;
    if (cache && c.set[dev] >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && cache) c.set[dev] = bytes;
    return e;
}
static inline int device_sms()
{
    static int n[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!n[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        n[dev] = v > 0 ? v : 148;
    }
    return n[dev];
}

template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                     Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace dsv4cu
