// tma_gemv.cuh - TMA-staged packed GEMV tile for sm_100a.
//
// A CTA = 8 consumer warps + 1 producer warp. Consumer warp w owns a "stream":
// 16 consecutive weight rows of one matrix, from byte kb0 of each row, L bytes
// long (the eight streams of a CTA share L). The producer warp moves the
// streams through shared memory in stages of 256 bytes per row with tensor-map
// TMA loads (cp.async.bulk.tensor.2d): per stage and stream, two 16-row x
// 128-byte boxes of weights (128-byte swizzle) and, for FP4 1x32 scales, one
// 16 x 16 box of scale bytes - 24 TMA instructions per stage for the whole
// CTA. Completion is counted on an mbarrier; STAGES stages are in flight.
//
// Consumers read a stage with the fragment mapping of gemv_core.cuh (lane
// (g, c): rows g and g+8, 16-byte chunk c of each 64-byte segment), widen
// e4m3 / e2m1 to f16 with the hardware converters, and reduce with mma.sync
// against the [hi | lo] activation operand; each chunk's exact partial is
// scaled by its E8M0 block scale in fp32.
//
// Every wait is bounded: a wait that exceeds its spin limit records an error
// code in *err and the CTA stops issuing work (no trap, no endless loop).
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "gemv_core.cuh"

namespace dsv4cu {

// ------------------------------------------------------------- PTX helpers
DSV4CU_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

DSV4CU_DEV void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

DSV4CU_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

DSV4CU_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

DSV4CU_DEV void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// A waiting thread is suspended until the phase completes or the hint (ns)
// runs out, so warps parked on a barrier leave the SM's issue slots to the
// warps that work (a dependent grid's CTAs wait beside the primary's).
constexpr uint32_t MBAR_SUSPEND_NS = 1000000u;

DSV4CU_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "n"(MBAR_SUSPEND_NS) : "memory");
    return ok != 0;
}

DSV4CU_DEV uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// A healthy stage lands in microseconds; 2 s means the pipeline is broken.
constexpr uint64_t MBAR_TIMEOUT_NS = 2000000000ull;

// Bounded wait: returns false (and records code in *err) once the barrier has
// not completed for MBAR_TIMEOUT_NS of wall time.
DSV4CU_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > MBAR_TIMEOUT_NS) break;
    }
    if (err) atomicCAS(err, 0, code);
    return false;
}

// L2 policy for streamed weights: evict first. Weights are read once per
// step and exceed the L2, so under the default policy they push out what
// the next kernels reuse (their code, routing tables, activations, partial
// buffers); with this hint those stay resident.
DSV4CU_DEV uint64_t l2_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

DSV4CU_DEV uint64_t l2_evict_normal()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 2-D tensor-map load with an L2 cache policy (l2_evict_first / l2_evict_normal). No multicast.
DSV4CU_DEV void tma_load_2d_hint(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar, uint64_t pol)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
                 " [%0], [%1, {%2, %3}], [%4], %5;"
                 ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
                 : "memory");
}

// 2-D tensor-map load of one box into shared memory; completion counted in
// bytes on `bar`. x (bytes) is always a multiple of 16. No multicast.
DSV4CU_DEV void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
                 : "memory");
}

// -------------------------------------------------------------- the tile
struct Stream {
    MatArgs m;              // the matrix (row_bytes, scales for the unstaged path)
    const CUtensorMap *tw;  // weight map, 16 x 128 B boxes, 128-byte swizzle
    const CUtensorMap *ts;  // FP4 1x32 scale map (16 x 16 boxes) or nullptr
    int row0;               // first of 16 rows
    int kb0;                // first byte of each row (a multiple of 16)
};

constexpr int TMA_SB = 256;                      // bytes per row per stage (two boxes)
constexpr int TMA_BOX_HALF = 128;
constexpr int TMA_STREAM_BYTES = 16 * TMA_SB;    // weight bytes per stream per stage
constexpr int TMA_SCALE_BYTES = 16 * 16;         // scale bytes per stream per stage

template <int STAGES>
struct TmaSmem {
    static constexpr int DATA = 8 * TMA_STREAM_BYTES;   // 32 KB, 1024-byte aligned boxes
    static constexpr int SCL = 8 * TMA_SCALE_BYTES;     // 2 KB
    static constexpr int BYTES = 1024 /* alignment slack */ + STAGES * (DATA + SCL) + 2 * STAGES * 8;
};

// Runs the 8 streams of a CTA over L bytes per row (L a multiple of 16; the
// last stage of a part may be partial and is masked by the consumers).
// Consumer warp w (w < 8) returns per-lane partials in acc (quad_sum still
// needed); the producer warp (w == 8) returns with acc untouched. Scale bytes
// are staged with the weights when every stream has a scale map (FP4 1x32);
// otherwise scales come through L1.
template <int FMT, int NT, int STAGES>
DSV4CU_DEV void tma_gemv_streams(unsigned char *smem_raw, const Stream *streams, int L, const XArgs &x, int nvalid,
                                 float (&acc)[NT][2], int *err)
{
    using SM = TmaSmem<STAGES>;
    unsigned char *base = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char *data = base;                                  // [STAGES][8][16 x 256] swizzled
    unsigned char *scl = base + STAGES * SM::DATA;               // [STAGES][8][16 x 16]
    uint64_t *full = reinterpret_cast<uint64_t *>(scl + STAGES * SM::SCL);
    uint64_t *empty = full + STAGES;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nst = (L + TMA_SB - 1) / TMA_SB;
    // Scale boxes start at byte/16 of the row: whole 16-byte runs need
    // stage-aligned (256-byte) part starts.
    bool staged = true;
#pragma unroll
    for (int w = 0; w < 8; w++) staged = staged && streams[w].ts != nullptr && (streams[w].kb0 % TMA_SB) == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 8);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 8) {
        // ---------------- producer: lane i < 8 loads stream i's boxes
        const bool live = lane < 8;
        const Stream st = streams[live ? lane : 0];
        const bool rows_in = live && st.row0 < st.m.rows;
        for (int k = 0; k < nst; k++) {
            const int s = k % STAGES;
            if (k >= STAGES) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(empty + s, ((k / STAGES) - 1) & 1, err, 0x101);
                ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
                if (!ok) {
                    if (lane == 0) abort_flag = 1;
                    break;
                }
            }
            const int x0 = st.kb0 + k * TMA_SB;
            const bool b0 = rows_in && x0 < st.m.row_bytes;
            const bool b1 = rows_in && x0 + TMA_BOX_HALF < st.m.row_bytes;
            uint32_t bytes = (b0 ? 2048u : 0u) + (b1 ? 2048u : 0u) + ((staged && b0) ? 256u : 0u);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) bytes += __shfl_xor_sync(0xFFFFFFFFu, bytes, o);
            if (lane == 0) mbar_arrive_expect_tx(full + s, bytes);
            __syncwarp();
            unsigned char *dst = data + s * SM::DATA + lane * TMA_STREAM_BYTES;
            if (b0) tma_load_2d(dst, st.tw, x0, st.row0, full + s);
            if (b1) tma_load_2d(dst + 2048, st.tw, x0 + TMA_BOX_HALF, st.row0, full + s);
            if (staged && b0)
                tma_load_2d(scl + s * SM::SCL + lane * TMA_SCALE_BYTES, st.ts, x0 / 16, st.row0, full + s);
        }
        return;
    }

    // ---------------- consumers
    const Stream st = streams[warp];
    const MatArgs &m = st.m;
    const int g = lane >> 2, c = lane & 3;
    const int r0 = st.row0 + g, r1 = r0 + 8;
    const bool v0 = r0 < m.rows, v1 = r1 < m.rows;
    const bool bact = (g >> 1) == c;
    const uint16_t *xsel = (g & 1) ? x.xl : x.xh;
    const int sr0 = (v0 ? r0 : 0) / m.blk_r, sr1 = (v1 ? r1 : 0) / m.blk_r;

    for (int k = 0; k < nst; k++) {
        const int s = k % STAGES;
        const bool ok = mbar_wait(full + s, (k / STAGES) & 1, err, 0x102);
        if (!__all_sync(0xFFFFFFFFu, ok) || abort_flag) break;
        const unsigned char *sd = data + s * SM::DATA + warp * TMA_STREAM_BYTES;
        const unsigned char *ss = scl + s * SM::SCL + warp * TMA_SCALE_BYTES;
        const int off = k * TMA_SB;
#pragma unroll
        for (int seg = 0; seg < TMA_SB / 64; seg++) {
            const int lb = seg * 64 + c * 16;                // byte within the stage row
            const int boff = st.kb0 + off + lb;              // byte within the matrix row
            const bool cvalid = (off + lb) < L && boff < m.row_bytes;
            if (!__any_sync(0xFFFFFFFFu, cvalid)) break;
            // box lb / 128, 16-byte chunk j of the 128-byte line, swizzled by row
            const int box = lb >> 7, j = (lb & 127) >> 4;
            const uint4 w0 = (cvalid && v0)
                ? *reinterpret_cast<const uint4 *>(sd + box * 2048 + g * 128 + ((j ^ (g & 7)) << 4))
                : make_uint4(0, 0, 0, 0);
            const uint4 w1 = (cvalid && v1)
                ? *reinterpret_cast<const uint4 *>(sd + box * 2048 + (g + 8) * 128 + ((j ^ ((g + 8) & 7)) << 4))
                : make_uint4(0, 0, 0, 0);
            const int k0 = Fmt<FMT>::elem(boff);
            float sc0 = 1.0f, sc1 = 1.0f;
            if constexpr (FMT == DSV4CU_WFP4) {
                if (staged) {
                    sc0 = (cvalid && v0) ? e8m0_to_f32(ss[g * 16 + (lb >> 4)]) : 0.0f;
                    sc1 = (cvalid && v1) ? e8m0_to_f32(ss[(g + 8) * 16 + (lb >> 4)]) : 0.0f;
                } else {
                    const int kb = cvalid ? k0 / m.blk_c : 0;
                    sc0 = (cvalid && v0) ? e8m0_to_f32(__ldg(m.s + (size_t)sr0 * m.s_cols + kb)) : 0.0f;
                    sc1 = (cvalid && v1) ? e8m0_to_f32(__ldg(m.s + (size_t)sr1 * m.s_cols + kb)) : 0.0f;
                }
            } else if constexpr (FMT == DSV4CU_WFP8) {
                const int kb = cvalid ? k0 / m.blk_c : 0;
                sc0 = (cvalid && v0) ? e8m0_to_f32(__ldg(m.s + (size_t)sr0 * m.s_cols + kb)) : 0.0f;
                sc1 = (cvalid && v1) ? e8m0_to_f32(__ldg(m.s + (size_t)sr1 * m.s_cols + kb)) : 0.0f;
            }
            // Per-token activation row and chunk partials C[.][2c] / C[.][2c+1].
            const uint16_t *xb[NT];
            float e[NT][4];
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const int xr = (t < nvalid) ? (x.tok ? __ldg(x.tok + t) : t) : 0;
                xb[t] = xsel + (size_t)xr * x.ldx + k0;
                e[t][0] = e[t][1] = e[t][2] = e[t][3] = 0.0f;
            }
            const uint32_t q0[4] = {w0.x, w0.y, w0.z, w0.w}, q1[4] = {w1.x, w1.y, w1.z, w1.w};
            // One 32-bit word at a time: widen the A fragments it holds and run
            // its MMAs for every token before widening the next word.
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if constexpr (FMT == DSV4CU_WFP4) {
                    uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
                    cvt_e2m1x8(q0[i], a0, a1, a2, a3);
                    cvt_e2m1x8(q1[i], b0, b1, b2, b3);
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        if (t >= nvalid) break;
                        uint4 b = make_uint4(0u, 0u, 0u, 0u);
                        if (bact && cvalid) b = __ldg(reinterpret_cast<const uint4 *>(xb[t] + 8 * i));
                        mma_f16_16816(e[t][0], e[t][1], e[t][2], e[t][3], a0, b0, a1, b1, b.x, b.y);
                        mma_f16_16816(e[t][0], e[t][1], e[t][2], e[t][3], a2, b2, a3, b3, b.z, b.w);
                    }
                } else {
                    static_assert(FMT == DSV4CU_WFP8, "the TMA GEMV streams FP4 or FP8 weights");
                    uint32_t glo, ghi, hlo, hhi;
                    cvt_e4m3x4(q0[i], glo, ghi);
                    cvt_e4m3x4(q1[i], hlo, hhi);
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        if (t >= nvalid) break;
                        uint2 b = make_uint2(0u, 0u);
                        if (bact && cvalid) b = __ldg(reinterpret_cast<const uint2 *>(xb[t] + 4 * i));
                        mma_f16_16816(e[t][0], e[t][1], e[t][2], e[t][3], glo, hlo, ghi, hhi, b.x, b.y);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t >= nvalid) break;
                const int xr = x.tok ? __ldg(x.tok + t) : t;
                const float xsv = cvalid ? __ldg(x.xs + (size_t)xr * (x.ldx >> 5) + (k0 >> 5)) : 0.0f;
                acc[t][0] = fmaf((e[t][0] + e[t][1]) * xsv, sc0, acc[t][0]);
                acc[t][1] = fmaf((e[t][2] + e[t][3]) * xsv, sc1, acc[t][1]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + s);
    }
}

}  // namespace dsv4cu
