// gemv_core.cuh - bandwidth-bound packed GEMV tile for sm_100a.
//
// One warp computes the dot products of 16 weight rows against up to NT token
// vectors over a contiguous range of 64-byte row segments.
//
//   * Weights stream from HBM as 16-byte loads per lane (ld.global.nc with no
//     L1 allocation): lane (g, c) = (lane/4, lane%4) reads chunk c of the
//     segment for rows g and g+8, so a warp load covers 16 rows x 64 bytes.
//   * The chunk is widened in registers with the exact hardware converters
//     (e4m3 / e2m1 -> f16) straight into mma.sync A fragments.
//     K positions inside an MMA are a free permutation of a dot product, so a
//     lane feeds its own contiguous chunk.
//   * The activation enters as B = [hi | lo] f16 pairs (x split exactly after
//     a power-of-two prescale per 32 elements). Column 2c of B carries the hi
//     part and column 2c+1 the lo part of THREAD-COLUMN c's chunk only, so the
//     accumulator C[r][2c] + C[r][2c+1] that lane (g, c) holds is exactly its
//     own chunk's partial dot product. One chunk never straddles a scale block,
//     so the E8M0 block scale (and the activation prescale) is applied to that
//     partial in fp32, per block, like the reference (dsv4_matmul_fp8.c:87-88,
//     dsv4_matmul_fp4.c:66-69): acc += part * 2^-P * scale.
//
// The tensor core is only the reduction engine here; the bound is HBM.
#pragma once

#include "common.cuh"

namespace dsv4cu {

struct MatArgs {
    const uint8_t *w;
    const uint8_t *s;
    int rows, cols;
    int blk_r, blk_c;
    int s_cols;     // ceil(cols / blk_c): scale grid row length
    int row_bytes;  // stored bytes per weight row (multiple of 16)
};

// Activation operand: per token row, f16 hi and lo halves and the
// per-32 power-of-two factor 2^-P that undoes the prescale.
struct XArgs {
    const uint16_t *xh;
    const uint16_t *xl;
    const float *xs;
    int ldx;        // elements per token row, multiple of 32
    const int *tok; // optional: tile token t reads activation row tok[t]
};

template <int FMT> struct Fmt {
    // Logical elements in one 16-byte chunk, and MMAs (4 elements each) per chunk.
    static_assert(FMT == DSV4CU_WFP4 || FMT == DSV4CU_WFP8, "FP4 or FP8 weights");
    static constexpr int CE = FMT == DSV4CU_WFP4 ? 32 : 16;
    static constexpr int MMAS = CE / 4;
    // element offset of byte offset b
    static DSV4CU_DEV int elem(int b) { return FMT == DSV4CU_WFP4 ? 2 * b : b; }
};

// Host-side check that the fast path covers a geometry (BF16 weights take
// the exact double path of gemv_bf16.cu instead).
static inline bool fast_geometry(int wdt, int cols, int blk_r, int blk_c)
{
    if (wdt == DSV4CU_WFP8) return cols % 16 == 0 && blk_c > 0 && blk_c % 16 == 0 && blk_r > 0;
    if (wdt == DSV4CU_WFP4) return cols % 32 == 0 && blk_c > 0 && blk_c % 32 == 0 && blk_r > 0;
    return false;
}

// A fragments of MMA j (elements 4j..4j+3 of the chunk) for one row.
template <int FMT>
DSV4CU_DEV void decode_chunk(const uint4 &q, uint32_t (&lo)[Fmt<FMT>::MMAS], uint32_t (&hi)[Fmt<FMT>::MMAS])
{
    const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
    if constexpr (FMT == DSV4CU_WFP4) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t h0, h1, h2, h3;
            cvt_e2m1x8(wv[i], h0, h1, h2, h3);
            lo[2 * i] = h0; hi[2 * i] = h1;
            lo[2 * i + 1] = h2; hi[2 * i + 1] = h3;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) cvt_e4m3x4(wv[i], lo[i], hi[i]);
    }
}

// Accumulate 16 rows [row0, row0+16) x segments [seg_begin, seg_end) into
// acc[t][0] (row g) and acc[t][1] (row g+8) for tokens t < min(NT, nt_valid).
// The caller still has to sum acc over the four lanes of a row (c = 0..3).
template <int FMT, int NT, int DEPTH>
DSV4CU_DEV void gemv_tile16(const MatArgs &m, int row0, int seg_begin, int seg_end,
                            const XArgs &x, int nt_valid, float (&acc)[NT][2])
{
    constexpr int MM = Fmt<FMT>::MMAS;
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int r0 = row0 + g, r1 = r0 + 8;
    const bool v0 = r0 < m.rows, v1 = r1 < m.rows;
    const uint8_t *p0 = m.w + (size_t)(v0 ? r0 : 0) * (size_t)m.row_bytes + c * 16;
    const uint8_t *p1 = m.w + (size_t)(v1 ? r1 : 0) * (size_t)m.row_bytes + c * 16;
    // B is nonzero only in columns 2c (hi) and 2c+1 (lo); lane (g, c) supplies
    // column g, which belongs to thread-column g/2.
    const bool bact = (g >> 1) == c;
    const uint16_t *xsel = (g & 1) ? x.xl : x.xh;
    const int sr0 = (v0 ? r0 : 0) / m.blk_r, sr1 = (v1 ? r1 : 0) / m.blk_r;

    uint4 q0[DEPTH], q1[DEPTH];
    const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int i = 0; i < DEPTH; i++) {
        const int s = seg_begin + i, off = s * 64 + c * 16;
        const bool cv = s < seg_end && off < m.row_bytes;
        q0[i] = (cv && v0) ? ld_stream16(p0 + s * 64) : z4;
        q1[i] = (cv && v1) ? ld_stream16(p1 + s * 64) : z4;
    }

    for (int sb = seg_begin; sb < seg_end; sb += DEPTH) {
#pragma unroll
        for (int i = 0; i < DEPTH; i++) {
            const int s = sb + i;
            if (s >= seg_end) break;
            const uint4 w0 = q0[i], w1 = q1[i];
            {
                const int sn = s + DEPTH, offn = sn * 64 + c * 16;
                const bool cvn = sn < seg_end && offn < m.row_bytes;
                q0[i] = (cvn && v0) ? ld_stream16(p0 + sn * 64) : z4;
                q1[i] = (cvn && v1) ? ld_stream16(p1 + sn * 64) : z4;
            }
            const int boff = s * 64 + c * 16;
            const bool cvalid = boff < m.row_bytes;
            const int k0 = Fmt<FMT>::elem(boff);

            uint32_t a0[MM], a2[MM], a1[MM], a3[MM];
            decode_chunk<FMT>(w0, a0, a2);
            decode_chunk<FMT>(w1, a1, a3);

            const int kb = cvalid ? k0 / m.blk_c : 0;
            const float sc0 = (cvalid && v0) ? e8m0_to_f32(__ldg(m.s + (size_t)sr0 * m.s_cols + kb)) : 0.0f;
            const float sc1 = (cvalid && v1) ? e8m0_to_f32(__ldg(m.s + (size_t)sr1 * m.s_cols + kb)) : 0.0f;
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t >= nt_valid) break;
                const int xr = x.tok ? __ldg(x.tok + t) : t;
                const uint16_t *xb = xsel + (size_t)xr * x.ldx + k0;
                float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
                for (int j = 0; j < MM; j++) {
                    uint2 b = make_uint2(0u, 0u);
                    if (bact && cvalid) b = __ldg(reinterpret_cast<const uint2 *>(xb + 4 * j));
                    mma_f16_16816(d0, d1, d2, d3, a0[j], a1[j], a2[j], a3[j], b.x, b.y);
                }
                const float xsv = cvalid ? __ldg(x.xs + (size_t)xr * (x.ldx >> 5) + (k0 >> 5)) : 0.0f;
                acc[t][0] = fmaf((d0 + d1) * xsv, sc0, acc[t][0]);
                acc[t][1] = fmaf((d2 + d3) * xsv, sc1, acc[t][1]);
            }
        }
    }
}

// Sum a per-lane partial over the four lanes (c = 0..3) of its row; the
// result is valid in lane c == 0.
DSV4CU_DEV float quad_sum(float v)
{
    v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
    v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
    return v;
}

}  // namespace dsv4cu
