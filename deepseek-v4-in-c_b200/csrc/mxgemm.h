// mxgemm.h - host side of the tcgen05 block-scaled GEMM shared by mxgemm.cu
// (dense products) and moe_mx.cu (the MoE layer).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/dsv4cu.h"

namespace dsv4cu {

// A packed matrix prepared for the tensor-core path: its TMA map (128 x 128
// element boxes, 128-byte swizzle) and its scale factors rearranged into the
// TMEM block layout: [tiles_m][kc][512] bytes, byte (m % 32) * 16 + (m / 32)
// * 4 + kb of block (row tile, K chunk) = scale of row m, K block kb.
struct MxMat {
    dsv4cu_qmat q;
    CUtensorMap ta;
    uint8_t *sfa;
    int fp4, kc, tiles_m;
    int owns_sfa;
};

// Column tiling of one launch: NB B columns per tile = terms x tpt tokens
// (rounded), KB 128-wide K chunks per pipeline stage.
struct MxTiling {
    int NB, tpt, tiles_n, KB;
};

// dsv4cu_mmq (and the reference-signature matmuls built on it) hands
// products of at least MX_MMQ_MIN_TOKENS tokens to the tensor-core GEMM with
// MX_MMQ_TERMS exact activation terms (results within ~1e-6 of fp32).
constexpr int MX_MMQ_MIN_TOKENS = 1;
constexpr int MX_MMQ_TERMS = 4;

bool mx_supported(const dsv4cu_qmat *q);
size_t mx_sfa_bytes(const dsv4cu_qmat *q);
// sfa_buf: caller-owned block of mx_sfa_bytes(q) device bytes, or NULL to
// allocate one owned by the MxMat.
int mx_prepare(MxMat *m, const dsv4cu_qmat *q, uint8_t *sfa_buf, cudaStream_t st);
void mx_release(MxMat *m);
int mx_encode_kmajor(CUtensorMap *map, const void *base, bool fp4, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_rows);
// The B-operand tensor map of an activation buffer (e4m3 rows of `inner`
// bytes, box_rows-row boxes), from a small per-process cache keyed by
// address, shape and device: workspace buffers repeat call after call.
int mx_cached_bmap(CUtensorMap *out, const void *base, uint64_t inner, uint64_t outer, uint32_t box);
MxTiling mx_tiling(int nt, int terms, int nb_req, int kb_req, int kc);
// Split-K segments of one dense product: at most MX_MAX_SEGMENTS.
constexpr int MX_MAX_SEGMENTS = 16;
int mx_device_sms();
size_t mx_workspace(const MxMat *m, int nt, int terms, int sms);
// ev (optional): three events recorded before the activation split, before
// the GEMM and after it.
int mx_gemm(const MxMat *m, float *y, const float *x, int nt, int terms, int nb_req, int kb_req, void *ws, int sms,
            int *err, cudaStream_t st, cudaEvent_t *ev = nullptr);

}  // namespace dsv4cu
