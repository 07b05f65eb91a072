// tmap.h - TMA tensor maps for packed weight matrices.
//
// Weight bytes: a 2-D uint8 map over [rows][row_bytes] with 16-row x 128-byte
// boxes and the 128-byte swizzle (conflict-free shared-memory reads).
// FP4 1x32 scales: a 2-D uint8 map over [rows][cols/32] with 16 x 16 boxes,
// used when the scale grid is stageable (tmap_scales_stageable).
#pragma once
#include <cuda.h>

#include "../../include/dsv4cu.h"

namespace dsv4cu {

constexpr int TMAP_BOX_ROWS = 16;
constexpr int TMAP_BOX_BYTES = 128;

// True when the fast TMA path can stream this matrix: 16-byte aligned base,
// rows of at least one box and a whole number of 16-byte chunks.
bool tmap_weights_ok(const dsv4cu_qmat *q);
// True when the FP4 1x32 scale grid can ride in the stages with the weights.
bool tmap_scales_stageable(const dsv4cu_qmat *q);

// Encode the weight map (and the scale map when stageable). Returns a
// DSV4CU_* status; *staged tells whether the scale map was written.
int tmap_encode(const dsv4cu_qmat *q, CUtensorMap *wmap, CUtensorMap *smap, int *staged);

// A 2-D map of any element type: `inner` elements per row, `outer` rows of
// `row_bytes`, boxes of box_inner x box_rows, the given swizzle, zero fill
// outside the tensor.
int tmap_encode_2d(CUtensorMap *map, CUtensorMapDataType type, const void *base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle);

}  // namespace dsv4cu
