// tmap.cu - host-side encoding of the TMA tensor maps (see tmap.h).
#include <string.h>

#include "common.cuh"
#include "gemv.h"
#include "tmap.h"
#include "stream_mv.cuh"

namespace dsv4cu {

// The driver entry point is looked up through the runtime, so the library has
// no link-time dependency on libcuda (it still loads on machines without a GPU).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

int tmap_encode_2d(CUtensorMap *map, CUtensorMapDataType type, const void *base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, type, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled(2-D): %d", (int)r);
    return DSV4CU_OK;
}

bool tmap_weights_ok(const dsv4cu_qmat *q)
{
    const int rb = row_bytes_of(q->wdt, q->cols);
    return q->w && ((uintptr_t)q->w & 15u) == 0 && rb >= TMAP_BOX_BYTES && rb % 16 == 0 && q->rows > 0;
}

bool tmap_scales_stageable(const dsv4cu_qmat *q)
{
    if (q->wdt != DSV4CU_WFP4 || q->blk_r != 1 || q->blk_c != 32 || !q->s) return false;
    const int s_cols = q->cols / 32;
    return q->cols % 32 == 0 && s_cols % 16 == 0 && ((uintptr_t)q->s & 15u) == 0;
}

int tmap_encode(const dsv4cu_qmat *q, CUtensorMap *wmap, CUtensorMap *smap, int *staged)
{
    *staged = 0;
    EncodeTiledFn cuTensorMapEncodeTiled = encode_fn();
    if (!cuTensorMapEncodeTiled) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if (!tmap_weights_ok(q)) return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "tensor map: matrix not streamable");
    const cuuint64_t rb = (cuuint64_t)row_bytes_of(q->wdt, q->cols);
    cuuint64_t dims[2] = {rb, (cuuint64_t)q->rows};
    cuuint64_t strides[1] = {rb};
    cuuint32_t box[2] = {TMAP_BOX_BYTES, TMAP_BOX_ROWS};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = cuTensorMapEncodeTiled(wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(q->w), dims,
                                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled(weights): %d", (int)r);
    if (smap && tmap_scales_stageable(q)) {
        const cuuint64_t sc = (cuuint64_t)(q->cols / 32);
        cuuint64_t sdims[2] = {sc, (cuuint64_t)q->rows};
        cuuint64_t sstr[1] = {sc};
        cuuint32_t sbox[2] = {16, TMAP_BOX_ROWS};
        r = cuTensorMapEncodeTiled(smap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(q->s), sdims, sstr,
                                   sbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled(scales): %d", (int)r);
        *staged = 1;
    }
    return DSV4CU_OK;
}

// Streamed GEMV maps (stream_mv.cuh). Weights: 3-D uint8 view of
// [rows][row_bytes] as (128-byte chunk piece, row, chunk) with strides
// (row_bytes, 128), box 128 x 32 x min(8, chunks), 128-byte swizzle: one copy
// moves 32 rows x up to 1 KB of row. FP4 scales of rows longer than one
// stage: 2-D [rows][cols / 32] with 64 x 32 boxes.
int smv_encode(const dsv4cu_qmat *q, CUtensorMap *wmap, CUtensorMap *smap)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const int rb = row_bytes_of(q->wdt, q->cols), chunks = rb / 128;
    cuuint64_t dims[3] = {128, (cuuint64_t)q->rows, (cuuint64_t)chunks};
    cuuint64_t strides[2] = {(cuuint64_t)rb, 128};
    cuuint32_t box[3] = {128, SMV_ROWS, (cuuint32_t)(chunks < 8 ? chunks : 8)}, es[3] = {1, 1, 1};
    CUresult r = enc(wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(q->w), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled(stream weights): %d", (int)r);
    memset(smap, 0, sizeof *smap);
    if (q->wdt == DSV4CU_WFP4 && rb > 1024) {
        const int sl = q->cols / 32;
        cuuint64_t sd[2] = {(cuuint64_t)sl, (cuuint64_t)q->rows};
        cuuint64_t ss[1] = {(cuuint64_t)sl};
        cuuint32_t sb[2] = {64, SMV_ROWS}, se[2] = {1, 1};
        r = enc(smap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(q->s), sd, ss, sb, se,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled(stream scales): %d", (int)r);
    }
    return DSV4CU_OK;
}

}  // namespace dsv4cu
