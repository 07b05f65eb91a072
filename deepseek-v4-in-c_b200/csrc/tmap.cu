// tmap.cu - host-side encoding of the TMA tensor maps (see tmap.h).
#include <string.h>

#include "common.cuh"
#include "gemv.h"
#include "tmap.h"

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

}  // namespace dsv4cu
