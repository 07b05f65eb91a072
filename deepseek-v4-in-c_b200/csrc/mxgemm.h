// mxgemm.h - the tcgen05 block-scaled GEMM (mxgemm.cu) for other translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/dsv4cu.h"

namespace dsv4cu {

// A packed matrix prepared for the tensor-core path: its TMA map and its
// scale factors rearranged into the TMEM block layout (owned).
struct MxMat {
    dsv4cu_qmat q;
    CUtensorMap ta;
    uint8_t *sfa;      // [tiles_m][kc][512]
    int fp4, kc, tiles_m;
};

struct MxArgs {
    const uint8_t *sfa;   // weight scale blocks [tiles_m][kc][512]
    const uint8_t *sfb;   // activation scale blocks [tiles_n][kc][NB/128 rounded up][512]
    int kc;               // K / 128
    int tiles_m, tiles_n;
    int rows, nt, tpt, terms;
    float *y;
    int ldy;
    uint32_t idesc;       // instruction descriptor, scale ids 0
    uint32_t a_tx;        // global bytes of one A box
    int *err;
};

bool mx_supported(const dsv4cu_qmat *q);
int mx_prepare(MxMat *m, const dsv4cu_qmat *q, cudaStream_t st);
void mx_release(MxMat *m);
size_t mx_workspace(const MxMat *m, int nt, int terms);
int mx_gemm(const MxMat *m, float *y, const float *x, int nt, int terms, void *ws, int sms, int *err,
            cudaStream_t st);

}  // namespace dsv4cu
