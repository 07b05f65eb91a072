// gemv.h - internal entry points of gemv.cu shared with other translation units.
#pragma once
#include <cuda_runtime.h>

#include "../../include/dsv4cu.h"
#include "gemv_core.cuh"

namespace dsv4cu {

int row_bytes_of(int wdt, int cols);
MatArgs mat_args(const dsv4cu_qmat *q);
int xprep_launch(const float *x, int cols, int ldx_in, int nt, int ldx, uint16_t *xh, uint16_t *xl, float *xs,
                 cudaStream_t st);
size_t mmq_workspace(const dsv4cu_qmat *q, int nt, int sm_count);
size_t bf16_chain_workspace(int cols, int nt);
int bf16_chain_run(float *y, const float *x, const dsv4cu_qmat *q, int nt, void *ws, int *err, cudaStream_t st);
int mmq_run(dsv4cu_ctx *ctx, float *y, const float *x, const dsv4cu_qmat *q, int nt,
            cudaStream_t st, void *ws, int *counters);

}  // namespace dsv4cu
