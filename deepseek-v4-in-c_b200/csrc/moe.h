// moe.h - the prepared MoE layer shared by the two decode paths:
// moe_decode.cu (CUDA-core GEMV tiles) and moe_mx.cu (tcgen05 block-scaled MMA).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/dsv4cu.h"

namespace dsv4cu {

// Device view for the CUDA-core path: expert e (e == n_experts is the shared
// expert) has matrices m = 0 (w1), 1 (w3), 2 (w2); maps[6e + 2m] is the weight
// map, maps[6e + 2m + 1] the FP4 scale map, valid when staged[3e + m].
struct MoeDev {
    const dsv4cu_expert *experts;   // [n_experts + 1], shared last
    const CUtensorMap *maps;
    const int *staged;
    int n_experts, has_shared;
};

// Device view for the tensor-core path, matrix index 3e + m as above: the
// A-operand tensor map (128 x 128 boxes), the scale blocks in TMEM layout and
// whether the matrix is FP4 (else FP8).
struct MoeMxDev {
    const CUtensorMap *maps;
    const uint8_t *const *sfa;
    const int *fp4;
};

}  // namespace dsv4cu

struct dsv4cu_moe {
    int n_experts, hidden, inter, has_shared, device;
    void *dev_block;                // experts + maps + staged, one allocation
    dsv4cu::MoeDev view;
    // Tensor-core path (mx_ok == 0 when a matrix does not qualify).
    int mx_ok;
    int sms;                        // SM count of the layer's device (sizes the tensor-core work split)
    // Streamed decode path (moe_stream.cu): every matrix readable by the
    // streamer (stream_mv.cuh); used for one or two tokens. smv_maps: per
    // matrix 3e + m (m = w1, w3, w2) its weight map and FP4 scale map.
    int smv_ok;
    int path;                       // DSV4CU_MOE_PATH_* chosen by dsv4cu_moe_set_path
    void *smv_block;
    const CUtensorMap *smv_maps;
    void *mx_block;                 // maps + scale blocks + pointer table, one allocation
    dsv4cu::MoeMxDev mx;
};

namespace dsv4cu {

// Prepares the tensor-core view of a layer whose n_experts + 1 experts
// (shared last, a copy of expert 0 when there is none) are given on the host.
int moe_mx_prepare(dsv4cu_moe *L, const dsv4cu_expert *hexp);
void moe_mx_release(dsv4cu_moe *L);
size_t moe_mx_workspace(const dsv4cu_moe *L, int topk, int nt);
int moe_mx_decode(const dsv4cu_moe *L, float *out, const float *x, const float *logits, const float *bias,
                  const int64_t *tid2eid, const int *token_ids, int topk, float route_scale, float limit, int nt,
                  int *idx_out, float *wts_out, void *ws, int *counters, int *status, int sms, cudaStream_t st,
                  cudaEvent_t *ev);

size_t moe_mx_prefill_workspace(const dsv4cu_moe *L, int topk, int nt, int terms);
int moe_mx_prefill(const dsv4cu_moe *L, float *out, const float *x, const float *logits, const float *bias,
                   const int64_t *tid2eid, const int *token_ids, int topk, float route_scale, float limit, int nt,
                   int terms, int *idx_out, float *wts_out, void *ws, int *status, int sms, cudaStream_t st,
                   cudaEvent_t *ev);

bool smv_moe_layer_ok(const dsv4cu_expert *hexp, int n_experts, int hidden, int inter);
int smv_moe_prepare(dsv4cu_moe *L, const dsv4cu_expert *hexp);
size_t smv_moe_workspace(const dsv4cu_moe *L, int topk, int nt);
int smv_moe_decode(const dsv4cu_moe *L, float *out, const float *x, const float *logits, const float *bias,
                   const int64_t *tid2eid, const int *token_ids, int topk, float route_scale, float limit, int nt,
                   int *idx_out, float *wts_out, void *ws, int *status, int sms, cudaStream_t st, cudaEvent_t *ev);

size_t moe_mx_rows_workspace(const dsv4cu_moe *L, int nrows, int live_rows);
int moe_mx_rows(const dsv4cu_moe *L, float *y, const float *x, long ldx, const int *ids, int nrows, int live_rows,
                float limit,
                void *ws, int *status, int sms, cudaStream_t st);

}  // namespace dsv4cu
