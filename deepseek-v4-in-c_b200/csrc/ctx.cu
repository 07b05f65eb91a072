// ctx.cu - library context (per-device workspace) and thread-local errors.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "ctx.h"

namespace dsv4cu {
const float *router_table_get();
}

static thread_local char g_err[512] = "no error";

extern "C" const char *dsv4cu_last_error(void) { return g_err; }

extern "C" int dsv4cu_set_error(int code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

extern "C" int dsv4cu_ctx_create(dsv4cu_ctx **out, int device)
{
    if (!out) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ctx_create: out is NULL");
    *out = nullptr;
    int prev = 0;
    DSV4CU_CUDA_TRY(cudaGetDevice(&prev));
    DSV4CU_CUDA_TRY(cudaSetDevice(device));
    dsv4cu_ctx *c = (dsv4cu_ctx *)calloc(1, sizeof *c);
    if (!c) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "ctx_create: host OOM");
    c->device = device;
    cudaDeviceProp p;
    cudaError_t e = cudaGetDeviceProperties(&p, device);
    if (e != cudaSuccess) {
        free(c);
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "ctx_create: %s", cudaGetErrorString(e));
    }
    c->sm_count = p.multiProcessorCount;
    // Counters for the last-block reductions must start at zero and are
    // returned to zero by the block that consumes them.
    e = cudaMalloc(&c->counters, (DSV4CU_MAX_COUNTERS + 64) * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->counters, 0, (DSV4CU_MAX_COUNTERS + 64) * sizeof(int));
    c->status = c->counters + DSV4CU_MAX_COUNTERS;
    if (e != cudaSuccess) {
        if (c->counters) cudaFree(c->counters);
        free(c);
        cudaSetDevice(prev);
        return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "ctx_create: %s", cudaGetErrorString(e));
    }
    // Build the router's bf16 score table now, so no later call has to.
    if (!dsv4cu::router_table_get()) {
        cudaFree(c->counters);
        free(c);
        cudaSetDevice(prev);
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "ctx_create: router table setup failed");
    }
    cudaSetDevice(prev);
    *out = c;
    return DSV4CU_OK;
}

extern "C" void dsv4cu_ctx_destroy(dsv4cu_ctx *c)
{
    if (!c) return;
    if (c->ws) cudaFree(c->ws);
    if (c->counters) cudaFree(c->counters);
    free(c);
}

extern "C" int dsv4cu_ctx_reserve(dsv4cu_ctx *c, size_t bytes)
{
    if (!c) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ctx_reserve: NULL ctx");
    if (bytes <= c->ws_bytes) return DSV4CU_OK;
    // The old buffer may still be read by queued work: wait before freeing.
    DSV4CU_CUDA_TRY(cudaDeviceSynchronize());
    if (c->ws) cudaFree(c->ws);
    c->ws = nullptr;
    c->ws_bytes = 0;
    bytes = (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;
    cudaError_t e = cudaMalloc(&c->ws, bytes);
    if (e != cudaSuccess) {
        c->ws = nullptr;
        return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "workspace of %zu bytes: %s", bytes,
                                cudaGetErrorString(e));
    }
    c->ws_bytes = bytes;
    return DSV4CU_OK;
}

extern "C" size_t dsv4cu_ctx_workspace_bytes(const dsv4cu_ctx *c)
{
    return c ? c->ws_bytes : 0;
}

extern "C" int dsv4cu_ctx_inject(dsv4cu_ctx *c, int what)
{
    if (!c) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ctx_inject: NULL context");
    if (what != 0 && what != DSV4CU_INJECT_WITHHOLD_STAGE)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "ctx_inject: unknown fault %d", what);
    c->inject = what;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_ctx_status(dsv4cu_ctx *c, void *stream, int *code)
{
    if (!c || !code) return dsv4cu_set_error(DSV4CU_ERR_ARG, "ctx_status: NULL argument");
    DSV4CU_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    DSV4CU_CUDA_TRY(cudaMemcpy(code, c->status, sizeof(int), cudaMemcpyDeviceToHost));
    if (*code) {
        // A kernel that gave up may have left its last-arriver counts behind.
        DSV4CU_CUDA_TRY(cudaMemset(c->counters, 0, DSV4CU_MAX_COUNTERS * sizeof(int)));
        DSV4CU_CUDA_TRY(cudaMemset(c->status, 0, sizeof(int)));
        return dsv4cu_set_error(DSV4CU_ERR_TIMEOUT, "a bounded device wait timed out (code 0x%x)", *code);
    }
    return DSV4CU_OK;
}

int dsv4cu_ws_get(dsv4cu_ctx *c, size_t bytes, void **out)
{
    if (!c) return dsv4cu_set_error(DSV4CU_ERR_ARG, "NULL context");
    if (bytes > c->ws_bytes) {
        int r = dsv4cu_ctx_reserve(c, bytes);
        if (r) return r;
    }
    *out = c->ws;
    return DSV4CU_OK;
}
