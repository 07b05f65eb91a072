// ctx.h - internal layout of dsv4cu_ctx.
#pragma once
#include <stddef.h>

#include "../../include/dsv4cu.h"

// Zero-initialised counters used by last-block-done reductions. Each launch
// that uses them takes a disjoint slice and leaves it at zero again.
#define DSV4CU_MAX_COUNTERS 65536

struct dsv4cu_ctx {
    int    device;
    int    sm_count;
    void  *ws;          // device workspace
    size_t ws_bytes;
    int   *counters;    // [DSV4CU_MAX_COUNTERS], zero between calls
    int   *status;      // device word: first bounded-wait timeout code, 0 = none
    int    inject;      // one-shot test fault for the next dsv4cu_gemv (DSV4CU_INJECT_*), 0 = none
};

// Returns a workspace of at least `bytes` (grows the buffer if needed).
int dsv4cu_ws_get(dsv4cu_ctx *c, size_t bytes, void **out);

static inline size_t dsv4cu_align256(size_t b) { return (b + 255) & ~(size_t)255; }
