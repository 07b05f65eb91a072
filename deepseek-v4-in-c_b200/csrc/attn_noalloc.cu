// attn_noalloc.cu - sparse attention that allocates nothing.
//
// dsv4cu_sparse_attn takes its per-chunk partials (max, exp-sum, partial
// output) from the context workspace, which grows with cudaMalloc on demand.
// Some callers cannot allocate at the moment they call in: code running while
// a CUDA graph is being captured (cudaMalloc is not a stream operation and
// breaks the capture's "no allocation" expectations), code inside a custom
// allocator's own callbacks, or an engine that has handed all remaining HBM to
// its KV/expert pools and must not fragment it. dsv4cu_sparse_attn_noalloc is
// the same computation with its partials in one fixed array that is part of
// the library image (a file-scope __device__ array), so no call allocates.
//
// Limits and sharing rules (also stated in include/dsv4cu.h):
//   - the partials need attn_workspace(h, d, topk) bytes and must fit in
//     DSV4CU_ATTN_NOALLOC_BYTES (12 MiB: h = 64, d = 576, topk = 2176 needs
//     9.6 MiB); larger shapes are rejected with DSV4CU_ERR_UNSUPPORTED;
//   - every call on a device shares that device's array; its contents are
//     whatever the last call left. Each call writes every element it later
//     reads, so nothing has to start at zero;
//   - two calls whose executions overlap on one device (different streams
//     without ordering, or different host threads) race on the array.
//     Serialise them on one stream.
//   - the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress with that device current), which loads the
//     library's module on that device if that has not happened yet. Make
//     the first call on each device before any stream capture begins.
#include <mutex>

#include "common.cuh"
#include "ctx.h"

#define DSV4CU_ATTN_NOALLOC_BYTES (12u << 20)
#define DSV4CU_NOALLOC_MAX_DEVICES 64

namespace dsv4cu {

size_t attn_workspace(int H, int D, int topk);
int attn_run(float *o, const float *q, const void *kv, int kv_bf16, const float *sink, const int *idxs, int H,
             int D, int topk, float scale, void *ws, cudaStream_t st);

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[DSV4CU_ATTN_NOALLOC_BYTES];

// Device address of g_attn_noalloc_scratch on `device`, looked up on every
// call (cheap once the module is loaded) so that a module reloaded after a
// device reset or a new primary context is followed. The last address found
// is kept only for a lookup that fails (e.g. one the runtime refuses during a
// stream capture); then the device must not have been reset since.
static int attn_noalloc_scratch(int device, void **out)
{
    static std::mutex mu;
    static void *addr[DSV4CU_NOALLOC_MAX_DEVICES];
    if (device < 0 || device >= DSV4CU_NOALLOC_MAX_DEVICES)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "sparse_attn_noalloc: device %d out of range", device);
    std::lock_guard<std::mutex> lk(mu);
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e == cudaSuccess) {
        addr[device] = p;
    } else {
        cudaGetLastError();
        if (!addr[device])
            return dsv4cu_set_error(DSV4CU_ERR_CUDA, "sparse_attn_noalloc: cudaGetSymbolAddress: %s",
                                    cudaGetErrorString(e));
    }
    *out = addr[device];
    return DSV4CU_OK;
}

}  // namespace dsv4cu

using namespace dsv4cu;

extern "C" int dsv4cu_sparse_attn_noalloc(float *o, const float *q, const void *kv, int kv_bf16, const float *sink,
                                          const int *idxs, int h, int d, int topk, float scale, void *stream)
{
    if (!o || !q || !kv || !sink) return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn_noalloc: NULL argument");
    if (h <= 0 || d <= 0 || topk < 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn_noalloc: bad shape");
    cudaStream_t st = (cudaStream_t)stream;
    if (topk == 0) {
        DSV4CU_CUDA_TRY(cudaMemsetAsync(o, 0, (size_t)h * d * sizeof(float), st));
        return DSV4CU_OK;
    }
    if (!idxs) return dsv4cu_set_error(DSV4CU_ERR_ARG, "sparse_attn_noalloc: NULL idxs");
    const size_t need = attn_workspace(h, d, topk);
    if (need > DSV4CU_ATTN_NOALLOC_BYTES)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED,
                                "sparse_attn_noalloc: h=%d d=%d topk=%d needs %zu scratch bytes, limit is %u", h, d,
                                topk, need, DSV4CU_ATTN_NOALLOC_BYTES);
    int device = 0;
    DSV4CU_CUDA_TRY(cudaGetDevice(&device));
    void *ws = nullptr;
    int r = attn_noalloc_scratch(device, &ws);
    if (r) return r;
    return attn_run(o, q, kv, kv_bf16, sink, idxs, h, d, topk, scale, ws, st);
}
