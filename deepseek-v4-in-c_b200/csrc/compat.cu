// compat.cu - the reference's own operator entry points over host pointers.
//
// These are the drop-in symbols: dsv4_mmq_n, fp8_n, fp4_n, bf16_n, dsv4_route,
// dsv4_swiglu, dsv4_expert_forward, dsv4_indexer_score, dsv4_topk,
// dsv4_indexer_offset, dsv4_sparse_attn, dsv4_window_idxs and the prefill GPU
// seam dsv4_prefill_vk_*, with the prototypes of src/10_compute/dsv4_matmul.h,
// src/10_compute/dsv4_kernels.h and src/80_prefill/dsv4_prefill_vk.h. All the
// arithmetic runs in this library's CUDA kernels; host code here only moves
// bytes and keeps the weight mirror.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <mutex>
#include <vector>

#include "../../include/dsv4_compat.h"
#include "common.cuh"
#include "ctx.h"
#include "mxgemm.h"

namespace {

struct RegEntry {
    size_t bytes;
    uint64_t fp;
    void *dev;
};

struct DevBuf {
    void *p = nullptr;
    size_t n = 0;
};

struct HostState {
    std::recursive_mutex mu;
    bool init = false;
    int device = 0;
    dsv4cu_ctx *ctx = nullptr;
    cudaStream_t st = nullptr;
    std::map<uintptr_t, RegEntry> reg;   // keyed by host start address
    size_t reg_bytes = 0;
    // Tensor-core preparations (TMA map + scale blocks) of mirrored
    // matrices, keyed by the device weight address.
    std::map<uintptr_t, dsv4cu::MxMat> mx;
    DevBuf buf[8];
    DevBuf pin[2];   // pinned host staging for activations in / results out
};

HostState &S()
{
    static HostState s;
    return s;
}

[[noreturn]] void die(const char *what)
{
    fprintf(stderr, "dsv4cu: %s: %s\n", what, dsv4cu_last_error());
    abort();
}

void must(int rc, const char *what)
{
    if (rc != DSV4CU_OK) die(what);
}

void must_cuda(cudaError_t e, const char *what)
{
    if (e != cudaSuccess) {
        dsv4cu_set_error(DSV4CU_ERR_CUDA, "%s", cudaGetErrorString(e));
        die(what);
    }
}

// Returns 0 or an error code (the prefill seam must not abort).
int ensure_init()
{
    HostState &s = S();
    if (s.init) return DSV4CU_OK;
    const char *env = getenv("DSV4CU_DEVICE");
    s.device = env ? atoi(env) : 0;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= s.device)
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "no CUDA device %d", s.device);
    if (cudaSetDevice(s.device) != cudaSuccess)
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cudaSetDevice(%d) failed", s.device);
    int r = dsv4cu_ctx_create(&s.ctx, s.device);
    if (r) return r;
    if (cudaStreamCreateWithFlags(&s.st, cudaStreamNonBlocking) != cudaSuccess)
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "stream creation failed");
    s.init = true;
    return DSV4CU_OK;
}

// Keeps the caller's current device across a call.
struct DeviceScope {
    int prev = -1;
    DeviceScope()
    {
        cudaGetDevice(&prev);
        if (S().init && prev != S().device) cudaSetDevice(S().device);
    }
    ~DeviceScope()
    {
        if (prev >= 0 && S().init && prev != S().device) cudaSetDevice(prev);
    }
};

// Content check of a mirrored host buffer. Sampled (the default): the first
// and last 64 bytes and the first 8-byte word of every 4 KiB page, so any two
// different experts (which differ almost everywhere) are told apart, but a
// rewrite confined to unsampled bytes is not seen - such a caller must call
// dsv4cu_host_forget, or switch to full checking (dsv4cu_host_verify(1):
// every word hashed on every call, exact but a pass over the weights per call).
static int g_verify_full = 0;

uint64_t fingerprint(const void *p, size_t bytes)
{
    const unsigned char *b = (const unsigned char *)p;
    uint64_t h = 0x9E3779B97F4A7C15ull ^ (uint64_t)bytes ^ (g_verify_full ? 1ull : 0ull);
    auto mix = [&](uint64_t w) {
        h ^= w;
        h *= 0xFF51AFD7ED558CCDull;
        h ^= h >> 32;
    };
    auto word = [&](size_t off) {
        uint64_t w;
        memcpy(&w, b + off, 8);
        mix(w);
    };
    if (g_verify_full || bytes <= 256) {
        size_t i = 0;
        for (; i + 8 <= bytes; i += 8) word(i);
        for (; i < bytes; i++) mix(b[i]);
        return h;
    }
    for (size_t i = 0; i < 64; i += 8) {
        word(i);
        word(bytes - 64 + i);
    }
    for (size_t pg = 4096; pg + 8 <= bytes; pg += 4096) word(pg);
    return h;
}

int reg_upload(const void *host, size_t bytes, void **dev)
{
    HostState &s = S();
    void *d = nullptr;
    cudaError_t e = cudaMalloc(&d, bytes);
    if (e != cudaSuccess) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "weight mirror of %zu bytes: %s", bytes, cudaGetErrorString(e));
    e = cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(d);
        return dsv4cu_set_error(DSV4CU_ERR_CUDA, "weight upload: %s", cudaGetErrorString(e));
    }
    s.reg[(uintptr_t)host] = RegEntry{bytes, fingerprint(host, bytes), d};
    s.reg_bytes += bytes;
    *dev = d;
    return DSV4CU_OK;
}

void reg_drop(std::map<uintptr_t, RegEntry>::iterator it)
{
    HostState &s = S();
    cudaStreamSynchronize(s.st);
    // Tensor-core preparations that read the dropped mirror go with it.
    const uintptr_t a = (uintptr_t)it->second.dev, b = a + it->second.bytes;
    for (auto jt = s.mx.begin(); jt != s.mx.end();) {
        const uintptr_t w = (uintptr_t)jt->second.q.w, sc = (uintptr_t)jt->second.q.s;
        if ((w >= a && w < b) || (sc >= a && sc < b)) {
            dsv4cu::mx_release(&jt->second);
            jt = s.mx.erase(jt);
        } else {
            ++jt;
        }
    }
    cudaFree(it->second.dev);
    s.reg_bytes -= it->second.bytes;
    s.reg.erase(it);
}

// Device address of [host, host + bytes): an existing mirror that contains
// the range (sub-matrix views such as dsv4_wo_a_group slices reuse the parent)
// or a fresh upload. A mirror whose host bytes changed is uploaded again.
int reg_lookup(const void *host, size_t bytes, const void **dev)
{
    HostState &s = S();
    const uintptr_t p = (uintptr_t)host;
    auto it = s.reg.upper_bound(p);
    if (it != s.reg.begin()) {
        --it;
        const uintptr_t start = it->first;
        if (p >= start && p + bytes <= start + it->second.bytes) {
            if (fingerprint((const void *)start, it->second.bytes) == it->second.fp) {
                *dev = (const char *)it->second.dev + (p - start);
                return DSV4CU_OK;
            }
            const size_t pb = it->second.bytes;
            reg_drop(it);
            void *d = nullptr;
            int r = reg_upload((const void *)start, pb, &d);
            if (r) return r;
            *dev = (const char *)d + (p - start);
            return DSV4CU_OK;
        }
    }
    // Remove mirrors that overlap the new range (a buffer was re-carved).
    for (auto jt = s.reg.lower_bound(p > 0 ? 0 : 0); jt != s.reg.end();) {
        const uintptr_t a = jt->first, b = a + jt->second.bytes;
        if (a < p + bytes && p < b) {
            auto nx = std::next(jt);
            reg_drop(jt);
            jt = nx;
        } else {
            ++jt;
        }
    }
    void *d = nullptr;
    int r = reg_upload(host, bytes, &d);
    if (r) return r;
    *dev = d;
    return DSV4CU_OK;
}

void *buf(int i, size_t bytes)
{
    DevBuf &b = S().buf[i];
    if (bytes == 0) bytes = 16;
    if (b.n < bytes) {
        if (b.p) {
            cudaStreamSynchronize(S().st);
            cudaFree(b.p);
        }
        b.p = nullptr;
        b.n = 0;
        if (cudaMalloc(&b.p, bytes) != cudaSuccess) return nullptr;
        b.n = bytes;
    }
    return b.p;
}

// Pinned host staging buffer i (grown on demand): a copy between it and the
// device is a plain DMA, where a pageable buffer costs a driver-side staging
// copy and synchronisation per call.
void *pinned(int i, size_t bytes)
{
    DevBuf &b = S().pin[i];
    if (bytes == 0) bytes = 16;
    if (b.n < bytes) {
        if (b.p) {
            cudaStreamSynchronize(S().st);
            cudaFreeHost(b.p);
        }
        b.p = nullptr;
        b.n = 0;
        if (cudaHostAlloc(&b.p, bytes, cudaHostAllocDefault) != cudaSuccess) return nullptr;
        b.n = bytes;
    }
    return b.p;
}

void *buf_or_die(int i, size_t bytes)
{
    void *p = buf(i, bytes);
    if (!p) {
        dsv4cu_set_error(DSV4CU_ERR_NOMEM, "staging buffer of %zu bytes", bytes);
        die("device memory");
    }
    return p;
}

size_t qmat_wbytes(const DSV4QMat *m)
{
    switch (m->wdt) {
    case DSV4_WBF16: return (size_t)m->rows * m->cols * 2;
    case DSV4_WFP8: return (size_t)m->rows * m->cols;
    case DSV4_WFP4: return (size_t)m->rows * (size_t)(m->cols / 2);
    default: return 0;
    }
}

size_t qmat_sbytes(const DSV4QMat *m)
{
    if (m->wdt != DSV4_WFP8 && m->wdt != DSV4_WFP4) return 0;
    const size_t sr = (size_t)((m->rows + m->blk_r - 1) / m->blk_r);
    const size_t sc = (size_t)((m->cols + m->blk_c - 1) / m->blk_c);
    return sr * sc;
}

// Host QMat -> device descriptor (weights mirrored in HBM).
int to_device(const DSV4QMat *m, dsv4cu_qmat *d)
{
    d->wdt = m->wdt;
    d->rows = m->rows;
    d->cols = m->cols;
    d->blk_r = m->blk_r;
    d->blk_c = m->blk_c;
    d->s = nullptr;
    int r = reg_lookup(m->w, qmat_wbytes(m), &d->w);
    if (r) return r;
    if (m->wdt == DSV4_WFP8 || m->wdt == DSV4_WFP4) r = reg_lookup(m->s, qmat_sbytes(m), &d->s);
    return r;
}

void unknown_wdt(const DSV4QMat *m)
{
    // Same message and outcome as the reference (src/10_compute/dsv4_matmul.c:56-60).
    fprintf(stderr, "dsv4_mmq_n: matrix has unimplemented wdt %d (%dx%d)\n", m->wdt, m->rows, m->cols);
    abort();
}

// y = x * W^T on device buffers, through the best available kernel.
int mmq_dev(float *dy, const float *dx, const dsv4cu_qmat *dq, int nt)
{
    HostState &s = S();
    if (nt >= dsv4cu::MX_MMQ_MIN_TOKENS && dsv4cu::mx_supported(dq)) {
        auto it = s.mx.find((uintptr_t)dq->w);
        if (it != s.mx.end() && (it->second.q.s != dq->s || it->second.q.rows != dq->rows ||
                                 it->second.q.cols != dq->cols || it->second.q.wdt != dq->wdt ||
                                 it->second.q.blk_r != dq->blk_r || it->second.q.blk_c != dq->blk_c)) {
            dsv4cu::mx_release(&it->second);
            s.mx.erase(it);
            it = s.mx.end();
        }
        if (it == s.mx.end()) {
            dsv4cu::MxMat m;
            int r = dsv4cu::mx_prepare(&m, dq, nullptr, s.st);
            if (r) return r;
            it = s.mx.emplace((uintptr_t)dq->w, m).first;
        }
        void *ws = nullptr;
        int r = dsv4cu_ws_get(s.ctx, dsv4cu::mx_workspace(&it->second, nt, dsv4cu::MX_MMQ_TERMS, s.ctx->sm_count),
                              &ws);
        if (r) return r;
        return dsv4cu::mx_gemm(&it->second, dy, dx, nt, dsv4cu::MX_MMQ_TERMS, 0, 0, ws, s.ctx->sm_count, s.ctx->status,
                               s.st);
    }
    return dsv4cu_mmq(s.ctx, dy, dx, dq, nt, s.st);
}

// y (host) = x (host) * W^T; returns a status instead of aborting.
int mmq_host(float *y, const float *x, const DSV4QMat *m, int nt)
{
    HostState &s = S();
    int r = ensure_init();
    if (r) return r;
    DeviceScope ds;
    dsv4cu_qmat dq;
    r = to_device(m, &dq);
    if (r) return r;
    const size_t xb = (size_t)nt * m->cols * 4, yb = (size_t)nt * m->rows * 4;
    float *dx = (float *)buf(0, xb), *dy = (float *)buf(1, yb);
    float *px = (float *)pinned(0, xb), *py = (float *)pinned(1, yb);
    if (!dx || !dy || !px || !py) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "staging");
    memcpy(px, x, xb);
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(dx, px, xb, cudaMemcpyHostToDevice, s.st));
    r = mmq_dev(dy, dx, &dq, nt);
    if (r) return r;
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(py, dy, yb, cudaMemcpyDeviceToHost, s.st));
    DSV4CU_CUDA_TRY(cudaStreamSynchronize(s.st));
    memcpy(y, py, yb);
    return DSV4CU_OK;
}

}  // namespace

// ======================================================== matmul entry points
extern "C" void dsv4_mmq_n(float *y, const float *x, const DSV4QMat *m, int nt)
{
    if (nt <= 0) return;
    if (m->wdt != DSV4_WBF16 && m->wdt != DSV4_WFP8 && m->wdt != DSV4_WFP4) unknown_wdt(m);
    std::lock_guard<std::recursive_mutex> lk(S().mu);
    must(mmq_host(y, x, m, nt), "dsv4_mmq_n");
}

extern "C" void dsv4_mmq(float *y, const float *x, const DSV4QMat *m) { dsv4_mmq_n(y, x, m, 1); }

extern "C" void bf16_n(float *y, const float *x, const uint16_t *W, int in, int out, int nt)
{
    DSV4QMat m = {W, nullptr, DSV4_WBF16, out, in, 0, 0};
    dsv4_mmq_n(y, x, &m, nt);
}

extern "C" void fp8_n(float *y, const float *x, const uint8_t *W, const uint8_t *Sc, int in, int out, int blk_r,
                      int blk_c, int nt)
{
    DSV4QMat m = {W, Sc, DSV4_WFP8, out, in, blk_r, blk_c};
    dsv4_mmq_n(y, x, &m, nt);
}

extern "C" void fp4_n(float *y, const float *x, const uint8_t *W, const uint8_t *Sc, int in, int out, int blk_r,
                      int blk_c, int nt)
{
    DSV4QMat m = {W, Sc, DSV4_WFP4, out, in, blk_r, blk_c};
    dsv4_mmq_n(y, x, &m, nt);
}

// ====================================================== router / expert ops
extern "C" void dsv4_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    if (n <= 0) return;
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    must(ensure_init(), "dsv4_rmsnorm");
    DeviceScope ds;
    const size_t b = (size_t)n * 4;
    float *dx = (float *)buf_or_die(0, b), *dw = (float *)buf_or_die(1, b), *dy = (float *)buf_or_die(2, b);
    must_cuda(cudaMemcpyAsync(dx, x, b, cudaMemcpyHostToDevice, s.st), "dsv4_rmsnorm");
    must_cuda(cudaMemcpyAsync(dw, w, b, cudaMemcpyHostToDevice, s.st), "dsv4_rmsnorm");
    must(dsv4cu_rmsnorm(dy, dx, dw, n, 1, eps, s.st), "dsv4_rmsnorm");
    must_cuda(cudaMemcpyAsync(y, dy, b, cudaMemcpyDeviceToHost, s.st), "dsv4_rmsnorm");
    must_cuda(cudaStreamSynchronize(s.st), "dsv4_rmsnorm");
}

extern "C" void dsv4_swiglu(float *y, const float *gate, const float *up, int n, float limit)
{
    if (n <= 0) return;
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    must(ensure_init(), "dsv4_swiglu");
    DeviceScope ds;
    const size_t b = (size_t)n * 4;
    float *dg = (float *)buf_or_die(0, b), *du = (float *)buf_or_die(1, b), *dy = (float *)buf_or_die(2, b);
    must_cuda(cudaMemcpyAsync(dg, gate, b, cudaMemcpyHostToDevice, s.st), "dsv4_swiglu");
    must_cuda(cudaMemcpyAsync(du, up, b, cudaMemcpyHostToDevice, s.st), "dsv4_swiglu");
    must(dsv4cu_swiglu(dy, dg, du, n, limit, s.st), "dsv4_swiglu");
    must_cuda(cudaMemcpyAsync(y, dy, b, cudaMemcpyDeviceToHost, s.st), "dsv4_swiglu");
    must_cuda(cudaStreamSynchronize(s.st), "dsv4_swiglu");
}

extern "C" void dsv4_route(int *idx, float *wts, float *scores, float *orig, const float *bias,
                           const int64_t *tid2eid, int token_id, int n_experts, int topk, float route_scale)
{
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    must(ensure_init(), "dsv4_route");
    DeviceScope ds;
    const size_t eb = (size_t)n_experts * 4;
    char *d = (char *)buf_or_die(0, 4 * eb + 4 * 64 + 512);
    float *dl = (float *)d, *dsc = (float *)(d + eb), *dor = (float *)(d + 2 * eb), *db = (float *)(d + 3 * eb);
    int *didx = (int *)(d + 4 * eb);
    float *dw = (float *)(d + 4 * eb + 64);
    int64_t *drow = (int64_t *)(d + 4 * eb + 128);
    int *dtok = (int *)(d + 4 * eb + 128 + 8 * 16);
    must_cuda(cudaMemcpyAsync(dl, scores, eb, cudaMemcpyHostToDevice, s.st), "dsv4_route");
    if (bias) must_cuda(cudaMemcpyAsync(db, bias, eb, cudaMemcpyHostToDevice, s.st), "dsv4_route");
    if (tid2eid) {
        // Only the token's own row of the hash table is needed.
        const int zero = 0;
        must_cuda(cudaMemcpyAsync(drow, tid2eid + (int64_t)token_id * topk, (size_t)topk * 8,
                                  cudaMemcpyHostToDevice, s.st), "dsv4_route");
        must_cuda(cudaMemcpyAsync(dtok, &zero, 4, cudaMemcpyHostToDevice, s.st), "dsv4_route");
    }
    must(dsv4cu_route(didx, dw, dsc, dor, dl, bias ? db : nullptr, tid2eid ? drow : nullptr,
                      tid2eid ? dtok : nullptr, n_experts, topk, route_scale, 1, s.st), "dsv4_route");
    must_cuda(cudaMemcpyAsync(idx, didx, (size_t)topk * 4, cudaMemcpyDeviceToHost, s.st), "dsv4_route");
    must_cuda(cudaMemcpyAsync(wts, dw, (size_t)topk * 4, cudaMemcpyDeviceToHost, s.st), "dsv4_route");
    must_cuda(cudaMemcpyAsync(scores, dsc, eb, cudaMemcpyDeviceToHost, s.st), "dsv4_route");
    must_cuda(cudaMemcpyAsync(orig, dor, eb, cudaMemcpyDeviceToHost, s.st), "dsv4_route");
    must_cuda(cudaStreamSynchronize(s.st), "dsv4_route");
}

// w2( swiglu(w1 x, w3 x) ), with the caller's gate/up/mid rows filled as the
// reference fills them (src/10_compute/dsv4_ops.c:85-93).
static int expert_host(float *out, const float *x, const DSV4ExpertW *e, float *gate, float *up, float *mid,
                       int n, int inter, float limit)
{
    HostState &s = S();
    int r = ensure_init();
    if (r) return r;
    DeviceScope ds;
    dsv4cu_qmat q1, q3, q2;
    if ((r = to_device(&e->w1, &q1)) || (r = to_device(&e->w3, &q3)) || (r = to_device(&e->w2, &q2))) return r;
    const int hid = e->w1.cols, hout = e->w2.rows;
    const size_t xb = (size_t)n * hid * 4, ib = (size_t)n * inter * 4, ob = (size_t)n * hout * 4;
    float *dx = (float *)buf(0, xb), *dg = (float *)buf(1, ib), *du = (float *)buf(2, ib);
    float *dm = (float *)buf(3, ib), *dy = (float *)buf(4, ob);
    if (!dx || !dg || !du || !dm || !dy) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "staging");
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, s.st));
    if ((r = dsv4cu_mmq(s.ctx, dg, dx, &q1, n, s.st))) return r;
    if ((r = dsv4cu_mmq(s.ctx, du, dx, &q3, n, s.st))) return r;
    if ((r = dsv4cu_swiglu(dm, dg, du, n * inter, limit, s.st))) return r;
    if ((r = dsv4cu_mmq(s.ctx, dy, dm, &q2, n, s.st))) return r;
    DSV4CU_CUDA_TRY(cudaMemcpyAsync(out, dy, ob, cudaMemcpyDeviceToHost, s.st));
    if (gate) DSV4CU_CUDA_TRY(cudaMemcpyAsync(gate, dg, ib, cudaMemcpyDeviceToHost, s.st));
    if (up) DSV4CU_CUDA_TRY(cudaMemcpyAsync(up, du, ib, cudaMemcpyDeviceToHost, s.st));
    if (mid) DSV4CU_CUDA_TRY(cudaMemcpyAsync(mid, dm, ib, cudaMemcpyDeviceToHost, s.st));
    DSV4CU_CUDA_TRY(cudaStreamSynchronize(s.st));
    return DSV4CU_OK;
}

extern "C" void dsv4_expert_forward(float *out, const float *x, const DSV4ExpertW *e, float *gate, float *up,
                                    float *mid, int inter, float limit)
{
    const DSV4QMat *ms[3] = {&e->w1, &e->w3, &e->w2};
    for (int i = 0; i < 3; i++)
        if (ms[i]->wdt != DSV4_WBF16 && ms[i]->wdt != DSV4_WFP8 && ms[i]->wdt != DSV4_WFP4) unknown_wdt(ms[i]);
    std::lock_guard<std::recursive_mutex> lk(S().mu);
    must(expert_host(out, x, e, gate, up, mid, 1, inter, limit), "dsv4_expert_forward");
}

// ======================================================== indexer / attention
extern "C" void dsv4_indexer_score(float *out, const float *q, const float *kv, const float *weights, int n_heads,
                                   int head_dim, int n_pos)
{
    if (n_pos <= 0) return;
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    must(ensure_init(), "dsv4_indexer_score");
    DeviceScope ds;
    const size_t qb = (size_t)n_heads * head_dim * 4, kb = (size_t)n_pos * head_dim * 4;
    float *dq = (float *)buf_or_die(0, qb), *dk = (float *)buf_or_die(1, kb);
    float *dw = (float *)buf_or_die(2, (size_t)n_heads * 4), *dout = (float *)buf_or_die(3, (size_t)n_pos * 4);
    must_cuda(cudaMemcpyAsync(dq, q, qb, cudaMemcpyHostToDevice, s.st), "dsv4_indexer_score");
    must_cuda(cudaMemcpyAsync(dk, kv, kb, cudaMemcpyHostToDevice, s.st), "dsv4_indexer_score");
    must_cuda(cudaMemcpyAsync(dw, weights, (size_t)n_heads * 4, cudaMemcpyHostToDevice, s.st), "dsv4_indexer_score");
    must(dsv4cu_indexer_score(dout, dq, dk, dw, n_heads, head_dim, n_pos, s.st), "dsv4_indexer_score");
    must_cuda(cudaMemcpyAsync(out, dout, (size_t)n_pos * 4, cudaMemcpyDeviceToHost, s.st), "dsv4_indexer_score");
    must_cuda(cudaStreamSynchronize(s.st), "dsv4_indexer_score");
}

extern "C" int dsv4_topk(int *idxs, const float *scores, int n, int k)
{
    if (k > n) k = n;
    if (k <= 0 || n <= 0) return k;
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    must(ensure_init(), "dsv4_topk");
    DeviceScope ds;
    float *dsx = (float *)buf_or_die(0, (size_t)n * 4);
    int *di = (int *)buf_or_die(1, (size_t)k * 4);
    must_cuda(cudaMemcpyAsync(dsx, scores, (size_t)n * 4, cudaMemcpyHostToDevice, s.st), "dsv4_topk");
    must(dsv4cu_topk(s.ctx, di, dsx, n, k, s.st), "dsv4_topk");
    must_cuda(cudaMemcpyAsync(idxs, di, (size_t)k * 4, cudaMemcpyDeviceToHost, s.st), "dsv4_topk");
    must_cuda(cudaStreamSynchronize(s.st), "dsv4_topk");
    return k;
}

extern "C" void dsv4_indexer_offset(int *idxs, int n, int offset)
{
    if (n <= 0) return;
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    must(ensure_init(), "dsv4_indexer_offset");
    DeviceScope ds;
    int *d = (int *)buf_or_die(0, (size_t)n * 4);
    must_cuda(cudaMemcpyAsync(d, idxs, (size_t)n * 4, cudaMemcpyHostToDevice, s.st), "dsv4_indexer_offset");
    must(dsv4cu_indexer_offset(d, n, offset, s.st), "dsv4_indexer_offset");
    must_cuda(cudaMemcpyAsync(idxs, d, (size_t)n * 4, cudaMemcpyDeviceToHost, s.st), "dsv4_indexer_offset");
    must_cuda(cudaStreamSynchronize(s.st), "dsv4_indexer_offset");
}

__global__ void window_kernel(int *idxs, int pos, int win)
{
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= win) return;
    const int n = min(pos + 1, win);
    idxs[k] = k < n ? (pos - k) % win : -1;
}

// src/10_compute/dsv4_attn.c:117-127: ring slots of the most recent
// min(pos+1, win) positions, newest first; -1 for unwritten slots.
extern "C" int dsv4_window_idxs(int *idxs, int pos, int win)
{
    int n = pos + 1;
    if (n > win) n = win;
    if (win <= 0) return n;
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    must(ensure_init(), "dsv4_window_idxs");
    DeviceScope ds;
    int *d = (int *)buf_or_die(0, (size_t)win * 4);
    window_kernel<<<(win + 127) / 128, 128, 0, s.st>>>(d, pos, win);
    must_cuda(cudaGetLastError(), "dsv4_window_idxs");
    must_cuda(cudaMemcpyAsync(idxs, d, (size_t)win * 4, cudaMemcpyDeviceToHost, s.st), "dsv4_window_idxs");
    must_cuda(cudaStreamSynchronize(s.st), "dsv4_window_idxs");
    return n;
}

// The host-pointer form cannot see the KV cache's length, so it ships only the
// selected rows: row j of the upload is kv[idxs[j]] (masked slots stay -1).
// Device-resident caches use dsv4cu_sparse_attn directly.
extern "C" void dsv4_sparse_attn(float *o, const float *q, const float *kv, const float *sink, const int *idxs,
                                 int h, int d, int topk, float scale, float *scratch)
{
    (void)scratch;
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    must(ensure_init(), "dsv4_sparse_attn");
    DeviceScope ds;
    std::vector<float> rows((size_t)(topk > 0 ? topk : 1) * d);
    std::vector<int> rid((size_t)(topk > 0 ? topk : 1));
    for (int j = 0; j < topk; j++) {
        rid[j] = idxs[j] < 0 ? -1 : j;
        if (idxs[j] >= 0) memcpy(&rows[(size_t)j * d], kv + (size_t)idxs[j] * d, (size_t)d * 4);
    }
    const size_t qb = (size_t)h * d * 4, kb = (size_t)topk * d * 4;
    float *dq = (float *)buf_or_die(0, qb), *dk = (float *)buf_or_die(1, kb);
    float *dsink = (float *)buf_or_die(2, (size_t)h * 4), *dout = (float *)buf_or_die(3, qb);
    int *di = (int *)buf_or_die(4, (size_t)(topk > 0 ? topk : 1) * 4);
    must_cuda(cudaMemcpyAsync(dq, q, qb, cudaMemcpyHostToDevice, s.st), "dsv4_sparse_attn");
    if (topk > 0) {
        must_cuda(cudaMemcpyAsync(dk, rows.data(), kb, cudaMemcpyHostToDevice, s.st), "dsv4_sparse_attn");
        must_cuda(cudaMemcpyAsync(di, rid.data(), (size_t)topk * 4, cudaMemcpyHostToDevice, s.st), "dsv4_sparse_attn");
    }
    must_cuda(cudaMemcpyAsync(dsink, sink, (size_t)h * 4, cudaMemcpyHostToDevice, s.st), "dsv4_sparse_attn");
    must(dsv4cu_sparse_attn(s.ctx, dout, dq, dk, 0, dsink, di, h, d, topk, scale, s.st), "dsv4_sparse_attn");
    must_cuda(cudaMemcpyAsync(o, dout, qb, cudaMemcpyDeviceToHost, s.st), "dsv4_sparse_attn");
    must_cuda(cudaStreamSynchronize(s.st), "dsv4_sparse_attn");
}

// ============================================================ prefill seam
struct DSV4PrefillVk {
    int dead;   // latched after a device error, as the Vulkan backend does
};

extern "C" int dsv4_prefill_vk_init(DSV4PrefillVk **out, const DSV4Cfg *cfg, struct DSV4Trunk *tr,
                                    struct DSV4Cache *cache)
{
    (void)cfg;
    (void)tr;
    (void)cache;
    if (!out) return -1;
    *out = nullptr;
    std::lock_guard<std::recursive_mutex> lk(S().mu);
    if (ensure_init() != DSV4CU_OK) return -1;
    DSV4PrefillVk *v = (DSV4PrefillVk *)calloc(1, sizeof *v);
    if (!v) return -1;
    *out = v;
    return 0;
}

extern "C" void dsv4_prefill_vk_free(DSV4PrefillVk *v) { free(v); }

extern "C" int dsv4_prefill_vk_gemm(DSV4PrefillVk *v, float *y, const float *x, const DSV4QMat *m, int n)
{
    if (!v || v->dead) return -1;
    if (n <= 0) return 0;
    if (m->wdt != DSV4_WBF16 && m->wdt != DSV4_WFP8 && m->wdt != DSV4_WFP4) return -1;
    std::lock_guard<std::recursive_mutex> lk(S().mu);
    if (mmq_host(y, x, m, n) != DSV4CU_OK) {
        fprintf(stderr, "dsv4cu: prefill gemm failed: %s\n", dsv4cu_last_error());
        v->dead = 1;
        return -1;
    }
    return 0;
}

extern "C" int dsv4_prefill_vk_expert_fused(DSV4PrefillVk *v, float *y, const float *x, const DSV4QMat *w1,
                                            const DSV4QMat *w3, const DSV4QMat *w2, int n, int inter, float limit,
                                            DSV4PrefillVkFillFn fill, void *fill_ctx)
{
    if (!v || v->dead) return -1;
    if (n <= 0) return 0;
    std::lock_guard<std::recursive_mutex> lk(S().mu);
    HostState &s = S();
    if (ensure_init() != DSV4CU_OK) return -1;
    DeviceScope ds;
    DSV4ExpertW e = {*w1, *w3, *w2};
    dsv4cu_qmat q1, q3, q2;
    if (to_device(&e.w1, &q1) || to_device(&e.w3, &q3) || to_device(&e.w2, &q2)) goto fail;
    {
        const int hid = w1->cols, hout = w2->rows;
        const size_t xb = (size_t)n * hid * 4, ib = (size_t)n * inter * 4, ob = (size_t)n * hout * 4;
        float *dx = (float *)buf(0, xb), *dg = (float *)buf(1, ib), *du = (float *)buf(2, ib);
        float *dm = (float *)buf(3, ib), *dy = (float *)buf(4, ob);
        if (!dx || !dg || !du || !dm || !dy) goto fail;
        if (cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, s.st) != cudaSuccess) goto fail;
        if (mmq_dev(dg, dx, &q1, n) || mmq_dev(du, dx, &q3, n) || dsv4cu_swiglu(dm, dg, du, n * inter, limit, s.st) ||
            mmq_dev(dy, dm, &q2, n))
            goto fail;
        if (cudaMemcpyAsync(y, dy, ob, cudaMemcpyDeviceToHost, s.st) != cudaSuccess) goto fail;
        // The CPU fill callback runs while the device is busy, until it reports
        // no more ready work (src/80_prefill/dsv4_prefill_vk.h:25-29).
        if (fill)
            while (cudaStreamQuery(s.st) == cudaErrorNotReady)
                if (!fill(fill_ctx)) break;
        if (cudaStreamSynchronize(s.st) != cudaSuccess) goto fail;
    }
    return 0;
fail:
    fprintf(stderr, "dsv4cu: prefill expert failed: %s\n", dsv4cu_last_error());
    v->dead = 1;
    return -1;
}

// ============================================================ registry admin
extern "C" void dsv4cu_host_forget(const void *host_ptr)
{
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    auto it = s.reg.find((uintptr_t)host_ptr);
    if (it != s.reg.end()) reg_drop(it);
}

extern "C" void dsv4cu_host_verify(int full)
{
    std::lock_guard<std::recursive_mutex> lk(S().mu);
    g_verify_full = full ? 1 : 0;
}

extern "C" void dsv4cu_host_forget_all(void)
{
    HostState &s = S();
    std::lock_guard<std::recursive_mutex> lk(s.mu);
    while (!s.reg.empty()) reg_drop(s.reg.begin());
}

extern "C" size_t dsv4cu_host_registry_count(void)
{
    std::lock_guard<std::recursive_mutex> lk(S().mu);
    return S().reg.size();
}

extern "C" size_t dsv4cu_host_registry_bytes(void)
{
    std::lock_guard<std::recursive_mutex> lk(S().mu);
    return S().reg_bytes;
}
