// trunk_loader.cu - the dense trunk (every layer's non-expert tensors) from
// the reference's pack straight into HBM.
//
// The reference reads trunk.bin into one host arena and binds pointers into
// it (src/50_loader/dsv4_trunk.c:37-131); the engine's kernels then read the
// weights across the bus, or through the host-pointer registry's mirrors.
// Here the layer runs go to one device arena once, and callers take device
// descriptors by (layer, slot).
//
// Format (written by the reference's tools/pack_trunk.py, read by
// src/50_loader/dsv4_trunk_manifest.c:24-110):
//   trunk.idx  text, blank lines ignored:
//              "DSV4TRUNK 2", "n_layers N", "layout 1", then per layer
//              "layer L file_off nbytes n_tensors widen_bytes" followed by
//              n_tensors lines "slot id off nbytes dtype rows cols wdt blk_r blk_c"
//              (off within the layer run; dtype the safetensors code 1..8 of
//              src/40_io/dsv4_st.h:25-33; wdt DSV4CU_W*);
//   trunk.bin  the layer runs at their file offsets.
// A packed matrix's scale tensor is the slot after the matrix's slot
// (dsv4_bind_layer.c:10-23, 36-47: X and X_S ids are consecutive).
//
// Host side: the file is read in 64 MiB pieces into two pinned staging
// buffers that alternate, so a read overlaps the copy of the piece before.
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"
#include "ctx.h"

namespace {

constexpr int64_t TRUNK_ALIGN = 4096;               // layer runs start on 4 KiB in the arena
constexpr size_t TRUNK_PIECE = (size_t)64 << 20;    // staging piece
enum { DT_U8 = 1, DT_BF16 = 2, DT_F32 = 4, DT_I64 = 8 };

struct TrunkLayer {
    int64_t file_off = 0, nbytes = 0, widen = 0;
    std::vector<dsv4cu_trunk_tensor> t;
    int64_t arena_off = -1;          // -1: not resident
};

struct Manifest {
    int n_layers = 0;
    std::vector<TrunkLayer> lay;
};

// Next line with something other than blanks, trailing CR / LF removed.
bool next_line(FILE *f, std::string &line)
{
    char buf[512];
    while (fgets(buf, sizeof buf, f)) {
        size_t n = strlen(buf);
        while (n && (buf[n - 1] == '\n' || buf[n - 1] == '\r')) buf[--n] = 0;
        const char *p = buf;
        while (*p == ' ' || *p == '\t') p++;
        if (*p) {
            line = buf;
            return true;
        }
    }
    return false;
}

int read_manifest(const char *dir, Manifest *m)
{
    const std::string path = std::string(dir) + "/trunk.idx";
    FILE *f = fopen(path.c_str(), "r");
    if (!f) return dsv4cu_set_error(DSV4CU_ERR_IO, "trunk: cannot open %s", path.c_str());
    std::string line;
    char magic[32];
    int version = 0, layout = 0;
    int rc = DSV4CU_OK;
    if (!next_line(f, line) || sscanf(line.c_str(), "%31s %d", magic, &version) != 2 ||
        strcmp(magic, "DSV4TRUNK") != 0 || version != 2)
        rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk: %s is not a version-2 trunk index", path.c_str());
    else if (!next_line(f, line) || sscanf(line.c_str(), "n_layers %d", &m->n_layers) != 1 || m->n_layers <= 0)
        rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk: %s: missing or invalid n_layers", path.c_str());
    else if (!next_line(f, line) || sscanf(line.c_str(), "layout %d", &layout) != 1 || layout != 1)
        rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk: %s: unsupported layer layout", path.c_str());
    if (!rc) m->lay.resize((size_t)m->n_layers);
    for (int L = 0; L < m->n_layers && !rc; L++) {
        TrunkLayer &lay = m->lay[(size_t)L];
        long long off = 0, nb = 0, widen = 0;
        int got = -1, nt = 0;
        if (!next_line(f, line) ||
            sscanf(line.c_str(), "layer %d %lld %lld %d %lld", &got, &off, &nb, &nt, &widen) != 5 || got != L ||
            off < 0 || nb < 0 || nt < 0 || widen < 0) {
            rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk: %s: bad layer %d line", path.c_str(), L);
            break;
        }
        lay.file_off = off;
        lay.nbytes = nb;
        lay.widen = widen;
        lay.t.resize((size_t)nt);
        for (int i = 0; i < nt; i++) {
            dsv4cu_trunk_tensor &t = lay.t[(size_t)i];
            long long toff = 0, tnb = 0;
            if (!next_line(f, line) ||
                sscanf(line.c_str(), "slot %d %lld %lld %d %d %d %d %d %d", &t.slot, &toff, &tnb, &t.dtype, &t.rows,
                       &t.cols, &t.wdt, &t.blk_r, &t.blk_c) != 9) {
                rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk: %s: bad tensor in layer %d", path.c_str(), L);
                break;
            }
            t.off = toff;
            t.nbytes = tnb;
            if (t.dtype < DT_U8 || t.dtype > DT_I64 || t.wdt < DSV4CU_WF32 || t.wdt > DSV4CU_WFP4) {
                rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk: %s: layer %d slot %d has an invalid dtype / format",
                                      path.c_str(), L, t.slot);
                break;
            }
            if (t.off < 0 || t.nbytes < 0 || t.off + t.nbytes > lay.nbytes) {
                rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk: %s: layer %d slot %d lies outside its run",
                                      path.c_str(), L, t.slot);
                break;
            }
        }
    }
    fclose(f);
    return rc;
}

const dsv4cu_trunk_tensor *find_slot(const TrunkLayer &lay, int slot)
{
    for (const dsv4cu_trunk_tensor &t : lay.t)
        if (t.slot == slot) return &t;
    return nullptr;
}

int pread_all(int fd, int64_t off, size_t nbytes, void *dst)
{
    char *p = (char *)dst;
    while (nbytes > 0) {
        const ssize_t n = pread(fd, p, std::min<size_t>(nbytes, (size_t)1 << 30), (off_t)off);
        if (n <= 0) return -1;
        p += n;
        off += n;
        nbytes -= (size_t)n;
    }
    return 0;
}

// bf16 -> f32 is exact: the bf16 bits are the top half of the float.
__global__ void trunk_widen_bf16_kernel(float *__restrict__ dst, const uint16_t *__restrict__ src, long n)
{
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        dst[i] = __uint_as_float((uint32_t)src[i] << 16);
}

}  // namespace

struct dsv4cu_trunk {
    Manifest m;
    char *dev = nullptr;             // the arena: resident layer runs, each 4 KiB aligned
    int device = 0;
    int64_t resident = 0;
};

extern "C" int dsv4cu_trunk_manifest(const char *dir, int *n_layers, int layer, int64_t *run, int *n_tensors,
                                     dsv4cu_trunk_tensor *tensors, int cap)
{
    if (!dir) return dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk manifest: NULL directory");
    Manifest m;
    int r = read_manifest(dir, &m);
    if (r) return r;
    if (n_layers) *n_layers = m.n_layers;
    if (layer < 0) return DSV4CU_OK;
    if (layer >= m.n_layers) return dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk manifest: layer %d of %d", layer, m.n_layers);
    const TrunkLayer &lay = m.lay[(size_t)layer];
    if (run) {
        run[0] = lay.file_off;
        run[1] = lay.nbytes;
        run[2] = lay.widen;
    }
    if (n_tensors) *n_tensors = (int)lay.t.size();
    for (int i = 0; tensors && i < cap && i < (int)lay.t.size(); i++) tensors[i] = lay.t[(size_t)i];
    return DSV4CU_OK;
}

extern "C" int dsv4cu_trunk_load(dsv4cu_trunk **out, const char *dir, int first, int count, void *stream)
{
    if (!out || !dir) return dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk_load: NULL argument");
    *out = nullptr;
    dsv4cu_trunk *T = new dsv4cu_trunk;
    int rc = read_manifest(dir, &T->m);
    if (!rc && count <= 0) count = T->m.n_layers - first;
    if (!rc && (first < 0 || count <= 0 || first + count > T->m.n_layers))
        rc = dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk_load: layers [%d, %d) outside the index (%d layers)", first,
                              first + count, T->m.n_layers);
    int64_t total = 0, biggest = 0;
    for (int L = first; !rc && L < first + count; L++) {
        TrunkLayer &lay = T->m.lay[(size_t)L];
        if (lay.nbytes == 0) continue;
        lay.arena_off = total;
        total += (lay.nbytes + TRUNK_ALIGN - 1) / TRUNK_ALIGN * TRUNK_ALIGN;
        biggest = std::max(biggest, lay.nbytes);
    }
    int fd = -1;
    if (!rc) {
        const std::string path = std::string(dir) + "/trunk.bin";
        fd = open(path.c_str(), O_RDONLY);
        if (fd < 0) rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk_load: cannot open %s", path.c_str());
    }
    cudaGetDevice(&T->device);
    if (!rc && total > 0) {
        const cudaError_t ce = cudaMalloc((void **)&T->dev, (size_t)total);
        if (ce != cudaSuccess)
            rc = dsv4cu_set_error(DSV4CU_ERR_NOMEM, "trunk_load: %lld bytes: %s", (long long)total,
                                  cudaGetErrorString(ce));
    }
    cudaStream_t st = (cudaStream_t)stream;
    const size_t piece = (size_t)std::min<int64_t>((int64_t)TRUNK_PIECE, std::max<int64_t>(biggest, 1));
    void *stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    for (int i = 0; i < 2 && !rc && total > 0; i++)
        if (cudaHostAlloc(&stage[i], piece, cudaHostAllocDefault) != cudaSuccess ||
            cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess)
            rc = dsv4cu_set_error(DSV4CU_ERR_NOMEM, "trunk_load: pinned staging of %zu bytes", piece);
    long k = 0;   // pieces issued
    for (int L = first; !rc && L < first + count; L++) {
        const TrunkLayer &lay = T->m.lay[(size_t)L];
        for (int64_t o = 0; o < lay.nbytes && !rc; o += (int64_t)piece, k++) {
            const int b = (int)(k & 1);
            const size_t len = (size_t)std::min<int64_t>((int64_t)piece, lay.nbytes - o);
            if (k >= 2 && cudaEventSynchronize(done[b]) != cudaSuccess) {   // the copy that last used it
                rc = dsv4cu_set_error(DSV4CU_ERR_CUDA, "trunk_load: staging copy failed");
                break;
            }
            if (pread_all(fd, lay.file_off + o, len, stage[b])) {
                rc = dsv4cu_set_error(DSV4CU_ERR_IO, "trunk_load: short read on layer %d at %lld", L,
                                      (long long)(lay.file_off + o));
                break;
            }
            if (cudaMemcpyAsync(T->dev + lay.arena_off + o, stage[b], len, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaEventRecord(done[b], st) != cudaSuccess)
                rc = dsv4cu_set_error(DSV4CU_ERR_CUDA, "trunk_load: copy to the device failed");
        }
    }
    if (total > 0 && cudaStreamSynchronize(st) != cudaSuccess && !rc)
        rc = dsv4cu_set_error(DSV4CU_ERR_CUDA, "trunk_load: copy to the device failed");
    for (int i = 0; i < 2; i++) {
        if (stage[i]) cudaFreeHost(stage[i]);
        if (done[i]) cudaEventDestroy(done[i]);
    }
    if (fd >= 0) close(fd);
    if (rc) {
        if (T->dev) cudaFree(T->dev);
        delete T;
        return rc;
    }
    T->resident = total;
    *out = T;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_trunk_slot(const dsv4cu_trunk *t, int layer, int slot, dsv4cu_trunk_tensor *desc, void **dev)
{
    if (dev) *dev = nullptr;
    if (!t) return dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk_slot: NULL trunk");
    if (layer < 0 || layer >= t->m.n_layers || t->m.lay[(size_t)layer].arena_off < 0)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk_slot: layer %d is not resident", layer);
    const TrunkLayer &lay = t->m.lay[(size_t)layer];
    const dsv4cu_trunk_tensor *x = find_slot(lay, slot);
    if (!x) return dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk_slot: layer %d has no slot %d", layer, slot);
    if (desc) *desc = *x;
    if (dev) *dev = t->dev + lay.arena_off + x->off;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_trunk_qmat(const dsv4cu_trunk *t, int layer, int slot, dsv4cu_qmat *q)
{
    if (!q) return dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk_qmat: NULL matrix");
    dsv4cu_trunk_tensor d;
    void *w = nullptr, *s = nullptr;
    int r = dsv4cu_trunk_slot(t, layer, slot, &d, &w);
    if (r) return r;
    if (d.wdt == DSV4CU_WFP8 || d.wdt == DSV4CU_WFP4) {
        r = dsv4cu_trunk_slot(t, layer, slot + 1, nullptr, &s);   // its scale tensor
        if (r) return r;
    }
    q->w = w;
    q->s = s;
    q->wdt = d.wdt;
    q->rows = d.rows;
    q->cols = d.cols;
    q->blk_r = d.blk_r;
    q->blk_c = d.blk_c;
    return DSV4CU_OK;
}

extern "C" int dsv4cu_trunk_widen(const dsv4cu_trunk *t, int layer, int slot, float *dst, void *stream)
{
    if (!dst) return dsv4cu_set_error(DSV4CU_ERR_ARG, "trunk_widen: NULL destination");
    dsv4cu_trunk_tensor d;
    void *src = nullptr;
    int r = dsv4cu_trunk_slot(t, layer, slot, &d, &src);
    if (r) return r;
    cudaStream_t st = (cudaStream_t)stream;
    if (d.dtype == DT_F32) {
        if (d.nbytes % 4) return dsv4cu_set_error(DSV4CU_ERR_IO, "trunk_widen: %lld bytes of f32", (long long)d.nbytes);
        DSV4CU_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)d.nbytes, cudaMemcpyDeviceToDevice, st));
        return DSV4CU_OK;
    }
    if (d.dtype != DT_BF16 || d.nbytes % 2)
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED, "trunk_widen: layer %d slot %d: dtype %d, %lld bytes", layer,
                                slot, d.dtype, (long long)d.nbytes);
    const long n = (long)(d.nbytes / 2);
    if (n == 0) return DSV4CU_OK;
    trunk_widen_bf16_kernel<<<(unsigned)std::min<long>(1024, (n + 255) / 256), 256, 0, st>>>(
        dst, (const uint16_t *)src, n);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

extern "C" int64_t dsv4cu_trunk_resident_bytes(const dsv4cu_trunk *t) { return t ? t->resident : 0; }

extern "C" void dsv4cu_trunk_free(dsv4cu_trunk *t)
{
    if (!t) return;
    if (t->dev) {
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(t->device);
        cudaFree(t->dev);
        cudaSetDevice(cur);
    }
    delete t;
}
