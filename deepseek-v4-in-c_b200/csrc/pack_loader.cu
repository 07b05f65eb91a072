// pack_loader.cu - routed experts from the reference's pack straight into HBM.
//
// The reference streams routed experts from disk through its expert cache
// (src/60_cache) every time a token routes to one. Here a layer's experts are
// read once and stay resident in HBM, partitioned over the ranks for expert
// parallelism (rank r holds experts [first, first + count)).
//
// Pack format (written by the reference's tools/pack_trunk.py, read by
// src/40_io/dsv4_st.c):
//   experts.idx  "DSV4EXP1", int32 n_layers, int32 n_experts, then for every
//                (layer, expert) six 24-byte records {int32 shard, int32 pad,
//                int64 off, int64 nbytes} in the order w1, w1 scales, w2,
//                w2 scales, w3, w3 scales (dsv4_st.h:36-55, dsv4_st.c:65-87);
//   shards       every *.safetensors file of the model directory, numbered
//                in strcmp order of their paths (dsv4_st.c:89-143); a record's
//                bytes are the raw tensor payload at `off`.
// The tensors are the reference's FP4 layout: w1/w3 [inter][hidden/2] e2m1
// (low nibble = even column), w2 [hidden][inter/2], one E8M0 byte per 1x32
// block (dsv4_weights.h:101 gives the 13,369,344-byte expert of config 2).
//
// Host side only: pread into two pinned staging buffers that alternate, so
// the disk read of one expert overlaps the host-to-device copy of the last.
#include <dirent.h>
#include <fcntl.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <vector>

#include "ctx.h"

namespace {

enum { EXP_W1W, EXP_W1S, EXP_W2W, EXP_W2S, EXP_W3W, EXP_W3S, EXP_TENSORS };

struct Loc {
    int32_t shard;
    int32_t pad;
    int64_t off;
    int64_t nbytes;
};
static_assert(sizeof(Loc) == 24, "experts.idx records are 24 bytes");

struct Index {
    int32_t n_layers = 0, n_experts = 0;
    std::vector<Loc> rec;     // [n_layers][n_experts][6]
};

int read_index(const char *index_dir, Index *ix)
{
    const std::string path = std::string(index_dir) + "/experts.idx";
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return dsv4cu_set_error(DSV4CU_ERR_IO, "experts index: cannot open %s", path.c_str());
    char magic[8];
    int32_t nl = 0, ne = 0;
    int rc = DSV4CU_OK;
    if (fread(magic, 1, 8, f) != 8 || memcmp(magic, "DSV4EXP1", 8) != 0) {
        rc = dsv4cu_set_error(DSV4CU_ERR_IO, "experts index: %s is not a DSV4EXP1 index", path.c_str());
    } else if (fread(&nl, 4, 1, f) != 1 || fread(&ne, 4, 1, f) != 1 || nl <= 0 || ne <= 0 || nl > 4096 ||
               ne > 65536) {
        rc = dsv4cu_set_error(DSV4CU_ERR_IO, "experts index: %s has a bad header", path.c_str());
    } else {
        ix->n_layers = nl;
        ix->n_experts = ne;
        ix->rec.resize((size_t)nl * ne * EXP_TENSORS);
        if (fread(ix->rec.data(), sizeof(Loc), ix->rec.size(), f) != ix->rec.size())
            rc = dsv4cu_set_error(DSV4CU_ERR_IO, "experts index: %s is truncated", path.c_str());
    }
    fclose(f);
    return rc;
}

// Sorted *.safetensors paths of model_dir, opened read-only.
struct Shards {
    std::vector<int> fd;
    ~Shards()
    {
        for (int d : fd)
            if (d >= 0) close(d);
    }
};

int open_shards(const char *model_dir, Shards *sh)
{
    DIR *d = opendir(model_dir);
    if (!d) return dsv4cu_set_error(DSV4CU_ERR_IO, "experts: cannot open directory %s", model_dir);
    std::vector<std::string> files;
    while (struct dirent *e = readdir(d)) {
        const size_t n = strlen(e->d_name);
        if (n >= 12 && strcmp(e->d_name + n - 12, ".safetensors") == 0)
            files.push_back(std::string(model_dir) + "/" + e->d_name);
    }
    closedir(d);
    if (files.empty()) return dsv4cu_set_error(DSV4CU_ERR_IO, "experts: no .safetensors files in %s", model_dir);
    std::sort(files.begin(), files.end(), [](const std::string &a, const std::string &b) {
        return strcmp(a.c_str(), b.c_str()) < 0;
    });
    for (const std::string &p : files) {
        const int fd = open(p.c_str(), O_RDONLY);
        if (fd < 0) return dsv4cu_set_error(DSV4CU_ERR_IO, "experts: cannot open %s", p.c_str());
        sh->fd.push_back(fd);
    }
    return DSV4CU_OK;
}

int read_all(int fd, int64_t off, int64_t nbytes, void *dst)
{
    char *p = (char *)dst;
    while (nbytes > 0) {
        const ssize_t n = pread(fd, p, (size_t)std::min<int64_t>(nbytes, 1 << 30), (off_t)off);
        if (n <= 0) return -1;
        p += n;
        off += n;
        nbytes -= n;
    }
    return 0;
}

}  // namespace

struct dsv4cu_expert_store {
    void *dev = nullptr;
    int device = 0;
};

extern "C" int dsv4cu_experts_index(const char *index_dir, int *n_layers, int *n_experts, int layer, int expert,
                                    int64_t *loc)
{
    if (!index_dir) return dsv4cu_set_error(DSV4CU_ERR_ARG, "experts index: NULL directory");
    Index ix;
    int r = read_index(index_dir, &ix);
    if (r) return r;
    if (n_layers) *n_layers = ix.n_layers;
    if (n_experts) *n_experts = ix.n_experts;
    if (loc) {
        if (layer < 0 || layer >= ix.n_layers || expert < 0 || expert >= ix.n_experts)
            return dsv4cu_set_error(DSV4CU_ERR_ARG, "experts index: (layer %d, expert %d) out of range", layer,
                                    expert);
        const Loc *l = &ix.rec[((size_t)layer * ix.n_experts + expert) * EXP_TENSORS];
        for (int t = 0; t < EXP_TENSORS; t++) {
            loc[3 * t] = l[t].shard;
            loc[3 * t + 1] = l[t].off;
            loc[3 * t + 2] = l[t].nbytes;
        }
    }
    return DSV4CU_OK;
}

extern "C" int dsv4cu_experts_load(dsv4cu_expert_store **out, dsv4cu_expert *experts, const char *model_dir,
                                   const char *index_dir, int layer, int first, int count, int hidden, int inter,
                                   void *stream)
{
    if (!out || !experts || !model_dir || !index_dir) return dsv4cu_set_error(DSV4CU_ERR_ARG, "experts_load: NULL");
    *out = nullptr;
    if (count <= 0 || first < 0 || hidden <= 0 || inter <= 0 || hidden % 32 || inter % 32)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "experts_load: bad range or shape");
    Index ix;
    int r = read_index(index_dir, &ix);
    if (r) return r;
    if (layer < 0 || layer >= ix.n_layers || first + count > ix.n_experts)
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "experts_load: layer %d experts [%d, %d) outside the index (%d x %d)",
                                layer, first, first + count, ix.n_layers, ix.n_experts);
    Shards sh;
    r = open_shards(model_dir, &sh);
    if (r) return r;

    // Expected payload sizes, in the record order.
    const int64_t want[EXP_TENSORS] = {
        (int64_t)inter * hidden / 2, (int64_t)inter * (hidden / 32),   // w1, its scales
        (int64_t)hidden * inter / 2, (int64_t)hidden * (inter / 32),   // w2
        (int64_t)inter * hidden / 2, (int64_t)inter * (hidden / 32)};  // w3
    size_t off[EXP_TENSORS + 1];
    off[0] = 0;
    for (int t = 0; t < EXP_TENSORS; t++) off[t + 1] = off[t] + dsv4cu_align256((size_t)want[t]);
    const size_t per = off[EXP_TENSORS];
    for (int e = first; e < first + count; e++) {
        const Loc *l = &ix.rec[((size_t)layer * ix.n_experts + e) * EXP_TENSORS];
        for (int t = 0; t < EXP_TENSORS; t++)
            if (l[t].nbytes != want[t] || l[t].shard < 0 || l[t].shard >= (int)sh.fd.size() || l[t].off < 0)
                return dsv4cu_set_error(DSV4CU_ERR_IO,
                                        "experts_load: layer %d expert %d tensor %d: shard %d, %lld bytes (want %lld)",
                                        layer, e, t, l[t].shard, (long long)l[t].nbytes, (long long)want[t]);
    }

    dsv4cu_expert_store *S = new dsv4cu_expert_store;
    cudaGetDevice(&S->device);
    cudaError_t ce = cudaMalloc(&S->dev, per * (size_t)count);
    if (ce != cudaSuccess) {
        delete S;
        return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "experts_load: %zu bytes: %s", per * (size_t)count,
                                cudaGetErrorString(ce));
    }
    cudaStream_t st = (cudaStream_t)stream;
    void *stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int rc = DSV4CU_OK;
    for (int i = 0; i < 2 && rc == DSV4CU_OK; i++) {
        if (cudaHostAlloc(&stage[i], per, cudaHostAllocDefault) != cudaSuccess ||
            cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess)
            rc = dsv4cu_set_error(DSV4CU_ERR_NOMEM, "experts_load: pinned staging of %zu bytes", per);
    }
    for (int i = 0; i < count && rc == DSV4CU_OK; i++) {
        const int b = i & 1;
        if (i >= 2 && cudaEventSynchronize(done[b]) != cudaSuccess) {   // the copy that last used this buffer
            rc = dsv4cu_set_error(DSV4CU_ERR_CUDA, "experts_load: staging copy failed");
            break;
        }
        const Loc *l = &ix.rec[((size_t)layer * ix.n_experts + first + i) * EXP_TENSORS];
        for (int t = 0; t < EXP_TENSORS && rc == DSV4CU_OK; t++)
            if (read_all(sh.fd[l[t].shard], l[t].off, l[t].nbytes, (char *)stage[b] + off[t]))
                rc = dsv4cu_set_error(DSV4CU_ERR_IO, "experts_load: short read, layer %d expert %d tensor %d", layer,
                                      first + i, t);
        if (rc) break;
        char *dst = (char *)S->dev + per * (size_t)i;
        if (cudaMemcpyAsync(dst, stage[b], per, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaEventRecord(done[b], st) != cudaSuccess) {
            rc = dsv4cu_set_error(DSV4CU_ERR_CUDA, "experts_load: copy to the device failed");
            break;
        }
        dsv4cu_expert &E = experts[i];
        const int rows[3] = {inter, inter, hidden}, cols[3] = {hidden, hidden, inter};
        dsv4cu_qmat *ms[3] = {&E.w1, &E.w3, &E.w2};
        const int wt[3] = {EXP_W1W, EXP_W3W, EXP_W2W};
        for (int m = 0; m < 3; m++) {
            ms[m]->w = dst + off[wt[m]];
            ms[m]->s = dst + off[wt[m] + 1];
            ms[m]->wdt = DSV4CU_WFP4;
            ms[m]->rows = rows[m];
            ms[m]->cols = cols[m];
            ms[m]->blk_r = 1;
            ms[m]->blk_c = 32;
        }
    }
    if (cudaStreamSynchronize(st) != cudaSuccess && rc == DSV4CU_OK)
        rc = dsv4cu_set_error(DSV4CU_ERR_CUDA, "experts_load: copy to the device failed");
    for (int i = 0; i < 2; i++) {
        if (stage[i]) cudaFreeHost(stage[i]);
        if (done[i]) cudaEventDestroy(done[i]);
    }
    if (rc) {
        cudaFree(S->dev);
        delete S;
        return rc;
    }
    *out = S;
    return DSV4CU_OK;
}

extern "C" void dsv4cu_experts_free(dsv4cu_expert_store *s)
{
    if (!s) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(s->device);
    cudaFree(s->dev);
    cudaSetDevice(cur);
    delete s;
}
