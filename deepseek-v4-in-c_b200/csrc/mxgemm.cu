// mxgemm.cu - packed-weight GEMM on the sm_100a tensor cores (dense case).
//
// y[t][o] = sum_k x[t][k] * W[o][k] for W in the reference pack layouts (FP4
// e2m1 with 1x32 E8M0 scales, FP8 e4m3 with 128x128 E8M0 scales), computed by
// tcgen05.mma.kind::mxf8f6f4.block_scale (mx_kernel.cuh): the tensor core
// reads the e2m1 / e4m3 weight bytes straight from shared memory and applies
// the E8M0 scales itself, so no CUDA-core instruction touches a weight element.
//
// Activations. The MMA's B operand is e4m3 with one E8M0 scale per 32 values
// and per column. An fp32 activation x is written as a sum of T e4m3 terms
// (mx_split128): each term is its own B column with its own scales and the
// epilogue sums a token's T columns. The remaining error per element is
// below 2^(-4T) of its block's magnitude: T = 3 keeps matmul results within
// the 1e-3 bar with margin, T = 4 is close to fp32, T = 1 is plain MXFP8.
//
// This file holds what every user of the kernel shares (scale-block
// preparation, tensor-map encoding, column tiling) and the dense problem: a
// grid of 128-row x NB-column tiles over one matrix.
#include <cuda.h>
#include <mutex>
#include <stdlib.h>
#include <string.h>

#include "ctx.h"
#include "gemv.h"
#include "mx_kernel.cuh"
#include "mxgemm.h"

namespace dsv4cu {

// Weight scale factors -> 512-byte blocks (128 rows x 4 K-blocks of 32).
__global__ void sfa_blocks_kernel(uint8_t *__restrict__ out, const uint8_t *__restrict__ s, int rows, int cols,
                                  int blk_r, int blk_c, int kc, int tiles_m)
{
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;   // one 32-bit word each
    if (i >= (long)tiles_m * kc * 128) return;
    const int blk = (int)(i >> 7), w = (int)(i & 127);
    const int rt = blk / kc, c = blk - rt * kc;
    const int m0 = w >> 2, m1 = w & 3;
    const int row = rt * 128 + m1 * 32 + m0;
    const int sc = (cols + blk_c - 1) / blk_c;
    uint32_t v = 0;
    if (row < rows) {
        for (int kb = 0; kb < 4; kb++) {
            const int k = (c * 4 + kb) * 32;
            v |= (uint32_t)s[(size_t)(row / blk_r) * sc + k / blk_c] << (8 * kb);
        }
    }
    ((uint32_t *)out)[(size_t)blk * 128 + m0 * 4 + m1] = v;
}

// Activation split for the dense problem: one warp per (token, 128-wide K
// chunk). Column n of column tile tn holds term n / tpt of token tn * tpt +
// n % tpt; columns past terms x tpt only feed accumulator columns that are
// never read.
// Also clears the ncnt split-K tile counters the GEMM after it counts with.
__global__ void __launch_bounds__(256) xsplit_kernel(const float *__restrict__ x, int nt, int K, int ldx, int terms,
                                                     int tpt, int NB, uint8_t *__restrict__ xq,
                                                     uint8_t *__restrict__ sfb, int *__restrict__ cnt, int ncnt)
{
    // The GEMM may launch at once and stream its weights while the previous
    // kernel finishes: weights and scale blocks were complete before this
    // kernel could start (the kernels that write them, the scale-block
    // preparation included, never release their dependents early). x and the
    // buffers written below belong to the previous kernel until it ends.
    pdl_trigger();
    pdl_wait();
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < ncnt; i += (long)gridDim.x * blockDim.x) cnt[i] = 0;
    const long gw = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31, kc = K >> 7;
    if (gw >= (long)nt * kc) return;
    const int tok = (int)(gw / kc), c = (int)(gw - (long)tok * kc);
    const int tn = tok / tpt, tl = tok - tn * tpt, nbb = (NB + 127) / 128;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = x[(size_t)tok * ldx + c * 128 + 4 * lane + i];
    uint32_t q[4];
    uint8_t sb[4];
    mx_split128(v, terms, q, sb);
    uint8_t *row[4], *sf[4];
    int step[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int n = j * tpt + tl;
        row[j] = xq + ((size_t)tn * NB + n) * K + c * 128;
        sf[j] = sfb + ((size_t)tn * kc + c) * nbb * 512 + mx_sfb_offset(n, 0);
        step[j] = 1;
    }
    mx_store128(q, sb, terms, row, sf, step);
}

// ------------------------------------------------------------ dense policy
// K is cut into S segments of whole granules (g = 4, 2 or 1 chunks, the
// largest dividing kc; segment s covers granules [s * kst / S, (s + 1) * kst /
// S) of kst = kc / g). S depends on the matrix and the SM count only, never
// on the token count, and y = ((p_0 + p_1) + p_2) + ... over the segment
// partials p_s in every case, so a token's result is the same bits in a
// batch of any size. Two ways of running it:
//   cross (few tiles): tile t = (seg * tiles_n + tn) * tiles_m + tm, one
//     segment per tile on its own CTA, partials to part[seg]; the CTA that
//     completes a (tm, tn) tile's last segment (a counter per tile) sums the
//     partials in segment order into y;
//   in-CTA (tiles fill the GPU): tile t = tn * tiles_m + tm with nseg = S;
//     the CTA accumulates each segment separately and its epilogue adds it
//     onto y in order (y = p_0, then y = y + p_s).
struct DenseMx {
    struct Params {
        CUtensorMap ta;
        const uint8_t *sfa, *sfb;
        int kc, gran, tiles_m, tiles_n, nb, nbb, S, cross;
        int rows, nt, tpt, terms;
        float *y;        // in-CTA or S == 1: the output; cross: partials [S][nt][ldy]
        float *out;      // cross: the output
        int *cnt;        // cross: completed segments per (tm, tn) tile, cleared by the split kernel
        int ldy;
        uint32_t idesc, a_tx;
        int *err;
        // The packed matrix, read only for a NaN result (ref_row_nan).
        const uint8_t *w, *s;
        int cols, blk_r, blk_c, s_cols, fp4;
    };
    static constexpr bool kPrefetchA = true;    // weights and tiles are known at launch
    DSV4CU_DEV static int ntiles_pre(const Params &p) { return ntiles(p); }
    DSV4CU_DEV static MxTile tile_pre(const Params &p, int t) { return tile(p, t); }
    DSV4CU_DEV static float final_value(const Params &p, int row, float v)
    {
        if (!isnan(v)) return v;
        return ref_row_nan(p.w + (size_t)row * (p.fp4 ? p.cols / 2 : p.cols),
                           p.s + (size_t)(row / p.blk_r) * p.s_cols, p.cols, p.blk_c, p.fp4 != 0);
    }
    DSV4CU_DEV static int ntiles(const Params &p) { return p.tiles_m * p.tiles_n * (p.cross ? p.S : 1); }
    DSV4CU_DEV static int *err(const Params &p) { return p.err; }
    DSV4CU_DEV static int terms(const Params &p) { return p.terms; }
    DSV4CU_DEV static int tpt(const Params &p) { return p.tpt; }
    DSV4CU_DEV static MxTile tile(const Params &p, int t)
    {
        MxTile T;
        const int tm = t % p.tiles_m, rest = t / p.tiles_m, tn = rest % p.tiles_n, seg = rest / p.tiles_n;
        T.ta = &p.ta;
        T.sfa = p.sfa + (size_t)tm * p.kc * 512;
        T.sfb = p.sfb + (size_t)tn * p.kc * p.nbb * 512;
        T.idesc = p.idesc;
        T.a_tx = p.a_tx;
        T.a_row = tm * 128;
        T.b_row = tn * p.nb;
        const int kst = p.kc / p.gran;
        if (p.cross) {
            const int s0 = seg * kst / p.S, s1 = (seg + 1) * kst / p.S;
            T.k0 = s0 * p.gran;
            T.kc = (s1 - s0) * p.gran;
            T.nseg = 1;
            T.kst = 1;
        } else {
            T.k0 = 0;
            T.kc = p.kc;
            T.nseg = p.S;
            T.kst = kst;
        }
        T.id0 = tm;
        T.id1 = tn;
        T.id2 = p.cross ? seg : 0;
        T.id3 = 0;
        T.once = p.tiles_n == 1;   // one column tile: these weights are read by this tile only
        return T;
    }
    DSV4CU_DEV static void store(const Params &p, const MxTile &T, int row_l, int tl, float v, int sg)
    {
        const int row = T.id0 * 128 + row_l, tok = T.id1 * p.tpt + tl;
        if (tl < p.tpt && row < p.rows && tok < p.nt) {
            float *dst = p.y + ((size_t)T.id2 * p.nt + tok) * p.ldy + row;
            // The same thread stored the previous segment's sum here.
            float r = sg ? __fadd_rn(*dst, v) : v;
            if (!p.cross && sg == p.S - 1) r = final_value(p, row, r);
            *dst = r;
        }
    }
    // Cross mode: after its partial stores the CTA counts the segment done;
    // the one that completes the tile sums part[0] + part[1] + ... in order.
    DSV4CU_DEV static void finish(const Params &p, const MxTile &T, int row_l, int *words)
    {
        if (!p.cross) return;
        __threadfence();
        epi_sync();
        if (row_l == 0) words[0] = atomicAdd(p.cnt + T.id1 * p.tiles_m + T.id0, 1) == p.S - 1;
        epi_sync();
        if (!words[0]) return;
        __threadfence();
        const int row = T.id0 * 128 + row_l;
        if (row >= p.rows) return;
        const size_t n = (size_t)p.nt * p.ldy;
        for (int tl = 0; tl < p.tpt; tl++) {
            const int tok = T.id1 * p.tpt + tl;
            if (tok >= p.nt) break;
            const float *src = p.y + (size_t)tok * p.ldy + row;
            float v = __ldcg(src);
            for (int sg = 1; sg < p.S; sg++) v = __fadd_rn(v, __ldcg(src + sg * n));
            p.out[(size_t)tok * p.ldy + row] = final_value(p, row, v);
        }
    }
    DSV4CU_DEV static void finish_all(const Params &, int, int, int *) {}
};

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn mx_encode_fn()
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

int mx_encode_kmajor(CUtensorMap *map, const void *base, bool fp4, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_rows)
{
    EncodeTiledFn enc = mx_encode_fn();
    if (!enc) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                     const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return dsv4cu_set_error(DSV4CU_ERR_CUDA, "cuTensorMapEncodeTiled: %d", (int)r);
    return DSV4CU_OK;
}

// The B-operand maps of a step depend only on the workspace address and the
// shape: encoded once and reused (the encode is a driver call per map).
int mx_cached_bmap(CUtensorMap *out, const void *base, uint64_t inner, uint64_t outer, uint32_t box)
{
    struct Entry {
        const void *base;
        uint64_t inner, outer;
        uint32_t box;
        int device;
        CUtensorMap map;
    };
    static std::mutex mu;
    static Entry cache[16];
    static int next = 0;
    int dev = 0;
    DSV4CU_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    for (const Entry &e : cache)
        if (e.base == base && e.inner == inner && e.outer == outer && e.box == box && e.device == dev) {
            *out = e.map;
            return DSV4CU_OK;
        }
    Entry &e = cache[next];
    int r = mx_encode_kmajor(&e.map, base, false, inner, outer, inner, box);
    if (r) {
        e.base = nullptr;
        return r;
    }
    e.base = base;
    e.inner = inner;
    e.outer = outer;
    e.box = box;
    e.device = dev;
    next = (next + 1) % 16;
    *out = e.map;
    return DSV4CU_OK;
}

bool mx_supported(const dsv4cu_qmat *q)
{
    if (!q || !q->w || !q->s || q->rows <= 0 || q->cols <= 0 || q->cols % 128) return false;
    if (q->blk_r <= 0 || q->blk_c <= 0 || q->blk_c % 32) return false;
    if (q->wdt == DSV4CU_WFP4) return ((uintptr_t)q->w & 31u) == 0 && (q->cols / 2) % 32 == 0;
    if (q->wdt == DSV4CU_WFP8) return ((uintptr_t)q->w & 15u) == 0;
    return false;
}

size_t mx_sfa_bytes(const dsv4cu_qmat *q) { return (size_t)((q->rows + 127) / 128) * (q->cols / 128) * 512; }

int mx_prepare(MxMat *m, const dsv4cu_qmat *q, uint8_t *sfa_buf, cudaStream_t st)
{
    memset(m, 0, sizeof(*m));
    if (!mx_supported(q))
        return dsv4cu_set_error(DSV4CU_ERR_UNSUPPORTED,
                                "mx matrix: needs FP4/FP8, cols %% 128 == 0, blk_c %% 32 == 0, aligned weights");
    m->q = *q;
    m->fp4 = q->wdt == DSV4CU_WFP4;
    m->kc = q->cols / 128;
    m->tiles_m = (q->rows + 127) / 128;
    const size_t rb = m->fp4 ? (size_t)q->cols / 2 : (size_t)q->cols;
    int r = mx_encode_kmajor(&m->ta, q->w, m->fp4, (uint64_t)q->cols, (uint64_t)q->rows, rb, 128);
    if (r) return r;
    if (sfa_buf) {
        m->sfa = sfa_buf;
    } else {
        DSV4CU_CUDA_TRY(cudaMalloc((void **)&m->sfa, mx_sfa_bytes(q)));
        m->owns_sfa = 1;
    }
    const long words = (long)m->tiles_m * m->kc * 128;
    sfa_blocks_kernel<<<(unsigned)((words + 255) / 256), 256, 0, st>>>(m->sfa, (const uint8_t *)q->s, q->rows,
                                                                       q->cols, q->blk_r, q->blk_c, m->kc, m->tiles_m);
    DSV4CU_LAUNCH_CHECK();
    return DSV4CU_OK;
}

void mx_release(MxMat *m)
{
    if (m && m->owns_sfa && m->sfa) cudaFree(m->sfa);
    if (m) m->sfa = nullptr;
}

MxTiling mx_tiling(int nt, int terms, int nb_req, int kb_req, int kc)
{
    MxTiling t;
    if (nb_req) t.NB = nb_req;
    else if (nt * terms <= 8) t.NB = 8;          // decode
    else if (nt * terms <= 16) t.NB = 16;
    else if (nt <= (32 / terms) / 8 * 8) t.NB = 32;
    else if (nt <= (64 / terms) / 8 * 8) t.NB = 64;
    else t.NB = (terms == 3) ? 192 : 256;
    // Tiles wider than 16 columns are read back 8 columns at a time per term.
    t.tpt = t.NB <= 16 ? t.NB / terms : (t.NB / terms) / 8 * 8;
    t.tiles_n = t.tpt > 0 ? (nt + t.tpt - 1) / t.tpt : 0;
    // K chunks per stage: narrow tiles stream many bytes per MMA, so fewer
    // barrier round trips per byte pay; wide tiles need the stage count.
    t.KB = kb_req ? kb_req : (t.NB <= 16 ? 4 : t.NB <= 64 ? 2 : 1);
    while (t.KB > 1 && kc % t.KB) t.KB >>= 1;
    return t;
}

// Granule of the K segmentation: the largest of 4, 2, 1 chunks dividing kc
// (every tiling's chunks per stage divide it).
static int dense_gran(int kc) { return kc % 4 == 0 ? 4 : kc % 2 == 0 ? 2 : 1; }

// K segments of a matrix, sized for the one-token product: S minimises the
// longest CTA's share, ceil(tiles_m * S / sms) tiles of ceil(kst / S)
// granules, and must beat one segment by 10 %.
static int dense_segments(int tiles_m, int kc, int sms)
{
    if (tiles_m >= sms) return 1;
    const int kst = kc / dense_gran(kc);
    int S = 1;
    long best = kst;
    for (int c = 2; c <= MX_MAX_SEGMENTS && c <= kst; c++) {
        const long cost = (long)(((long)tiles_m * c + sms - 1) / sms) * ((kst + c - 1) / c);
        if (cost * 10 < best * 9 && (S == 1 || cost < best)) {
            best = cost;
            S = c;
        }
    }
    return S;
}

// Segments run on separate CTAs (partials + reduction) while the tiles leave SMs idle.
static bool dense_cross(int tiles, int S, int sms) { return S > 1 && tiles < sms; }

int mx_device_sms()
{
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return 148;
    return n;
}

// Workspace: B terms, B scale blocks, and in cross mode (S > 1) the partials
// [S][nt][rows] and one counter per tile.
static size_t dense_ws(int K, int kc, const MxTiling &t, int nt, int rows, int S)
{
    const size_t cols = (size_t)t.tiles_n * t.NB;
    size_t b = dsv4cu_align256(cols * K) + dsv4cu_align256((size_t)t.tiles_n * kc * ((t.NB + 127) / 128) * 512);
    if (S > 1)
        b += dsv4cu_align256((size_t)S * nt * rows * 4) + dsv4cu_align256((size_t)((rows + 127) / 128) * t.tiles_n * 4);
    return b;
}

size_t mx_workspace(const MxMat *m, int nt, int terms, int sms)
{
    // The widest tiling any configuration of this call may pick.
    size_t best = 0;
    const int nbs[7] = {8, 16, 32, 64, 128, 192, 256};
    for (int i = 0; i < 7; i++) {
        for (int kb = 1; kb <= 4; kb *= 2) {
            const MxTiling t = mx_tiling(nt, terms, nbs[i], kb, m->kc);
            if (t.tpt <= 0) continue;
            const int S = dense_segments(m->tiles_m, m->kc, sms);
            const int Sx = dense_cross(m->tiles_m * t.tiles_n, S, sms) ? S : 1;
            const size_t b = dense_ws(m->q.cols, m->kc, t, nt, m->q.rows, Sx);
            if (b > best) best = b;
        }
    }
    return best;
}

template <int NB, int KB, int STG = 0>
static int dense_launch(const CUtensorMap &tb, const DenseMx::Params &p, int sms, cudaStream_t st)
{
    int r = mx_kernel_prepare<NB, KB, DenseMx, STG>();
    if (r) return r;
    const int tiles = p.tiles_m * p.tiles_n * (p.cross ? p.S : 1);
    DSV4CU_CUDA_TRY(launch_pdl(mx_kernel<NB, KB, DenseMx, STG>, dim3(tiles < sms ? tiles : sms), dim3(MX_THREADS),
                               MxCfg<NB, KB, STG>::SMEM, st, tb, p));
    return DSV4CU_OK;
}

// One- and two-token products with the automatic tiling: 8-column tiles with
// a 5-stage ring of single K chunks (91 KB), one CTA per SM. The SM keeps
// room for the next product's CTA, which fetches its first weight tiles
// while this one finishes (the weights never depend on the previous kernel).
constexpr int MX_GEMV_STAGES = 5;

static int dense_dispatch(const MxTiling &t, const CUtensorMap &tb, const DenseMx::Params &p, int sms,
                          cudaStream_t st);

int mx_gemm(const MxMat *m, float *y, const float *x, int nt, int terms, int nb_req, int kb_req, void *ws, int sms,
            int *err, cudaStream_t st, cudaEvent_t *ev)
{
    if (terms < 1 || terms > 4) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mx gemm: terms must be 1..4");
    if (nt <= 0) return DSV4CU_OK;
    const MxTiling t = mx_tiling(nt, terms, nb_req, kb_req, m->kc);
    if (t.tpt <= 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mx gemm: %d columns cannot hold %d terms", t.NB, terms);
    const int K = m->q.cols;
    DenseMx::Params p;
    memset(&p, 0, sizeof(p));
    p.ta = m->ta;
    p.kc = m->kc;
    p.gran = dense_gran(m->kc);
    p.tiles_m = m->tiles_m;
    p.tiles_n = t.tiles_n;
    p.nb = t.NB;
    p.nbb = (t.NB + 127) / 128;
    p.S = dense_segments(m->tiles_m, m->kc, sms);
    p.cross = dense_cross(m->tiles_m * t.tiles_n, p.S, sms) ? 1 : 0;
    p.rows = m->q.rows;
    p.nt = nt;
    p.tpt = t.tpt;
    p.terms = terms;
    p.ldy = m->q.rows;
    p.idesc = umma::idesc_mx(m->fp4 ? umma::FMT_E2M1 : umma::FMT_E4M3, umma::FMT_E4M3, 128, t.NB);
    p.a_tx = m->fp4 ? 128 * 64 : 128 * 128;
    p.err = err;
    p.w = (const uint8_t *)m->q.w;
    p.s = (const uint8_t *)m->q.s;
    p.cols = K;
    p.blk_r = m->q.blk_r;
    p.blk_c = m->q.blk_c;
    p.s_cols = (K + m->q.blk_c - 1) / m->q.blk_c;
    p.fp4 = m->fp4 ? 1 : 0;
    uint8_t *xq = (uint8_t *)ws;
    uint8_t *sfb = xq + dsv4cu_align256((size_t)t.tiles_n * t.NB * K);
    p.sfa = m->sfa;
    p.sfb = sfb;
    float *part = (float *)(sfb + dsv4cu_align256((size_t)t.tiles_n * m->kc * p.nbb * 512));
    int *cnt = p.cross ? (int *)((char *)part + dsv4cu_align256((size_t)p.S * nt * m->q.rows * 4)) : nullptr;
    const int ncnt = p.cross ? m->tiles_m * t.tiles_n : 0;
    p.y = p.cross ? part : y;
    p.out = y;
    p.cnt = cnt;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[0], st));
    {
        const long warps = (long)nt * (K / 128);
        DSV4CU_CUDA_TRY(launch_pdl(xsplit_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, st, x,
                                   nt, K, K, terms, t.tpt, t.NB, xq, sfb, cnt, ncnt));
    }
    CUtensorMap tb;
    int r = mx_cached_bmap(&tb, xq, (uint64_t)K, (uint64_t)t.tiles_n * t.NB, (uint32_t)t.NB);
    if (r) return r;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[1], st));
    if (t.NB == 8 && nb_req == 0 && kb_req == 0) r = dense_launch<8, 1, MX_GEMV_STAGES>(tb, p, sms, st);
    else r = dense_dispatch(t, tb, p, sms, st);
    if (r) return r;
    if (ev) DSV4CU_CUDA_TRY(cudaEventRecord(ev[2], st));
    return DSV4CU_OK;
}

static int dense_dispatch(const MxTiling &t, const CUtensorMap &tb, const DenseMx::Params &p, int sms, cudaStream_t st)
{
    switch (t.NB * 8 + t.KB) {
    case 8 * 8 + 1: return dense_launch<8, 1>(tb, p, sms, st);
    case 8 * 8 + 2: return dense_launch<8, 2>(tb, p, sms, st);
    case 8 * 8 + 4: return dense_launch<8, 4>(tb, p, sms, st);
    case 16 * 8 + 1: return dense_launch<16, 1>(tb, p, sms, st);
    case 16 * 8 + 2: return dense_launch<16, 2>(tb, p, sms, st);
    case 16 * 8 + 4: return dense_launch<16, 4>(tb, p, sms, st);
    case 32 * 8 + 1: return dense_launch<32, 1>(tb, p, sms, st);
    case 32 * 8 + 2: return dense_launch<32, 2>(tb, p, sms, st);
    case 64 * 8 + 1: return dense_launch<64, 1>(tb, p, sms, st);
    case 64 * 8 + 2: return dense_launch<64, 2>(tb, p, sms, st);
    case 128 * 8 + 1: return dense_launch<128, 1>(tb, p, sms, st);
    case 192 * 8 + 1: return dense_launch<192, 1>(tb, p, sms, st);
    case 256 * 8 + 1: return dense_launch<256, 1>(tb, p, sms, st);
    default:
        return dsv4cu_set_error(DSV4CU_ERR_ARG, "mx gemm: no kernel for %d columns x %d K chunks per stage", t.NB,
                                t.KB);
    }
}

}  // namespace dsv4cu

// ------------------------------------------------------------ C ABI
using namespace dsv4cu;

struct dsv4cu_mat {
    MxMat m;
    int device;
};

extern "C" int dsv4cu_mat_create(dsv4cu_mat **out, const dsv4cu_qmat *q, void *stream)
{
    if (!out || !q) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mat_create: NULL argument");
    *out = nullptr;
    dsv4cu_mat *h = (dsv4cu_mat *)calloc(1, sizeof(dsv4cu_mat));
    if (!h) return dsv4cu_set_error(DSV4CU_ERR_NOMEM, "mat_create: host allocation failed");
    DSV4CU_CUDA_TRY(cudaGetDevice(&h->device));
    int r = mx_prepare(&h->m, q, nullptr, (cudaStream_t)stream);
    if (r) {
        mx_release(&h->m);
        free(h);
        return r;
    }
    *out = h;
    return DSV4CU_OK;
}

extern "C" void dsv4cu_mat_destroy(dsv4cu_mat *h)
{
    if (!h) return;
    mx_release(&h->m);
    free(h);
}

extern "C" size_t dsv4cu_mat_workspace(const dsv4cu_mat *h, int nt, int terms)
{
    return h ? mx_workspace(&h->m, nt, terms, mx_device_sms()) : 0;
}

extern "C" int dsv4cu_mat_gemm_cfg(dsv4cu_ctx *ctx, const dsv4cu_mat *h, float *y, const float *x, int nt, int terms,
                                   int nb, int kb, void *stream)
{
    if (!ctx || !h || !y || !x) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mat_gemm: NULL argument");
    if (nt < 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mat_gemm: nt < 0");
    if (nt == 0) return DSV4CU_OK;
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, mx_workspace(&h->m, nt, terms, ctx->sm_count), &ws);
    if (r) return r;
    return mx_gemm(&h->m, y, x, nt, terms, nb, kb, ws, ctx->sm_count, ctx->status, (cudaStream_t)stream);
}

extern "C" int dsv4cu_mat_gemm(dsv4cu_ctx *ctx, const dsv4cu_mat *h, float *y, const float *x, int nt, int terms,
                               void *stream)
{
    return dsv4cu_mat_gemm_cfg(ctx, h, y, x, nt, terms, 0, 0, stream);
}

extern "C" int dsv4cu_mat_gemm_ev(dsv4cu_ctx *ctx, const dsv4cu_mat *h, float *y, const float *x, int nt, int terms,
                                  void *stream, void **events)
{
    if (!ctx || !h || !y || !x || !events) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mat_gemm_ev: NULL argument");
    if (nt < 0) return dsv4cu_set_error(DSV4CU_ERR_ARG, "mat_gemm_ev: nt < 0");
    if (nt == 0) return DSV4CU_OK;
    void *ws = nullptr;
    int r = dsv4cu_ws_get(ctx, mx_workspace(&h->m, nt, terms, ctx->sm_count), &ws);
    if (r) return r;
    return mx_gemm(&h->m, y, x, nt, terms, 0, 0, ws, ctx->sm_count, ctx->status, (cudaStream_t)stream,
                   (cudaEvent_t *)events);
}
