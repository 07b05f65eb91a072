// stream_mv.cuh - the streamed packed GEMV core for decode-sized products
// (one or two tokens per weight row) on sm_100a.
//
// HBM is the bound at decode, and three things decide how close a kernel
// gets to it: the bytes each SM keeps in flight, long sequential DRAM runs,
// and few, large copy requests (a bulk copy costs about 80 cycles of the SM's
// TMA unit however small it is, so 1 KB copies cap a CTA near half of HBM).
// This core moves each pipeline stage - 32 weight rows x 1 KB of row, eight
// 128-byte chunks per row - with ONE 3-D tensor-map copy (dims: 128 bytes,
// rows, chunks; box 128 x 32 x 8; 128-byte swizzle), 4-6 stages (about
// 130-190 KB) in flight per SM. A probe of this copy pattern streams at the
// measured HBM copy peak.
//
// CTA roles (persistent, one CTA per SM):
//   warps 0-15  consumers: warp w takes 64-byte group w of every stage's 32
//               rows (two 16-row MMA tiles sharing one activation load),
//               widens e2m1 / e4m3 to f16 with the hardware converters and
//               reduces with mma.sync against the activation;
//   warp 16     producer (one thread): job queue, stage descriptors, the
//               copies (weight box, the FP4 1x32 scale bytes of the same
//               rows, and each job's activation operand into a shared-memory
//               buffer);
//   warp 17     epilogue: takes each finished job's row values from shared
//               memory and does the policy's stores (and any cross-CTA
//               signalling), so no consumer ever waits on a global fence.
//
// MMA operand mapping (m16n8k16, f16 -> f32; see mma_f16_16816). Lane
// (g, t) = (lane / 4, lane % 4) loads 16 bytes of tile rows pi(g) and
// pi(g) + 8 at byte 16 t of a 64-byte group: its "chunk" (32 FP4 or 16 FP8
// elements, inside one scale block). pi(g) = 4 (g & 1) + g / 2 puts the two
// rows of every quarter-warp in different halves of the swizzle pattern, so
// the 16-byte loads are free of bank conflicts. MMA j of the group takes
// chunk elements 4j .. 4j + 3 of every lane (K positions inside an MMA are a
// free permutation of the dot product, the same for A and B). The activation
// enters as B columns 2c (f16 hi part) and 2c + 1 (lo part) that are nonzero
// only on chunk c's K positions, so the accumulator pair (c0 + c1) of lane
// (g, t) is exactly the row's dot product over chunk t. That partial gets its
// chunk's weight scale (E8M0) and activation factor in fp32: acc += part *
// (s_w * s_x), like the reference applies its block scales to block partials
// (dsv4_matmul_fp4.c:66-69, dsv4_matmul_fp8.c:87-88).
//
// Activations: f16 hi / lo arrays with one power-of-two factor per 32
// elements (value = (hi + lo) * factor): hi = RN_f16(v 2^P), lo =
// RN_f16(v 2^P - hi), max |v| 2^P in [2^14, 2^15) over the block, so about 22
// significant bits survive. A job's operand (its tokens' rows over the whole
// K) is copied once into a shared-memory buffer; two buffers alternate, and a
// job whose operand equals the previous job's reuses its buffer.
//
// Every wait is bounded (MBAR_TIMEOUT_NS of %globaltimer): a wait that runs
// out records an error code in the context status word and the roles stop.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "tma_gemv.cuh"

namespace dsv4cu {

constexpr int SMV_CW = 16;                                 // consumer warps (one 64-byte group each)
constexpr int SMV_THREADS = 32 * (SMV_CW + 2);             // + producer + epilogue
constexpr int SMV_SEG = 1024;                              // weight bytes per row per stage
constexpr int SMV_ROWS = 32;                               // weight rows per stage (two MMA tiles)
constexpr int SMV_WBYTES = SMV_ROWS * SMV_SEG;             // weight box of a stage
constexpr int SMV_SLOT = SMV_WBYTES + SMV_ROWS * 64;       // + FP4 scale bytes (32 rows x 64)
constexpr int SMV_MAXNS = 8;                               // ring stages at most
constexpr int SMV_MAXT = 2;                                // tokens per job
constexpr int SMV_MATS = 2;                                // accumulator parts per job
constexpr int SMV_MAXK = 8192;                             // activation length a buffer holds
constexpr int SMV_SMEM_BUDGET = 227 * 1024;

enum { SMV_E_FULL = 51, SMV_E_EMPTY = 52, SMV_E_EPI = 53, SMV_E_DEP = 54, SMV_E_EPIFREE = 55, SMV_E_BUF = 56 };

// One packed matrix as the streamer reads it: its weight map (3-D, see
// above), for FP4 rows longer than one stage a 2-D map of its scale bytes
// (box 64 x 32), and the raw pointers. FP4: s is [rows][cols / 32]
// (s_ld = cols / 32); FP8: s is the [ceil(rows / blk_r)][s_ld] block grid.
struct SmvMat {
    const CUtensorMap *wmap, *smap;
    const uint8_t *w, *s;
    int rows, cols, row_bytes, fp4, s_ld, blk_r, blk_c;
};

// Stage descriptor, written by the producer into the stage's slot.
struct __align__(16) SmvDesc {
    int job;                       // CTA-local job sequence number, -1: end
    int combo;                     // accumulator part of the job (0 or 1)
    int flags;                     // SMV_F_*
    int fp4;
    int segbytes, kseg0, blk_c, sstr;
    const uint8_t *s8;             // FP8: scale row of this stage's 32 rows
    int bbuf, bk;                  // activation buffer and its row length (K)
    int ntok, e0, e1, e2;          // tokens; policy job coordinates (epilogue)
    int e3;
    int sc_ok;                     // FP8 with 128-column blocks: sc holds the stage's scales
    uint32_t sc[2];                // byte c: E8M0 scale of 128-column chunk c of the segment
};
enum { SMV_F_FLUSH = 1, SMV_F_LAST = 2, SMV_F_FIRST = 4, SMV_F_LOAD = 8 };
// SMV_F_LOAD on a job's first stage: the job copied its activation operand
// into buffer bbuf; the consumers wait for it on bfull[bbuf].

// Finished job handed to the epilogue warp.
struct SmvEpi {
    int job, ncombo, ntok, flags;
    int e0, e1, e2, e3;
};

// Launch geometry shared by every policy: ring depth, activation buffers
// (count and bytes per token), computed on the host (smv_geometry).
struct SmvGeom {
    int ns, nbuf, bstride;
};

// Shared state after the ring and the activation buffers. Consumer warps
// never wait for one another: each writes its partials of a job into
// red[b][warp] and arrives on epi_full[b] (16 arrivals); the epilogue warp
// sums them in warp order, then frees the buffer (epi_empty[b]).
template <int NT>
struct SmvSmem {
    uint64_t full[SMV_MAXNS], empty[SMV_MAXNS];
    uint64_t epi_full[2], epi_empty[2];
    uint64_t bfull[2];                 // activation operand of buffer b landed
    SmvDesc desc[SMV_MAXNS];
    SmvEpi epi[2];
    float red[2][SMV_CW][SMV_MATS][SMV_ROWS][NT];
    uint4 zero[4];                     // B operand of the lanes that supply none
    int bdone[2];                      // consumer-warp job completions per activation buffer
    uint32_t drain_valid, drain_par;   // producer's last stage per slot, stored when it stops
    uint32_t drain_b;                  // bit b: buffer b was loaded; bit 2 + b: parity of its last load
    int abort_flag;
};

// Bytes of one token's activation operand in a buffer: hi, lo (2 bytes each
// per element) and the per-32 factors, rounded to 128 bytes.
static inline __host__ __device__ int smv_bytes_per_token(int K) { return ((4 * K + K / 8) + 127) / 128 * 128; }

template <int NT>
static inline SmvGeom smv_geometry(int kmax, int nbuf)
{
    SmvGeom g;
    g.nbuf = nbuf;
    g.bstride = smv_bytes_per_token(kmax);
    const int fixed = 1024 + nbuf * NT * g.bstride + (int)((sizeof(SmvSmem<NT>) + 127) / 128 * 128);
    g.ns = (SMV_SMEM_BUDGET - fixed) / SMV_SLOT;
    if (g.ns > SMV_MAXNS) g.ns = SMV_MAXNS;
    return g;
}
template <int NT>
static inline int smv_smem_bytes(const SmvGeom &g)
{
    return 1024 + g.ns * SMV_SLOT + g.nbuf * NT * g.bstride + (int)((sizeof(SmvSmem<NT>) + 127) / 128 * 128);
}

DSV4CU_DEV int smv_aborted(const int *f) { return *(const volatile int *)f; }

DSV4CU_DEV void smv_bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Tensor-map copies (no multicast); the innermost coordinate is 0 or a
// multiple of 64 bytes.
// Weights stream with the L2 evict-first policy (l2_evict_first).
DSV4CU_DEV void smv_tma_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint32_t bar, uint64_t pol)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
                 " [%0], [%1, {%2, %3, %4}], [%5], %6;"
                 ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(pol)
                 : "memory");
}
DSV4CU_DEV void smv_tma_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar, uint64_t pol)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
                 " [%0], [%1, {%2, %3}], [%4], %5;"
                 ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar), "l"(pol)
                 : "memory");
}

DSV4CU_DEV uint4 smv_lds128(uint32_t a)
{
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    return r;
}
DSV4CU_DEV uint32_t smv_lds8(uint32_t a)
{
    uint32_t r;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(r) : "r"(a));
    return r;
}
DSV4CU_DEV float smv_ldsf(uint32_t a)
{
    float r;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(a));
    return r;
}

// A fragments of one 64-byte group for this lane: rows pi(g) (q0) and
// pi(g) + 8 (q1), 16 bytes each. FP4: byte b of the chunk holds elements 2b
// (low nibble) and 2b + 1; MMA j takes bytes 2j (-> a0 / a1) and 2j + 1
// (-> a2 / a3). FP8: MMA j takes bytes 4j, 4j + 1 (-> a0 / a1) and 4j + 2,
// 4j + 3 (-> a2 / a3).
template <bool FP4>
DSV4CU_DEV void smv_decode(const uint4 &q0, const uint4 &q1, uint32_t (&a)[FP4 ? 8 : 4][4])
{
    const uint32_t w0[4] = {q0.x, q0.y, q0.z, q0.w}, w1[4] = {q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        if constexpr (FP4) {
            cvt_e2m1x8(w0[i], a[2 * i][0], a[2 * i][2], a[2 * i + 1][0], a[2 * i + 1][2]);
            cvt_e2m1x8(w1[i], a[2 * i][1], a[2 * i][3], a[2 * i + 1][1], a[2 * i + 1][3]);
        } else {
            cvt_e4m3x4(w0[i], a[i][0], a[i][2]);
            cvt_e4m3x4(w1[i], a[i][1], a[i][3]);
        }
    }
}

// Tile row held by MMA row g (g < 8) of a lane; row g + 8 is that + 8.
DSV4CU_DEV int smv_pi(int g) { return ((g & 1) << 2) | (g >> 1); }

// Byte address, in a stage's weight box, of 16-byte unit u (0..7) of chunk
// c of stage row r (128-byte swizzle: the unit index XOR the row's low 3 bits).
DSV4CU_DEV uint32_t smv_box_addr(uint32_t wsm, int c, int r, int u)
{
    return wsm + c * (SMV_ROWS * 128) + r * 128 + ((u ^ (r & 7)) << 4);
}

// One stage's share of one consumer warp: 64-byte group `warp` of the
// stage's 32 rows, every token of the job, accumulated into acc[t][2 h + j]
// (tile h = rows 16 h ..; j = 0: row pi(g), j = 1: row pi(g) + 8) of this
// lane's chunk. All operands are in shared memory: weight box, FP4 scales,
// activation buffer; a token's activation is loaded once for both tiles
// (lanes that supply no B column read a zero block).
template <bool FP4, int NT>
DSV4CU_DEV void smv_consume(uint32_t wsm, uint32_t ssm, uint32_t bsm, uint32_t zsm, int bstride, const SmvDesc &d,
                            int warp, float (&acc)[NT][4])
{
    constexpr int MM = FP4 ? 8 : 4, NV = MM / 2;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    if (warp >= (d.segbytes >> 6)) return;
    const bool bact = t == (g >> 1);                // this lane supplies B column g
    const int pr = smv_pi(g);
    const int boff = warp * 64 + 16 * t;            // byte of this lane's chunk in the row segment
    const int kc = d.kseg0 + (FP4 ? 2 * boff : boff);   // first element of the chunk
    const int c = boff >> 7, u = (boff >> 4) & 7;
    const int K = d.bk, ntok = d.ntok;
    float fp8s = 0.0f;
    if constexpr (!FP4)
        fp8s = e8m0_to_f32(d.sc_ok ? (uint8_t)(d.sc[c >> 2] >> (8 * (c & 3))) : __ldg(d.s8 + kc / d.blk_c));
    // Activation of every token of the job for this lane's chunk: one token
    // is loaded once for both tiles, two tokens per tile (the 96-register
    // budget of 576 threads).
    constexpr bool ONCE = NT == 1;
    const uint32_t boffb = ((g & 1) ? 2u * K : 0u) + 2u * kc;     // hi, or lo after hi
    uint4 bv[1][NV];
    float sx[NT];
    auto load_b = [&](int i) {
        const uint32_t tb = bsm + i * bstride;
        const uint32_t src = (bact && i < ntok) ? tb + boffb : zsm;
        const uint32_t step = (bact && i < ntok) ? 16u : 0u;
#pragma unroll
        for (int v = 0; v < NV; v++) bv[0][v] = smv_lds128(src + v * step);
    };
#pragma unroll
    for (int i = 0; i < NT; i++) sx[i] = smv_ldsf(bsm + i * bstride + 4u * K + 4u * (kc >> 5));
    if constexpr (ONCE) load_b(0);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int r0 = 16 * h + pr, r1 = r0 + 8;
        const uint4 q0 = smv_lds128(smv_box_addr(wsm, c, r0, u));
        const uint4 q1 = smv_lds128(smv_box_addr(wsm, c, r1, u));
        float sw0, sw1;
        if constexpr (FP4) {
            sw0 = e8m0_to_f32(smv_lds8(ssm + r0 * d.sstr + (boff >> 4)));
            sw1 = e8m0_to_f32(smv_lds8(ssm + r1 * d.sstr + (boff >> 4)));
        } else {
            sw0 = sw1 = fp8s;
        }
        uint32_t a[MM][4];
        smv_decode<FP4>(q0, q1, a);
#pragma unroll
        for (int i = 0; i < NT; i++) {
            if (i >= ntok) break;
            if constexpr (!ONCE) load_b(i);
            float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f, q0f = 0.f, q1f = 0.f, q2f = 0.f, q3f = 0.f;
#pragma unroll
            for (int j = 0; j < MM; j++) {
                const uint32_t b0 = (j & 1) ? bv[0][j >> 1].z : bv[0][j >> 1].x;
                const uint32_t b1 = (j & 1) ? bv[0][j >> 1].w : bv[0][j >> 1].y;
                if (j & 1) mma_f16_16816(q0f, q1f, q2f, q3f, a[j][0], a[j][1], a[j][2], a[j][3], b0, b1);
                else mma_f16_16816(p0, p1, p2, p3, a[j][0], a[j][1], a[j][2], a[j][3], b0, b1);
            }
            acc[i][2 * h] = fmaf((p0 + p1) + (q0f + q1f), sw0 * sx[i], acc[i][2 * h]);
            acc[i][2 * h + 1] = fmaf((p2 + p3) + (q2f + q3f), sw1 * sx[i], acc[i][2 * h + 1]);
        }
    }
}

// Split 32 values of one block (one per lane) into the f16 hi / lo operand
// with its power-of-two factor.
DSV4CU_DEV void smv_split32(float v, uint16_t &hi, uint16_t &lo, float &fac)
{
    // block maximum of |v| as an unsigned warp max of the bit patterns
    const float a =
        __uint_as_float(__reduce_max_sync(0xFFFFFFFFu, __float_as_uint(isfinite(v) ? fabsf(v) : 0.0f)));
    // P = 15 - e with a = m 2^e, m in [0.5, 1) (frexp's exponent, read from
    // the bits: a subnormal a counts its leading zeros), clamped to +-125, so
    // that 2^P and 2^-P are normal floats and the scalings below are exact
    // (a product that lands below the normal range rounds as ldexp does).
    int P = 0;
    if (a > 0.0f) {
        const uint32_t b = __float_as_uint(a), ef = b >> 23;
        const int e = ef ? (int)ef - 126 : -117 - __clz((int)(b & 0x7FFFFFu));
        P = min(125, max(-125, 15 - e));
    }
    const float vs = __fmul_rn(v, __uint_as_float((uint32_t)(P + 127) << 23));
    const __half hh = __float2half_rn(vs);
    const float hf = __half2float(hh);
    const __half lh = isfinite(hf) ? __float2half_rn(vs - hf) : __float2half_rn(0.0f);
    hi = __half_as_ushort(hh);
    lo = __half_as_ushort(lh);
    fac = __uint_as_float((uint32_t)(127 - P) << 23);
}

// smv_split32 for N blocks of a warp at once (lane holds element `lane` of
// block j in v[j]; live[j] false: skipped), every step as in smv_split32.
template <int N>
DSV4CU_DEV void smv_split32_n(const float (&v)[N], const bool (&live)[N], uint16_t (&hi)[N], uint16_t (&lo)[N],
                              float (&fac)[N])
{
    // Block maxima of |v|: non-negative floats order like their bit patterns,
    // so one unsigned warp max (redux.sync) per block gives the same value as
    // a shuffle tree.
    float a[N];
#pragma unroll
    for (int j = 0; j < N; j++)
        a[j] = __uint_as_float(
            __reduce_max_sync(0xFFFFFFFFu, __float_as_uint(isfinite(v[j]) ? fabsf(v[j]) : 0.0f)));
#pragma unroll
    for (int j = 0; j < N; j++) {
        if (!live[j]) continue;
        int P = 0;
        if (a[j] > 0.0f) {
            const uint32_t b = __float_as_uint(a[j]), ef = b >> 23;
            const int e = ef ? (int)ef - 126 : -117 - __clz((int)(b & 0x7FFFFFu));
            P = min(125, max(-125, 15 - e));
        }
        const float vs = __fmul_rn(v[j], __uint_as_float((uint32_t)(P + 127) << 23));
        const __half hh = __float2half_rn(vs);
        const float hf = __half2float(hh);
        const __half lh = isfinite(hf) ? __float2half_rn(vs - hf) : __float2half_rn(0.0f);
        hi[j] = __half_as_ushort(hh);
        lo[j] = __half_as_ushort(lh);
        fac[j] = __uint_as_float((uint32_t)(127 - P) << 23);
    }
}

// ---------------------------------------------------------------- producer
// Segments of a row and the descriptor fields that depend on one.
DSV4CU_DEV int smv_nseg(const SmvMat &m) { return (m.row_bytes + SMV_SEG - 1) / SMV_SEG; }
DSV4CU_DEV void smv_seg_fields(SmvDesc &d, const SmvMat &m, int row0, int seg)
{
    d.fp4 = m.fp4;
    d.segbytes = min(SMV_SEG, m.row_bytes - seg * SMV_SEG);
    d.kseg0 = seg * (m.fp4 ? 2 * SMV_SEG : SMV_SEG);
    d.blk_c = m.blk_c;
    d.sstr = m.row_bytes <= SMV_SEG ? m.s_ld : SMV_SEG / 16;
    d.s8 = m.fp4 ? nullptr : m.s + (size_t)(row0 / m.blk_r) * m.s_ld;
    // FP8 scales of the segment's (at most 8) 128-column chunks, loaded by the
    // producer before it waits for the slot, so the consumers read them from
    // the descriptor instead of each stage starting with a global load.
    d.sc_ok = !m.fp4 && m.blk_c == 128;
    if (d.sc_ok) {
        const uint8_t *sp = d.s8 + d.kseg0 / 128;
        const int nc = d.segbytes >> 7;
        uint32_t lo = 0u, hi = 0u;
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const uint32_t b = c < nc ? (uint32_t)__ldg(sp + c) : 0u;
            if (c < 4) lo |= b << (8 * c);
            else hi |= b << (8 * (c - 4));
        }
        d.sc[0] = lo;
        d.sc[1] = hi;
    }
}

// Wait (bounded) for a ring slot to be free; the producer thread, which then
// writes the slot, waits.
template <int NT>
DSV4CU_DEV bool smv_slot_free(SmvSmem<NT> &sm, int slot, uint32_t phase, int *status)
{
    return mbar_wait(&sm.empty[slot], phase ^ 1u, status, SMV_E_EMPTY);
}

// Activation operand of a job into buffer b (producer thread): rows row[i]
// of the hi / lo / factor arrays (row length K) for i < ntok, counted on
// bfull[b]. The caller has made sure the buffer is free (smv_buf_pick).
template <int NT>
DSV4CU_DEV void smv_put_operand(uint8_t *bufs, int bstride, int b, SmvSmem<NT> &sm, const uint16_t *hi,
                                const uint16_t *lo, const float *fac, int K, const int *row, int ntok)
{
    const uint32_t bar = smem_u32(&sm.bfull[b]);
    // Phase of this load: one more than the last (the consumers count them).
    const uint32_t par = (sm.drain_b >> b) & 1u ? ((sm.drain_b >> (2 + b)) & 1u) ^ 1u : 0u;
    sm.drain_b = (sm.drain_b & ~(4u << b)) | (1u << b) | (par << (2 + b));
    mbar_arrive_expect_tx(&sm.bfull[b], (uint32_t)ntok * (uint32_t)(4 * K + K / 8));
    for (int i = 0; i < ntok; i++) {
        const uint32_t dst = smem_u32(bufs + (size_t)(b * NT + i) * bstride);
        const size_t r = (size_t)row[i];
        smv_bulk_load(dst, hi + r * K, 2u * K, bar);
        smv_bulk_load(dst + 2u * K, lo + r * K, 2u * K, bar);
        smv_bulk_load(dst + 4u * K, fac + r * (K / 32), K / 8, bar);
    }
}

// Producer bookkeeping of the last stage issued into each slot (parity of
// its fill), kept in registers and stored in shared memory when the
// producer stops, for the drain after an abort.
struct SmvDrain {
    uint32_t valid, par;
};

// Producer side of one stage (producer thread; the slot is free:
// smv_slot_free came first): the descriptor, the expected bytes, the weight
// box and the FP4 scale bytes of its 32 rows.
template <int NT>
DSV4CU_DEV void smv_put_stage(uint8_t *ring, SmvSmem<NT> &sm, SmvDrain &dr, int slot, uint32_t phase,
                              const SmvDesc &d, const SmvMat &m, int row0, int seg)
{
    sm.desc[slot] = d;
    dr.valid |= 1u << slot;
    dr.par = (dr.par & ~(1u << slot)) | (phase << slot);
    const int boxc = min(8, m.row_bytes >> 7);
    const uint32_t sbytes = !m.fp4 ? 0u : (m.row_bytes <= SMV_SEG ? (uint32_t)(SMV_ROWS * m.s_ld) : SMV_ROWS * 64u);
    mbar_arrive_expect_tx(&sm.full[slot], SMV_ROWS * 128u * (uint32_t)boxc + sbytes);
    const uint32_t base = smem_u32(ring + (size_t)slot * SMV_SLOT), bar = smem_u32(&sm.full[slot]);
    const uint64_t pol = l2_evict_first();
    smv_tma_3d(base, m.wmap, 0, row0, seg * 8, bar, pol);
    if (m.fp4) {
        if (m.row_bytes <= SMV_SEG) smv_bulk_load(base + SMV_WBYTES, m.s + (size_t)row0 * m.s_ld, sbytes, bar);
        else smv_tma_2d(base + SMV_WBYTES, m.smap, seg * 64, row0, bar, pol);
    }
}

// Host-side check: can the streamer read this matrix? FP4 with 1x32 scales,
// FP8 with blk_r % 32 == 0 and blk_c % 64 == 0; rows a multiple of 32; rows
// of a multiple of 128 bytes (FP4 cols % 256, FP8 cols % 128); for FP4 rows
// longer than one stage a scale row of a multiple of 16 bytes; 16-byte
// aligned weights and FP4 scales; cols up to SMV_MAXK.
static inline bool smv_ok(int wdt, const void *w, const void *s, int rows, int cols, int blk_r, int blk_c)
{
    if (rows <= 0 || rows % SMV_ROWS || cols <= 0 || cols > SMV_MAXK || cols % 128) return false;
    if ((uintptr_t)w % 16) return false;
    if (wdt == DSV4CU_WFP4) {
        if (blk_r != 1 || blk_c != 32 || cols % 256) return false;
        if (cols / 2 > SMV_SEG && (cols / 32) % 16) return false;
        return (uintptr_t)s % 16 == 0;
    }
    if (wdt == DSV4CU_WFP8) return blk_r > 0 && blk_r % SMV_ROWS == 0 && blk_c > 0 && blk_c % 64 == 0;
    return false;
}

// Host-side: the weight map (and the FP4 scale map when rows span stages).
int smv_encode(const dsv4cu_qmat *q, CUtensorMap *wmap, CUtensorMap *smap);

// A reference-layout matrix descriptor as the streamer reads it.
__host__ __device__ __forceinline__ SmvMat smv_mat(const dsv4cu_qmat &q, const CUtensorMap *wmap,
                                                   const CUtensorMap *smap)
{
    SmvMat m;
    m.wmap = wmap;
    m.smap = smap;
    m.w = (const uint8_t *)q.w;
    m.s = (const uint8_t *)q.s;
    m.rows = q.rows;
    m.cols = q.cols;
    m.fp4 = q.wdt == DSV4CU_WFP4;
    m.row_bytes = m.fp4 ? q.cols / 2 : q.cols;
    m.blk_r = q.blk_r;
    m.blk_c = q.blk_c;
    m.s_ld = m.fp4 ? q.cols / 32 : (q.cols + q.blk_c - 1) / q.blk_c;
    return m;
}

// ----------------------------------------------------- generic role loops
// A policy P supplies: Params (with members SmvGeom geom and int *status),
// producer<NT> (one thread: the job queue - operands, stage descriptors and
// copies, then an end marker) and epilogue<NT> (one finished job, epilogue
// warp).

// Wait (every lane, bounded) for job buffer b to be free; warp-uniform result.
template <int NT>
DSV4CU_DEV bool smv_epi_free(SmvSmem<NT> &sm, int b, uint32_t eph, int *status)
{
    const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.epi_empty[b], eph ^ 1u, status, SMV_E_EPIFREE));
    if (!ok && (threadIdx.x & 31) == 0) atomicExch(&sm.abort_flag, 1);
    return ok;
}

// Job value (part c, row r of 32, token i): the consumer warps' partials in
// order.
template <int NT>
DSV4CU_DEV float smv_job_value(const SmvSmem<NT> &sm, int b, int c, int r, int i)
{
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < SMV_CW; w++) s += sm.red[b][w][c][r][i];
    return s;
}

// Consumer warps. Each runs the stages on its own: no consumer waits for
// another (a job's partials meet in the epilogue warp), and every wait is
// bounded.
template <int NT, class P>
DSV4CU_DEV void smv_consumers(uint8_t *ring, uint8_t *bufs, SmvSmem<NT> &sm, const typename P::Params &p)
{
    const int NS = p.geom.ns, bstride = p.geom.bstride;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int pr = smv_pi(g);
    const uint32_t zsm = smem_u32(&sm.zero[0]);
    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    int slot = 0, eb = 0;
    uint32_t ph = 0, eph = 0, bph = 0;       // bph bit b: phase of bfull[b]
    for (;;) {
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.full[slot], ph, p.status, SMV_E_FULL));
        if (!ok) {
            if (lane == 0) atomicExch(&sm.abort_flag, 1);
            break;
        }
        if (smv_aborted(&sm.abort_flag)) break;
        const SmvDesc d = sm.desc[slot];
        if (d.job < 0) break;
        // The job's partials go to buffer eb: wait until it is free.
        if ((d.flags & SMV_F_FIRST) && !smv_epi_free(sm, eb, eph, p.status)) break;
        if ((d.flags & SMV_F_FIRST) && (d.flags & SMV_F_LOAD)) {
            const int b = d.bbuf;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&sm.bfull[b], (bph >> b) & 1u, p.status, SMV_E_BUF))) {
                if (lane == 0) atomicExch(&sm.abort_flag, 1);
                break;
            }
            bph ^= 1u << b;
        }
        const uint32_t wsm = smem_u32(ring + (size_t)slot * SMV_SLOT);
        const uint32_t bsm = smem_u32(bufs + (size_t)d.bbuf * NT * bstride);
        if (d.fp4) smv_consume<true, NT>(wsm, wsm + SMV_WBYTES, bsm, zsm, bstride, d, warp, acc);
        else smv_consume<false, NT>(wsm, wsm + SMV_WBYTES, bsm, zsm, bstride, d, warp, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
        if (++slot == NS) {
            slot = 0;
            ph ^= 1u;
        }
        if (d.flags & SMV_F_FLUSH) {
            // The four lanes of a row hold its chunk partials: add them, and
            // lane t == 0 writes the rows of this warp's group.
#pragma unroll
            for (int i = 0; i < NT; i++) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float v = acc[i][j];
                    v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
                    v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
                    if (t == 0) sm.red[eb][warp][d.combo][16 * (j >> 1) + pr + 8 * (j & 1)][i] = v;
                    acc[i][j] = 0.0f;
                }
            }
        }
        if (d.flags & SMV_F_LAST) {
            if (warp == 0 && lane == 0) sm.epi[eb] = SmvEpi{d.job, d.e3, d.ntok, 0, d.e0, d.e1, d.e2, 0};
            __syncwarp();
            if (lane == 0) {
                // This warp is done with the job's activation buffer too.
                asm volatile("red.release.cta.shared::cta.add.s32 [%0], 1;" ::"r"(smem_u32(&sm.bdone[d.bbuf]))
                             : "memory");
                mbar_arrive(&sm.epi_full[eb]);
            }
            if (++eb == 2) {
                eb = 0;
                eph ^= 1u;
            }
        }
    }
    // Tell the epilogue warp to stop (every warp arrives once more).
    if (smv_epi_free(sm, eb, eph, p.status)) {
        if (warp == 0 && lane == 0) sm.epi[eb].job = -1;
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.epi_full[eb]);
    }
}

template <int NT, class P>
DSV4CU_DEV void smv_epilogue_loop(SmvSmem<NT> &sm, const typename P::Params &p)
{
    const int lane = threadIdx.x & 31;
    pdl_wait();
    int eb = 0;
    uint32_t eph = 0;
    for (;;) {
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.epi_full[eb], eph, p.status, SMV_E_EPI));
        if (!ok) {
            if (lane == 0) atomicExch(&sm.abort_flag, 1);
            break;
        }
        const SmvEpi e = sm.epi[eb];
        if (e.job < 0) break;
        P::template epilogue<NT>(p, sm, eb, e);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.epi_empty[eb]);
        if (++eb == 2) {
            eb = 0;
            eph ^= 1u;
        }
    }
}

// Producer-side bookkeeping of the activation buffers: which operand each
// holds (a policy key) and how many jobs have used it. Every consumer warp
// counts each finished job once on the counter of the buffer that job used
// (sm.bdone), and no warp can count a job the producer has not issued, so
// bdone[b] == 16 * uses[b] means every warp is done with every job on b.
struct SmvBufState {
    long long key[2];
    int uses[2];
    int cur;
};
DSV4CU_DEV void smv_buf_init(SmvBufState &s)
{
    s.key[0] = s.key[1] = -1;
    s.uses[0] = s.uses[1] = 0;
    s.cur = 0;
}

// Pick the buffer for a job whose operand has key `key` (producer thread):
// the current buffer when it already holds that operand (no copy), else the
// other buffer once every consumer warp has finished every job that used it
// (bounded wait). Returns the buffer (-1 on timeout) and sets *load when the
// operand must be copied.
template <int NT>
DSV4CU_DEV int smv_buf_pick(SmvBufState &s, SmvSmem<NT> &sm, int nbuf, long long key, bool *load, int *status)
{
    if (s.key[s.cur] == key) {
        s.uses[s.cur]++;
        *load = false;
        return s.cur;
    }
    const int b = nbuf > 1 ? s.cur ^ 1 : 0;
    const int need = SMV_CW * s.uses[b];
    if (need > 0) {
        int v;
        asm volatile("ld.acquire.cta.shared::cta.s32 %0, [%1];" : "=r"(v) : "r"(smem_u32(&sm.bdone[b])) : "memory");
        const uint64_t t0 = v < need ? globaltimer_ns() : 0;
        while (v < need) {
            asm volatile("ld.acquire.cta.shared::cta.s32 %0, [%1];" : "=r"(v) : "r"(smem_u32(&sm.bdone[b]))
                         : "memory");
            if (v < need && globaltimer_ns() - t0 > MBAR_TIMEOUT_NS) {
                atomicCAS(status, 0, SMV_E_BUF);
                atomicExch(&sm.abort_flag, 1);
                *load = false;
                return -1;
            }
        }
        // The consumers' reads of the buffer come before the copy's writes.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    s.key[b] = key;
    s.uses[b]++;
    s.cur = b;
    *load = true;
    return b;
}

// End marker for the consumers (also after a producer timeout, which then
// only raises the abort flag), and the producer's drain record. Producer
// thread.
template <int NT>
DSV4CU_DEV void smv_end_marker(SmvSmem<NT> &sm, const SmvDrain &dr, int slot, uint32_t ph, int *status)
{
    sm.drain_valid = dr.valid;
    sm.drain_par = dr.par;
    if (smv_slot_free(sm, slot, ph, status)) {
        sm.desc[slot].job = -1;
        mbar_arrive(&sm.full[slot]);
    } else {
        atomicExch(&sm.abort_flag, 1);
    }
}

// The kernel: warps 0-15 consume, warp 16 produces (one thread), warp 17
// runs epilogues. The consumers touch nothing the previous kernel writes
// except through the producer's operand copies (which come after its
// griddepcontrol.wait), so they need no dependency wait of their own.
template <int NT, class P>
__global__ void __launch_bounds__(SMV_THREADS, 1) smv_kernel(const __grid_constant__ typename P::Params p)
{
    const int NS = p.geom.ns;
    extern __shared__ uint8_t smv_raw[];
    uint8_t *ring = (uint8_t *)(((uintptr_t)smv_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *bufs = ring + (size_t)NS * SMV_SLOT;
    SmvSmem<NT> &sm = *reinterpret_cast<SmvSmem<NT> *>(bufs + (size_t)p.geom.nbuf * NT * p.geom.bstride);
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x < 4) sm.zero[threadIdx.x] = make_uint4(0u, 0u, 0u, 0u);
    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], SMV_CW);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&sm.epi_full[i], SMV_CW);
            mbar_init(&sm.epi_empty[i], 1);
            mbar_init(&sm.bfull[i], 1);
        }
        sm.bdone[0] = sm.bdone[1] = 0;
        sm.abort_flag = 0;
        sm.drain_valid = 0;
        sm.drain_par = 0;
        sm.drain_b = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == SMV_CW) {
        // The producer is one thread: its per-stage path is short and serial.
        if ((threadIdx.x & 31) == 0) P::template producer<NT>(ring, bufs, sm, p);
    } else if (warp == SMV_CW + 1) {
        smv_epilogue_loop<NT, P>(sm, p);
    } else {
        // The policy may build the activation operand in shared memory here
        // (after its dependency wait); the consumer warps then sync once.
        if (P::template consumer_prologue<NT>(bufs, sm, p)) asm volatile("bar.sync 1, %0;" ::"n"(SMV_CW * 32) : "memory");
        smv_consumers<NT, P>(ring, bufs, sm, p);
    }
    // Normally the consumers waited for every stage and operand the producer
    // issued. After a timeout, wait (bounded) for the last copies issued into
    // each slot and buffer, so no copy lands in the shared memory of a CTA
    // that has left.
    __syncthreads();
    if (smv_aborted(&sm.abort_flag) && threadIdx.x == 32 * SMV_CW) {
        for (int i = 0; i < NS; i++)
            if (sm.drain_valid & (1u << i)) mbar_wait(&sm.full[i], (sm.drain_par >> i) & 1u, nullptr, 0);
        for (int b = 0; b < 2; b++)
            if (sm.drain_b & (1u << b)) mbar_wait(&sm.bfull[b], (sm.drain_b >> (2 + b)) & 1u, nullptr, 0);
    }
}

}  // namespace dsv4cu
