// mx_kernel.cuh - the persistent tcgen05 block-scaled GEMM kernel template.
//
// One kernel body serves every packed-weight product of the library: a
// problem policy P says how many tiles there are, where each tile's operands
// live and what its epilogue does with the fp32 results.
//
// A tile is 128 weight rows (the MMA's M) x NB activation columns (N). The
// A operand is a packed matrix in the reference pack layout (FP4 e2m1 or FP8
// e4m3), loaded by TMA from a tensor map in 128-row x 128-element boxes with
// 128-byte swizzle; FP4 boxes use the TMA type that spreads 16 values over 16
// shared-memory bytes, the operand form kind::mxf8f6f4 reads. The B operand
// is the activation written as e4m3 terms (mx_split128): NB rows of a term
// buffer, same box shape. Scale factors come as prepared 512-byte blocks (one
// per 128 rows x 128 K) by 1-D bulk copy and reach TMEM through tcgen05.cp.
//
// Roles (192 threads, one CTA per SM, persistent over tiles):
//   warp 0      producer: KB consecutive 128-wide K chunks per stage (A, B
//               and both scale blocks per chunk) into a STAGES-deep ring;
//   warp 1      TMEM owner and single-thread MMA issuer: per chunk two
//               scale copies and four K = 32 MMAs, then the stage goes back
//               to the producer (tcgen05.commit); after a tile's last stage
//               the accumulator goes to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld (TMEM lane = tile row), the terms of a
//               token summed, then P::store per value and P::finish per tile;
//               after the CTA's last tile P::finish_all (cross-CTA reductions).
// Two accumulators in TMEM (when they fit) let tile i's epilogue overlap tile
// i+1's MMAs. Waits are bounded by 2 s of %globaltimer: a timeout records an
// error code, the roles stop, in-flight copies and MMAs drain, TMEM is freed.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "tma_gemv.cuh"
#include "umma.cuh"

namespace dsv4cu {

// Operands of one tile, as the policy describes them.
struct MxTile {
    const CUtensorMap *ta;   // A tensor map (global or parameter memory)
    const uint8_t *sfa;      // A scale blocks of this row tile: [kc][512]
    const uint8_t *sfb;      // B scale blocks of this column tile: [kc][NBB][512]
    uint32_t idesc;          // MMA instruction descriptor (formats, M, N)
    uint32_t a_tx;           // global bytes of one A box
    int a_row;               // first weight row
    int b_row;               // first row of the B term buffer
    int k0;                  // first 128-wide K chunk (a K segment of a split tile)
    int kc;                  // 128-wide K chunks of this tile
    // K segments accumulated separately, in order, each handed to the
    // epilogue on its own: the tile's kc chunks form kst equal granules and
    // segment s covers granules [s * kst / nseg, (s + 1) * kst / nseg).
    int nseg, kst;
    int id0, id1, id2, id3;  // problem-specific tile coordinates
    int once;                // 1: no other tile reads these weights (they stream with L2 evict-first)
};

constexpr int MX_THREADS = 192;
constexpr int MX_TCACHE = 32;
// Dynamic shared memory for the stage ring: 227 KB less the 1 KB alignment
// slack and 4 KB for the kernel's static shared variables.
constexpr int MX_SMEM_BUDGET = 227 * 1024 - 1024 - 4096;

// STG: ring stages (0 = as many as the shared-memory budget holds). A small
// ring (a few stages) leaves room on the SM for the next kernel's CTA, which
// can then fetch its first weight tiles while this kernel finishes.
template <int NB, int KB, int STG = 0>
struct MxCfg {
    static constexpr int NBB = (NB + 127) / 128;          // 128-column scale blocks of B
    static constexpr int A_BOX = 128 * 128;
    static constexpr int B_BOX = NB * 128;
    static constexpr int SFA_BOX = 512;
    static constexpr int SFB_BOX = NBB * 512;
    // Stage: [A x KB][B x KB][SFA x KB][SFB x KB].
    static constexpr int OFF_B = KB * A_BOX;
    static constexpr int OFF_SFA = OFF_B + KB * B_BOX;
    static constexpr int OFF_SFB = OFF_SFA + KB * SFA_BOX;
    static constexpr int STAGE = ((OFF_SFB + KB * SFB_BOX + 1023) / 1024) * 1024;
    static constexpr int FIT = (MX_SMEM_BUDGET / STAGE) < 16 ? (MX_SMEM_BUDGET / STAGE) : 16;
    static constexpr int STAGES = STG > 0 && STG < FIT ? STG : FIT;
    static constexpr int SMEM = STAGES * STAGE + 1024;
    static constexpr int SF_SLOTS = 2 * KB < 4 ? 4 : 2 * KB;
    static constexpr int SFB_COLS = 4 * NBB;
    static constexpr int SF_COLS = SF_SLOTS * (4 + SFB_COLS);
    static constexpr int ACC_BUFS = (2 * NB + SF_COLS <= 512) ? 2 : 1;
    static constexpr int SFA_COL = ACC_BUFS * NB;
    static constexpr int SFB_COL = SFA_COL + 4 * SF_SLOTS;
    static constexpr int USED = SFB_COL + SFB_COLS * SF_SLOTS;
    static constexpr int TMEM_COLS = USED <= 32 ? 32 : USED <= 64 ? 64 : USED <= 128 ? 128 : USED <= 256 ? 256 : 512;
    static_assert(NB == 8 || NB == 16 || (NB % 32 == 0 && NB >= 32 && NB <= 256), "NB: 8, 16 or 32..256 by 32");
    static_assert(KB == 1 || KB == 2 || KB == 4, "KB: 1, 2 or 4");
    static_assert(STAGES >= 2, "at least two stages");
    static_assert(USED <= 512, "TMEM budget");
};

enum { MXE_EMPTY = 21, MXE_FULL = 22, MXE_ACC_EMPTY = 23, MXE_ACC_FULL = 24, MXE_DRAIN = 25, MXE_BAD_EXPERT = 26 };

DSV4CU_DEV void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Named barrier of the four epilogue warps.
DSV4CU_DEV void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Exact split of 128 consecutive fp32 values (one 128-wide K chunk; lane l
// holds values 4l .. 4l+3, so lanes 8b .. 8b+7 hold 32-block b) into `terms`
// (<= 4) e4m3 terms with one E8M0 scale per 32-block and term:
//   s_0   = the smallest power of two with max|x| <= 448 s_0 over the block,
//   s_j   = s_0 * 2^(-4j),
//   q_j   = RNE_e4m3(r_j / s_j),   r_0 = x,   r_{j+1} = r_j - q_j s_j (exact).
// |r_j| <= 448 s_j holds for every j (after a term the residual is at most
// half an e4m3 step, 16 s_j = 256 s_{j+1}), so no term saturates, and the
// remaining error is at most 16 s_{T-1}: about 2^(-4T) of the block maximum.
// q[j] returns this lane's 4 bytes of term j (byte i = value 4l + i);
// sb[j] the block's scale byte. Non-finite values stay out of the block
// maximum: NaN stays NaN, infinities saturate. Whole warp.
DSV4CU_DEV void mx_split128(const float (&v)[4], int terms, uint32_t (&q)[4], uint8_t (&sb)[4])
{
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) a = fmaxf(a, isfinite(v[i]) ? fabsf(v[i]) : 0.0f);
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 2));
    a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 4));
    int e0 = 0;
    if (a > 0.0f) {
        int E;
        const float f = frexpf(a, &E);
        e0 = max(-127, min(127, E - 9 + (f > 0.875f ? 1 : 0)));
    }
    float r[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (j >= terms) break;
        const int e = max(-127, e0 - 4 * j);
        const float inv = ldexpf(1.0f, -e), sc = ldexpf(1.0f, e);
        uint16_t lo, hi;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(r[1] * inv), "f"(r[0] * inv));
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(r[3] * inv), "f"(r[2] * inv));
        q[j] = (uint32_t)lo | ((uint32_t)hi << 16);
        sb[j] = (uint8_t)(127 + e);
        uint32_t h01, h23;
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h01) : "h"(lo));
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h23) : "h"(hi));
        const float2 f01 = __half22float2(*reinterpret_cast<const __half2 *>(&h01));
        const float2 f23 = __half22float2(*reinterpret_cast<const __half2 *>(&h23));
        r[0] = r[0] - f01.x * sc;
        r[1] = r[1] - f01.y * sc;
        r[2] = r[2] - f23.x * sc;
        r[3] = r[3] - f23.y * sc;
    }
}

// Writes the terms of one 128-value chunk: term j goes to row_j[j] (bytes
// 4l .. 4l+3 of the chunk from lane l) and its scale to sf_j[j][kb] with kb =
// lane / 8 (the lane that starts each 32-block writes it).
DSV4CU_DEV void mx_store128(const uint32_t (&q)[4], const uint8_t (&sb)[4], int terms, uint8_t *const (&row)[4],
                            uint8_t *const (&sf)[4], const int (&sf_step)[4])
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (j >= terms) break;
        *reinterpret_cast<uint32_t *>(row[j] + 4 * lane) = q[j];
        if ((lane & 7) == 0) sf[j][(lane >> 3) * sf_step[j]] = sb[j];
    }
}

// Byte offset of column n's scale for K block kb inside a [NBB][512] group.
DSV4CU_DEV int mx_sfb_offset(int n, int kb)
{
    return (n >> 7) * 512 + (n & 31) * 16 + ((n & 127) >> 5) * 4 + kb;
}

template <int NB, int KB, class P, int STG = 0>
__global__ void __launch_bounds__(MX_THREADS, 1)
    mx_kernel(const __grid_constant__ CUtensorMap tb, const __grid_constant__ typename P::Params p)
{
    using C = MxCfg<NB, KB, STG>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t mx_smem_raw[];
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], accf[2], acce[2], drain;
    __shared__ uint32_t tmem_holder;
    __shared__ volatile int abort_flag;
    // The epilogue warps' own stop decision, one slot per segment parity: a
    // slot is written only before the named barrier of its segment and read
    // after it, so the four warps always agree on it.
    __shared__ volatile int epi_stop[2];
    __shared__ int epi_words[64];    // policy scratch (epilogue warps only)
    // Descriptors of this CTA's first MX_TCACHE tiles, resolved once up front
    // (a policy's tile() may chase table entries in global memory).
    __shared__ MxTile tcache[MX_TCACHE];

    uint8_t *smem = (uint8_t *)(((uintptr_t)mx_smem_raw + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = P::err(p);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], 4);
        }
        mbar_init(&drain, 1);
        abort_flag = 0;
        epi_stop[0] = epi_stop[1] = 0;
        fence_mbar_init();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    // Stages whose A operand (weights + scale blocks) is requested before the
    // previous kernel has finished: a policy whose A side and tile list do not
    // depend on that kernel's output fills the first ring's worth early.
    int pre = 0;
    // Weights read by one tile only stream with L2 evict-first; weights that
    // several column tiles share keep the normal policy (they are re-read).
    const uint64_t pol_once = l2_evict_first(), pol_shared = l2_evict_normal();
    if constexpr (P::kPrefetchA) {
        if (threadIdx.x == 0) {
            const int nt0 = P::ntiles_pre(p);   // tiles whose A side is known before the wait
            for (int t = blockIdx.x; t < nt0 && pre < STAGES; t += gridDim.x) {
                const MxTile T = P::tile_pre(p, t);
                const uint32_t tx = KB * (T.a_tx + C::B_BOX + C::SFA_BOX + C::SFB_BOX);
                const int nst = T.kc / KB;
                for (int c = 0; c < nst && pre < STAGES; c++, pre++) {
                    uint8_t *st = smem + pre * C::STAGE;
                    mbar_arrive_expect_tx(&full[pre], tx);
#pragma unroll
                    for (int b = 0; b < KB; b++) {
                        const int kc = T.k0 + c * KB + b;
                        tma_load_2d_hint(st + b * C::A_BOX, T.ta, kc * 128, T.a_row, &full[pre],
                                         T.once ? pol_once : pol_shared);
                        bulk_load(st + C::OFF_SFA + b * C::SFA_BOX, T.sfa + (size_t)kc * C::SFA_BOX, C::SFA_BOX,
                                  &full[pre]);
                    }
                }
            }
        }
    }
    if (warp == 1) {
        umma::tmem_alloc(&tmem_holder, C::TMEM_COLS);
        umma::tmem_relinquish();
    }
    // Set-up above overlaps the previous kernel; its outputs are read below.
    pdl_wait();
    pdl_trigger();
    const int ntiles = P::ntiles(p);
    if (warp >= 2) {
        const int j = threadIdx.x - 64, t = blockIdx.x + j * gridDim.x;
        if (j < MX_TCACHE && t < ntiles) {
            const MxTile T = P::tile(p, t);
            tcache[j] = T;
            // A tile switch usually changes matrices: have the TMA unit fetch
            // the descriptor now rather than on the tile's first load.
            asm volatile("prefetch.tensormap [%0];" ::"l"(T.ta) : "memory");
        }
    }
    umma::fence_before();
    __syncthreads();
    // k-th tile of this CTA (tile index t).
    auto tile_of = [&](int t, int k) -> MxTile { return k < MX_TCACHE ? tcache[k] : P::tile(p, t); };
    umma::fence_after();
    const uint32_t tmem = tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int it = 0, k = 0;
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tb) : "memory");
            for (int t = blockIdx.x; t < ntiles && !abort_flag; t += gridDim.x, k++) {
                const MxTile T = tile_of(t, k);
                const uint32_t tx = KB * (T.a_tx + C::B_BOX + C::SFA_BOX + C::SFB_BOX);
                const int nst = T.kc / KB;
                for (int c = 0; c < nst; c++, it++) {
                    const int s = it % STAGES, r = it / STAGES;
                    uint8_t *st = smem + s * C::STAGE;
                    if (it >= pre) {
                        if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, err, MXE_EMPTY)) {
                            abort_flag = 1;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
                        for (int b = 0; b < KB; b++) {
                            const int kc = T.k0 + c * KB + b;
                            tma_load_2d_hint(st + b * C::A_BOX, T.ta, kc * 128, T.a_row, &full[s],
                                             T.once ? pol_once : pol_shared);
                            bulk_load(st + C::OFF_SFA + b * C::SFA_BOX, T.sfa + (size_t)kc * C::SFA_BOX, C::SFA_BOX,
                                      &full[s]);
                        }
                    }
#pragma unroll
                    for (int b = 0; b < KB; b++) {
                        const int kc = T.k0 + c * KB + b;
                        tma_load_2d(st + C::OFF_B + b * C::B_BOX, &tb, kc * 128, T.b_row, &full[s]);
                        bulk_load(st + C::OFF_SFB + b * C::SFB_BOX, T.sfb + (size_t)kc * C::SFB_BOX, C::SFB_BOX,
                                  &full[s]);
                    }
                }
            }
            // Every issued copy lands before the CTA can exit. (After an abort
            // a stage requested early may lack its B half: its bounded wait
            // gives up long after the A copy has landed.)
            const int hi = it > pre ? it : pre;
            for (int j = max(0, hi - STAGES); j < hi; j++)
                mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int it = 0, tcount = 0, kt = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok && !abort_flag; t += gridDim.x, kt++) {
                const MxTile T = tile_of(t, kt);
                const int gs = T.kc / KB / T.kst;     // stages per granule
                for (int sg = 0; sg < T.nseg && ok; sg++, tcount++) {
                const int ab = tcount % C::ACC_BUFS, use = tcount / C::ACC_BUFS;
                if (use > 0 && !mbar_wait(&acce[ab], (use - 1) & 1, err, MXE_ACC_EMPTY)) {
                    ok = false;
                    break;
                }
                umma::fence_after();
                const uint32_t dacc = tmem + ab * NB;
                const int c0 = sg * T.kst / T.nseg * gs, c1 = (sg + 1) * T.kst / T.nseg * gs;
                for (int c = c0; c < c1; c++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&full[s], (it / STAGES) & 1, err, MXE_FULL)) {
                        ok = false;
                        break;
                    }
                    umma::fence_after();
                    const uint8_t *st = smem + s * C::STAGE;
#pragma unroll
                    for (int b = 0; b < KB; b++) {
                        const int slot = (it * KB + b) % C::SF_SLOTS;
                        const uint32_t tsfa = tmem + C::SFA_COL + 4 * slot;
                        const uint32_t tsfb = tmem + C::SFB_COL + C::SFB_COLS * slot;
                        umma::cp_sf(tsfa, umma::desc_sf(st + C::OFF_SFA + b * C::SFA_BOX));
#pragma unroll
                        for (int j = 0; j < C::NBB; j++)
                            umma::cp_sf(tsfb + 4 * j, umma::desc_sf(st + C::OFF_SFB + b * C::SFB_BOX + 512 * j));
                        const uint8_t *sa = st + b * C::A_BOX, *sb = st + C::OFF_B + b * C::B_BOX;
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const uint32_t id = T.idesc | ((uint32_t)k << 4) | ((uint32_t)k << 29);
                            umma::mma_mx(dacc, umma::desc_sw128(sa + 32 * k), umma::desc_sw128(sb + 32 * k), id,
                                         ((c - c0) | b | k) ? 1u : 0u, tsfa | ((uint32_t)k << 30),
                                         tsfb | ((uint32_t)k << 30));
                        }
                    }
                    umma::commit(&empty[s]);
                }
                if (ok) umma::commit(&accf[ab]);
                }
            }
            if (!ok) abort_flag = 1;
            // Every MMA / copy this thread issued completes before TMEM is freed.
            umma::commit(&drain);
            mbar_wait(&drain, 0, err, MXE_DRAIN);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue
        const int q = warp & 3;             // the TMEM lane quarter this warp may read
        const int row_l = q * 32 + lane;
        const int terms = P::terms(p), tpt = P::tpt(p);
        // A stopped MMA warp commits no more accumulators, so the epilogue
        // learns of any abort through its own bounded wait.
        int tcount = 0, kt = 0;
        bool stop = false;
        for (int t = blockIdx.x; t < ntiles && !stop; t += gridDim.x, kt++) {
            const MxTile T = tile_of(t, kt);
            for (int sg = 0; sg < T.nseg; sg++, tcount++) {
            const int ab = tcount % C::ACC_BUFS, use = tcount / C::ACC_BUFS;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&accf[ab], use & 1, err, MXE_ACC_FULL);
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) {
                epi_stop[tcount & 1] = 1;
                abort_flag = 1;
            }
            epi_sync();
            if (epi_stop[tcount & 1]) {
                stop = true;            // every epilogue warp leaves at the same segment
                break;
            }
            umma::fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + ab * NB;
            if constexpr (NB <= 16) {
                // Narrow tiles: all NB columns at once, then per token; the
                // terms of token tl are columns tl, tpt + tl, 2 tpt + tl, ...
                float v[NB];
#pragma unroll
                for (int c8 = 0; c8 < NB; c8 += 8) {
                    float w[8];
                    umma::ld_x8(tbase + c8, w);
#pragma unroll
                    for (int i = 0; i < 8; i++) v[c8 + i] = w[i];
                }
                for (int tl = 0; tl < tpt; tl++) {
                    float a = 0.0f;
                    bool first = true;
#pragma unroll
                    for (int c = 0; c < NB; c++) {
                        if (c % tpt == tl && c / tpt < terms) {
                            a = first ? v[c] : a + v[c];
                            first = false;
                        }
                    }
                    P::store(p, T, row_l, tl, a, sg);
                }
            } else {
                for (int tb = 0; tb < tpt; tb += 8) {
                    float acc[8];
                    umma::ld_x8(tbase + tb, acc);
                    for (int j = 1; j < terms; j++) {
                        float v[8];
                        umma::ld_x8(tbase + j * tpt + tb, v);
#pragma unroll
                        for (int i = 0; i < 8; i++) acc[i] += v[i];
                    }
#pragma unroll
                    for (int i = 0; i < 8; i++) P::store(p, T, row_l, tb + i, acc[i], sg);
                }
            }
            // The accumulator is free once every epilogue warp has read it.
            umma::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[ab]);
            }
            if (stop) break;
            P::finish(p, T, row_l, epi_words);
        }
        if (!stop) P::finish_all(p, row_l, ntiles, epi_words);
    }

    umma::fence_before();
    __syncthreads();
    if (warp == 1) {
        umma::fence_after();
        umma::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// Dynamic shared memory of mx_kernel<NB, KB, P>, set once per device.
template <int NB, int KB, class P, int STG = 0>
static int mx_kernel_prepare()
{
    static volatile int done[64];
    int dev = 0;
    DSV4CU_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && done[dev]) return DSV4CU_OK;
    DSV4CU_CUDA_TRY(cudaFuncSetAttribute(mx_kernel<NB, KB, P, STG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         MxCfg<NB, KB, STG>::SMEM));
    if (dev >= 0 && dev < 64) done[dev] = 1;
    return DSV4CU_OK;
}

}  // namespace dsv4cu
