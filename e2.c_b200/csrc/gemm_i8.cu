// gemm_i8.cu — W8A8 GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
//   y[m, n] = sum over activation blocks b of  float(dot_b(m, n)) * (as[m, b] * ws[n])
//
// dot_b is the exact int32 dot of the signed int8 activation row and weight row over block b; the
// fold is f = fma(float(dot_b), as*ws, f), blocks in order, as in the reference's AVX512-VNNI kernel
// (src/kernels_i8_avx512_vnni.c:113-119,276-307), so per-row (one block = K) and per-block outputs
// are bit-identical to it. With per-row scales the whole K accumulates in TMEM and the epilogue
// runs once per tile; with per-block scales the accumulator is drained after every block into a
// register-resident fp32 fold while the tensor core fills the other TMEM buffer.
//
// Structure (one CTA per SM, persistent over 128 x BN output tiles):
//   warp 0      TMA producer: A [128 x 128] and B [BN x 128] int8 tiles, 128-byte swizzle,
//               a ring of shared-memory stages guarded by full/empty mbarriers;
//   warp 1      TMEM owner and MMA issuer: 4 x tcgen05.mma (K = 32) per stage into one of two
//               TMEM accumulators (2 x BN columns of int32), tcgen05.commit frees stages;
//   warps 2..17 epilogue, four warps per TMEM lane quadrant, each owning a quarter of the tile's
//               columns: tcgen05.ld, dequant (the columns' weight scales, fetched a tile ahead, read
//               back from shared memory by broadcast loads) and the fused tail (residual, clamp,
//               GELU-gate, per-head RMSNorm + RoPE), results staged in per-warp 64-byte-swizzled
//               shared-memory tiles (two, alternating) and written by TMA stores.
// Tile widths BN = 256, 192 or 128: the launcher picks the one whose waves of tiles over the SMs
// cost least (N = 768 takes 192: 4 column tiles, so 7 nearly full waves of 148 instead of 6 with
// the last one at a fifth).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "launch.h"
#include "epi_math.cuh"
#include "devstate.cuh"
#include "pdl.h"
#include "ptx.cuh"
#include "tmap.h"

namespace {

constexpr int BM = 128;   // tile rows (tokens) = TMEM lanes
constexpr int BK = 128;   // bytes of K per stage = one 128-byte swizzle row
constexpr int EPI_WARPS = 16;
constexpr int NTHREADS = 64 + 32 * EPI_WARPS;
constexpr int STG_WARP = 2048;  // staging bytes per epilogue warp and store (32 rows x 64 bytes)

template <int BN, int STAGES, bool PERBLOCK, int EPI, int CG>
struct GemmSmem {
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = (BN / CG) * BK;  // a CTA pair splits B's rows between its CTAs
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // staging tiles per epilogue warp: QKV stages the two halves of a head; the other epilogues
    // without the per-block fold alternate between two, so a store overlaps the next chunk's math
    static constexpr int STG_BUFS = (EPI == E2C_EPI_QKV || (!PERBLOCK && EPI != E2C_EPI_I32 && CG == 1)) ? 2 : 1;
    // (the per-block GELU-quantise and q|k|v epilogues store from registers)
    static constexpr bool SUBT = EPI == E2C_EPI_GELUQ || EPI == E2C_EPI_QKVPB;
    static constexpr int STG_PER_WARP = SUBT ? 0 : STG_BUFS * STG_WARP;
    static constexpr int STG_OFF = STAGES * STAGE_BYTES;
    // per-warp column constants (weight scales, norm gains): 128 floats (QKV: 256, 64 pairs a warp;
    // per-block mode: the 32 weight scales of the warp; per-block GELU-quantise: its 16 gate and 16
    // up weight scales of each of the two sub-tiles)
    // per-block q|k|v: the weight scales and norm gains of its 32 columns in each half of the head)
    static constexpr int CST_FLOATS = EPI == E2C_EPI_QKV ? 256 : EPI == E2C_EPI_GELUQ ? 64 : EPI == E2C_EPI_QKVPB ? 128
                                    : PERBLOCK ? 32 : 128;
    static constexpr int CST_OFF = STG_OFF + EPI_WARPS * STG_PER_WARP;
    static constexpr int CST_BYTES = EPI == E2C_EPI_I32 ? 0 : EPI_WARPS * CST_FLOATS * 4;
    static constexpr int SSQ_OFF = CST_OFF + CST_BYTES;
    // QKV: [group][part2][row] row sums of squares; per-block GELU-quantise and q|k|v: [tile
    // parity][part][row] row maxima of |h| or sums of squares
    static constexpr int SSQ_BYTES = EPI == E2C_EPI_QKV ? 2 * 2 * BM * 4 : SUBT ? 2 * 4 * BM * 4 : 0;
    static constexpr int BAR_OFF = SSQ_OFF + SSQ_BYTES;
    // TMEM accumulators: per-block mode keeps four (the tensor core runs up to three 128-deep blocks
    // ahead of the drain; the GELU-quantise epilogue three, columns 384.. holding the first
    // sub-tile's h; the q|k|v epilogue two, columns 256.. holding both halves of the head), the
    // others two
    static constexpr int NACC = EPI == E2C_EPI_QKVPB ? 2 : SUBT ? 3 : PERBLOCK ? 4 : 2;
    // full[S], empty[S], tfull[NACC], tempty[NACC], pair[2][4] (the QKV row-norm and per-block
    // GELU-quantise row-maximum exchanges), tmem slot
    static constexpr int NBAR = 2 * STAGES + 2 * NACC + 8;
    static constexpr int BYTES = BAR_OFF + NBAR * 8 + 16;
    static constexpr int ALLOC = BYTES + 1024;  // slack for 1024-byte alignment
    static_assert(ALLOC <= 232448, "shared memory");
};

// ---------------------------------------------------------------------------------- epilogue math
__device__ __forceinline__ float dq(uint32_t acc, float s) { return __fmul_rn(__int2float_rn((int)acc), s); }

// Staging tiles are 32 rows x 64 bytes in the TMA 64-byte-swizzle layout (512-byte aligned): the
// 16-byte chunk c of row r lives at chunk c ^ ((r >> 1) & 3). Row `lane` = the thread's TMEM lane.
__device__ __forceinline__ void stage_f32x16(uint8_t *buf, int lane, const float (&v)[16]) {
    uint8_t *row = buf + lane * 64;
#pragma unroll
    for (int c = 0; c < 4; c++)
        *reinterpret_cast<float4 *>(row + ((c ^ ((lane >> 1) & 3)) << 4)) =
            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}
// hand a staged tile to the TMA engine (one lane), after every lane's writes are visible to it
__device__ __forceinline__ void stage_store(const CUtensorMap *m, uint8_t *buf, int x, int y, int lane) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(m, smem_u32(buf), x, y);
        bulk_commit();
    }
}
// ---------------------------------------------------------------------------------- kernel
template <int BN, int STAGES, bool PERBLOCK, int EPI, int CG>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm_i8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmO0, const __grid_constant__ CUtensorMap tmO1, const e2c_gemm_args p,
              const int tma_out) {
    using L = GemmSmem<BN, STAGES, PERBLOCK, EPI, CG>;
    extern __shared__ uint8_t smem_raw[];
    griddep_launch_dependents();
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    constexpr int NACC = L::NACC;
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + NACC + a); };
    auto pair_bar = [&](int a, int q) { return bar0 + 8u * (2 * STAGES + 2 * NACC + 4 * a + q); };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + L::BAR_OFF + L::NBAR * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = p.M, K = p.K;
    const int ncols = p.n1 - p.n0;
    // A CTA pair (CG = 2, a cluster of two) shares 256-row tiles: rank r owns rows 128 r .. +127.
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
    const int tfirst = CG == 2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int tstride = CG == 2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    // Per-block GELU-quantise: a tile is 256 weight rows (128 gate + 128 up = one 128-column block
    // of h) taken as two sub-tiles of 128 columns, each the gate and up rows of 64 h columns.
    // Per-block q|k|v: a tile is one head of 256 weight rows, taken as its two halves.
    constexpr bool GQ = EPI == E2C_EPI_GELUQ;
    constexpr bool QP = EPI == E2C_EPI_QKVPB;
    constexpr int NSUB = (GQ || QP) ? 2 : 1;
    constexpr int TW = BN * NSUB;                        // weight rows per tile
    static_assert(!(GQ || QP) || (PERBLOCK && BN == 128), "sub-tiled epilogues are per-block ones");
    const int tiles_m = (M + BM * CG - 1) / (BM * CG), tiles_n = (ncols + TW - 1) / TW;
    const int ntiles = tiles_m * tiles_n;
    const int nk = (K + BK - 1) / BK;                    // stages per (sub-)tile
    const int kpu = PERBLOCK ? p.ablk / BK : nk;         // stages per accumulation unit
    const int nunits = PERBLOCK ? K / p.ablk : 1;
    const int nb = K / p.ablk;                           // scale blocks per row
    static_assert(!PERBLOCK || BN == 128, "per-block mode: four 128-column accumulators");
    constexpr uint32_t TMEM_COLS = PERBLOCK ? 512 : BN == 192 ? 512 : 2 * BN;  // a power of two

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < NACC; a++) {
            mbar_init(tfull_bar(a), 1);
            // one arrival per epilogue warp of the pair (QKV: per warp of the group that owns it)
            mbar_init(tempty_bar(a), (EPI == E2C_EPI_QKV ? EPI_WARPS / 2 : EPI_WARPS) * CG);
        }
        // QKV: the quadrant's 2 warps of a group; GELU-quantise: the quadrant's 4 warps
        for (int a = 0; a < 2; a++)
            for (int q = 0; q < 4; q++) mbar_init(pair_bar(a, q), (GQ || QP) ? 128 : 64);
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        __syncwarp();
        if constexpr (CG == 2) {
            tmem_alloc_pair(sbase + L::BAR_OFF + L::NBAR * 8, TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(sbase + L::BAR_OFF + L::NBAR * 8, TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    // a pair: the leader's barriers are initialised before the other CTA signals them
    if constexpr (CG == 2) cluster_sync();
    else __syncthreads();
    tc_fence_after();
    griddep_wait();  // the stream's earlier kernels are done with what this one reads and writes
    const uint32_t tmem_base = *tmem_slot;
    // the accumulator is free again: one arrival per warp on the leader's barrier
    auto release_acc = [&](int a) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            if constexpr (CG == 2) mbar_arrive_cluster(mapa_shared(tempty_bar(a), 0));
            else mbar_arrive(tempty_bar(a));
        }
    };

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (elect_one()) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;  // loads in flight that nobody consumed (drained on failure)
            bool ok = true;
            for (int t = tfirst; t < ntiles && ok; t += tstride) {
                const int m0 = (t / tiles_n) * (BM * CG) + (int)rank * BM, c0 = p.n0 + (t % tiles_n) * TW;
                for (int kb2 = 0; kb2 < NSUB * nk; kb2++) {
                    const int kb = NSUB > 1 ? kb2 % nk : kb2, sub = NSUB > 1 ? kb2 / nk : 0;
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.status, E2C_ERR_WAIT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = sbase + stage * L::STAGE_BYTES, sb = sa + L::A_BYTES;
                    if constexpr (CG == 2) {
                        // both halves complete on the leader's full barrier, which expects both
                        const uint32_t fb = mapa_shared(full_bar(stage), 0);
                        if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * L::STAGE_BYTES);
                        tma_load_2d_pair(sa, &tmA, kb * BK, m0, fb);
                        // GELU-quantise: the first CTA holds the sub-tile's 64 gate rows, the second
                        // its 64 up rows
                        tma_load_2d_pair(sb, &tmB, kb * BK,
                                         GQ ? c0 + 128 * (int)rank + 64 * sub : c0 + BN * sub + (int)rank * (BN / 2), fb);
                    } else {
                        mbar_arrive_expect_tx(full_bar(stage), L::STAGE_BYTES);
                        tma_load_2d(sa, &tmA, kb * BK, m0, full_bar(stage));
                        if constexpr (GQ) {
                            // 64 gate rows, then their 64 up rows (boxes of 64 rows)
                            tma_load_2d(sb, &tmB, kb * BK, c0 + 64 * sub, full_bar(stage));
                            tma_load_2d(sb + 64 * BK, &tmB, kb * BK, c0 + 128 + 64 * sub, full_bar(stage));
                        } else {
                            tma_load_2d(sb, &tmB, kb * BK, c0 + BN * sub, full_bar(stage));
                        }
                    }
                    issued++;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok && rank == 0) {
                // let the copies this thread started land before the CTA's shared memory goes away
                // (a pair's second CTA cannot observe its copies: they complete on the leader)
                int s = stage, ph = phase;
                for (int i = 0; i < (issued < STAGES ? issued : STAGES); i++) {
                    if (--s < 0) {
                        s = STAGES - 1;
                        ph ^= 1;
                    }
                    mbar_wait(full_bar(s), (uint32_t)ph, nullptr, E2C_ERR_WAIT_DRAIN);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        // commits arrive on a barrier of this CTA, or for a pair on that barrier in both CTAs
        auto commit = [&](uint32_t bar) {
            if constexpr (CG == 2) {
                mma_commit_pair(mapa_shared(bar, 0));
                mma_commit_pair(mapa_shared(bar, 1));
            } else {
                mma_commit(bar);
            }
        };
        if (rank == 0 && elect_one()) {
            constexpr uint32_t idesc = idesc_i8(BN, BM * CG);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = tfirst; t < ntiles && ok; t += tstride) {
                for (int u = 0; u < NSUB * nunits && ok; u++) {
                    if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.status, E2C_ERR_WAIT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                    for (int kk = 0; kk < kpu; kk++) {
                        if (!mbar_wait(full_bar(stage), phase, p.status, E2C_ERR_WAIT_MMA)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = sbase + stage * L::STAGE_BYTES, sb = sa + L::A_BYTES;
#pragma unroll
                        for (int k = 0; k < BK / 32; k++) {
                            if constexpr (CG == 2)
                                mma_i8_pair(d, smem_desc_sw128(sa + 32 * k), smem_desc_sw128(sb + 32 * k), idesc,
                                            (kk | k) != 0);
                            else
                                mma_i8(d, smem_desc_sw128(sa + 32 * k), smem_desc_sw128(sb + 32 * k), idesc,
                                       (kk | k) != 0);
                        }
                        commit(empty_bar(stage));
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    commit(tfull_bar(acc));
                    if (++acc == NACC) {
                        acc = 0;
                        acc_phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // every MMA issued so far must finish before the accumulator is released
                const uint32_t drain = tfull_bar(acc);
                if constexpr (CG == 2) mma_commit_pair(mapa_shared(drain, 0));
                else mma_commit(drain);
                mbar_wait(drain, acc_phase, nullptr, E2C_ERR_WAIT_DRAIN);
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int q = warp & 3;                  // TMEM lane quadrant this warp may access
        const int part = (warp - 2) >> 2;        // which quarter of the tile's columns it owns
        const int row = q * 32 + lane;           // row of the tile = TMEM lane
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        uint8_t *stg = smem + L::STG_OFF + (warp - 2) * L::STG_PER_WARP;
        constexpr int QCOLS = BN / 4;            // columns per warp
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        int nst = 0;  // store groups this warp committed
        // the staging tile for the next fp32 store: tiles alternate, and the store that last read
        // the chosen one must have finished reading it
        auto stg_next = [&]() -> uint8_t * {
            uint8_t *buf = stg + (nst % L::STG_BUFS) * STG_WARP;
            if (nst >= L::STG_BUFS) {
                if (lane == 0) {
                    if constexpr (L::STG_BUFS == 2) bulk_wait_read1();
                    else bulk_wait_read0();
                }
                __syncwarp();
            }
            return buf;
        };
        // stage 16 fp32 columns of this warp's 32 rows and store them at (x, y0)
        auto put16 = [&](const float (&v)[16], int x, int y0) {
            uint8_t *buf = stg_next();
            stage_f32x16(buf, lane, v);
            stage_store(&tmO0, buf, x, y0, lane);
            ++nst;
        };
        // Per-tile values that do not depend on the accumulator, fetched one tile ahead: the row's
        // activation scale, and per lane the weight scales (and for QKV the norm gains) of the
        // columns this warp owns. They reach the math through a per-warp shared array (`cst`) read
        // back by broadcast loads, four columns per instruction.
        struct Pre {
            float w0, w1, g0, g1, as;
        };
        auto fetch = [&](int t) -> Pre {
            Pre r{0.f, 0.f, 1.f, 1.f, 0.f};
            if (PERBLOCK || t >= ntiles) return r;
            const int m = (t / tiles_n) * (BM * CG) + (int)rank * BM + row, c0 = p.n0 + (t % tiles_n) * TW;
            if (m < M) r.as = __ldg(p.a_scale + (size_t)m * nb);
            if constexpr (EPI == E2C_EPI_F32 || EPI == E2C_EPI_RESID) {
                const int cw = c0 + part * QCOLS;
                if (lane < QCOLS && cw + lane < p.n1) r.w0 = __ldg(p.w_scale + cw + lane);
                if (32 + lane < QCOLS && cw + 32 + lane < p.n1) r.w1 = __ldg(p.w_scale + cw + 32 + lane);
            } else if constexpr (EPI == E2C_EPI_GELU) {
                // gate | up of this warp's 32 columns
                r.w0 = __ldg(p.w_scale + c0 + 32 * part + lane);
                r.w1 = __ldg(p.w_scale + c0 + 128 + 32 * part + lane);
            }
            return r;
        };
        float *cst = reinterpret_cast<float *>(smem + L::CST_OFF) + (warp - 2) * L::CST_FLOATS;
        // 16 consecutive floats of cst from `off` (a broadcast: every lane reads the same address)
        auto cst16 = [&](int off, float (&o)[16]) {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float4 w = *reinterpret_cast<const float4 *>(cst + off + 4 * k);
                o[4 * k] = w.x, o[4 * k + 1] = w.y, o[4 * k + 2] = w.z, o[4 * k + 3] = w.w;
            }
        };
        if constexpr (EPI == E2C_EPI_QKV) {
            // One 256-column tile = one head (q heads, then k, then v):
            //   x = float(acc) * as * ws;  y = x * inv * gamma, inv = 1/sqrt(mean(x^2) + eps) (v: no
            //   gamma), computed as float(acc) * (ws * gamma) * (as * inv); then RoPE and bf16.
            // Two groups of eight warps take alternate tiles of this CTA (group g: its tiles g, g + 2,
            // ..., accumulator g), so one group's waits (the row-norm exchange, the RoPE loads, TMEM)
            // overlap the other group's arithmetic. In a group, two warps per TMEM lane quadrant:
            // warp part2 owns rotate-half pairs i in [64 part2, 64 part2 + 64) with partners i + 128.
            const int grp = (warp - 2) >> 3;
            const int part2 = ((warp - 2) >> 2) & 1;
            float *cst2 = reinterpret_cast<float *>(smem + L::CST_OFF) + (warp - 2) * L::CST_FLOATS;
            // [0, 64) ws of pairs i, [64, 128) ws of partners, [128, 192) and [192, 256) ws * gamma
            auto c16 = [&](int off, float (&o)[16]) {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const float4 w = *reinterpret_cast<const float4 *>(cst2 + off + 4 * k);
                    o[4 * k] = w.x, o[4 * k + 1] = w.y, o[4 * k + 2] = w.z, o[4 * k + 3] = w.w;
                }
            };
            // the row's activation scale, fetched a tile of this group ahead
            auto fetch_as = [&](int t) -> float {
                if (t >= ntiles) return 0.f;
                const int m = (t / tiles_n) * (BM * CG) + (int)rank * BM + row;
                return m < M ? __ldg(p.a_scale + (size_t)m * nb) : 0.f;
            };
            float *ssq = reinterpret_cast<float *>(smem + L::SSQ_OFF);  // [group][part2][row]
            int nst2 = 0;  // store groups this warp committed
            int j = 0;     // tiles this group finished
            float as_next = fetch_as(tfirst + grp * tstride);
            for (int t = tfirst + grp * tstride; t < ntiles && ok; t += 2 * tstride, j++) {
                const float as = as_next;
                as_next = fetch_as(t + 2 * tstride);
                const uint32_t aph = (uint32_t)(j & 1);
                const int mt = (t / tiles_n) * (BM * CG) + (int)rank * BM;
                const int m = mt + row;
                const int c0 = p.n0 + (t % tiles_n) * TW;
                const bool mrow = m < M;
                const int y0 = mt + q * 32;
                const int head = (c0 - p.n0) / 256;
                const bool is_k = head == p.nq, is_v = head == p.nq + 1;
                const int pos = mrow ? m % p.seq_len : 0;
                // the column constants of the head (per lane: columns lane and lane + 32 of the
                // warp's pairs and of their partners)
                {
                    const float *gamma = is_v ? nullptr : (is_k ? p.k_gamma : p.q_gamma);
                    float wv[4], gv[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int col = (k >> 1) * 128 + 64 * part2 + 32 * (k & 1) + lane;
                        wv[k] = __ldg(p.w_scale + c0 + col);
                        gv[k] = gamma ? __ldg(gamma + col) : 1.f;
                    }
                    __syncwarp();  // every lane is done reading the previous tile's constants
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int o = (k >> 1) * 64 + 32 * (k & 1) + lane;
                        cst2[o] = wv[k];
                        cst2[128 + o] = __fmul_rn(wv[k], gv[k]);
                    }
                    __syncwarp();
                }
                if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(grp), aph, p.status, E2C_ERR_WAIT_EPI))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t tbase = tmem_base + lane_addr + (uint32_t)(grp * BN);
                // pass 1: sum over this warp's 128 columns of (float(acc) * ws)^2, in four independent
                // partial sums (a single fma chain would issue one step per fma latency)
                float ssp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    uint32_t ra[16], rb[16];
                    tmem_ld16(tbase + 64 * part2 + 16 * c, ra);
                    tmem_ld16(tbase + 128 + 64 * part2 + 16 * c, rb);
                    tmem_wait_ld();
                    float wa[16], wb[16];
                    c16(16 * c, wa);
                    c16(64 + 16 * c, wb);
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const float a = __fmul_rn(__int2float_rn((int)ra[e]), wa[e]);
                        const float b = __fmul_rn(__int2float_rn((int)rb[e]), wb[e]);
                        ssp[e & 3] = __fmaf_rn(b, b, __fmaf_rn(a, a, ssp[e & 3]));
                    }
                }
                const float ss = __fadd_rn(__fadd_rn(ssp[0], ssp[1]), __fadd_rn(ssp[2], ssp[3]));
                // the row's sum of squares over the two warps of this quadrant in the group
                ssq[(grp * 2 + part2) * BM + row] = ss;
                mbar_arrive(pair_bar(grp, q));
                // RoPE cos / sin come from pair-major tables ([128][ldrope]: a warp's 32 consecutive
                // positions of one pair are one coalesced 128-byte read), each step's 8 pairs loaded a
                // step ahead, the first step's before the row-norm exchange
                float csn[8], snn[8];
                if (!is_v) {
                    const float *cp = p.rope_cos + (size_t)(64 * part2) * p.ldrope + pos;
                    const float *sp = p.rope_sin + (size_t)(64 * part2) * p.ldrope + pos;
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        csn[k] = __ldg(cp + (size_t)k * p.ldrope);
                        snn[k] = __ldg(sp + (size_t)k * p.ldrope);
                    }
                }
                if (!__all_sync(0xffffffffu, mbar_wait(pair_bar(grp, q), aph, p.status, E2C_ERR_WAIT_EPI))) {
                    ok = false;
                    break;
                }
                const float sst = __fadd_rn(ssq[(grp * 2) * BM + row], ssq[(grp * 2 + 1) * BM + row]);
                const float ms = __fmul_rn(__fmul_rn(as, as), __fdiv_rn(sst, 256.0f));
                const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
                const float rs = __fmul_rn(as, inv);
                // pass 2: eight steps of 8 pairs (8-column TMEM loads, constants four at a time, outputs
                // packed to bf16 pairs at once: few registers live). The two staging tiles (pairs |
                // partners) take 32 pairs each and leave by TMA.
#pragma unroll 1
                for (int c8 = 0; c8 < 8; c8++) {
                    const int ia = 64 * part2 + 8 * c8;  // rotate-half index of these 8 pairs
                    if (!is_v && tma_out && (c8 & 3) == 0 && nst2 > 0) {
                        // the stores that last read the staging tiles have finished reading them
                        if (lane == 0) bulk_wait_read0();
                        __syncwarp();
                    }
                    uint32_t ra[8], rb[8];
                    tmem_ld8(tbase + ia, ra);
                    tmem_ld8(tbase + 128 + ia, rb);
                    float cs[8], sn[8];
#pragma unroll
                    for (int k = 0; k < 8; k++) cs[k] = csn[k], sn[k] = snn[k];
                    if (!is_v && c8 < 7) {
                        const float *cp = p.rope_cos + (size_t)(ia + 8) * p.ldrope + pos;
                        const float *sp = p.rope_sin + (size_t)(ia + 8) * p.ldrope + pos;
#pragma unroll
                        for (int k = 0; k < 8; k++) {
                            csn[k] = __ldg(cp + (size_t)k * p.ldrope);
                            snn[k] = __ldg(sp + (size_t)k * p.ldrope);
                        }
                    }
                    tmem_wait_ld();
                    if (c8 == 7) release_acc(grp);  // every TMEM column this warp reads has been read
                    uint32_t pa[4], pb[4];  // bf16 pairs of the 8 outputs of each side
                    float va[8], vb[8];
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        const float4 ca = *reinterpret_cast<const float4 *>(cst2 + 128 + 8 * c8 + 4 * k);
                        const float4 cb = *reinterpret_cast<const float4 *>(cst2 + 192 + 8 * c8 + 4 * k);
                        const float cav[4] = {ca.x, ca.y, ca.z, ca.w}, cbv[4] = {cb.x, cb.y, cb.z, cb.w};
                        // two pairs per packed f32x2 operation; lane for lane the scalar operations
                        // (a = float(acc) (ws g) rs; va = fma(a, cos, -(b sin)), vb = fma(a, sin, b cos)),
                        // no packed product feeding a packed add
                        const float2 rs2 = make_float2(rs, rs);
#pragma unroll
                        for (int e = 0; e < 4; e += 2) {
                            const int i = 4 * k + e;
                            const float2 a = mul2_rn(mul2_rn(make_float2(__int2float_rn((int)ra[i]), __int2float_rn((int)ra[i + 1])),
                                                             make_float2(cav[e], cav[e + 1])),
                                                     rs2);
                            const float2 b = mul2_rn(mul2_rn(make_float2(__int2float_rn((int)rb[i]), __int2float_rn((int)rb[i + 1])),
                                                             make_float2(cbv[e], cbv[e + 1])),
                                                     rs2);
                            if (!is_v) {
                                const float2 c2 = make_float2(cs[i], cs[i + 1]), s2 = make_float2(sn[i], sn[i + 1]);
                                const float2 x = fma2_rn(a, c2, mul2_rn(b, make_float2(-s2.x, -s2.y)));
                                const float2 y = fma2_rn(a, s2, mul2_rn(b, c2));
                                va[i] = x.x, va[i + 1] = x.y;
                                vb[i] = y.x, vb[i + 1] = y.y;
                            } else {
                                va[i] = a.x, va[i + 1] = a.y;
                                vb[i] = b.x, vb[i + 1] = b.y;
                            }
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const __nv_bfloat162 ha = __floats2bfloat162_rn(va[2 * k], va[2 * k + 1]);
                        const __nv_bfloat162 hb = __floats2bfloat162_rn(vb[2 * k], vb[2 * k + 1]);
                        pa[k] = *reinterpret_cast<const uint32_t *>(&ha);
                        pb[k] = *reinterpret_cast<const uint32_t *>(&hb);
                    }
                    if (is_v) {
                        if (mrow) {
                            __nv_bfloat16 *vt = reinterpret_cast<__nv_bfloat16 *>(p.vt_out) +
                                                (size_t)(m / p.seq_len) * 256 * p.ldvt + pos;
#pragma unroll
                            for (int i = 0; i < 8; i++) {
                                vt[(size_t)(ia + i) * p.ldvt] = reinterpret_cast<const __nv_bfloat16 *>(pa)[i];
                                vt[(size_t)(128 + ia + i) * p.ldvt] = reinterpret_cast<const __nv_bfloat16 *>(pb)[i];
                            }
                        }
                    } else if (tma_out) {
                        // 16-byte chunk (c8 & 3) of the row's 64 bytes, in the 64-byte swizzle
                        const int ch = ((c8 & 3) ^ ((lane >> 1) & 3)) << 4;
                        *reinterpret_cast<uint4 *>(stg + lane * 64 + ch) = make_uint4(pa[0], pa[1], pa[2], pa[3]);
                        *reinterpret_cast<uint4 *>(stg + STG_WARP + lane * 64 + ch) = make_uint4(pb[0], pb[1], pb[2], pb[3]);
                        if ((c8 & 3) == 3) {
                            const CUtensorMap *tm = is_k ? &tmO1 : &tmO0;
                            const int xb = (is_k ? 0 : head * 256) + 64 * part2 + 32 * (c8 >> 2);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                tma_store_2d(tm, smem_u32(stg), xb, y0);
                                tma_store_2d(tm, smem_u32(stg + STG_WARP), xb + 128, y0);
                                bulk_commit();
                            }
                            ++nst2;
                        }
                    } else if (mrow) {
                        __nv_bfloat16 *dst = is_k ? reinterpret_cast<__nv_bfloat16 *>(p.k_out) + (size_t)m * 256
                                                  : reinterpret_cast<__nv_bfloat16 *>(p.q_out) +
                                                        (size_t)m * (256 * p.nq) + head * 256;
                        *reinterpret_cast<uint4 *>(dst + ia) = make_uint4(pa[0], pa[1], pa[2], pa[3]);
                        *reinterpret_cast<uint4 *>(dst + 128 + ia) = make_uint4(pb[0], pb[1], pb[2], pb[3]);
                    }
                }
            }
        } else {
            Pre pre = fetch(tfirst);
            int jt = 0;  // tiles this CTA finished (GELU-quantise: the row-maximum slot and phase)
            for (int t = tfirst; t < ntiles && ok; t += tstride, jt++) {
                const int mt = (t / tiles_n) * (BM * CG) + (int)rank * BM;
                const int m = mt + row;
                const int c0 = p.n0 + (t % tiles_n) * TW;
                const bool mrow = m < M;
                const int y0 = mt + q * 32;  // first row of this warp's 32
                const int cw = c0 + part * QCOLS;  // first column of this warp (F32 / I32 / per-block)
                if constexpr (GQ) {
                    // Sub-tile s holds h columns [64 s, 64 s + 64) of the tile's block of 128: TMEM
                    // columns 0..63 their gate rows, 64..127 their up rows. This warp folds h columns
                    // 16 part .. 16 part + 15 of each sub-tile, g and u as the F32 epilogue does
                    // (f = fma(float(dot), as * ws, f) per 128-deep block, then the clamp), then
                    // h = gelu(g) * u; the block's quantiser follows the row maximum over the
                    // quadrant's four warps.
                    const int hb = (c0 - p.n0) / TW;  // the tile's block of 128 h columns
                    __syncwarp();  // every lane is done with the previous tile's weight scales
                    {
                        const int s = lane >> 4, j = lane & 15;
                        cst[32 * s + j] = __ldg(p.w_scale + c0 + 64 * s + 16 * part + j);
                        cst[32 * s + 16 + j] = __ldg(p.w_scale + c0 + 128 + 64 * s + 16 * part + j);
                    }
                    __syncwarp();
                    // h of the first sub-tile waits in TMEM columns 384 + 16 part .. (registers hold
                    // the second's)
                    const uint32_t park = tmem_base + lane_addr + (uint32_t)(3 * BN + 16 * part);
                    float hv[16];
#pragma unroll 1
                    for (int s = 0; s < 2; s++) {
                        float f[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) f[j] = 0.f;
                        float as_next = mrow ? __ldg(p.a_scale + (size_t)m * nb) : 0.f;
                        for (int u = 0; u < nunits; u++) {
                            const float as = as_next;
                            if (u + 1 < nunits) as_next = mrow ? __ldg(p.a_scale + (size_t)m * nb + u + 1) : 0.f;
                            if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(acc), acc_phase, p.status, E2C_ERR_WAIT_EPI))) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t ta = tmem_base + lane_addr + (uint32_t)(acc * BN + 16 * part);
                            const float2 as2 = make_float2(as, as);
                            // the gate columns, then the up columns (16 loaded values live at a time)
#pragma unroll
                            for (int gu = 0; gu < 2; gu++) {
                                uint32_t r[16];
                                tmem_ld16(ta + 64 * gu, r);
                                tmem_wait_ld();
                                if (gu == 1) release_acc(acc);
#pragma unroll
                                for (int j4 = 0; j4 < 4; j4++) {
                                    const float4 w4 = *reinterpret_cast<const float4 *>(cst + 32 * s + 16 * gu + 4 * j4);
#pragma unroll
                                    for (int h = 0; h < 2; h++) {
                                        const int j = 4 * j4 + 2 * h, jf = 16 * gu + j;
                                        const float2 s2 = mul2_rn(as2, h ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y));
                                        const float2 d2 = make_float2(__int2float_rn((int)r[j]), __int2float_rn((int)r[j + 1]));
                                        const float2 o = fma2_rn(d2, s2, make_float2(f[jf], f[jf + 1]));
                                        f[jf] = o.x;
                                        f[jf + 1] = o.y;
                                    }
                                }
                            }
                            if (++acc == NACC) {
                                acc = 0;
                                acc_phase ^= 1u;
                            }
                        }
                        if (!ok) break;
#pragma unroll
                        for (int j = 0; j < 16; j += 2) {
                            const float2 g = make_float2(fminf(fmaxf(f[j], p.out_min), p.out_max),
                                                         fminf(fmaxf(f[j + 1], p.out_min), p.out_max));
                            const float2 u = make_float2(fminf(fmaxf(f[16 + j], p.out_min), p.out_max),
                                                         fminf(fmaxf(f[17 + j], p.out_min), p.out_max));
                            const float2 h = mul2_rn(gelu_tanh2(g), u);
                            hv[j] = h.x;
                            hv[j + 1] = h.y;
                        }
                        if (s == 0) tmem_st16(park, reinterpret_cast<const uint32_t (&)[16]>(hv));
                    }
                    if (!ok) break;
                    float h0[16];
                    tmem_wait_st();
                    tmem_ld16(park, reinterpret_cast<uint32_t (&)[16]>(h0));
                    tmem_wait_ld();
                    // the row's max |h| over the block: this warp's 32 columns, then the quadrant's
                    // four warps through shared memory (two slots, alternating by tile)
                    float am = 0.f;
#pragma unroll
                    for (int j = 0; j < 16; j++) am = fmaxf(am, fmaxf(fabsf(h0[j]), fabsf(hv[j])));
                    float *xm = reinterpret_cast<float *>(smem + L::SSQ_OFF) + (jt & 1) * 4 * BM;
                    xm[part * BM + row] = am;
                    mbar_arrive(pair_bar(0, q));
                    if (!__all_sync(0xffffffffu, mbar_wait(pair_bar(0, q), (uint32_t)(jt & 1), p.status, E2C_ERR_WAIT_EPI))) {
                        ok = false;
                        break;
                    }
                    am = fmaxf(fmaxf(xm[row], xm[BM + row]), fmaxf(xm[2 * BM + row], xm[3 * BM + row]));
                    // the reference quantiser: scale = amax fl(1/127), q = rint(h fl(127 / amax)) (|q| <= 127
                    // without a clamp: h fl(127 / amax) <= 127 (1 + 2^-24))
                    const float inv = am > 0.f ? __fdiv_rn(127.0f, am) : 1.0f;
                    if (mrow) {
                        int8_t *qr = p.q8 + (size_t)m * p.ldq + 128 * hb + 16 * part;
#pragma unroll
                        for (int s = 0; s < 2; s++) {
                            const float *hs = s ? hv : h0;
                            uint32_t w[4];
#pragma unroll
                            for (int k = 0; k < 4; k++)
                                w[k] = pack_low_bytes(rint_low_byte(__fmul_rn(hs[4 * k], inv)),
                                                      rint_low_byte(__fmul_rn(hs[4 * k + 1], inv)),
                                                      rint_low_byte(__fmul_rn(hs[4 * k + 2], inv)),
                                                      rint_low_byte(__fmul_rn(hs[4 * k + 3], inv)));
                            *reinterpret_cast<uint4 *>(qr + 64 * s) = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                        if (part == 0) p.q8_scale[(size_t)m * tiles_n + hb] = am > 0.f ? __fmul_rn(am, 0x1.020408p-7f) : 1.0f;
                    }
                } else if constexpr (QP) {
                    // One tile = one head of 256 columns, its halves [0, 128) and [128, 256) the two
                    // sub-tiles. This warp folds columns 32 part .. 32 part + 31 of each half, so the
                    // rotate-half pairs (i, i + 128) of RoPE meet in one thread; both folded halves
                    // wait in TMEM columns 256 + 64 part .. + 63 for the norm. The row's sum of
                    // squares over the head combines the quadrant's four warps through shared memory.
                    // Arithmetic per element as the per-block F32 GEMM followed by the q|k|v finish
                    // (x = float(acc) fold, clamp; y = (x * inv) * gain; RoPE; bf16), the norm's sum
                    // of squares in its own order.
                    const int head = (c0 - p.n0) / TW;
                    const int nkv = (ncols / 256 - p.nq) / 2;
                    const int kind = head < p.nq ? 0 : head < p.nq + nkv ? 1 : 2;  // q, k, v
                    __syncwarp();  // every lane is done with the previous tile's constants
                    {
                        const float *gam = kind == 0 ? p.q_gamma : kind == 1 ? p.k_gamma : nullptr;
#pragma unroll
                        for (int s = 0; s < 2; s++) {
                            cst[32 * s + lane] = __ldg(p.w_scale + c0 + 128 * s + 32 * part + lane);
                            cst[64 + 32 * s + lane] = gam ? __ldg(gam + 128 * s + 32 * part + lane) : 1.f;
                        }
                    }
                    __syncwarp();
                    const uint32_t park = tmem_base + lane_addr + (uint32_t)(2 * BN + 64 * part);
                    float ssh = 0.f;  // the warp's sum of squares over the halves folded so far
#pragma unroll 1
                    for (int s = 0; s < 2; s++) {
                        float f[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) f[j] = 0.f;
                        float as_next = mrow ? __ldg(p.a_scale + (size_t)m * nb) : 0.f;
                        for (int u = 0; u < nunits; u++) {
                            const float as = as_next;
                            if (u + 1 < nunits) as_next = mrow ? __ldg(p.a_scale + (size_t)m * nb + u + 1) : 0.f;
                            if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(acc), acc_phase, p.status, E2C_ERR_WAIT_EPI))) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t ta = tmem_base + lane_addr + (uint32_t)(acc * BN + 32 * part);
                            const float2 as2 = make_float2(as, as);
                            // 16 columns at a time (16 loaded values live)
#pragma unroll
                            for (int hh = 0; hh < 2; hh++) {
                                uint32_t r[16];
                                tmem_ld16(ta + 16 * hh, r);
                                tmem_wait_ld();
                                if (hh == 1) release_acc(acc);
#pragma unroll
                                for (int j4 = 0; j4 < 4; j4++) {
                                    const float4 w4 = *reinterpret_cast<const float4 *>(cst + 32 * s + 16 * hh + 4 * j4);
#pragma unroll
                                    for (int h = 0; h < 2; h++) {
                                        const int j = 4 * j4 + 2 * h, jf = 16 * hh + j;
                                        const float2 s2 = mul2_rn(as2, h ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y));
                                        const float2 d2 = make_float2(__int2float_rn((int)r[j]), __int2float_rn((int)r[j + 1]));
                                        const float2 o = fma2_rn(d2, s2, make_float2(f[jf], f[jf + 1]));
                                        f[jf] = o.x;
                                        f[jf + 1] = o.y;
                                    }
                                }
                            }
                            if (++acc == NACC) {
                                acc = 0;
                                acc_phase ^= 1u;
                            }
                        }
                        if (!ok) break;
                        float ssp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            f[j] = fminf(fmaxf(f[j], p.out_min), p.out_max);
                            ssp[j & 3] = __fmaf_rn(f[j], f[j], ssp[j & 3]);
                        }
                        ssh = __fadd_rn(ssh, __fadd_rn(__fadd_rn(ssp[0], ssp[1]), __fadd_rn(ssp[2], ssp[3])));
                        tmem_st32(park + 32 * s, reinterpret_cast<const uint32_t (&)[32]>(f));
                    }
                    if (!ok) break;
                    float *xs = reinterpret_cast<float *>(smem + L::SSQ_OFF) + (jt & 1) * 4 * BM;
                    xs[part * BM + row] = ssh;
                    mbar_arrive(pair_bar(0, q));
                    const int bseq = mrow ? m / p.seq_len : 0, pos = mrow ? m - bseq * p.seq_len : 0;
                    // q, k: the RoPE coefficients of the first step's 8 pairs, requested before the
                    // row-norm exchange (each later step's one step ahead)
                    const float *rc = p.rope_cos + (size_t)pos * p.ldrope, *rs = p.rope_sin + (size_t)pos * p.ldrope;
                    float4 cnx[2] = {make_float4(1.f, 1.f, 1.f, 1.f), make_float4(1.f, 1.f, 1.f, 1.f)};
                    float4 snx[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
                    if (kind < 2) {
#pragma unroll
                        for (int h4 = 0; h4 < 2; h4++) {
                            cnx[h4] = __ldg(reinterpret_cast<const float4 *>(rc + 32 * part + 4 * h4));
                            snx[h4] = __ldg(reinterpret_cast<const float4 *>(rs + 32 * part + 4 * h4));
                        }
                    }
                    if (!__all_sync(0xffffffffu, mbar_wait(pair_bar(0, q), (uint32_t)(jt & 1), p.status, E2C_ERR_WAIT_EPI))) {
                        ok = false;
                        break;
                    }
                    const float ss = __fadd_rn(__fadd_rn(xs[row], xs[BM + row]), __fadd_rn(xs[2 * BM + row], xs[3 * BM + row]));
                    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 256.0f), p.eps)));
                    tmem_wait_st();
                    if (kind < 2) {
                        // q, k: 8 pairs a step from TMEM, RoPE on 4 at a time; 16-byte bf16 runs of
                        // each half
                        __nv_bfloat16 *dst = kind == 0
                            ? reinterpret_cast<__nv_bfloat16 *>(p.q_out) + (size_t)m * (256 * p.nq) + head * 256
                            : reinterpret_cast<__nv_bfloat16 *>(p.k_out) + (size_t)m * (256 * nkv) + (head - p.nq) * 256;
#pragma unroll 1
                        for (int c = 0; c < 4; c++) {
                            uint32_t r0[8], r1[8];
                            tmem_ld8(park + 8 * c, r0);
                            tmem_ld8(park + 32 + 8 * c, r1);
                            const int i0 = 32 * part + 8 * c;  // rotate-half index of the first pair
                            const float4 cur_c[2] = {cnx[0], cnx[1]}, cur_s[2] = {snx[0], snx[1]};
                            if (c < 3) {
#pragma unroll
                                for (int h4 = 0; h4 < 2; h4++) {
                                    cnx[h4] = __ldg(reinterpret_cast<const float4 *>(rc + i0 + 8 + 4 * h4));
                                    snx[h4] = __ldg(reinterpret_cast<const float4 *>(rs + i0 + 8 + 4 * h4));
                                }
                            }
                            tmem_wait_ld();
                            uint32_t px[4], pz[4];
#pragma unroll
                            for (int h4 = 0; h4 < 2; h4++) {
                                const float4 c4 = cur_c[h4];
                                const float4 s4 = cur_s[h4];
                                const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
                                float xo[4], zo[4];
#pragma unroll
                                for (int jj = 0; jj < 4; jj++) {
                                    const int j = 4 * h4 + jj;
                                    const float x = __fmul_rn(__fmul_rn(__uint_as_float(r0[j]), inv), cst[64 + 8 * c + j]);
                                    const float z = __fmul_rn(__fmul_rn(__uint_as_float(r1[j]), inv), cst[96 + 8 * c + j]);
                                    xo[jj] = __fmaf_rn(x, cs[jj], -__fmul_rn(z, sn[jj]));
                                    zo[jj] = __fmaf_rn(x, sn[jj], __fmul_rn(z, cs[jj]));
                                }
#pragma unroll
                                for (int k = 0; k < 2; k++) {
                                    const __nv_bfloat162 hx = __floats2bfloat162_rn(xo[2 * k], xo[2 * k + 1]);
                                    const __nv_bfloat162 hz = __floats2bfloat162_rn(zo[2 * k], zo[2 * k + 1]);
                                    px[2 * h4 + k] = *reinterpret_cast<const uint32_t *>(&hx);
                                    pz[2 * h4 + k] = *reinterpret_cast<const uint32_t *>(&hz);
                                }
                            }
                            if (mrow) {
                                *reinterpret_cast<uint4 *>(dst + i0) = make_uint4(px[0], px[1], px[2], px[3]);
                                *reinterpret_cast<uint4 *>(dst + 128 + i0) = make_uint4(pz[0], pz[1], pz[2], pz[3]);
                            }
                        }
                    } else {
                        // v: V^T [B][256 nkv][ldvt]; the warp's 32 consecutive positions of one dimension
                        // are one contiguous run
                        __nv_bfloat16 *vt = reinterpret_cast<__nv_bfloat16 *>(p.vt_out) +
                                            ((size_t)bseq * 256 * nkv + (size_t)(head - p.nq - nkv) * 256) * p.ldvt + pos;
#pragma unroll 1
                        for (int c = 0; c < 4; c++) {
                            uint32_t r0[8], r1[8];
                            tmem_ld8(park + 8 * c, r0);
                            tmem_ld8(park + 32 + 8 * c, r1);
                            tmem_wait_ld();
                            const int i0 = 32 * part + 8 * c;
                            if (mrow)
#pragma unroll
                                for (int j = 0; j < 8; j++) {
                                    vt[(size_t)(i0 + j) * p.ldvt] =
                                        __float2bfloat16_rn(__fmul_rn(__fmul_rn(__uint_as_float(r0[j]), inv), cst[64 + 8 * c + j]));
                                    vt[(size_t)(128 + i0 + j) * p.ldvt] =
                                        __float2bfloat16_rn(__fmul_rn(__fmul_rn(__uint_as_float(r1[j]), inv), cst[96 + 8 * c + j]));
                                }
                        }
                    }
                } else if constexpr (PERBLOCK) {
                    float f[QCOLS];
    #pragma unroll
                    for (int j = 0; j < QCOLS; j++) f[j] = 0.f;
                    if constexpr (EPI != E2C_EPI_I32) {
                        // the warp's 32 weight scales, read back by broadcast loads four at a time
                        const int nl = cw + lane;
                        __syncwarp();  // every lane is done with the previous tile's
                        cst[lane] = nl < p.n1 ? __ldg(p.w_scale + nl) : 0.f;
                        __syncwarp();
                    }
                    // the row's activation scale of block u, loaded a block ahead
                    float as_next = mrow ? __ldg(p.a_scale + (size_t)m * nb) : 0.f;
                    for (int u = 0; u < nunits; u++) {
                        const float as = as_next;
                        if (u + 1 < nunits) as_next = mrow ? __ldg(p.a_scale + (size_t)m * nb + u + 1) : 0.f;
                        // warp-uniform outcome: tcgen05.ld below is .sync.aligned
                        if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(acc), acc_phase, p.status, E2C_ERR_WAIT_EPI))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        uint32_t r[32];
                        tmem_ld32(tmem_base + lane_addr + (uint32_t)(acc * BN + part * QCOLS), r);
                        tmem_wait_ld();
                        release_acc(acc);
                        if constexpr (EPI == E2C_EPI_I32) {
                            if (mrow)
                                for (int j = 0; j < 32; j++)
                                    if (cw + j < p.n1) p.dots[((size_t)m * p.ldd + cw + j) * nb + u] = (int32_t)r[j];
                        } else {
                            // f = fma(float(dot), as * ws, f) per column, two columns per packed
                            // f32x2 multiply and fma
                            const float2 as2 = make_float2(as, as);
    #pragma unroll
                            for (int j4 = 0; j4 < 8; j4++) {
                                const float4 w4 = *reinterpret_cast<const float4 *>(cst + 4 * j4);
    #pragma unroll
                                for (int h = 0; h < 2; h++) {
                                    const int j = 4 * j4 + 2 * h;
                                    const float2 s2 = mul2_rn(as2, h ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y));
                                    const float2 d2 = make_float2(__int2float_rn((int)r[j]), __int2float_rn((int)r[j + 1]));
                                    const float2 o = fma2_rn(d2, s2, make_float2(f[j], f[j + 1]));
                                    f[j] = o.x;
                                    f[j + 1] = o.y;
                                }
                            }
                        }
                        if (++acc == NACC) {
                            acc = 0;
                            acc_phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    if constexpr (EPI != E2C_EPI_I32) {
    #pragma unroll
                        for (int h2 = 0; h2 < 2; h2++) {
                            float v[16];
    #pragma unroll
                            for (int j = 0; j < 16; j++) {
                                const int n = cw + 16 * h2 + j;
                                v[j] = fminf(fmaxf(f[16 * h2 + j], p.out_min), p.out_max);
                                if constexpr (EPI == E2C_EPI_RESID)
                                    if (mrow && n < p.n1) v[j] = __fadd_rn(v[j], p.resid[(size_t)m * p.ldr + n]);
                            }
                            if (tma_out) {
                                put16(v, cw + 16 * h2 - p.n0, y0);
                            } else if (mrow) {
                                for (int j = 0; j < 16; j++)
                                    if (cw + 16 * h2 + j < p.n1) p.y[(size_t)m * p.ldy + cw + 16 * h2 + j] = v[j];
                            }
                        }
                    }
                } else {
                    const Pre cur = pre;
                    pre = fetch(t + tstride);
                    const float as = cur.as;
                    __syncwarp();  // every lane is done reading the previous tile's cst
                    if constexpr (EPI == E2C_EPI_F32 || EPI == E2C_EPI_RESID) {
                        if (lane < QCOLS) cst[lane] = cur.w0;
                        if (32 + lane < QCOLS) cst[32 + lane] = cur.w1;
                    } else if constexpr (EPI == E2C_EPI_GELU) {
                        cst[lane] = cur.w0;
                        cst[32 + lane] = cur.w1;
                    }
                    __syncwarp();
                    if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(acc), acc_phase, p.status, E2C_ERR_WAIT_EPI))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t tbase = tmem_base + lane_addr + (uint32_t)(acc * BN);
                    if constexpr (EPI == E2C_EPI_I32) {
    #pragma unroll 1
                        for (int c = 0; c < QCOLS / 16; c++) {
                            uint32_t r[16];
                            tmem_ld16(tbase + part * QCOLS + 16 * c, r);
                            tmem_wait_ld();
                            const int nbase = cw + 16 * c;
                            if (mrow)
                                for (int j = 0; j < 16; j++)
                                    if (nbase + j < p.n1) p.dots[(size_t)m * p.ldd + nbase + j] = (int32_t)r[j];
                        }
                    } else if constexpr (EPI == E2C_EPI_F32 || EPI == E2C_EPI_RESID) {
                        // y = float(acc) * (as * ws), the reference's single-block fold; the clamp only
                        // when the weight carries one (the defaults +-1e31 bound no finite output)
                        constexpr int NCH = QCOLS / 16;
                        const bool clamp = p.out_min > -1e30f || p.out_max < 1e30f;
    #pragma unroll
                        for (int c2 = 0; c2 < NCH; c2 += 2) {
                            uint32_t r[2][16];
                            tmem_ld16(tbase + part * QCOLS + 16 * c2, r[0]);
                            if (c2 + 1 < NCH) tmem_ld16(tbase + part * QCOLS + 16 * (c2 + 1), r[1]);
                            tmem_wait_ld();
    #pragma unroll
                            for (int h = 0; h < 2; h++) {
                                if (c2 + h < NCH) {
                                    const int nbase = cw + 16 * (c2 + h);
                                    float w[16], v[16];
                                    cst16(16 * (c2 + h), w);
    #pragma unroll
                                    for (int j = 0; j < 16; j++) v[j] = dq(r[h][j], __fmul_rn(as, w[j]));
                                    if (clamp)
    #pragma unroll
                                        for (int j = 0; j < 16; j++) v[j] = fminf(fmaxf(v[j], p.out_min), p.out_max);
                                    if constexpr (EPI == E2C_EPI_RESID) {
                                        if (mrow) {
                                            const float *rr = p.resid + (size_t)m * p.ldr + nbase;
                                            for (int j = 0; j < 16; j++)
                                                if (nbase + j < p.n1) v[j] = __fadd_rn(v[j], rr[j]);
                                        }
                                    }
                                    if (tma_out) {
                                        put16(v, nbase - p.n0, y0);
                                    } else if (mrow && nbase < p.n1) {
                                        float *yr = p.y + (size_t)m * p.ldy + nbase;
                                        for (int j = 0; j < 16; j++)
                                            if (nbase + j < p.n1) yr[j] = v[j];
                                    }
                                }
                            }
                        }
                    } else if constexpr (EPI == E2C_EPI_GELU) {
                        // weight rows are interleaved per 128: [gate c0/2 .. +128 | up c0/2 .. +128];
                        // this warp produces outputs [32 part, 32 part + 32) of the tile's 128, 16 at a time
                        const int h0 = (c0 - p.n0) / 2;
    #pragma unroll
                        for (int h2 = 0; h2 < 2; h2++) {
                            const int oc = 32 * part + 16 * h2;
                            uint32_t rg[16], ru[16];
                            tmem_ld16(tbase + oc, rg);
                            tmem_ld16(tbase + 128 + oc, ru);
                            tmem_wait_ld();
                            float wg[16], wu[16], h[16];
                            cst16(16 * h2, wg);
                            cst16(32 + 16 * h2, wu);
    #pragma unroll
                            for (int j = 0; j < 16; j++) {
                                const float g = dq(rg[j], __fmul_rn(as, wg[j]));
                                const float u = dq(ru[j], __fmul_rn(as, wu[j]));
                                h[j] = __fmul_rn(gelu_tanh(g), u);
                            }
                            if (tma_out) {
                                put16(h, h0 + oc, y0);
                            } else if (mrow) {
                                float4 *y4 = reinterpret_cast<float4 *>(p.y + (size_t)m * p.ldy + h0 + oc);
    #pragma unroll
                                for (int j = 0; j < 4; j++) y4[j] = make_float4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
                            }
                        }
                    }
                    release_acc(acc);
                    if (++acc == NACC) {
                        acc = 0;
                        acc_phase ^= 1u;
                    }
                }
            }
        }
        // the global writes of every store this warp issued complete before the kernel ends
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }

    tc_fence_before();
    // a pair: neither CTA leaves while the other may still signal its barriers
    if constexpr (CG == 2) cluster_sync();
    else __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if constexpr (CG == 2) tmem_dealloc_pair(tmem_base, TMEM_COLS);
        else tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <int BN, int STAGES, bool PERBLOCK, int EPI, int CG>
int launch(const e2c_gemm_args *a, cudaStream_t st, int dev, int num_sms) {
    using L = GemmSmem<BN, STAGES, PERBLOCK, EPI, CG>;
    auto kern = k_gemm_i8<BN, STAGES, PERBLOCK, EPI, CG>;
    static E2cPerDev attr_set;   // the shared-memory opt-in, per device
    static E2cPerDev max_pairs;  // CTA pairs the device holds at once (CG = 2)
    if (!attr_set.get(dev)) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) != cudaSuccess) {
            e2c_set_msg("gemm: cannot reserve %d bytes of shared memory", L::ALLOC);
            return -2;
        }
        attr_set.set(dev, 1);
    }
    CUtensorMap ta, tb, t0, t1;
    if (e2c_tmap_2d(&ta, a->a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->M, (uint64_t)a->lda,
                    BK, BM) ||
        e2c_tmap_2d(&tb, a->w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->wrows,
                    (uint64_t)a->ldw, BK, EPI == E2C_EPI_GELUQ ? 64 : BN / CG))
        return -3;
    memset(&t0, 0, sizeof t0);
    memset(&t1, 0, sizeof t1);
    int tma_out = 0;
    if (EPI == E2C_EPI_F32 || EPI == E2C_EPI_RESID) {
        // TMA stores need 16-byte aligned rows and column starts; the tensor ends at n1 so nothing
        // right of the requested range is written
        if (a->ldy % 4 == 0 && a->n0 % 4 == 0 && ((uintptr_t)a->y & 15) == 0)
            tma_out = !e2c_tmap_2d_sw64(&t0, a->y + a->n0, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)(a->n1 - a->n0),
                                        (uint64_t)a->M, (uint64_t)a->ldy * 4, 16, 32);
    } else if (EPI == E2C_EPI_GELU) {
        const int width = (a->n1 - a->n0) / 2;
        if (a->ldy % 4 == 0 && ((uintptr_t)a->y & 15) == 0)
            tma_out = !e2c_tmap_2d_sw64(&t0, a->y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)width, (uint64_t)a->M,
                                        (uint64_t)a->ldy * 4, 16, 32);
    } else if (EPI == E2C_EPI_QKV) {
        if ((((uintptr_t)a->q_out | (uintptr_t)a->k_out) & 15) == 0)
            tma_out = !e2c_tmap_2d_sw64(&t0, a->q_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)256 * a->nq,
                                        (uint64_t)a->M, (uint64_t)512 * a->nq, 32, 32) &&
                      !e2c_tmap_2d_sw64(&t1, a->k_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 256, (uint64_t)a->M, 512, 32, 32);
    }
    constexpr int TW = (EPI == E2C_EPI_GELUQ || EPI == E2C_EPI_QKVPB) ? 2 * BN : BN;  // weight rows per tile
    const int tiles = ((a->M + BM * CG - 1) / (BM * CG)) * ((a->n1 - a->n0 + TW - 1) / TW);
    cudaError_t e;
    if constexpr (CG == 1) {
        const int grid = tiles < num_sms ? tiles : num_sms;
        e = e2c_launch(kern, dim3(grid), dim3(NTHREADS), L::ALLOC, st, ta, tb, t0, t1, *a, tma_out);
    } else {
        cudaLaunchConfig_t cfg;
        memset(&cfg, 0, sizeof cfg);
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.blockDim = dim3(NTHREADS);
        cfg.dynamicSmemBytes = L::ALLOC;
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int pairs = max_pairs.get(dev);
        if (!pairs) {
            cfg.gridDim = dim3(2 * (num_sms / 2));
            if (cudaOccupancyMaxActiveClusters(&pairs, kern, &cfg) != cudaSuccess || pairs <= 0) {
                cudaGetLastError();
                e2c_set_msg("gemm: the device cannot hold a pair of GEMM CTAs");
                return -2;
            }
            max_pairs.set(dev, pairs);
        }
        cfg.gridDim = dim3(2 * (tiles < pairs ? tiles : pairs));
        cfg.numAttrs = e2c_pdl_attr(attr, 1);
        e = cudaLaunchKernelEx(&cfg, kern, ta, tb, t0, t1, *a, tma_out);
    }
    if (e != cudaSuccess) {
        e2c_set_msg("gemm launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}

// the kernel family e2c_gemm last chose on this thread (for benchmark reports)
thread_local const char *g_last_kernel = "";

// E2C_GEMM_STREAM=0 turns the weight-streaming path off (the split-K and persistent kernels then
// take short activation matrices), for comparisons
bool stream_path_on() {
    static int on = -1;
    if (on < 0) {
        const char *v = getenv("E2C_GEMM_STREAM");
        on = !(v && v[0] == '0');
    }
    return on != 0;
}

// Tile plan: width BN and whether CTA pairs (M = 256 per pair, each SM loading half of the weight
// tile: a third less operand traffic per MAC) share tiles.
struct Plan {
    int bn, cg;
};

Plan pick_plan(const e2c_gemm_args *a, int num_sms) {
    const int ncols = a->n1 - a->n0;
    if (a->ablk != a->K) {
        // per-block fold: BN 128 (four 128-column accumulators); CTA pairs on the same rule (the
        // GELU-quantise epilogue's tiles are 256 weight rows)
        const int tw = (a->epi == E2C_EPI_GELUQ || a->epi == E2C_EPI_QKVPB) ? 256 : 128;
        const long pairs128 = (long)((a->M + 2 * BM - 1) / (2 * BM)) * ((ncols + tw - 1) / tw);
        return {128, (pairs128 >= num_sms / 2 && a->M > 2 * BM) ? 2 : 1};
    }
    const long pairs256 = (long)((a->M + 2 * BM - 1) / (2 * BM)) * ((ncols + 255) / 256);
    // pairs pay off once they fill the device (a full wave of 256-row tiles) and both CTAs of a
    // pair have rows of their own: with M <= 256 the second one would only multiply zeros
    const int cg = (pairs256 >= num_sms / 2 && a->M > 2 * BM) ? 2 : 1;
    if (a->epi == E2C_EPI_GELU || a->epi == E2C_EPI_QKV) return {256, cg};
    // the width whose waves of persistent tiles cost least: a tile's time ~ BN + a fixed 32
    const int slots = cg == 2 ? num_sms / 2 : num_sms;
    const long tm = (a->M + BM * cg - 1) / (BM * cg);
    int best = 256;
    long best_cost = -1;
    for (int bn : {256, 192, 128}) {
        const long units = tm * ((ncols + bn - 1) / bn);
        const long cost = (units + slots - 1) / slots * (bn + 32);
        if (best_cost < 0 || cost < best_cost) {
            best = bn;
            best_cost = cost;
        }
    }
    return {best, cg};
}

}  // namespace

extern "C" const char *e2c_gemm_last_kernel(void) { return g_last_kernel; }

extern "C" size_t e2c_gemm_ws_bytes(int M) {
    const int num_sms = e2c_sm_count(e2c_device());
    return (num_sms && M >= 1 && M <= 256) ? e2c_gemm_stream_ws_bytes(M, num_sms) : 0;
}

extern "C" void e2c_gemm_tile(const e2c_gemm_args *a, int *bm, int *bn) {
    int num_sms = e2c_sm_count(e2c_device());
    if (!num_sms) num_sms = 148;
    const Plan pl = pick_plan(a, num_sms);
    *bm = BM * pl.cg;
    *bn = pl.bn;
}

extern "C" int e2c_gemm(const e2c_gemm_args *a, void *stream) {
    const int dev = e2c_device();
    const int num_sms = e2c_sm_count(dev);
    if (!num_sms) {
        e2c_set_msg("gemm: no CUDA device");
        return -2;
    }
    if (a->M < 0 || a->K <= 0 || a->K % 16 || a->lda % 16 || a->ldw % 16 || a->n0 < 0 || a->n1 > a->wrows ||
        a->n0 > a->n1) {
        e2c_set_msg("gemm: bad geometry (M=%d K=%d lda=%d ldw=%d n0=%d n1=%d wrows=%d): K and strides must be multiples of 16",
                    a->M, a->K, a->lda, a->ldw, a->n0, a->n1, a->wrows);
        return -1;
    }
    if (a->ablk <= 0 || a->K % a->ablk || (a->ablk != a->K && a->ablk % BK)) {
        e2c_set_msg("gemm: activation block %d must be K (per-row) or a multiple of 128 dividing K=%d", a->ablk, a->K);
        return -1;
    }
    if (((uintptr_t)a->a | (uintptr_t)a->w) & 15) {
        e2c_set_msg("gemm: operands must be 16-byte aligned");
        return -1;
    }
    if (a->M == 0 || a->n1 == a->n0) return 0;
    cudaStream_t st = (cudaStream_t)stream;
    const bool perblock = a->ablk != a->K;
    if (stream_path_on() && a->ws && !perblock && (a->epi == E2C_EPI_F32 || a->epi == E2C_EPI_RESID) && a->M <= 256 &&
        a->ws_bytes >= e2c_gemm_stream_ws_bytes(a->M, num_sms) && !((uintptr_t)a->ws & 127)) {
        // short activation matrices against a long weight: stream the weight over every SM (the
        // weight in the MMA's M slot). It pays where each CTA streams at least 8 of the 16 KB weight
        // tiles, so its fixed costs (launch ramp, the split tiles' reductions) amortise; shorter
        // weights go to the split-K kernel below, which measured faster there (4-17 MB at M <= 128).
        const Plan pp = pick_plan(a, num_sms);
        const long ptiles = (long)((a->M + BM * pp.cg - 1) / (BM * pp.cg)) * ((a->n1 - a->n0 + pp.bn - 1) / pp.bn);
        const long wtiles = (long)((a->n1 - a->n0 + 127) / 128) * ((a->K + 127) / 128);
        if (wtiles >= 8L * num_sms && (a->M <= 64 || ptiles * pp.cg < num_sms)) {
            g_last_kernel = "stream";
            return e2c_gemm_stream(a, stream);
        }
        // Short weights at a few tokens run co-resident (two CTAs per SM) under programmatic
        // dependent launch, on by default for these launches (E2C_PDL_SMALL=0: off): the next
        // launch's weight tiles are requested while this one finishes, which hides the fixed costs
        // a chain of short launches pays one after another.
        if (e2c_pdl_small_on() && a->M <= 32) {
            // Up to K = 4096 the co-resident split-K kernel, whose partials are reduced in a
            // cluster's shared memory rather than through the workspace, measured faster in a chain
            // (2048 x 8192 at M = 1: 6.45 against 6.84 us); deeper K balances better streamed
            // (8192 x 2048: 7.07 against 8.32 us). E2C_PDL_SPLITK=0 keeps the streaming kernel.
            static int splitk = -1;
            if (splitk < 0) {
                const char *v = getenv("E2C_PDL_SPLITK");
                splitk = !(v && v[0] == '0');
            }
            if (splitk && a->K <= 4096) {
                const int rc = e2c_gemm_splitk_co(a, stream);
                if (rc != -1) {
                    g_last_kernel = "splitk_coresident";
                    return rc;
                }
            }
            g_last_kernel = "stream_coresident";
            return e2c_gemm_stream(a, stream);
        }
    }
    {
        // short activation matrices: when the persistent kernel would leave most SMs idle, split K
        // over a cluster so every SM streams a slice of the weight
        int sbn = 0, S = 1;
        const int split_ctas = e2c_gemm_splitk_plan(a, num_sms, &sbn, &S);
        if (split_ctas) {
            const Plan pp = pick_plan(a, num_sms);
            const long ptiles = (long)((a->M + BM * pp.cg - 1) / (BM * pp.cg)) * ((a->n1 - a->n0 + pp.bn - 1) / pp.bn);
            const long pctas = (ptiles < num_sms / pp.cg ? ptiles : num_sms / pp.cg) * pp.cg;
            if (split_ctas >= 2 * pctas) {
                g_last_kernel = "splitk";
                return e2c_gemm_splitk(a, sbn, S, stream);
            }
        }
    }
    const Plan pl = pick_plan(a, num_sms);
    const bool pair = pl.cg == 2;
    g_last_kernel = pair ? "persistent_pair" : "persistent";
    switch (a->epi) {
    case E2C_EPI_F32:
        if (perblock)
            return pair ? launch<128, 6, true, E2C_EPI_F32, 2>(a, st, dev, num_sms)
                        : launch<128, 5, true, E2C_EPI_F32, 1>(a, st, dev, num_sms);
        if (pair)
            return pl.bn == 128   ? launch<128, 6, false, E2C_EPI_F32, 2>(a, st, dev, num_sms)
                   : pl.bn == 192 ? launch<192, 6, false, E2C_EPI_F32, 2>(a, st, dev, num_sms)
                                  : launch<256, 5, false, E2C_EPI_F32, 2>(a, st, dev, num_sms);
        return pl.bn == 128   ? launch<128, 4, false, E2C_EPI_F32, 1>(a, st, dev, num_sms)
               : pl.bn == 192 ? launch<192, 3, false, E2C_EPI_F32, 1>(a, st, dev, num_sms)
                              : launch<256, 3, false, E2C_EPI_F32, 1>(a, st, dev, num_sms);
    case E2C_EPI_RESID:
        if (perblock)
            return pair ? launch<128, 6, true, E2C_EPI_RESID, 2>(a, st, dev, num_sms)
                        : launch<128, 5, true, E2C_EPI_RESID, 1>(a, st, dev, num_sms);
        if (pair)
            return pl.bn == 128   ? launch<128, 6, false, E2C_EPI_RESID, 2>(a, st, dev, num_sms)
                   : pl.bn == 192 ? launch<192, 6, false, E2C_EPI_RESID, 2>(a, st, dev, num_sms)
                                  : launch<256, 5, false, E2C_EPI_RESID, 2>(a, st, dev, num_sms);
        return pl.bn == 128   ? launch<128, 4, false, E2C_EPI_RESID, 1>(a, st, dev, num_sms)
               : pl.bn == 192 ? launch<192, 3, false, E2C_EPI_RESID, 1>(a, st, dev, num_sms)
                              : launch<256, 3, false, E2C_EPI_RESID, 1>(a, st, dev, num_sms);
    case E2C_EPI_I32:
        if (perblock)
            return pair ? launch<128, 6, true, E2C_EPI_I32, 2>(a, st, dev, num_sms)
                        : launch<128, 6, true, E2C_EPI_I32, 1>(a, st, dev, num_sms);
        if (pair)
            return pl.bn == 128   ? launch<128, 6, false, E2C_EPI_I32, 2>(a, st, dev, num_sms)
                   : pl.bn == 192 ? launch<192, 6, false, E2C_EPI_I32, 2>(a, st, dev, num_sms)
                                  : launch<256, 6, false, E2C_EPI_I32, 2>(a, st, dev, num_sms);
        return pl.bn == 128   ? launch<128, 6, false, E2C_EPI_I32, 1>(a, st, dev, num_sms)
               : pl.bn == 192 ? launch<192, 4, false, E2C_EPI_I32, 1>(a, st, dev, num_sms)
                              : launch<256, 4, false, E2C_EPI_I32, 1>(a, st, dev, num_sms);
    case E2C_EPI_GELU:
        if (perblock || (a->n1 - a->n0) % 256 || a->n0 % 256 || a->ldy % 4) {
            e2c_set_msg("gemm: the GELU-gate epilogue needs per-row scales and 256-column (gate|up) groups");
            return -1;
        }
        return pair ? launch<256, 5, false, E2C_EPI_GELU, 2>(a, st, dev, num_sms) : launch<256, 3, false, E2C_EPI_GELU, 1>(a, st, dev, num_sms);
    case E2C_EPI_QKV:
        if (perblock || a->n0 != 0 || a->n1 != 256 * (a->nq + 2) || a->seq_len <= 0 || a->M % a->seq_len ||
            a->ldrope < a->seq_len) {
            e2c_set_msg("gemm: the QKV epilogue needs per-row scales, whole heads of 256, M a multiple of seq_len "
                        "and RoPE tables of ldrope >= seq_len positions");
            return -1;
        }
        // (single CTAs only for short activation matrices: two stages leave room for the constants)
        return pair ? launch<256, 4, false, E2C_EPI_QKV, 2>(a, st, dev, num_sms) : launch<256, 2, false, E2C_EPI_QKV, 1>(a, st, dev, num_sms);
    case E2C_EPI_NORMADD: {
        // the residual norms in the epilogue: its own kernel (gemm_i8_norm.cu); with per-128-block
        // activation scales the int8 output is quantised per 128-column block (q8_scale [M][N/128])
        // Three forms: q8 with norm_g2 (quantise rmsnorm(x) g2), q8 alone (quantise x), or norm_gf
        // without q8 (res = rmsnorm(x) gf after the last layer).
        const int ncols = a->n1 - a->n0;
        const bool quant = a->q8 != nullptr;
        if ((perblock && a->ablk != 128) || a->n0 != 0 || ncols % 128 || ncols / 128 > 8 || !a->res || !a->norm_g1 ||
            (quant ? (!a->q8_scale || a->ldq % 16 || ((uintptr_t)a->q8 & 15) || a->norm_gf) : !a->norm_gf || a->norm_g2) ||
            a->ldres % 4 || ((uintptr_t)a->res & 15)) {
            e2c_set_msg("gemm: the norm epilogue needs per-row or 128-wide block scales, whole rows of 128 x (1..8) columns, a 16-byte "
                        "aligned res, the first gain, and either 16-byte aligned int8 rows with their scales (and "
                        "optionally a second gain) or a final gain");
            return -1;
        }
        return e2c_gemm_norm(a, stream);
    }
    case E2C_EPI_GELUQ: {
        const int ncols = a->n1 - a->n0;
        if (perblock) {
            // GELU-gate and h's per-128-block quantiser in the per-block kernel's epilogue: each tile's
            // 256 weight rows are one block of h
            if (a->ablk != 128 || a->n0 != 0 || ncols % 256 || !a->q8 || !a->q8_scale || a->ldq % 16 ||
                a->ldq < ncols / 2 || ((uintptr_t)a->q8 & 15)) {
                e2c_set_msg("gemm: the per-block GELU-quantise epilogue needs 128-wide activation blocks, gate|up rows "
                            "in groups of 256 from row 0 and 16-byte aligned int8 rows of ldq >= N/2 with their scales");
                return -1;
            }
            return pair ? launch<128, 8, true, E2C_EPI_GELUQ, 2>(a, st, dev, num_sms)
                        : launch<128, 6, true, E2C_EPI_GELUQ, 1>(a, st, dev, num_sms);
        }
        // GELU-gate and the per-token quantiser of h in the epilogue: its own kernel (gemm_i8_gelu.cu)
        if ( a->n0 != 0 || ncols % 256 || ncols / 256 > 16 || !a->q8 || !a->q8_scale || a->ldq % 16 ||
            ((uintptr_t)a->q8 & 15)) {
            e2c_set_msg("gemm: the GELU-quantise epilogue needs per-row scales, gate|up rows in groups of 256 "
                        "(1..16) from row 0 and 16-byte aligned int8 rows with their scales");
            return -1;
        }
        return e2c_gemm_gelu_quant(a, stream);
    }
    case E2C_EPI_QKVPB: {
        // the per-block q|k|v finish of heads of 256 in the per-block kernel's epilogue
        const int ncols = a->n1 - a->n0, heads = ncols / 256, nkv2 = heads - a->nq;
        if (!perblock || a->n0 != 0 || ncols % 256 || a->nq < 1 || nkv2 < 2 || nkv2 % 2 || a->seq_len <= 0 ||
            a->M % a->seq_len || a->ldvt < a->seq_len || a->ldrope < 128 || a->ldrope % 4 || !a->q_out || !a->k_out ||
            !a->vt_out || !a->rope_cos || !a->rope_sin ||
            (((uintptr_t)a->q_out | (uintptr_t)a->k_out | (uintptr_t)a->rope_cos | (uintptr_t)a->rope_sin) & 15)) {
            e2c_set_msg("gemm: the per-block q|k|v epilogue needs per-block scales, whole heads of 256 (nq q heads, then "
                        "as many k as v heads), M a multiple of seq_len, ldvt >= seq_len, position-major RoPE tables "
                        "of ldrope >= 128 (a multiple of 4) and 16-byte aligned Q, K and tables");
            return -1;
        }
        return pair ? launch<128, 8, true, E2C_EPI_QKVPB, 2>(a, st, dev, num_sms)
                    : launch<128, 6, true, E2C_EPI_QKVPB, 1>(a, st, dev, num_sms);
    }
    default:
        e2c_set_msg("gemm: unknown epilogue %d", a->epi);
        return -1;
    }
}

// sizeof(e2c_gemm_args), for the bindings' layout check
extern "C" int e2c_gemm_args_size(void) { return (int)sizeof(e2c_gemm_args); }
