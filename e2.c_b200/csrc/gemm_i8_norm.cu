// gemm_i8_norm.cu — W8A8 GEMM with an encoder layer's residual norms in its epilogue.
//
//   t  = float(acc) * (as[m] * ws[n])                        the projection (o_proj or down)
//   x  = rmsnorm(t) * g1 + res ;  res <- x                   e2.c src/text.c:947,954 (norm_add)
//   q8 = quantise(rmsnorm(x) * g2) per token                 the next projection's int8 input
//   or, after the last layer (g2 NULL):  res <- rmsnorm(x) * gf
//   or, with int8 rows but no g2:          q8 = quantise(x)    (e2.c's text tower, after the FFN)
// with x optionally multiplied by a layer scalar after the residual add (the text tower's
// per-layer-embedding step, src/text.c:966-975).
//
// with rmsnorm(v) = v / sqrt(mean(v^2) + eps) over the D = 128 x (1..8) columns of a row
// (src/kernels.c:144-171) and the per-token quantiser of src/int8.c:178-209. The GEMM output t
// never reaches memory: HBM sees the int8 activations, the residual read and written once, and
// the int8 rows with their scales.
//
// Layout: a cluster of D / 128 CTAs owns 128-row blocks, one 128-column block per CTA (the
// CTA's block is fixed for the kernel), persistent over the row blocks. Per CTA:
//   warp 0      TMA producer of A [128 x 128] and B [128 x 128] int8 stages (128-byte swizzle);
//   warp 1      MMA issuer, tcgen05.mma kind::i8 into one of four TMEM accumulators (all 512
//               columns), so the tensor core runs up to two row blocks ahead of the epilogue;
//   warps 2-17  epilogue: four per TMEM lane quadrant, each owning 32 rows x 32 columns.
// A row's statistics span the cluster: each needs a sum over its D columns, reduced in two
// rounds (sum t^2, then sum x^2 with max |x g2|). In a round the quadrant's four warps combine
// their columns in shared memory and one of them sends the CTA's partial to every CTA of the
// cluster by st.async, counted in bytes on the receiver's mbarrier (two slots and barriers,
// alternating by row block, so a fast CTA's next round never lands on a slot still being read).
//
// The epilogue is software-pipelined over row blocks so both rounds' latency hides behind work
// of a neighbouring block: while block n's second round travels, the warp runs block n+1's first
// pass; while block n+1's first round travels, it runs block n's last pass. Per block n:
//   pass 1   acc(n) -> sum (acc ws)^2, and v = acc (ws g1) back into acc(n)'s TMEM columns
//                                                                    -> round 0 send
//   pass 2   x = fma(v, as inv1, res) into the residual tiles (then TMA store); sum x^2, and
//            y = x g2 back into TMEM with max |y|                   -> round 1 send
//   pass 3   y from TMEM -> q8 = rint(y 127 / max|y|), staged and TMA-stored
// The residual tiles of a warp (32 x 32 fp32, 64-byte swizzle) are reloaded for block n+1 as
// soon as block n's x store has read them. fp32 is reassociated relative to the two-kernel path
// (sum t^2 = as^2 sum (acc ws)^2, x = (acc (ws g1)) (as inv1) + res); results agree with it
// to a few ulp, within the norms' tolerance.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "epi_math.cuh"
#include "launch.h"
#include "devstate.cuh"
#include "pdl.h"
#include "ptx.cuh"
#include "tmap.h"

namespace {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int NACC = 4;                    // TMEM accumulators of BN columns
constexpr int EPI_WARPS = 16;
constexpr int NTHREADS = 64 + 32 * EPI_WARPS;
constexpr int QCOLS = BN / 4;              // columns per epilogue warp
constexpr int NCH = QCOLS / 16;            // 16-column chunks per warp
constexpr int MAXCL = 8;                   // CTAs per cluster: D <= 1024
// Column constants per column part (the quadrants' four warps of a part share them): ws, ws g1, g2
// (or gf); then per warp the activation scales of four row blocks (rows differ by quadrant)
constexpr int CSTC_FLOATS = 3 * QCOLS;
constexpr int CSTA_FLOATS = 4 * 32;
constexpr int RES_TILE = 32 * 16 * 4;      // 32 rows x 16 fp32, 64-byte swizzle
constexpr int C_WG1 = QCOLS, C_G2 = 2 * QCOLS;

// STG mainloop stages; exchange slots for clusters of up to XMAX CTAs. Four stages fit beside the
// epilogue's buffers for clusters of up to 6 (D <= 768); wider clusters keep three.
template <int STG, int XMAX>
struct Smem {
    static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE = A_BYTES + B_BYTES;
    static constexpr int RES_OFF = STG * STAGE;
    static constexpr int CSTC_OFF = RES_OFF + EPI_WARPS * NCH * RES_TILE;  // [4 parts][3 x 32] float
    static constexpr int CSTA_OFF = CSTC_OFF + 4 * CSTC_FLOATS * 4;        // [16 warps][4 x 32] float
    static constexpr int XL0_OFF = CSTA_OFF + EPI_WARPS * CSTA_FLOATS * 4;  // [4 parts][BM] float
    static constexpr int XL1_OFF = XL0_OFF + 4 * BM * 4;                   // [4 parts][BM] float2
    static constexpr int XR0_OFF = XL1_OFF + 4 * BM * 8;                   // [2][XMAX][BM] float
    static constexpr int XR1_OFF = XR0_OFF + 2 * XMAX * BM * 4;            // [2][XMAX][BM] float2
    static constexpr int BAR_OFF = XR1_OFF + 2 * XMAX * BM * 8;
    // full[S], empty[S], tfull[NACC], tempty[NACC], lbar[2 rounds][4], xbar[2 rounds][2][4], rbar[16]
    static constexpr int NBAR = 2 * STG + 2 * NACC + 8 + 16 + EPI_WARPS;
    static constexpr int BYTES = BAR_OFF + NBAR * 8 + 16;
    // No alignment slack: the dynamic shared memory of a kernel without static shared variables
    // starts 1024-byte aligned, which the kernel checks before using it (the swizzled tiles need it).
    static constexpr int ALLOC = BYTES;
    static_assert(RES_OFF % 1024 == 0, "swizzled TMA tiles");
    static_assert(ALLOC <= 232448, "shared memory");
};

// QUANT: the next layer's int8 input is produced (g2 given); otherwise the final norm (gf).
// PB: activations with per-128-block scales (the per-block fold, e2.c's default recipe): the MMA
// fills a ring of two 128-deep-block accumulators (TMEM columns 0..255), the first pass folds a
// row block's blocks into t = sum fl(as ws) float(dot) (then the F32 epilogue's clamp) and keeps
// v = t g1 in one of two row-block slots (columns 256..511), and the int8 output is quantised per
// 128-column block, the CTA's own: its maximum comes from the quadrant's four warps, not the
// cluster. The second pass's factor is inv1 alone.
template <bool QUANT, int STAGES, int XMAX, bool PB>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm_norm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmR,
                const e2c_gemm_args p) {
    using L = Smem<STAGES, XMAX>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    griddep_launch_dependents();
    if (smem_u32(smem_raw) & 1023) {  // never expected; every CTA of the launch sees the same base
        griddep_wait();
        if (threadIdx.x == 0) record_status(p.status, E2C_ERR_SMEM_ALIGN);
        return;
    }
    uint8_t *smem = smem_raw;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + NACC + a); };
    auto lbar = [&](int r, int q) { return bar0 + 8u * (2 * STAGES + 2 * NACC + 4 * r + q); };
    auto xbar = [&](int r, int b, int q) { return bar0 + 8u * (2 * STAGES + 2 * NACC + 8 + 8 * r + 4 * b + q); };
    auto rbar = [&](int w) { return bar0 + 8u * (2 * STAGES + 2 * NACC + 24 + w); };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + L::BAR_OFF + L::NBAR * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = p.M, K = p.K, D = p.n1 - p.n0;
    const int ncl = D / BN;                      // CTAs of a cluster (the launch's cluster width)
    const int rank = (int)(blockIdx.x % (unsigned)ncl);  // = cluster rank = this CTA's column block
    const int cid = (int)(blockIdx.x / (unsigned)ncl), ncls = (int)(gridDim.x / (unsigned)ncl);
    const int tiles_m = (M + BM - 1) / BM;
    const int ntl = cid < tiles_m ? (tiles_m - 1 - cid) / ncls + 1 : 0;  // row blocks of this CTA
    const int nk = (K + BK - 1) / BK;
    const int kpu = PB ? p.ablk / BK : nk;  // k-blocks per accumulation unit
    const int nb = PB ? K / p.ablk : 1;     // units (activation scale blocks) per row block
    auto row0 = [&](int n) { return (cid + n * ncls) * BM; };

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < NACC; a++) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), EPI_WARPS);
        }
        for (int r = 0; r < 2; r++)
            for (int q = 0; q < 4; q++) {
                mbar_init(lbar(r, q), 128);  // the quadrant's 4 warps
                for (int b = 0; b < 2; b++) mbar_init(xbar(r, b, q), 1);  // own expect_tx; bytes by st.async
            }
        for (int w = 0; w < EPI_WARPS; w++) mbar_init(rbar(w), 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        __syncwarp();
        tmem_alloc(sbase + L::BAR_OFF + L::NBAR * 8, NACC * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    cluster_sync();  // every CTA's barriers exist before another CTA signals them
    tc_fence_after();
    griddep_wait();  // the stream's earlier kernels are done with what this one reads and writes
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (elect_one()) {
            int stage = 0, issued = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int n = 0; n < ntl && ok; n++) {
                for (int kb = 0; kb < nk; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.status, E2C_ERR_WAIT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = sbase + stage * L::STAGE, sb = sa + L::A_BYTES;
                    mbar_arrive_expect_tx(full_bar(stage), L::STAGE);
                    tma_load_2d(sa, &tmA, kb * BK, row0(n), full_bar(stage));
                    tma_load_2d(sb, &tmB, kb * BK, p.n0 + rank * BN, full_bar(stage));
                    issued++;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // the copies this thread started land before the CTA's shared memory goes away
                int s = stage, ph = (int)phase;
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
        if (PB && elect_one()) {
            // a ring of two accumulators of one 128-deep block each, drained by the first pass
            constexpr uint32_t idesc = idesc_i8(BN, BM);
            int stage = 0, ua = 0;
            uint32_t phase = 0, uph = 0;
            bool ok = true;
            for (int n = 0; n < ntl && ok; n++) {
                for (int u = 0; u < nb && ok; u++) {
                    if (!mbar_wait(tempty_bar(ua), uph ^ 1u, p.status, E2C_ERR_WAIT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(ua * BN);
                    for (int kk = 0; kk < kpu; kk++) {
                        if (!mbar_wait(full_bar(stage), phase, p.status, E2C_ERR_WAIT_MMA)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = sbase + stage * L::STAGE, sb = sa + L::A_BYTES;
#pragma unroll
                        for (int k = 0; k < BK / 32; k++)
                            mma_i8(d, smem_desc_sw128(sa + 32 * k), smem_desc_sw128(sb + 32 * k), idesc, (kk | k) != 0);
                        mma_commit(empty_bar(stage));
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    mma_commit(tfull_bar(ua));
                    ua ^= 1;
                    if (ua == 0) uph ^= 1u;
                }
            }
            if (!ok) {
                // every MMA issued so far finishes before the accumulators are released
                const uint32_t drain = tfull_bar(ua);
                mma_commit(drain);
                mbar_wait(drain, uph, nullptr, E2C_ERR_WAIT_DRAIN);
            }
        } else if (!PB && elect_one()) {
            constexpr uint32_t idesc = idesc_i8(BN, BM);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int n = 0;
            for (; n < ntl && ok; n++) {
                const int a = n % NACC;
                if (!mbar_wait(tempty_bar(a), (uint32_t)((n / NACC) & 1) ^ 1u, p.status, E2C_ERR_WAIT_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(a * BN);
                for (int kb = 0; kb < nk; kb++) {
                    if (!mbar_wait(full_bar(stage), phase, p.status, E2C_ERR_WAIT_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = sbase + stage * L::STAGE, sb = sa + L::A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 32; k++)
                        mma_i8(d, smem_desc_sw128(sa + 32 * k), smem_desc_sw128(sb + 32 * k), idesc, (kb | k) != 0);
                    mma_commit(empty_bar(stage));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(tfull_bar(a));
            }
            if (!ok) {
                // every MMA issued so far finishes before the accumulators are released
                const uint32_t drain = tfull_bar(n % NACC);
                mma_commit(drain);
                mbar_wait(drain, (uint32_t)((n / NACC) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int q = warp & 3;             // TMEM lane quadrant this warp may access
        const int part = (warp - 2) >> 2;   // which 32 of the CTA's 128 columns
        const int row = q * 32 + lane;      // row of the block = TMEM lane
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        const int cl0 = rank * BN + part * QCOLS;  // first column of this warp within the row
        constexpr bool quant = QUANT;
        float *cst = reinterpret_cast<float *>(smem + L::CSTC_OFF) + part * CSTC_FLOATS;   // shared by the part's warps
        float *csta = reinterpret_cast<float *>(smem + L::CSTA_OFF) + (warp - 2) * CSTA_FLOATS;
        uint8_t *resb = smem + L::RES_OFF + (warp - 2) * NCH * RES_TILE;
        const uint32_t resb_s = smem_u32(resb);
        const uint32_t rb = rbar(warp - 2);
        {
            // (quantising x itself: g2 = 1)
            const float *gb = quant ? p.norm_g2 : p.norm_gf;
            for (int j = lane; j < QCOLS; j += 32) {
                const float w = __ldg(p.w_scale + p.n0 + cl0 + j);
                cst[j] = w;
                // per-block: the gain alone (t is scaled by the fold)
                cst[C_WG1 + j] = PB ? __ldg(p.norm_g1 + cl0 + j) : __fmul_rn(w, __ldg(p.norm_g1 + cl0 + j));
                cst[C_G2 + j] = gb ? __ldg(gb + cl0 + j) : 1.0f;
            }
            __syncwarp();
        }
        bool ok = true, xok = true;
        // the rows' activation scales of block n land in slot n & 3 by cp.async (one group per call)
        const uint32_t as_slot = smem_u32(csta + lane);
        auto load_as = [&](int n) {
            if (!PB && n < ntl) {  // (per-block: the fold reads its scales itself; an empty group)
                const int mr = row0(n) + row;
                cp_async_4(as_slot + (uint32_t)((n & 3) * 128), p.a_scale + (mr < M ? (size_t)mr : 0), mr < M ? 4u : 0u);
            }
            cp_async_commit();
        };
        // the residual of block n: this warp's 32 rows x 32 columns, two 64-byte-swizzled tiles
        bool rpend = false;
        uint32_t rpar = 0;
        auto load_res = [&](int n) {
            if (lane == 0) {
                mbar_arrive_expect_tx(rb, (uint32_t)(NCH * RES_TILE));
#pragma unroll
                for (int c = 0; c < NCH; c++) tma_load_2d(resb_s + c * RES_TILE, &tmR, cl0 + 16 * c, row0(n) + q * 32, rb);
            }
            rpend = true;
            rpar = (uint32_t)(n & 1);
        };
        auto store_res = [&](int n) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
#pragma unroll
                for (int c = 0; c < NCH; c++) tma_store_2d(&tmR, resb_s + c * RES_TILE, cl0 + 16 * c, row0(n) + q * 32);
                bulk_commit();
            }
        };
        // element (lane, 4 k .. 4 k + 3) of residual tile c (the TMA map's 64-byte swizzle)
        auto rp = [&](int c, int k) -> float4 * {
            return reinterpret_cast<float4 *>(resb + c * RES_TILE + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4));
        };
        float *xl0 = reinterpret_cast<float *>(smem + L::XL0_OFF);
        // round 1's per-warp partials; per-block mode reads them again for the block maximum in
        // pass 3, so they alternate by row block (odd blocks in the row-scale area it does not use)
        auto xl1b = [&](int n) {
            return reinterpret_cast<float2 *>(smem + ((PB && (n & 1)) ? L::CSTA_OFF : L::XL1_OFF));
        };
        // round r of block n: this warp's partial (sum in .x, max in .y) to the quadrant, and from
        // part 0 the CTA's partial to every CTA of the cluster
        auto send = [&](int r, int n, float2 v) {
            float2 *xl1 = xl1b(n);
            if (r == 0) xl0[part * BM + row] = v.x;
            else xl1[part * BM + row] = v;
            mbar_arrive(lbar(r, q));
            if (part != 0) return;
            xok = xok && __all_sync(0xffffffffu, mbar_wait(lbar(r, q), (uint32_t)(n & 1), p.status, E2C_ERR_WAIT_EPI));
            float2 c = make_float2(0.f, 0.f);
#pragma unroll
            for (int w = 0; w < 4; w++) {
                if (r == 0) {
                    c.x = __fadd_rn(c.x, xl0[w * BM + row]);
                } else {
                    const float2 o = xl1[w * BM + row];
                    c.x = __fadd_rn(c.x, o.x);
                    c.y = fmaxf(c.y, o.y);
                }
            }
            const int b = n & 1;
            const uint32_t xb = xbar(r, b, q);
            if (lane == 0) mbar_arrive_expect_tx(xb, (uint32_t)(ncl * 32 * (r == 0 ? 4 : 8)));
            const uint32_t slot = r == 0 ? sbase + L::XR0_OFF + (uint32_t)(((b * XMAX + rank) * BM + row) * 4)
                                         : sbase + L::XR1_OFF + (uint32_t)(((b * XMAX + rank) * BM + row) * 8);
            for (int d = 0; d < ncl; d++) {
                if (r == 0) st_async_f32(mapa_shared(slot, (uint32_t)d), c.x, mapa_shared(xb, (uint32_t)d));
                else st_async_f32x2(mapa_shared(slot, (uint32_t)d), c.x, c.y, mapa_shared(xb, (uint32_t)d));
            }
        };
        auto recv = [&](int r, int n) -> float2 {
            const int b = n & 1;
            xok = xok && __all_sync(0xffffffffu, mbar_wait(xbar(r, b, q), (uint32_t)((n >> 1) & 1), p.status, E2C_ERR_WAIT_EPI));
            float2 tot = make_float2(0.f, 0.f);
            for (int d = 0; d < ncl; d++) {
                if (r == 0) {
                    tot.x = __fadd_rn(tot.x, reinterpret_cast<const float *>(smem + L::XR0_OFF)[(b * XMAX + d) * BM + row]);
                } else {
                    const float2 o = reinterpret_cast<const float2 *>(smem + L::XR1_OFF)[(b * XMAX + d) * BM + row];
                    tot.x = __fadd_rn(tot.x, o.x);
                    tot.y = fmaxf(tot.y, o.y);
                }
            }
            return tot;
        };
        // the block's TMEM columns: its accumulator, or per-block its slot (columns 256..511)
        auto tcols = [&](int n) {
            return tmem_base + lane_addr + (uint32_t)((PB ? 2 + (n & 1) : n % NACC) * BN + part * QCOLS);
        };
        int ua = 0;  // per-block: the accumulator ring, in step with the MMA issuer
        uint32_t uph = 0;
        // per-block pass 1: block n's 128-deep blocks folded in registers, f = fma(float(dot),
        // fl(as ws), f) block by block (the per-block F32 epilogue's arithmetic) and clamped to t;
        // returns sum t^2 over the warp's columns and leaves v = t g1 in the block's slot
        auto pass1_pb = [&](int n) -> float {
            const int m = row0(n) + row;
            const bool mrow = m < M;
            float f[QCOLS];
#pragma unroll
            for (int j = 0; j < QCOLS; j++) f[j] = 0.f;
            float as_next = mrow ? __ldg(p.a_scale + (size_t)m * nb) : 0.f;
            for (int u = 0; u < nb; u++) {
                const float as = as_next;
                if (u + 1 < nb) as_next = mrow ? __ldg(p.a_scale + (size_t)m * nb + u + 1) : 0.f;
                if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(ua), uph, p.status, E2C_ERR_WAIT_EPI))) {
                    ok = false;
                    return 0.f;
                }
                tc_fence_after();
                const uint32_t ta = tmem_base + lane_addr + (uint32_t)(ua * BN + part * QCOLS);
                const float2 as2 = make_float2(as, as);
#pragma unroll
                for (int c = 0; c < NCH; c++) {
                    uint32_t r[16];
                    tmem_ld16(ta + 16 * c, r);
                    tmem_wait_ld();
                    if (c == NCH - 1) {
                        // every column of the accumulator this warp reads has been read
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(tempty_bar(ua));
                    }
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const float4 w4 = *reinterpret_cast<const float4 *>(cst + 16 * c + 4 * k);
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int e = 4 * k + 2 * h, j = 16 * c + e;
                            const float2 s2 = mul2_rn(as2, h ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y));
                            const float2 d2 = make_float2(__int2float_rn((int)r[e]), __int2float_rn((int)r[e + 1]));
                            const float2 o = fma2_rn(d2, s2, make_float2(f[j], f[j + 1]));
                            f[j] = o.x;
                            f[j + 1] = o.y;
                        }
                    }
                }
                ua ^= 1;
                if (ua == 0) uph ^= 1u;
            }
            float2 ssp[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
            for (int c = 0; c < NCH; c++) {
                uint32_t r[16];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const float4 g4 = *reinterpret_cast<const float4 *>(cst + C_WG1 + 16 * c + 4 * k);
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int e = 4 * k + 2 * h, j = 16 * c + e;
                        const float2 t = make_float2(fminf(fmaxf(f[j], p.out_min), p.out_max),
                                                     fminf(fmaxf(f[j + 1], p.out_min), p.out_max));
                        ssp[h] = fma2_rn(t, t, ssp[h]);
                        const float2 v = mul2_rn(t, h ? make_float2(g4.z, g4.w) : make_float2(g4.x, g4.y));
                        r[e] = __float_as_uint(v.x);
                        r[e + 1] = __float_as_uint(v.y);
                    }
                }
                tmem_st16(tcols(n) + 16 * c, r);
            }
            tmem_wait_st();
            return __fadd_rn(__fadd_rn(ssp[0].x, ssp[0].y), __fadd_rn(ssp[1].x, ssp[1].y));
        };
        // pass 1: as^2 sum over the warp's columns of (acc ws)^2, once block n's accumulator is full;
        // v = acc (ws g1) replaces the accumulator for pass 2
        auto pass1 = [&](int n) -> float {
            if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(n % NACC), (uint32_t)((n / NACC) & 1), p.status, E2C_ERR_WAIT_EPI))) {
                ok = false;
                return 0.f;
            }
            tc_fence_after();
            uint32_t r[NCH][16];
#pragma unroll
            for (int c = 0; c < NCH; c++) tmem_ld16(tcols(n) + 16 * c, r[c]);
            tmem_wait_ld();
            // four independent partial sums (a single fma chain would issue one step per fma latency),
            // two per packed f32x2 register: ssp[h] = (sum of columns 4i + 2h, of columns 4i + 2h + 1)
            float2 ssp[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
            for (int c = 0; c < NCH; c++) {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(cst + 16 * c + 4 * k);
                    const float4 c4 = *reinterpret_cast<const float4 *>(cst + C_WG1 + 16 * c + 4 * k);
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int e = 4 * k + 2 * h;
                        const float2 f = make_float2(__int2float_rn((int)r[c][e]), __int2float_rn((int)r[c][e + 1]));
                        const float2 u = mul2_rn(f, h ? make_float2(w4.z, w4.w) : make_float2(w4.x, w4.y));
                        ssp[h] = fma2_rn(u, u, ssp[h]);
                        // v = acc (ws g1), for pass 2
                        const float2 v = mul2_rn(f, h ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y));
                        r[c][e] = __float_as_uint(v.x);
                        r[c][e + 1] = __float_as_uint(v.y);
                    }
                }
                tmem_st16(tcols(n) + 16 * c, r[c]);
            }
            tmem_wait_st();
            const float ss = __fadd_rn(__fadd_rn(ssp[0].x, ssp[0].y), __fadd_rn(ssp[1].x, ssp[1].y));
            const float as = csta[(n & 3) * 32 + lane];
            return __fmul_rn(__fmul_rn(as, as), ss);
        };
        auto pass1x = [&](int n) -> float {
            if constexpr (PB) return pass1_pb(n);
            else return pass1(n);
        };
        auto release = [&](int n) {
            if (PB) return;  // (per-block: the slots belong to the epilogue; the ring is released by pass 1)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(n % NACC));
        };

        if (ntl > 0) {
            load_as(0);
            load_as(1);
            load_res(0);
            cp_async_wait_1();
            const float s0 = pass1x(0);
            if (ok) send(0, 0, make_float2(s0, 0.f));
        }
        for (int n = 0; n < ntl && ok && xok; n++) {
            load_as(n + 2);
            const float s1 = recv(0, n).x;
            if (!xok) break;
            const float inv1 = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s1, (float)D), p.eps)));
            const float sr = PB ? inv1 : __fmul_rn(csta[(n & 3) * 32 + lane], inv1);
            // the layer scalar after the residual add (text tower's per-layer-embedding step)
            const bool ls_on = p.norm_ls != 0.f && p.norm_ls != 1.f;
            const float2 ls2 = make_float2(p.norm_ls, p.norm_ls);
            // pass 2: x = fma(v, as inv1, res) into the residual tiles; y = x g2 into the accumulator
            if (!__all_sync(0xffffffffu, mbar_wait(rb, rpar, p.status, E2C_ERR_WAIT_EPI))) {
                ok = false;
                break;
            }
            rpend = false;
            // independent partials, the sums two per packed f32x2 register (as in pass 1)
            float2 s2p[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            float mxp[4] = {0.f, 0.f, 0.f, 0.f};
            const float2 sr2 = make_float2(sr, sr);
#pragma unroll
            for (int c = 0; c < NCH; c++) {
                uint32_t r[16];
                tmem_ld16(tcols(n) + 16 * c, r);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    float4 *p4 = rp(c, k);
                    const float4 r4 = *p4;
                    float2 xa = fma2_rn(make_float2(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1])), sr2,
                                        make_float2(r4.x, r4.y));
                    float2 xb = fma2_rn(make_float2(__uint_as_float(r[4 * k + 2]), __uint_as_float(r[4 * k + 3])), sr2,
                                        make_float2(r4.z, r4.w));
                    if (ls_on) {
                        xa = mul2_rn(xa, ls2);
                        xb = mul2_rn(xb, ls2);
                    }
                    *p4 = make_float4(xa.x, xa.y, xb.x, xb.y);
                    s2p[0] = fma2_rn(xa, xa, s2p[0]);
                    s2p[1] = fma2_rn(xb, xb, s2p[1]);
                    if constexpr (quant) {
                        // y = x g2 goes back to TMEM for the int8 pass
                        const float4 g4 = *reinterpret_cast<const float4 *>(cst + C_G2 + 16 * c + 4 * k);
                        const float2 ya = mul2_rn(xa, make_float2(g4.x, g4.y)), yb = mul2_rn(xb, make_float2(g4.z, g4.w));
                        const float y[4] = {ya.x, ya.y, yb.x, yb.y};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            mxp[e] = fmaxf(mxp[e], fabsf(y[e]));
                            r[4 * k + e] = __float_as_uint(y[e]);
                        }
                    }
                }
                if constexpr (quant) tmem_st16(tcols(n) + 16 * c, r);
            }
            tmem_wait_st();
            const float ss2 = __fadd_rn(__fadd_rn(s2p[0].x, s2p[0].y), __fadd_rn(s2p[1].x, s2p[1].y));
            const float mx = fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3]));
            if constexpr (quant) store_res(n);  // the new residual is x
            send(1, n, make_float2(ss2, mx));
            if constexpr (quant) {
                // block n+1's first pass and residual load while block n's second round travels
                if (n + 1 < ntl) {
                    cp_async_wait_1();
                    const float s0 = pass1x(n + 1);
                    if (!ok) break;
                    send(0, n + 1, make_float2(s0, 0.f));
                    if (lane == 0) bulk_wait_read0();  // block n's x store has read the tiles
                    __syncwarp();
                    load_res(n + 1);
                }
                const float2 t2 = recv(1, n);
                if (!xok) break;
                // pass 3: the quantiser of src/int8.c:178-209 on z = x inv2 g2, amax = inv2 max|y| with
                // y = x g2, scale = amax / 127, q = rint(z 127 / amax) = rint(y 127 / max|y|); |q| <= 127
                // needs no clamp, and rint is the round-to-nearest-even of adding 1.5 2^23, whose low
                // byte is q
                // (quantising x itself: no second norm)
                const float inv2 = p.norm_g2 ? __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t2.x, (float)D), p.eps))) : 1.0f;
                // the quantiser's max|y|: the row's (cluster), or per-block the CTA's 128 columns (the
                // quadrant's four warps, whose round-1 partials this warp waits for too)
                float mxy = t2.y;
                if constexpr (PB) {
                    xok = xok && __all_sync(0xffffffffu, mbar_wait(lbar(1, q), (uint32_t)(n & 1), p.status, E2C_ERR_WAIT_EPI));
                    if (!xok) break;
                    const float2 *xb = xl1b(n);
                    mxy = fmaxf(fmaxf(xb[row].y, xb[BM + row].y), fmaxf(xb[2 * BM + row].y, xb[3 * BM + row].y));
                }
                const float amax = __fmul_rn(mxy, inv2);
                const float s = mxy > 0.f ? __fdiv_rn(127.0f, mxy) : 0.f;
                const int m = row0(n) + row;
                if ((PB || rank == 0) && part == 0 && m < M)
                    p.q8_scale[PB ? (size_t)m * ncl + rank : (size_t)m] = amax > 0.f ? __fmul_rn(amax, 0x1.020408p-7f) : 1.0f;
                uint4 *qrow = reinterpret_cast<uint4 *>(p.q8 + (size_t)(m < M ? m : 0) * p.ldq + cl0);
#pragma unroll
                for (int c = 0; c < NCH; c++) {
                    uint32_t r[16];
                    tmem_ld16(tcols(n) + 16 * c, r);
                    tmem_wait_ld();
                    uint32_t pk[4];
                    const float2 s2 = make_float2(s, s), mg = make_float2(12582912.0f, 12582912.0f);
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const float2 ba = fma2_rn(make_float2(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1])), s2, mg);
                        const float2 bb = fma2_rn(make_float2(__uint_as_float(r[4 * k + 2]), __uint_as_float(r[4 * k + 3])), s2, mg);
                        pk[k] = __byte_perm(__byte_perm(__float_as_uint(ba.x), __float_as_uint(ba.y), 0x0040),
                                            __byte_perm(__float_as_uint(bb.x), __float_as_uint(bb.y), 0x0040), 0x5410);
                    }
                    // 16 bytes of row m straight from registers (chunks 0 and 1 fill the row's 32-byte sector)
                    if (m < M) qrow[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                release(n);
            } else {
                // the final norm: res = x inv2 gf, written over x in the tiles; then block n+1
                const float2 t2 = recv(1, n);
                if (!xok) break;
                const float inv2 = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t2.x, (float)D), p.eps)));
#pragma unroll
                for (int c = 0; c < NCH; c++)
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        float4 *p4 = rp(c, k);
                        const float4 x4 = *p4;
                        const float4 g4 = *reinterpret_cast<const float4 *>(cst + C_G2 + 16 * c + 4 * k);
                        *p4 = make_float4(__fmul_rn(__fmul_rn(x4.x, inv2), g4.x), __fmul_rn(__fmul_rn(x4.y, inv2), g4.y),
                                          __fmul_rn(__fmul_rn(x4.z, inv2), g4.z), __fmul_rn(__fmul_rn(x4.w, inv2), g4.w));
                    }
                release(n);
                store_res(n);
                if (n + 1 < ntl) {
                    cp_async_wait_1();
                    const float s0 = pass1x(n + 1);
                    if (!ok) break;
                    send(0, n + 1, make_float2(s0, 0.f));
                    if (lane == 0) bulk_wait_read0();
                    __syncwarp();
                    load_res(n + 1);
                }
            }
        }
        // copies into this warp's shared memory land, and its stores complete, before the CTA ends
        cp_async_wait_all();
        if (rpend) {
            if (lane == 0) mbar_wait(rb, rpar, nullptr, E2C_ERR_WAIT_DRAIN);
            __syncwarp();
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }

    tc_fence_before();
    // no CTA leaves while another may still signal its barriers or write its shared memory
    cluster_sync();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, NACC * BN);
    }
}

template <int STG, int XMAX, bool PB>
int launch_norm(const e2c_gemm_args *a, int ncl, bool quant, cudaStream_t st, int dev, int num_sms) {
    using L = Smem<STG, XMAX>;
    static E2cPerDev attr_set;                    // the shared-memory opt-in, per device
    static E2cPerDev max_clusters[2][MAXCL + 1];  // resident clusters per (quantise, width), per device
    if (!attr_set.get(dev)) {
        if (cudaFuncSetAttribute(k_gemm_norm<true, STG, XMAX, PB>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) !=
                cudaSuccess ||
            cudaFuncSetAttribute(k_gemm_norm<false, STG, XMAX, PB>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) !=
                cudaSuccess) {
            cudaGetLastError();
            e2c_set_msg("gemm_norm: cannot reserve %d bytes of shared memory", L::ALLOC);
            return -2;
        }
        attr_set.set(dev, 1);
    }
    const int D = a->n1 - a->n0;
    CUtensorMap ta, tb, tr;
    if (e2c_tmap_2d(&ta, a->a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->M, (uint64_t)a->lda, BK, BM) ||
        e2c_tmap_2d(&tb, a->w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->wrows, (uint64_t)a->ldw, BK, BN) ||
        e2c_tmap_2d_sw64(&tr, a->res, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)D, (uint64_t)a->M,
                         (uint64_t)a->ldres * 4, 16, 32))
        return -3;
    const int tiles_m = (a->M + BM - 1) / BM;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ncl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = L::ALLOC;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    auto kern = quant ? k_gemm_norm<true, STG, XMAX, PB> : k_gemm_norm<false, STG, XMAX, PB>;
    int maxc = max_clusters[quant][ncl].get(dev);
    if (!maxc) {
        cfg.gridDim = dim3((unsigned)(ncl * (num_sms / ncl)));
        if (cudaOccupancyMaxActiveClusters(&maxc, kern, &cfg) != cudaSuccess || maxc <= 0) {
            cudaGetLastError();
            e2c_set_msg("gemm_norm: the device cannot hold a cluster of %d CTAs", ncl);
            return -2;
        }
        max_clusters[quant][ncl].set(dev, maxc);
    }
    cfg.gridDim = dim3((unsigned)(ncl * (tiles_m < maxc ? tiles_m : maxc)));
    cfg.numAttrs = e2c_pdl_attr(attr, 1);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tr, *a);
    if (e != cudaSuccess) {
        e2c_set_msg("gemm_norm launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}

}  // namespace

// The GEMM + norms launch: geometry checked by e2c_gemm (per-row scales, n0 = 0, D = 128 x (1..8)).
extern "C" int e2c_gemm_norm(const e2c_gemm_args *a, void *stream) {
    const int dev = e2c_device();
    const int num_sms = e2c_sm_count(dev);
    if (!num_sms) {
        e2c_set_msg("gemm_norm: no CUDA device");
        return -2;
    }
    const int D = a->n1 - a->n0;
    const int ncl = D / BN;
    if (a->n0 != 0 || D % BN || ncl < 1 || ncl > MAXCL) {
        e2c_set_msg("gemm_norm: rows of 128 x (1..8) columns starting at column 0");
        return -1;
    }
    const bool quant = a->q8 != nullptr;
    cudaStream_t st = (cudaStream_t)stream;
    if (a->ablk != a->K)  // per-128-block activation scales
        return ncl <= 6 ? launch_norm<4, 6, true>(a, ncl, quant, st, dev, num_sms)
                        : launch_norm<3, MAXCL, true>(a, ncl, quant, st, dev, num_sms);
    return ncl <= 6 ? launch_norm<4, 6, false>(a, ncl, quant, st, dev, num_sms)
                    : launch_norm<3, MAXCL, false>(a, ncl, quant, st, dev, num_sms);
}
