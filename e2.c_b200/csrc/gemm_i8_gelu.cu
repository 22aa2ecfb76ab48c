// gemm_i8_gelu.cu — the FFN's gate|up W8A8 GEMM with GELU-gate and the per-token quantiser of its
// output in the epilogue:
//
//   g, u  = float(acc) * (as[m] * ws[n])  over the gate and up weight rows (interleaved per 128)
//   h     = gelu_tanh(g) * u                                 e2.c src/text.c:950-953 (GELU-gate)
//   q8[m] = rint(h * fl(127 / amax)), scale = amax fl(1/127), amax = max |h| over the row's I
//           columns                                           src/int8.c:178-209, per token
//
// The bits are those of the GELU epilogue followed by the quantiser kernel (same element function,
// same order of operations; the row maximum does not depend on the order it is taken in), so the
// down projection's input is bit-identical to the two-kernel path while h, fp32 [M][I], never
// reaches memory: HBM sees the int8 activations and the int8 h with its scales.
//
// Layout: a cluster of I / 128 CTAs (9 for I = 1152: a non-portable cluster size) owns 128-row
// blocks; each CTA one 256-row block of the interleaved weight (128 gate + 128 up rows = 128 h
// columns, fixed for the kernel), persistent over the row blocks. Per CTA:
//   warp 0      TMA producer of A [128 x 128] and B [256 x 128] int8 stages (128-byte swizzle);
//   warp 1      MMA issuer into one of two TMEM accumulators of 256 columns;
//   warps 2-17  epilogue: four per TMEM lane quadrant, each owning 32 rows x 32 h columns.
// Per row block: h = gelu(g) u from TMEM, written back over the gate columns; the row's maximum
// |h| over the cluster (the quadrant's 4 warps combine in shared memory, one sends the CTA's value
// to every CTA by st.async, counted on the receiver's mbarrier; two slots alternating by block);
// then h from TMEM -> int8, staged in the 32-byte swizzle and written by TMA. The accumulator is
// released after the second pass, so the tensor core fills the other one meanwhile.
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

constexpr int BM = 128, BN = 256, BK = 128;  // BN weight rows = 128 h columns
constexpr int HC = BN / 2;                   // h columns per CTA
constexpr int STAGES = 3;
constexpr int NACC = 2;
constexpr int EPI_WARPS = 16;
constexpr int NTHREADS = 64 + 32 * EPI_WARPS;
constexpr int QH = HC / 4;                   // h columns per epilogue warp
constexpr int MAXCL = 16;
constexpr int Q8_WARP = 32 * QH;             // 32 rows x 32 int8, 32-byte swizzle
constexpr int C_WU = QH, C_AS = 2 * QH;
constexpr int CST_FLOATS = C_AS + 2 * 32;    // gate and up weight scales; two blocks' activation scales
constexpr float kInv127 = 0x1.020408p-7f;    // fl(1/127)

struct Smem {
    static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE = A_BYTES + B_BYTES;
    static constexpr int Q8_OFF = STAGES * STAGE;
    static constexpr int CST_OFF = Q8_OFF + EPI_WARPS * Q8_WARP;
    static constexpr int XL_OFF = CST_OFF + EPI_WARPS * CST_FLOATS * 4;  // [4 parts][BM]
    static constexpr int XR_OFF = XL_OFF + 4 * BM * 4;                  // [2][MAXCL][BM]
    static constexpr int BAR_OFF = XR_OFF + 2 * MAXCL * BM * 4;
    // full[S], empty[S], tfull[2], tempty[2], lbar[4], xbar[2][4]
    static constexpr int NBAR = 2 * STAGES + 2 * NACC + 4 + 8;
    static constexpr int BYTES = BAR_OFF + NBAR * 8 + 16;
    static constexpr int ALLOC = BYTES + 1024;
    static_assert(Q8_OFF % 1024 == 0, "swizzled TMA tiles");
    static_assert(ALLOC <= 232448, "shared memory");
};

__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm_gelu_quant(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmQ, const e2c_gemm_args p) {
    using L = Smem;
    extern __shared__ uint8_t smem_raw[];
    griddep_launch_dependents();
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + NACC + a); };
    auto lbar = [&](int q) { return bar0 + 8u * (2 * STAGES + 2 * NACC + q); };
    auto xbar = [&](int b, int q) { return bar0 + 8u * (2 * STAGES + 2 * NACC + 4 + 4 * b + q); };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + L::BAR_OFF + L::NBAR * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = p.M, K = p.K;
    const int ncl = (p.n1 - p.n0) / BN;                  // CTAs of a cluster
    const int rank = (int)(blockIdx.x % (unsigned)ncl);  // = cluster rank = weight row block
    const int cid = (int)(blockIdx.x / (unsigned)ncl), ncls = (int)(gridDim.x / (unsigned)ncl);
    const int tiles_m = (M + BM - 1) / BM;
    const int ntl = cid < tiles_m ? (tiles_m - 1 - cid) / ncls + 1 : 0;
    const int nk = (K + BK - 1) / BK;
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
        for (int q = 0; q < 4; q++) {
            mbar_init(lbar(q), 128);
            for (int b = 0; b < 2; b++) mbar_init(xbar(b, q), 1);
        }
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
    cluster_sync();
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
        if (elect_one()) {
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
                const uint32_t drain = tfull_bar(n % NACC);
                mma_commit(drain);
                mbar_wait(drain, (uint32_t)((n / NACC) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const int part = (warp - 2) >> 2;
        const int row = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        const int hc0 = rank * HC + part * QH;  // first h column of this warp
        float *cst = reinterpret_cast<float *>(smem + L::CST_OFF) + (warp - 2) * CST_FLOATS;
        uint8_t *q8s = smem + L::Q8_OFF + (warp - 2) * Q8_WARP;
        {
            // gate row r and up row r + 128 of the CTA's weight block give h column r
            const int wr = p.n0 + rank * BN + part * QH;
            for (int j = lane; j < QH; j += 32) {
                cst[j] = __ldg(p.w_scale + wr + j);
                cst[C_WU + j] = __ldg(p.w_scale + wr + HC + j);
            }
            __syncwarp();
        }
        const uint32_t as_slot = smem_u32(cst + C_AS + lane);
        auto load_as = [&](int n) {
            if (n < ntl) {
                const int mr = row0(n) + row;
                cp_async_4(as_slot + (uint32_t)((n & 1) * 128), p.a_scale + (mr < M ? (size_t)mr : 0), mr < M ? 4u : 0u);
            }
            cp_async_commit();
        };
        float *xl = reinterpret_cast<float *>(smem + L::XL_OFF);
        bool ok = true;
        if (ntl > 0) load_as(0);
        for (int n = 0; n < ntl && ok; n++) {
            const int a = n % NACC;
            const int y0 = row0(n) + q * 32;
            cp_async_wait_all();
            const float as = cst[C_AS + (n & 1) * 32 + lane];
            load_as(n + 1);
            if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(a), (uint32_t)((n / NACC) & 1), p.status, E2C_ERR_WAIT_EPI))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t tg = tmem_base + lane_addr + (uint32_t)(a * BN + part * QH);  // gate columns; up at + HC
            // pass 1: h = gelu(g) u (the GELU epilogue's bits), back over the gate columns; max |h| in
            // four independent partial maxima
            float amp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < QH / 16; c++) {
                uint32_t rg[16], ru[16];
                tmem_ld16(tg + 16 * c, rg);
                tmem_ld16(tg + HC + 16 * c, ru);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    // columns j, j + 1 per packed f32x2 operation (lane for lane the scalar epilogue's
                    // operations: the same bits)
                    const int j = 2 * k;
                    const float2 wg = *reinterpret_cast<const float2 *>(cst + 16 * c + j);
                    const float2 wu = *reinterpret_cast<const float2 *>(cst + C_WU + 16 * c + j);
                    const float2 as2 = make_float2(as, as);
                    const float2 g = mul2_rn(make_float2(__int2float_rn((int)rg[j]), __int2float_rn((int)rg[j + 1])),
                                             mul2_rn(as2, wg));
                    const float2 u = mul2_rn(make_float2(__int2float_rn((int)ru[j]), __int2float_rn((int)ru[j + 1])),
                                             mul2_rn(as2, wu));
                    const float2 h = mul2_rn(gelu_tanh2(g), u);
                    amp[j & 3] = fmaxf(amp[j & 3], fabsf(h.x));
                    amp[(j + 1) & 3] = fmaxf(amp[(j + 1) & 3], fabsf(h.y));
                    rg[j] = __float_as_uint(h.x);
                    rg[j + 1] = __float_as_uint(h.y);
                }
                tmem_st16(tg + 16 * c, rg);
            }
            tmem_wait_st();
            const float amax = fmaxf(fmaxf(amp[0], amp[1]), fmaxf(amp[2], amp[3]));
            // the row's maximum over the cluster
            xl[part * BM + row] = amax;
            mbar_arrive(lbar(q));
            const int b = n & 1;
            if (part == 0) {
                if (!__all_sync(0xffffffffu, mbar_wait(lbar(q), (uint32_t)(n & 1), p.status, E2C_ERR_WAIT_EPI))) {
                    ok = false;
                    break;
                }
                const float cm = fmaxf(fmaxf(xl[row], xl[BM + row]), fmaxf(xl[2 * BM + row], xl[3 * BM + row]));
                const uint32_t xb = xbar(b, q);
                if (lane == 0) mbar_arrive_expect_tx(xb, (uint32_t)(ncl * 32 * 4));
                const uint32_t slot = sbase + L::XR_OFF + (uint32_t)(((b * MAXCL + rank) * BM + row) * 4);
                for (int d = 0; d < ncl; d++) st_async_f32(mapa_shared(slot, (uint32_t)d), cm, mapa_shared(xb, (uint32_t)d));
            }
            if (!__all_sync(0xffffffffu, mbar_wait(xbar(b, q), (uint32_t)((n >> 1) & 1), p.status, E2C_ERR_WAIT_EPI))) {
                ok = false;
                break;
            }
            const float *xr = reinterpret_cast<const float *>(smem + L::XR_OFF) + b * MAXCL * BM + row;
            float rmax = 0.f;
            for (int d = 0; d < ncl; d++) rmax = fmaxf(rmax, xr[d * BM]);
            // pass 2: the quantiser on h from TMEM
            const float inv = rmax > 0.f ? __fdiv_rn(127.0f, rmax) : 1.0f;
            const int m = row0(n) + row;
            if (rank == 0 && part == 0 && m < M) p.q8_scale[m] = rmax > 0.f ? __fmul_rn(rmax, kInv127) : 1.0f;
            if (lane == 0) bulk_wait_read0();  // the previous block's int8 store has read the staging rows
            __syncwarp();
#pragma unroll
            for (int c = 0; c < QH / 16; c++) {
                uint32_t r[16];
                tmem_ld16(tg + 16 * c, r);
                tmem_wait_ld();
                uint32_t pk[4];
#pragma unroll
                for (int k = 0; k < 4; k++)
                    pk[k] = pack_low_bytes(rint_low_byte(__fmul_rn(__uint_as_float(r[4 * k]), inv)),
                                           rint_low_byte(__fmul_rn(__uint_as_float(r[4 * k + 1]), inv)),
                                           rint_low_byte(__fmul_rn(__uint_as_float(r[4 * k + 2]), inv)),
                                           rint_low_byte(__fmul_rn(__uint_as_float(r[4 * k + 3]), inv)));
                *reinterpret_cast<uint4 *>(q8s + lane * 32 + ((c ^ ((lane >> 2) & 1)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(a));
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&tmQ, smem_u32(q8s), hc0, y0);
                bulk_commit();
            }
        }
        cp_async_wait_all();
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }

    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, NACC * BN);
    }
}

E2cPerDev g_max_clusters[MAXCL + 1];  // resident clusters per width, per device (-1: none)

// Per-device set-up and the launch configuration; *maxc_out is the clusters the device holds.
int prepare(int ncl, cudaLaunchConfig_t *cfg, cudaLaunchAttribute *attr, cudaStream_t st, int *maxc_out) {
    using L = Smem;
    static E2cPerDev attr_set;  // the shared-memory and cluster-size opt-ins, per device
    const int dev = e2c_device();
    const int num_sms = e2c_sm_count(dev);
    if (!num_sms) {
        e2c_set_msg("gemm_gelu_quant: no CUDA device");
        return -2;
    }
    if (!attr_set.get(dev)) {
        if (cudaFuncSetAttribute(k_gemm_gelu_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemm_gelu_quant, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
            cudaGetLastError();
            e2c_set_msg("gemm_gelu_quant: cannot reserve %d bytes of shared memory or clusters above 8", L::ALLOC);
            return -2;
        }
        attr_set.set(dev, 1);
    }
    memset(cfg, 0, sizeof *cfg);
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ncl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg->blockDim = dim3(NTHREADS);
    cfg->dynamicSmemBytes = L::ALLOC;
    cfg->stream = st;
    cfg->attrs = attr;
    cfg->numAttrs = 1;
    int maxc = g_max_clusters[ncl].get(dev);
    if (!maxc) {
        cfg->gridDim = dim3((unsigned)(ncl * (num_sms / ncl)));
        if (cudaOccupancyMaxActiveClusters(&maxc, k_gemm_gelu_quant, cfg) != cudaSuccess || maxc <= 0) {
            cudaGetLastError();
            maxc = -1;
        }
        g_max_clusters[ncl].set(dev, maxc);
    }
    if (maxc < 0) {
        e2c_set_msg("gemm_gelu_quant: the device cannot hold a cluster of %d CTAs", ncl);
        return -2;
    }
    *maxc_out = maxc;
    return 0;
}

}  // namespace

// 1 when the fused gate|up + quantiser kernel can run with I = 128 ncl h columns on this device
extern "C" int e2c_gemm_gelu_quant_supported(int ncl) {
    if (ncl < 1 || ncl > MAXCL) return 0;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    int maxc = 0;
    return prepare(ncl, &cfg, attr, 0, &maxc) == 0;
}

// The launch: geometry checked by e2c_gemm (per-row scales, n0 = 0, N = 256 x (1..16)).
extern "C" int e2c_gemm_gelu_quant(const e2c_gemm_args *a, void *stream) {
    const int ncl = (a->n1 - a->n0) / BN;
    if (a->n0 != 0 || (a->n1 - a->n0) % BN || ncl < 1 || ncl > MAXCL) {
        e2c_set_msg("gemm_gelu_quant: gate|up rows in groups of 256 (1..16 groups) from row 0");
        return -1;
    }
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    int maxc = 0;
    const int rc = prepare(ncl, &cfg, attr, (cudaStream_t)stream, &maxc);
    if (rc) return rc;
    CUtensorMap ta, tb, tq;
    if (e2c_tmap_2d(&ta, a->a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->M, (uint64_t)a->lda, BK, BM) ||
        e2c_tmap_2d(&tb, a->w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->wrows, (uint64_t)a->ldw, BK, BN) ||
        e2c_tmap_2d_sw32(&tq, a->q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(HC * ncl), (uint64_t)a->M, (uint64_t)a->ldq,
                         QH, 32))
        return -3;
    const int tiles_m = (a->M + BM - 1) / BM;
    cfg.gridDim = dim3((unsigned)(ncl * (tiles_m < maxc ? tiles_m : maxc)));
    cfg.numAttrs = e2c_pdl_attr(attr, 1);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_gelu_quant, ta, tb, tq, *a);
    if (e != cudaSuccess) {
        e2c_set_msg("gemm_gelu_quant launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}
