// gemm_i8_splitk.cu — the W8A8 GEMM for short activation matrices: K split over a thread-block
// cluster, partial products reduced through distributed shared memory.
//
// With few output tiles (a handful of tokens against a weight of a few thousand rows) the
// persistent kernel leaves most SMs idle and the weight streams from HBM at a fraction of its
// bandwidth. Here a cluster of S CTAs (S = 2 .. 16) shares one 128 x BN output tile (BN = 128 or
// 256): CTA r of the cluster streams k-blocks [r kpc, (r + 1) kpc) of the tile's weight rows and
// accumulates them in TMEM with tcgen05.mma kind::i8. Stages are packed: the A part of a stage holds
// only the activation rows that exist (16 rows: 2 KB), so up to 16 stages are in flight per SM.
// The int32 partials go to the CTA's shared memory; after a cluster barrier CTA r sums columns
// [r BN/S, (r + 1) BN/S) of the tile over the S partials (ld.shared::cluster) and writes
//     y[m, n] = clamp(float(sum) * (as[m] * ws[n])) (+ residual)
// — per-row activation scales only, the reference's single-block fold
// (src/kernels_i8_avx512_vnni.c:113-122,276-307): int32 sums are exact in any order, so the output
// is bit-identical to the persistent kernel's.
//
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer, 2..5 TMEM -> shared partials and the reduction.
// Every wait is bounded; no TMA load uses multicast.
//
// The co-resident variant (CO, up to 32 rows, BN 128) keeps its stages in under half of an SM's
// shared memory and is launched with at most one CTA per SM, so under programmatic dependent launch
// the next GEMM's CTAs become resident beside this one's. Its producer requests the first stages'
// weight tiles before griddepcontrol.wait (the weight is never written by the stream's kernels):
// they stream while the previous kernel finishes; the activation tiles, the scales and the output
// wait for it.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "launch.h"
#include "devstate.cuh"
#include "pdl.h"
#include "ptx.cuh"
#include "tmap.h"

namespace {

constexpr int BM = 128, BK = 128;
constexpr int MAXST = 16;
constexpr int NTHREADS = 192;
// shared memory: a pool for the stages (and, once the MMAs are done, the partials), then barriers.
// The MMA reads 128 rows of A from a stage's A base; past the rows a packed stage holds it reads
// whatever follows (never used), so the pool keeps 16 KB of slack past the last stage.
constexpr int POOL_1 = 200 * 1024, POOL_CO = 108 * 1024;
constexpr int CO_ROWS = 32;  // rows the co-resident variant takes (its partials: CO_ROWS x BN int32)
constexpr int A_FULL = BM * BK;
constexpr int NBAR = 2 * MAXST + 1;  // full[MAXST], empty[MAXST], tfull; then the TMEM address slot
__host__ __device__ constexpr int pool_of(bool co) { return co ? POOL_CO : POOL_1; }
__host__ __device__ constexpr int smem_alloc(bool co) { return pool_of(co) + NBAR * 8 + 16 + 1024; }

E2C_DEV uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
E2C_DEV int4 ld_dsmem_v4(uint32_t cluster_addr) {
    int4 v;
    asm volatile("ld.shared::cluster.v4.s32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(cluster_addr)
                 : "memory");
    return v;
}
// The partials, [rows][BN / 4 chunks of 4 int32], at the pool's start. Chunk c of row r sits at
// chunk c ^ (r & 7): the lanes of a warp (consecutive rows) store to distinct bank groups.
template <int BN>
E2C_DEV uint32_t red_off(int row, int chunk) {
    return (uint32_t)(row * (BN * 4) + ((chunk ^ (row & 7)) << 4));
}

// stages that fit for a packed stage of `stage_bytes`
__host__ __device__ constexpr int stages_for(int stage_bytes, bool co) {
    return (pool_of(co) - A_FULL) / stage_bytes < MAXST ? (pool_of(co) - A_FULL) / stage_bytes : MAXST;
}

template <int BN, bool CO>
__global__ void __launch_bounds__(NTHREADS, CO ? 2 : 1)
    k_gemm_splitk(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const e2c_gemm_args p, const int a_rows) {
    constexpr int POOL = pool_of(CO), BAR_OFF = POOL;
    static_assert((CO ? CO_ROWS : BM) * BN * 4 <= POOL, "partials fit in the pool");
    extern __shared__ uint8_t smem_raw[];
    griddep_launch_dependents();
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (MAXST + s); };
    const uint32_t tfull = bar0 + 8u * (2 * MAXST);
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + BAR_OFF + NBAR * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = (int)cluster_nctarank(), rank = (int)cluster_ctarank();
    const int tile = blockIdx.x / S;
    const int ncols = p.n1 - p.n0;
    const int tiles_n = (ncols + BN - 1) / BN;
    const int mt = (tile / tiles_n) * BM, c0 = p.n0 + (tile % tiles_n) * BN;
    const int nk = (p.K + BK - 1) / BK;
    const int kpc = (nk + S - 1) / S;
    const int kb0 = rank * kpc, kb1 = min(nk, kb0 + kpc);
    const int nkb = kb1 > kb0 ? kb1 - kb0 : 0;  // k-blocks of this CTA (the last rank may have none)
    const int a_bytes = a_rows * BK;            // a multiple of 1024: a_rows is a multiple of 8
    const int stage_bytes = a_bytes + BN * BK;
    const int nst = stages_for(stage_bytes, CO);

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < MAXST; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(tfull, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        __syncwarp();
        tmem_alloc(sbase + BAR_OFF + NBAR * 8, BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // the stream's earlier kernels are done with what this one reads and writes (co-resident: each
    // role waits where it first touches the stream's data)
    if constexpr (!CO) griddep_wait();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (elect_one()) {
            int i0 = 0;
            if constexpr (CO) {
                // the first stages' weight tiles before the wait, their activation tiles after it
                const int pre = nkb < nst ? nkb : nst;
                for (int i = 0; i < pre; i++) {
                    const uint32_t sa = sbase + i * stage_bytes, sb = sa + a_bytes;
                    mbar_arrive_expect_tx(full_bar(i), (uint32_t)stage_bytes);
                    tma_load_2d(sb, &tmB, (kb0 + i) * BK, c0, full_bar(i));
                }
                griddep_wait();
                for (int i = 0; i < pre; i++)
                    tma_load_2d(sbase + i * stage_bytes, &tmA, (kb0 + i) * BK, mt, full_bar(i));
                i0 = pre;
            }
            for (int i = i0; i < nkb; i++) {
                const int s = i % nst;
                const uint32_t par = (uint32_t)((i / nst) & 1);
                if (!mbar_wait(empty_bar(s), par ^ 1u, p.status, E2C_ERR_WAIT_PRODUCER)) break;
                const uint32_t sa = sbase + s * stage_bytes, sb = sa + a_bytes;
                mbar_arrive_expect_tx(full_bar(s), (uint32_t)stage_bytes);
                tma_load_2d(sa, &tmA, (kb0 + i) * BK, mt, full_bar(s));
                tma_load_2d(sb, &tmB, (kb0 + i) * BK, c0, full_bar(s));
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_i8(BN);
            for (int i = 0; i < nkb; i++) {
                const int s = i % nst;
                if (!mbar_wait(full_bar(s), (uint32_t)((i / nst) & 1), p.status, E2C_ERR_WAIT_MMA)) break;
                tc_fence_after();
                const uint32_t sa = sbase + s * stage_bytes, sb = sa + a_bytes;
#pragma unroll
                for (int k = 0; k < BK / 32; k++)
                    mma_i8(tmem, smem_desc_sw128(sa + 32 * k), smem_desc_sw128(sb + 32 * k), idesc, (i | k) != 0);
                mma_commit(empty_bar(s));
            }
            // tfull completes once every MMA issued above has (none: at once)
            mma_commit(tfull);
        }
    } else {
        // ---------------------------------------------------------------- TMEM -> shared partials
        if constexpr (CO) griddep_wait();  // (the reduction reads the scales and writes y)
        const int q = warp & 3;
        const int row = q * 32 + lane;
        if (mt + q * 32 < p.M) {  // warp-uniform: this quadrant holds rows of the output
            if (!__all_sync(0xffffffffu, mbar_wait(tfull, 0, p.status, E2C_ERR_WAIT_EPI))) {
                ok = false;
            } else {
                tc_fence_after();
                const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(tmem + lane_addr + (uint32_t)c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int4 v = nkb ? make_int4((int)r[4 * j], (int)r[4 * j + 1], (int)r[4 * j + 2], (int)r[4 * j + 3])
                                           : make_int4(0, 0, 0, 0);
                        *reinterpret_cast<int4 *>(smem + red_off<BN>(row, c / 4 + j)) = v;
                    }
                }
            }
        }
    }
    // every CTA's partials are in its shared memory
    tc_fence_before();
    cluster_sync();

    if (warp >= 2 && ok) {
        // ---------------------------------------------------------------- reduction over the cluster
        // CTA r owns chunks [r ch, (r + 1) ch) of every row: 4 columns per thread and step, summed
        // over the S partials with 16-byte loads from each CTA's shared memory
        const int tid = threadIdx.x - 64;
        const int ch = BN / 4 / S, cbase = rank * ch;
        const int mv = min(BM, p.M - mt);
        const bool clamp = p.out_min > -1e30f || p.out_max < 1e30f;
        const bool vec = (p.ldy % 4 == 0) && (p.n0 % 4 == 0) && (((uintptr_t)p.y & 15) == 0) && p.epi == E2C_EPI_F32;
        uint32_t peer[16];
#pragma unroll
        for (int s = 0; s < 16; s++)
            if (s < S) peer[s] = mapa_shared(sbase, (uint32_t)s);
        for (int idx = tid; idx < ch * mv; idx += 128) {
            const int m = idx / ch, cc = cbase + idx % ch;
            const int n = c0 + 4 * cc;
            if (n >= p.n1) continue;
            const uint32_t off = red_off<BN>(m, cc);
            int4 acc = make_int4(0, 0, 0, 0);
#pragma unroll
            for (int s = 0; s < 16; s++) {
                if (s < S) {
                    const int4 v = ld_dsmem_v4(peer[s] + off);
                    acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
                }
            }
            const int gm = mt + m;
            const float as = __ldg(p.a_scale + (size_t)gm * (p.K / p.ablk));
            const int sums[4] = {acc.x, acc.y, acc.z, acc.w};
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int nj = n + j < p.n1 ? n + j : n;
                v[j] = __fmul_rn(__int2float_rn(sums[j]), __fmul_rn(as, __ldg(p.w_scale + nj)));
                if (clamp) v[j] = fminf(fmaxf(v[j], p.out_min), p.out_max);
            }
            float *yr = p.y + (size_t)gm * p.ldy + n;
            if (vec && n + 4 <= p.n1) {
                *reinterpret_cast<float4 *>(yr) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
                for (int j = 0; j < 4 && n + j < p.n1; j++) {
                    float o = v[j];
                    if (p.epi == E2C_EPI_RESID) o = __fadd_rn(o, p.resid[(size_t)gm * p.ldr + n + j]);
                    yr[j] = o;
                }
            }
        }
    }
    // no CTA leaves while the others may still read its partials
    cluster_sync();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

// the shared-memory and cluster-size opt-ins on the current device: 0 unset, 1 ok, -1 failed
template <int BN, bool CO>
bool configure() {
    static E2cPerDev state;
    const int dev = e2c_device();
    if (dev < 0) return false;
    int s = state.get(dev);
    if (!s) {
        s = (cudaFuncSetAttribute(k_gemm_splitk<BN, CO>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_alloc(CO)) ==
                 cudaSuccess &&
             cudaFuncSetAttribute(k_gemm_splitk<BN, CO>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess)
                ? 1
                : -1;
        if (s < 0) cudaGetLastError();
        state.set(dev, s);
    }
    return s > 0;
}

// clusters of S CTAs the current device holds at once (0: none), per device and S
template <int BN, bool CO>
int clusters(int S) {
    static E2cPerDev cache[5];  // value + 1; 0 = not yet asked
    int i = 0;
    while ((2 << i) < S && i < 4) i++;
    if (S < 2 || S > 16 || (2 << i) != S || !configure<BN, CO>()) return 0;
    const int dev = e2c_device();
    const int c = cache[i].get(dev);
    if (c > 0) return c - 1;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)S;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)S);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem_alloc(CO);
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_gemm_splitk<BN, CO>, &cfg) != cudaSuccess || n < 0) {
        cudaGetLastError();
        n = 0;
    }
    cache[i].set(dev, n + 1);
    return n;
}

template <int BN, bool CO>
int launch_bn(const e2c_gemm_args *a, int S, cudaStream_t st) {
    if (!configure<BN, CO>()) {
        e2c_set_msg("gemm_splitk: cannot configure the kernel (%d bytes of shared memory, clusters of 16)", smem_alloc(CO));
        return -2;
    }
    // A: as many rows as the output tile has (rounded up to 8); the MMA's other rows are never read
    const int a_rows = a->M >= BM ? BM : (a->M + 7) / 8 * 8;
    CUtensorMap ta, tb;
    if (e2c_tmap_2d(&ta, a->a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->M, (uint64_t)a->lda, BK,
                    (uint32_t)a_rows) ||
        e2c_tmap_2d(&tb, a->w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->wrows, (uint64_t)a->ldw, BK,
                    BN))
        return -3;
    const int tiles = ((a->M + BM - 1) / BM) * ((a->n1 - a->n0 + BN - 1) / BN);
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr_c[2];
    attr_c[0].id = cudaLaunchAttributeClusterDimension;
    attr_c[0].val.clusterDim.x = (unsigned)S;
    attr_c[0].val.clusterDim.y = 1;
    attr_c[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(tiles * S));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem_alloc(CO);
    cfg.stream = st;
    cfg.attrs = attr_c;
    cfg.numAttrs = e2c_pdl_attr(attr_c, 1, CO);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_splitk<BN, CO>, ta, tb, *a, a_rows);
    if (e != cudaSuccess) {
        e2c_set_msg("gemm_splitk launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}

}  // namespace

extern "C" int e2c_gemm_splitk_plan(const e2c_gemm_args *a, int num_sms, int *bn, int *S) {
    *bn = 0;
    *S = 1;
    if (a->ablk != a->K || (a->epi != E2C_EPI_F32 && a->epi != E2C_EPI_RESID) || a->M > 2 * BM) return 0;
    const int nk = (a->K + BK - 1) / BK;
    const long mtiles = (a->M + BM - 1) / BM;
    int best = 0;
    for (int w : {256, 128}) {
        const long tiles = mtiles * ((a->n1 - a->n0 + w - 1) / w);
        for (int s2 = 2; s2 <= 16 && s2 <= nk && tiles * s2 <= num_sms; s2 *= 2) {
            const int c = w == 256 ? clusters<256, false>(s2) : clusters<128, false>(s2);
            if (c >= tiles && tiles * s2 > best) {
                best = (int)(tiles * s2);
                *bn = w;
                *S = s2;
            }
        }
    }
    return best;
}

extern "C" int e2c_gemm_splitk(const e2c_gemm_args *a, int bn, int S, void *stream) {
    if (a->ablk != a->K || (a->epi != E2C_EPI_F32 && a->epi != E2C_EPI_RESID) || S < 2 || S > 16 || (S & (S - 1)) ||
        (bn != 128 && bn != 256)) {
        e2c_set_msg("gemm_splitk: per-row scales, the F32 or residual epilogue, BN 128 or 256, a cluster of 2..16");
        return -1;
    }
    return bn == 256 ? launch_bn<256, false>(a, S, (cudaStream_t)stream) : launch_bn<128, false>(a, S, (cudaStream_t)stream);
}

// The co-resident variant for up to 32 rows: BN 128, the widest power-of-two split with one CTA per
// SM at most and every cluster resident at once. Returns -1 (nothing launched) where it does not
// apply.
extern "C" int e2c_gemm_splitk_co(const e2c_gemm_args *a, void *stream) {
    if (a->ablk != a->K || (a->epi != E2C_EPI_F32 && a->epi != E2C_EPI_RESID) || a->M < 1 || a->M > CO_ROWS) return -1;
    const int dev = e2c_device();
    const int num_sms = e2c_sm_count(dev);
    const int nk = (a->K + BK - 1) / BK;
    const long tiles = (a->n1 - a->n0 + 127) / 128;
    int best = 0;
    for (int s2 = 2; s2 <= 16 && s2 <= nk && tiles * s2 <= num_sms; s2 *= 2)
        if (clusters<128, true>(s2) >= tiles) best = s2;
    if (!best) return -1;
    return launch_bn<128, true>(a, best, (cudaStream_t)stream);
}
