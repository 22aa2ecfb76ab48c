// gemm_i8_stream.cu — the W8A8 GEMM for short activation matrices (M <= 256 tokens): weight
// streaming over every SM, the weight in the MMA's M slot.
//
// With few tokens the GEMM is a stream of the weight from HBM: N x K bytes against M x K of
// activations. The weight's rows therefore fill the MMA's 128-row A operand and the tokens its B
// operand (N slot = MT, the token count rounded up to 16, 32, 64, 128 or 256):
//     D[n][m] = sum_k W[n][k] X[m][k]          (TMEM lane = weight row, column = token)
// The work is the list of (128-row weight tile j, 128-byte k-block kb) pairs in tile-major order,
// T = ceil(N / 128) x ceil(K / 128) of them, cut into G contiguous ranges of equal length, one per
// CTA (G <= the SM count; stream-K). A CTA accumulates each run of k-blocks of one weight tile in
// TMEM (two accumulators, so the next run's MMAs overlap this run's drain), then:
//   - a run that covers all of K is the output: y[m][n] = clamp(float(acc) * (as[m] * ws[n]))
//     (+ residual), the reference's single-block fold (src/kernels_i8_avx512_vnni.c:113-122,276-307);
//   - a run that covers part of K adds its int32 partials into a zeroed workspace slot with
//     red.global.add and counts its k-blocks on the tile's counter; the CTA whose count completes
//     the tile reads the sums back, writes the output as above and returns the slot and the counter
//     to zero for the next launch. int32 sums are exact in any order, so the output is bit-identical
//     to the other GEMM kernels'.
// No CTA waits on another CTA: the counter decides who finishes a tile, so nothing here depends on
// which CTAs are resident at once.
//
// Workspace: a weight tile is split by at most the G - 1 range boundaries, and the slot of a split
// tile is the index of the first boundary inside it, so G slots of M x 128 int32 plus G counters
// suffice (e2c_gemm_stream_ws_bytes). It must be zero before the first launch; every launch that
// completes leaves it zero. A launch that fails (a bounded wait that gave up) may leave partial sums
// behind: the owner of the workspace clears it before reusing it.
//
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer, 2..5 epilogue (warp w drains TMEM lanes
// 32 (w % 4) .. +31). Every wait is bounded; no TMA load uses multicast.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "devstate.cuh"
#include "launch.h"
#include "pdl.h"
#include "ptx.cuh"
#include "tmap.h"

namespace {

constexpr int BW = 128;  // weight rows per tile (the MMA's M, TMEM lanes)
constexpr int BK = 128;  // K bytes per k-block (one 128-byte swizzle row)
constexpr int NTHREADS = 192;
constexpr int EPI_THREADS = 128;

// CO = 1: a ring short enough (about 110 KB) for two CTAs per SM, so that under programmatic
// dependent launch the next launch's CTAs are resident, and stream their first weight tiles, while
// this launch finishes (short weights at a few tokens, where a launch's fixed costs exceed its
// streaming time)
template <int MT, int CO = 0>
struct StreamSmem {
    static constexpr int W_BYTES = BW * BK;
    static constexpr int X_BYTES = MT * BK;
    static constexpr int STAGE = W_BYTES + X_BYTES;
    // deep rings (180-200 KB in flight per SM): a CTA's whole range of a 4-17 MB weight is requested
    // at once, and a long stream keeps enough bytes in flight to cover HBM latency
    static constexpr int STAGES = CO ? (MT <= 16 ? 6 : MT <= 32 ? 5 : 4)
                                     : MT <= 16 ? 10 : MT <= 32 ? 9 : MT <= 64 ? 8 : MT <= 128 ? 6 : 4;
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int NBAR = 2 * STAGES + 5;  // full[S], empty[S], tfull[2], tempty[2], mma_done
    static constexpr int SLOT_OFF = BAR_OFF + NBAR * 8;  // TMEM address, then the "last" flag
    static constexpr int BYTES = SLOT_OFF + 16;
    static constexpr int ALLOC = BYTES + 1024;  // slack for 1024-byte alignment
    static constexpr uint32_t TMEM_COLS = 2 * MT < 32 ? 32 : 2 * MT;
    static_assert(ALLOC <= (CO ? 232448 / 2 - 1024 : 232448), "shared memory");
    static_assert(STAGE % 1024 == 0, "stages stay 1024-byte aligned");
};

// first CTA range boundary strictly inside weight tile j: the tile's workspace slot (range b
// starts at floor(b T / G))
__device__ __forceinline__ int split_slot(int j, int nk, long long T, int G) {
    const long long lo = (long long)j * nk;
    long long b = ((lo + 1) * G + T - 1) / T;  // smallest b with floor(b T / G) > lo
    if (b < 1) b = 1;
    return (int)b;
}

__device__ __forceinline__ void red_add_s32(int *p, int v) {
    asm volatile("red.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float fold(int acc, float as, float wsn, const e2c_gemm_args &p, bool clamp, int m, int n) {
    float o = __fmul_rn(__int2float_rn(acc), __fmul_rn(as, wsn));
    if (clamp) o = fminf(fmaxf(o, p.out_min), p.out_max);
    if (p.epi == E2C_EPI_RESID) o = __fadd_rn(o, p.resid[(size_t)m * p.ldr + n]);
    return o;
}

template <int MT, int CO>
__global__ void __launch_bounds__(NTHREADS, CO ? 2 : 1)
    k_gemm_stream(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const e2c_gemm_args p) {
    using L = StreamSmem<MT, CO>;
    constexpr int ST = L::STAGES;
    extern __shared__ uint8_t smem_raw[];
    griddep_launch_dependents();
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (ST + s); };
    auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * ST + b); };
    auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * ST + 2 + b); };
    const uint32_t mma_done = bar0 + 8u * (2 * ST + 4);
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + L::SLOT_OFF);
    volatile int *last_flag = reinterpret_cast<volatile int *>(smem + L::SLOT_OFF + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = (int)gridDim.x;
    const int ncols = p.n1 - p.n0;
    const int nt = (ncols + BW - 1) / BW;
    const int nk = (p.K + BK - 1) / BK;
    const long long T = (long long)nt * nk;
    const long long t0 = (long long)blockIdx.x * T / G, t1 = (long long)(blockIdx.x + 1) * T / G;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < ST; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), EPI_THREADS / 32);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
    }
    if (warp == 1) {
        __syncwarp();
        tmem_alloc(sbase + L::SLOT_OFF, L::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (elect_one()) {
            // The weight is never written by the kernels of this stream, so the first stages' weight
            // tiles are requested before griddep_wait: under programmatic dependent launch they
            // stream while the previous kernel finishes. The activations wait for it.
            const long long pre = t1 - t0 < ST ? t1 - t0 : ST;
            for (long long i = 0; i < pre; i++) {
                const long long t = t0 + i;
                const int j = (int)(t / nk), kb = (int)(t % nk);
                mbar_arrive_expect_tx(full_bar((int)i), (uint32_t)L::STAGE);
                tma_load_2d(sbase + (uint32_t)(i * L::STAGE), &tmW, kb * BK, p.n0 + j * BW, full_bar((int)i));
            }
            griddep_wait();
            for (long long i = 0; i < pre; i++) {
                const int kb = (int)((t0 + i) % nk);
                tma_load_2d(sbase + (uint32_t)(i * L::STAGE + L::W_BYTES), &tmX, kb * BK, 0, full_bar((int)i));
            }
            long long issued = pre;
            for (long long i = pre; i < t1 - t0; i++) {
                const long long t = t0 + i;
                const int j = (int)(t / nk), kb = (int)(t % nk);
                const int s = (int)(i % ST);
                if (!mbar_wait(empty_bar(s), (uint32_t)(((i / ST) & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) break;
                const uint32_t sw = sbase + (uint32_t)(s * L::STAGE);
                mbar_arrive_expect_tx(full_bar(s), (uint32_t)L::STAGE);
                tma_load_2d(sw, &tmW, kb * BK, p.n0 + j * BW, full_bar(s));
                tma_load_2d(sw + L::W_BYTES, &tmX, kb * BK, 0, full_bar(s));
                issued = i + 1;
            }
            // no copy may still be landing in this CTA's shared memory when it exits (after a failed
            // wait elsewhere); on the normal path the MMA issuer has waited on each of these already
            for (long long i = issued > ST ? issued - ST : 0; i < issued; i++)
                if (!mbar_wait(full_bar((int)(i % ST)), (uint32_t)((i / ST) & 1), nullptr, E2C_ERR_WAIT_DRAIN)) break;
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_i8(MT, BW);
            long long i = 0;
            int g = 0;
            bool live = true;
            for (long long t = t0; t < t1 && live; g++) {
                const int j = (int)(t / nk);
                const long long tend = (long long)(j + 1) * nk < t1 ? (long long)(j + 1) * nk : t1;
                const int b = g & 1;
                if (!mbar_wait(tempty_bar(b), (uint32_t)(((g >> 1) & 1) ^ 1), p.status, E2C_ERR_WAIT_MMA)) break;
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * MT);
                for (long long u = t; u < tend; u++, i++) {
                    const int s = (int)(i % ST);
                    if (!mbar_wait(full_bar(s), (uint32_t)((i / ST) & 1), p.status, E2C_ERR_WAIT_MMA)) {
                        live = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sw = sbase + (uint32_t)(s * L::STAGE), sx = sw + L::W_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 32; k++)
                        mma_i8(acc, smem_desc_sw128(sw + 32 * k), smem_desc_sw128(sx + 32 * k), idesc,
                               (u != t || k != 0) ? 1u : 0u);
                    mma_commit(empty_bar(s));
                }
                if (!live) break;
                mma_commit(tfull_bar(b));
                t = tend;
            }
            // every MMA issued above completes before the TMEM is released
            mma_commit(mma_done);
            mbar_wait(mma_done, 0, p.status, E2C_ERR_WAIT_DRAIN);
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        griddep_wait();  // the scales, the residual, y and the workspace belong to the stream
        const int q = warp & 3;
        const int r = q * 32 + lane;  // this thread's row of the weight tile
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        const int M = p.M;
        const int nbs = p.K / p.ablk;  // activation scales per row (1: per token)
        const bool clamp = p.out_min > -1e30f || p.out_max < 1e30f;
        const bool leader = warp == 2 && lane == 0;
        int *cnt = p.ws;                        // [G] counters
        int *slots = p.ws + ((G + 31) & ~31);  // [G][M][128] partial sums, 128-byte aligned
        int g = 0;
        for (long long t = t0; t < t1; g++) {
            const int j = (int)(t / nk);
            const long long tend = (long long)(j + 1) * nk < t1 ? (long long)(j + 1) * nk : t1;
            const int kb0 = (int)(t - (long long)j * nk), kb1 = (int)(tend - (long long)j * nk);
            const bool whole = kb0 == 0 && kb1 == nk;
            const int b = g & 1;
            const int n = p.n0 + j * BW + r;
            const bool nok = n < p.n1;
            const float wsn = nok ? __ldg(p.w_scale + n) : 0.f;
            // every epilogue warp takes the same branch (the named barriers below need all four)
            const bool got = __all_sync(0xffffffffu, mbar_wait(tfull_bar(b), (uint32_t)((g >> 1) & 1), p.status,
                                                                E2C_ERR_WAIT_EPI));
            if (!named_barrier_and(1, EPI_THREADS, got)) break;
            tc_fence_after();
            const int slot = whole ? 0 : split_slot(j, nk, T, G);
            int *part = slots + (size_t)slot * M * BW + r;
#pragma unroll 1
            for (int c = 0; c < MT; c += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + lane_addr + (uint32_t)(b * MT + c), v);
                tmem_wait_ld();
                if (c + 16 >= MT) {
                    // the accumulator is read: the MMA may refill it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty_bar(b));
                }
                if (whole) {
                    if (nok) {
                        // the chunk's scales first: loads issued back to back, not one per store
                        float as16[16];
#pragma unroll
                        for (int u = 0; u < 16; u++) as16[u] = c + u < M ? __ldg(p.a_scale + (size_t)(c + u) * nbs) : 0.f;
#pragma unroll
                        for (int u = 0; u < 16; u++) {
                            const int m = c + u;
                            if (m < M) p.y[(size_t)m * p.ldy + n] = fold((int)v[u], as16[u], wsn, p, clamp, m, n);
                        }
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 16; u++)
                        if (c + u < M) red_add_s32(part + (size_t)(c + u) * BW, (int)v[u]);
                }
            }
            if (!whole) {
                // count this run's k-blocks on the tile; the run that completes the count finishes it
                __threadfence();
                named_barrier(1, EPI_THREADS);
                if (leader) {
                    const int before = atomicAdd(cnt + slot, kb1 - kb0);
                    *last_flag = before + (kb1 - kb0) == nk;
                }
                named_barrier(1, EPI_THREADS);
                const bool last = *last_flag != 0;
                named_barrier(1, EPI_THREADS);  // the flag is read before the next run rewrites it
                if (last) {
                    __threadfence();
                    // 16 rows at a time: the sums and scales are loaded back to back before any of
                    // the stores (which could alias them as far as the compiler knows) is issued
#pragma unroll 1
                    for (int m0 = 0; m0 < M; m0 += 16) {
                        int sum[16];
                        float as16[16];
#pragma unroll
                        for (int u = 0; u < 16; u++) {
                            sum[u] = m0 + u < M ? __ldcg(part + (size_t)(m0 + u) * BW) : 0;
                            as16[u] = m0 + u < M ? __ldg(p.a_scale + (size_t)(m0 + u) * nbs) : 0.f;
                        }
#pragma unroll
                        for (int u = 0; u < 16; u++) {
                            const int m = m0 + u;
                            if (m < M) {
                                __stcg(part + (size_t)m * BW, 0);
                                if (nok) p.y[(size_t)m * p.ldy + n] = fold(sum[u], as16[u], wsn, p, clamp, m, n);
                            }
                        }
                    }
                    if (leader) atomicExch(cnt + slot, 0);
                }
            }
            t = tend;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

template <int MT, int CO = 0>
int launch_mt(const e2c_gemm_args *a, int G, cudaStream_t st, int dev) {
    using L = StreamSmem<MT, CO>;
    static E2cPerDev attr_set;
    if (!attr_set.get(dev)) {
        if (cudaFuncSetAttribute(k_gemm_stream<MT, CO>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) != cudaSuccess) {
            cudaGetLastError();
            e2c_set_msg("gemm_stream: cannot reserve %d bytes of shared memory", L::ALLOC);
            return -2;
        }
        attr_set.set(dev, 1);
    }
    CUtensorMap tw, tx;
    if (e2c_tmap_2d(&tw, a->w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->wrows, (uint64_t)a->ldw,
                    BK, BW) ||
        e2c_tmap_2d(&tx, a->a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a->K, (uint64_t)a->M, (uint64_t)a->lda, BK,
                    (uint32_t)MT))
        return -3;
    const cudaError_t e = e2c_launch_as(CO != 0, k_gemm_stream<MT, CO>, dim3((unsigned)G), dim3(NTHREADS), L::ALLOC, st, tw, tx, *a);
    if (e != cudaSuccess) {
        e2c_set_msg("gemm_stream launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}

}  // namespace

// CTAs of a launch over these arguments: every SM, or one per (tile, k-block) when there are fewer
extern "C" int e2c_gemm_stream_ctas(const e2c_gemm_args *a, int num_sms) {
    const long long T = (long long)((a->n1 - a->n0 + BW - 1) / BW) * ((a->K + BK - 1) / BK);
    return (int)(T < num_sms ? T : num_sms);
}

extern "C" size_t e2c_gemm_stream_ws_bytes(int M, int num_sms) {
    const size_t g = (size_t)((num_sms + 31) & ~31);
    return 4 * (g + (size_t)num_sms * (size_t)M * BW);
}

extern "C" int e2c_gemm_stream(const e2c_gemm_args *a, void *stream) {
    const int dev = e2c_device();
    const int num_sms = e2c_sm_count(dev);
    if (!num_sms) {
        e2c_set_msg("gemm_stream: no CUDA device");
        return -2;
    }
    if (a->ablk != a->K || (a->epi != E2C_EPI_F32 && a->epi != E2C_EPI_RESID) || a->M < 1 || a->M > 256 || !a->ws ||
        a->ws_bytes < e2c_gemm_stream_ws_bytes(a->M, num_sms) || ((uintptr_t)a->ws & 127) || a->K % 16 ||
        a->lda % 16 || a->ldw % 16 || (((uintptr_t)a->a | (uintptr_t)a->w) & 15) || a->n0 < 0 || a->n1 > a->wrows ||
        a->n0 >= a->n1) {
        e2c_set_msg("gemm_stream: per-row scales, the F32 or residual epilogue, 1..256 rows, 16-byte aligned operands "
                    "and a zeroed, 128-byte aligned workspace of e2c_gemm_stream_ws_bytes");
        return -1;
    }
    const int G = e2c_gemm_stream_ctas(a, num_sms);
    cudaStream_t st = (cudaStream_t)stream;
    // under programmatic dependent launch, short weights at a few tokens take the co-resident ring
    const long long T = (long long)((a->n1 - a->n0 + BW - 1) / BW) * ((a->K + BK - 1) / BK);
    if (e2c_pdl_small_on() && a->M <= 32 && T < 8LL * num_sms)
        return a->M <= 16 ? launch_mt<16, 1>(a, G, st, dev) : launch_mt<32, 1>(a, G, st, dev);
    if (a->M <= 16) return launch_mt<16>(a, G, st, dev);
    if (a->M <= 32) return launch_mt<32>(a, G, st, dev);
    if (a->M <= 64) return launch_mt<64>(a, G, st, dev);
    if (a->M <= 128) return launch_mt<128>(a, G, st, dev);
    return launch_mt<256>(a, G, st, dev);
}
