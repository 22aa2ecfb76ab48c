// attention_wide.cu — attention for head dim 512 (e2.c's full-attention text layers: head_dim 512,
// one KV head, src/text.c:470-481), bf16 QK^T and PV on the tcgen05 tensor cores.
//
// A 128 x 512 fp32 O accumulator would fill all 512 TMEM columns and leave none for S, so a work
// unit owns half of the value dimensions: unit = (sequence, query head, 128-query tile, value half),
// the two halves of a tile adjacent so their Q and K reads meet in L2. Each unit computes the full
// S = Q K^T over all 512 dimensions and O[:, 256 h .. +255] = P V[:, 256 h .. +255].
//
// Shared memory (one CTA per SM): Q as 8 panels of [128 q][64 d] (128 KB, 128-byte swizzle), K tiles
// of 32 keys as 8 panels of [32 k][64 d] (32 KB, two buffers), V^T tiles [256 d][32 k] (16 KB, rows of
// 64 bytes, 64-byte swizzle, two buffers). TMEM: four S buffers of 32 columns (P written back over
// each as bf16 pairs, the PV product's A operand), O in columns 256..511.
//
// Warps: 0 = TMA for Q and K, 1 = TMA for V^T, 2 = MMA issuer (+TMEM owner), 3..6 = softmax, one per
// TMEM lane quadrant (32 query rows x every key of a tile), 7..10 = epilogue, ctx = O / rowsum stored
// row per lane. The tile order, the S/P/PV barrier sets (four, index g & 3) and the K/V sets (two)
// follow attention.cu; the online softmax is the same (running max moved only when a row's max grows
// by more than 2^8, then its O row is rescaled in TMEM). Masking: keys past the sequence end, keys
// with valid == 0 and, with a window, keys farther than `window` from the query get probability 0;
// query rows with valid == 0 get ctx 0 (src/text.c:639-701).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "devstate.cuh"
#include "launch.h"
#include "pdl.h"
#include "ptx.cuh"
#include "tmap.h"

namespace {

constexpr int HD = 512;   // query/key head dim
constexpr int DV = 256;   // value columns of one unit
constexpr int TQ = 128;   // queries per unit
constexpr int TKV = 32;   // keys per tile
constexpr int SM_WARPS = 4;
constexpr int EP_WARPS = 4;
constexpr int NTHREADS = 96 + 32 * (SM_WARPS + EP_WARPS);
constexpr float kRescaleLog2 = 8.0f;

enum {
    B_Q,
    B_QE,
    B_OE,
    B_KF,
    B_KE = B_KF + 2,
    B_VF = B_KE + 2,
    B_VE = B_VF + 2,
    B_PV = B_VE + 2,
    B_SF = B_PV + 4,
    B_PF = B_SF + 4,
    B_DRAIN = B_PF + 4,
    B_UD,  // [2 unit parities][4 quadrants]
    B_NUM = B_UD + 8
};

constexpr int Q_OFF = 0;
constexpr int K_TILE = TKV * HD * 2;   // 8 panels of TKV x 128 bytes
constexpr int V_TILE = DV * TKV * 2;   // 256 rows of 64 bytes
constexpr int K_OFF = Q_OFF + TQ * HD * 2;
constexpr int V_OFF = K_OFF + 2 * K_TILE;
constexpr int INV_OFF = V_OFF + 2 * V_TILE;  // 1 / rowsum [2 unit parities][128]
constexpr int BAR_OFF = INV_OFF + 2 * TQ * 4;
constexpr int SMEM_BYTES = BAR_OFF + B_NUM * 8 + 16;
static_assert(SMEM_BYTES <= 232448, "shared memory");
static_assert(K_OFF % 1024 == 0 && V_OFF % 1024 == 0 && (TKV * 128) % 1024 == 0 && V_TILE % 512 == 0, "atom alignment");

struct WideArgs {
    const uint8_t *valid;
    float *ctx;
    int S, H, KV, nkt, nqt, units, window;
    float scale_log2;
    int *status;
};

E2C_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct Unit {
    int b, h, qt, half;
};
E2C_DEV Unit unit_of(int u, const WideArgs &p) {
    const int per_seq = p.H * p.nqt * 2;
    const int b = u / per_seq, rem = u - b * per_seq;
    const int h = rem / (p.nqt * 2), r2 = rem - h * (p.nqt * 2);
    return {b, h, r2 >> 1, r2 & 1};
}
E2C_DEV void tile_range(const Unit &w, const WideArgs &p, int &j0, int &nt) {
    if (p.window < 0) {
        j0 = 0;
        nt = p.nkt;
        return;
    }
    const int q0 = w.qt * TQ, q1 = min(q0 + TQ, p.S) - 1;
    const int lo = max(0, q0 - p.window), hi = min(p.S - 1, q1 + p.window);
    j0 = lo / TKV;
    nt = hi / TKV + 1 - j0;
}

__global__ void __launch_bounds__(NTHREADS, 1)
    k_attention_wide(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const WideArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    griddep_launch_dependents();
    if (smem_u32(smem_raw) & 1023) {  // never expected; refuse rather than misplace the swizzled tiles
        griddep_wait();
        if (threadIdx.x == 0) record_status(p.status, E2C_ERR_SMEM_ALIGN);
        return;
    }
    uint8_t *smem = smem_raw;
    const uint32_t sbase = smem_u32(smem);
    auto bar = [&](int i) { return sbase + BAR_OFF + 8u * i; };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + BAR_OFF + B_NUM * 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.S;

    if (warp == 0 && lane == 0) {
        mbar_init(bar(B_Q), 1);
        mbar_init(bar(B_QE), 1);
        mbar_init(bar(B_OE), 32 * EP_WARPS);
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(B_KF + i), 1);
            mbar_init(bar(B_KE + i), 1);
            mbar_init(bar(B_VF + i), 1);
            mbar_init(bar(B_VE + i), 1);
        }
        for (int i = 0; i < 4; i++) {
            mbar_init(bar(B_SF + i), 1);
            mbar_init(bar(B_PV + i), 1);
            mbar_init(bar(B_PF + i), 32 * SM_WARPS);
        }
        mbar_init(bar(B_DRAIN), 1);
        for (int i = 0; i < 8; i++) mbar_init(bar(B_UD + i), 32);
        fence_mbar_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 2) {
        tmem_alloc(sbase + BAR_OFF + B_NUM * 8, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_wait();
    const uint32_t tmem = *tmem_slot;  // S buffer i: cols 32 i .. +31 (i < 4), O: 256..511

    if (warp == 0) {
        // ---------------------------------------------------------------- Q and K loads
        if (elect_one()) {
            int g = 0, nu = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, nu++) {
                const Unit w = unit_of(u, p);
                const int row0 = w.b * S, kvh = w.h / (p.H / p.KV);
                int j0, nt;
                tile_range(w, p, j0, nt);
                if (!mbar_wait(bar(B_QE), (uint32_t)((nu & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) break;
                mbar_arrive_expect_tx(bar(B_Q), TQ * HD * 2);
                for (int i = 0; i < HD / 64; i++)
                    tma_load_2d(sbase + Q_OFF + i * (TQ * 128), &tmQ, w.h * HD + 64 * i, row0 + w.qt * TQ, bar(B_Q));
                for (int j = j0; j < j0 + nt; j++, g++) {
                    const int kb = g & 1;
                    if (!mbar_wait(bar(B_KE + kb), (uint32_t)(((g >> 1) & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(B_KF + kb), K_TILE);
                    for (int i = 0; i < HD / 64; i++)
                        tma_load_2d(sbase + K_OFF + kb * K_TILE + i * (TKV * 128), &tmK, kvh * HD + 64 * i, row0 + j * TKV,
                                    bar(B_KF + kb));
                }
            }
            if (nu > 0) mbar_wait(bar(B_Q), (uint32_t)((nu - 1) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
            for (int i = g - 2 < 0 ? 0 : g - 2; i < g; i++)
                mbar_wait(bar(B_KF + (i & 1)), (uint32_t)((i >> 1) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- V^T loads
        if (elect_one()) {
            int g = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                const Unit w = unit_of(u, p);
                const int vrow = (w.b * p.KV + w.h / (p.H / p.KV)) * HD + w.half * DV;
                int j0, nt;
                tile_range(w, p, j0, nt);
                for (int j = j0; j < j0 + nt; j++, g++) {
                    const int vb = g & 1;
                    if (!mbar_wait(bar(B_VE + vb), (uint32_t)(((g >> 1) & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(B_VF + vb), V_TILE);
                    tma_load_2d(sbase + V_OFF + vb * V_TILE, &tmV, j * TKV, vrow, bar(B_VF + vb));
                }
            }
            for (int i = g - 2 < 0 ? 0 : g - 2; i < g; i++)
                mbar_wait(bar(B_VF + (i & 1)), (uint32_t)((i >> 1) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
        }
    } else if (warp == 2) {
        // ---------------------------------------------------------------- MMA issuer
        // per unit QK0, QK1, then per tile j: QK(j+2), PV(j)
        if (elect_one()) {
            constexpr uint32_t id_s = idesc_bf16(TKV), id_o = idesc_bf16(DV);
            int g0 = 0, nu = 0, nt = 0;
            bool ok = true;
            auto issue_qk = [&](int g, int last) -> bool {
                const int kb = g & 1, s4 = g & 3;
                if (!mbar_wait(bar(B_KF + kb), (uint32_t)((g >> 1) & 1), p.status, E2C_ERR_WAIT_MMA)) return false;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(s4 * TKV);
                const uint32_t kbase = sbase + K_OFF + kb * K_TILE;
#pragma unroll
                for (int k = 0; k < HD / 16; k++) {
                    const uint32_t qoff = (uint32_t)((k >> 2) * (TQ * 128) + (k & 3) * 32);
                    const uint32_t koff = (uint32_t)((k >> 2) * (TKV * 128) + (k & 3) * 32);
                    mma_bf16(d, smem_desc_sw128(sbase + Q_OFF + qoff), smem_desc_sw128(kbase + koff), id_s, k != 0);
                }
                mma_commit(bar(B_SF + s4));
                mma_commit(bar(B_KE + kb));
                if (last) mma_commit(bar(B_QE));
                return true;
            };
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, nu++, g0 += nt) {
                int j0;
                tile_range(unit_of(u, p), p, j0, nt);
                if (!mbar_wait(bar(B_Q), (uint32_t)(nu & 1), p.status, E2C_ERR_WAIT_MMA) || !issue_qk(g0, nt == 1) ||
                    (nt > 1 && !issue_qk(g0 + 1, nt == 2))) {
                    ok = false;
                    break;
                }
                for (int j = 0; j < nt; j++) {
                    const int g = g0 + j, vb = g & 1, s4 = g & 3;
                    if (j + 2 < nt && !(ok = issue_qk(g + 2, j + 2 == nt - 1))) break;
                    if (!mbar_wait(bar(B_PF + s4), (uint32_t)((g >> 2) & 1), p.status, E2C_ERR_WAIT_MMA) ||
                        !mbar_wait(bar(B_VF + vb), (uint32_t)((g >> 1) & 1), p.status, E2C_ERR_WAIT_MMA) ||
                        (j == 0 && !mbar_wait(bar(B_OE), (uint32_t)((nu & 1) ^ 1), p.status, E2C_ERR_WAIT_MMA))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t pa = tmem + (uint32_t)(s4 * TKV);  // P(g): 16 columns of bf16 pairs
                    const uint32_t vbase = sbase + V_OFF + vb * V_TILE;
#pragma unroll
                    for (int k = 0; k < TKV / 16; k++)
                        mma_bf16_ts(tmem + 256, pa + 8 * k, smem_desc_sw64(vbase + (uint32_t)(k * 32)), id_o, (j | k) != 0);
                    mma_commit(bar(B_PV + s4));
                    mma_commit(bar(B_VE + vb));
                }
            }
            if (!ok) {
                mma_commit(bar(B_DRAIN));
                mbar_wait(bar(B_DRAIN), 0, nullptr, E2C_ERR_WAIT_DRAIN);
            }
        }
    } else if (warp < 3 + SM_WARPS) {
        // ---------------------------------------------------------------- softmax
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        float *invs = reinterpret_cast<float *>(smem + INV_OFF);
        bool ok = true;
        int g0 = 0, nu = 0, nt = 0;
        for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, nu++, g0 += nt) {
            const Unit w = unit_of(u, p);
            const int row0 = w.b * S, q0 = w.qt * TQ, qrow = q0 + r, wq0 = q0 + quad * 32;
            const bool row_in = qrow < S;
            int j0;
            tile_range(w, p, j0, nt);
            float m_used = -INFINITY, l = 0.f;
            for (int jj = 0; jj < nt; jj++) {
                const int j = j0 + jj, g = g0 + jj, s4 = g & 3;
                if (!__all_sync(0xffffffffu, mbar_wait(bar(B_SF + s4), (uint32_t)((g >> 2) & 1), p.status, E2C_ERR_WAIT_ATTN))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float s[32];
                {
                    uint32_t rr[32];
                    tmem_ld32(tmem + lane_addr + (uint32_t)(s4 * TKV), rr);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) s[i] = __uint_as_float(rr[i]);
                }
                const int k0 = j * TKV;
                if (p.valid || k0 + TKV > S) {
                    const int key = k0 + lane;
                    const uint32_t keep = __ballot_sync(0xffffffffu, key < S && (!p.valid || p.valid[row0 + key]));
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (!((keep >> i) & 1u)) s[i] = -INFINITY;
                }
                if (p.window >= 0 && (k0 < wq0 + 31 - p.window || k0 + 31 > wq0 + p.window)) {
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (k0 + i < qrow - p.window || k0 + i > qrow + p.window) s[i] = -INFINITY;
                }
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < 32; i++) mx = fmaxf(mx, s[i]);
                mx *= p.scale_log2;
                float alpha = 1.f;
                if (mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx > -INFINITY)) {
                    alpha = m_used == -INFINITY ? 0.f : exp2f(m_used - mx);
                    l *= alpha;
                    m_used = mx;
                }
                if (jj > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                    // O may be touched only once PV of tile g-1 completed (tcgen05.ld/st are warp-collective)
                    if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PV + ((g - 1) & 3)), (uint32_t)(((g - 1) >> 2) & 1),
                                                           p.status, E2C_ERR_WAIT_ATTN))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < DV / 32; c++) {
                        uint32_t o[32];
                        const uint32_t ta = tmem + lane_addr + (uint32_t)(256 + c * 32);
                        tmem_ld32(ta, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(ta, o);
                    }
                    tmem_wait_st();
                }
                const float c = p.scale_log2, mneg = -m_used;
                const bool live = m_used != -INFINITY;
                uint32_t pk[16];
                float lsum = 0.f;
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const float e0 = live ? ex2_approx(__fmaf_rn(s[2 * i], c, mneg)) : 0.f;
                    const float e1 = live ? ex2_approx(__fmaf_rn(s[2 * i + 1], c, mneg)) : 0.f;
                    lsum += e0 + e1;
                    const __nv_bfloat162 hv = __floats2bfloat162_rn(e0, e1);
                    pk[i] = *reinterpret_cast<const uint32_t *>(&hv);
                }
                l += lsum;
                tmem_st16(tmem + lane_addr + (uint32_t)(s4 * TKV), pk);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(bar(B_PF + s4));
            }
            if (!ok) break;
            // 1 / rowsum for the epilogue warp of this quadrant; the slot is written again two units
            // on, after that warp has released O of the unit between (see attention.cu)
            const bool keep = row_in && (!p.valid || p.valid[row0 + qrow]) && l > 0.f;
            invs[(nu & 1) * TQ + r] = keep ? __fdiv_rn(1.0f, l) : 0.f;
            mbar_arrive(bar(B_UD + (nu & 1) * 4 + quad));
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const float *invs = reinterpret_cast<const float *>(smem + INV_OFF);
        bool ok = true;
        int g0 = 0, nu = 0, nt = 0;
        for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, nu++, g0 += nt) {
            const Unit w = unit_of(u, p);
            const int row0 = w.b * S, qrow = w.qt * TQ + r;
            const bool row_in = qrow < S;
            int j0;
            tile_range(w, p, j0, nt);
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_UD + (nu & 1) * 4 + quad), (uint32_t)((nu >> 1) & 1), p.status,
                                                   E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            const float inv = invs[(nu & 1) * TQ + r];
            const int gl = g0 + nt - 1;
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PV + (gl & 3)), (uint32_t)((gl >> 2) & 1), p.status, E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float *out = p.ctx + ((size_t)row0 + qrow) * (size_t)(p.H * HD) + (size_t)w.h * HD + w.half * DV;
#pragma unroll 1
            for (int cp = 0; cp < DV / 32; cp++) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(256 + 32 * cp), o);
                tmem_wait_ld();
                if (cp == DV / 32 - 1) {  // every O column of this quadrant has been read
                    tc_fence_before();
                    mbar_arrive(bar(B_OE));
                }
                if (row_in) {
                    float4 *o4 = reinterpret_cast<float4 *>(out + 32 * cp);
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        o4[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                            __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

extern "C" int e2c_attention_wide(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                                  int B, int S, int H, int KV, float scale, int window, int *status, void *stream) {
    if (B <= 0 || S <= 0) return 0;
    const int dev = e2c_device();
    const int num_sms = e2c_sm_count(dev);
    if (!num_sms) {
        e2c_set_msg("attention_wide: no CUDA device");
        return -2;
    }
    static E2cPerDev attr;
    if (!attr.get(dev)) {
        if (cudaFuncSetAttribute(k_attention_wide, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess) {
            cudaGetLastError();
            e2c_set_msg("attention_wide: cannot reserve %d bytes of shared memory", SMEM_BYTES);
            return -2;
        }
        attr.set(dev, 1);
    }
    CUtensorMap tq, tk, tv;
    const uint64_t rows = (uint64_t)B * S;
    if (e2c_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H * HD, rows, (uint64_t)H * HD * 2, 64, TQ) ||
        e2c_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)KV * HD, rows, (uint64_t)KV * HD * 2, 64, TKV) ||
        e2c_tmap_2d_sw64(&tv, vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)S, (uint64_t)B * KV * HD, (uint64_t)ldvt * 2,
                         TKV, DV))
        return -3;
    WideArgs a;
    a.valid = valid;
    a.ctx = ctx;
    a.S = S;
    a.H = H;
    a.KV = KV;
    a.nkt = (S + TKV - 1) / TKV;
    a.nqt = (S + TQ - 1) / TQ;
    a.units = B * H * a.nqt * 2;
    a.window = window;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.status = status;
    const int grid = a.units < num_sms ? a.units : num_sms;
    e2c_launch(k_attention_wide, dim3(grid), dim3(NTHREADS), SMEM_BYTES, (cudaStream_t)stream, tq, tk, tv, a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        e2c_set_msg("attention_wide launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}
