// attention.cu — bidirectional GQA attention on the sm_100a tensor cores (tcgen05.mma kind::f16).
//
// One CTA per (sequence, query head, 128-query tile). Keys are swept in tiles of 64, K and V^T
// double-buffered in shared memory so the next tile's loads overlap the current tile's products.
// Per key tile j:
//   S_j = Q K_j^T        bf16 x bf16 -> fp32 in TMEM (two S buffers, so QK of tile j+1 overlaps the
//                        softmax of tile j)
//   P_j = exp2(S_j * scale * log2e - m)   online softmax in registers; the running max m moves only
//                        when a row's max grows by more than 2^8 (then its O row is rescaled in
//                        TMEM). P is written back as bf16 into the S buffer it came from, and the PV
//                        product reads its A operand from tensor memory.
//   O  += P_j V_j        fp32 accumulator in TMEM (256 columns)
// and at the end ctx = O / rowsum in fp32. Keys past the sequence end or with valid == 0 get
// probability 0; query rows with valid == 0 get ctx 0 (the reference's masking, src/text.c:661-701).
//
// Operands: Q [B*S][H*256] and K [B*S][256] bf16 row-major (head dim contiguous, K-major for QK^T),
// V^T [B][256][ldvt] bf16 (keys contiguous, K-major for PV) — the QKV GEMM epilogue writes them so.
//
// Warps: 0 = TMA for Q and K, 1 = TMA for V^T, 2 = MMA issuer (+TMEM owner), 3..10 = softmax,
// rescale and epilogue: warp w owns TMEM lanes 32*(w%4) .. +31 and, with its partner of the same
// quadrant, half of every key tile (keys 32*kh .. +31) and half of the output columns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "launch.h"
#include "ptx.cuh"
#include "tmap.h"

namespace {

constexpr int HD = 256;        // head dim
constexpr int TQ = 128;        // queries per CTA
constexpr int TKV = 64;        // keys per tile
constexpr int SM_WARPS = 8;    // softmax warps
constexpr int NTHREADS = 96 + 32 * SM_WARPS;
constexpr float kRescaleLog2 = 8.0f;

// shared memory map (bytes, from a 1024-aligned base)
constexpr int Q_OFF = 0;                           // 4 x [128 q][64 d]   (16 KB each)
constexpr int K_TILE = TKV * HD * 2;               // 4 x [64 k][64 d]    (8 KB each)
constexpr int V_TILE = HD * TKV * 2;               // [256 d][64 k]       (32 KB)
constexpr int K_OFF = Q_OFF + TQ * HD * 2;         // 2 buffers
constexpr int V_OFF = K_OFF + 2 * K_TILE;          // 2 buffers
constexpr int X_OFF = V_OFF + 2 * V_TILE;          // row-max / row-sum exchange [2][2][128] floats
constexpr int BAR_OFF = X_OFF + 2 * 2 * TQ * 4;
// Q, K full x2, K empty x2, V full x2, V empty x2, PV done x2, S full x2, P full x2, pair [2][4],
// final [4], drain. Every per-tile barrier comes in two, indexed by tile parity: a waiter may then
// trail the arriving side by up to one tile without two phases completing under it.
enum {
    B_Q,
    B_KF,
    B_KE = B_KF + 2,
    B_VF = B_KE + 2,
    B_VE = B_VF + 2,
    B_PV = B_VE + 2,
    B_SF = B_PV + 2,
    B_PF = B_SF + 2,
    B_PAIR = B_PF + 2,
    B_FIN = B_PAIR + 8,
    B_DRAIN = B_FIN + 4,
    B_NUM
};
constexpr int SMEM_BYTES = BAR_OFF + B_NUM * 8 + 16;
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;

struct AttnArgs {
    const uint8_t *valid;
    float *ctx;
    int S, H, nkt;
    float scale_log2;
    int *status;
};

E2C_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(NTHREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const AttnArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    auto bar = [&](int i) { return sbase + BAR_OFF + 8u * i; };
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + BAR_OFF + B_NUM * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int S = p.S, nkt = p.nkt;
    const int q0 = qt * TQ;
    const int row0 = b * S;  // first token row of this sequence

    if (warp == 0 && lane == 0) {
        mbar_init(bar(B_Q), 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(B_KF + i), 1);
            mbar_init(bar(B_KE + i), 1);
            mbar_init(bar(B_VF + i), 1);
            mbar_init(bar(B_VE + i), 1);
            mbar_init(bar(B_SF + i), 1);
            mbar_init(bar(B_PV + i), 1);
            mbar_init(bar(B_PF + i), 32 * SM_WARPS);
        }
        mbar_init(bar(B_DRAIN), 1);
        for (int i = 0; i < 8; i++) mbar_init(bar(B_PAIR + i), 64);
        for (int i = 0; i < 4; i++) mbar_init(bar(B_FIN + i), 64);
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
    const uint32_t tmem = *tmem_slot;  // S0: cols 0..63, S1: 64..127, O: 256..511

    if (warp == 0) {
        // ---------------------------------------------------------------- Q and K loads
        if (elect_one()) {
            mbar_arrive_expect_tx(bar(B_Q), TQ * HD * 2);
            for (int i = 0; i < 4; i++)
                tma_load_2d(sbase + Q_OFF + i * (TQ * 128), &tmQ, h * HD + 64 * i, row0 + q0, bar(B_Q));
            int issued = 0;
            for (int j = 0; j < nkt; j++) {
                const int kb = j & 1;
                // buffer kb is free once QK of tile j-2 completed
                if (!mbar_wait(bar(B_KE + kb), (uint32_t)(((j >> 1) & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) break;
                mbar_arrive_expect_tx(bar(B_KF + kb), K_TILE);
                for (int i = 0; i < 4; i++)
                    tma_load_2d(sbase + K_OFF + kb * K_TILE + i * (TKV * 128), &tmK, 64 * i, row0 + j * TKV, bar(B_KF + kb));
                issued = j + 1;
            }
            // the last loads (and Q) must have landed before the CTA may exit
            mbar_wait(bar(B_Q), 0, nullptr, E2C_ERR_WAIT_DRAIN);
            for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; j++)
                mbar_wait(bar(B_KF + (j & 1)), (uint32_t)((j >> 1) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- V^T loads
        if (elect_one()) {
            int issued = 0;
            for (int j = 0; j < nkt; j++) {
                const int vb = j & 1;
                // buffer vb is free once PV of tile j-2 completed
                if (!mbar_wait(bar(B_VE + vb), (uint32_t)(((j >> 1) & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) break;
                mbar_arrive_expect_tx(bar(B_VF + vb), V_TILE);
                tma_load_2d(sbase + V_OFF + vb * V_TILE, &tmV, j * TKV, b * HD, bar(B_VF + vb));
                issued = j + 1;
            }
            for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; j++)
                mbar_wait(bar(B_VF + (j & 1)), (uint32_t)((j >> 1) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
        }
    } else if (warp == 2) {
        // ---------------------------------------------------------------- MMA issuer
        // Issue order QK0, QK1, PV0, QK2, PV1, QK3, ...: tcgen05.mma from one thread runs in order,
        // so QK(j+2) overwrites S buffer j%2 only after PV(j) has read P(j) out of it.
        if (elect_one()) {
            constexpr uint32_t id_s = idesc_bf16(TKV), id_o = idesc_bf16(HD);
            bool ok = mbar_wait(bar(B_Q), 0, p.status, E2C_ERR_WAIT_MMA);
            auto issue_qk = [&](int j) -> bool {
                const int sb = j & 1;
                if (!mbar_wait(bar(B_KF + sb), (uint32_t)((j >> 1) & 1), p.status, E2C_ERR_WAIT_MMA)) return false;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(sb * TKV);
                const uint32_t kbase = sbase + K_OFF + sb * K_TILE;
#pragma unroll
                for (int k = 0; k < HD / 16; k++) {
                    const uint32_t qoff = (uint32_t)((k >> 2) * (TQ * 128) + (k & 3) * 32);
                    const uint32_t koff = (uint32_t)((k >> 2) * (TKV * 128) + (k & 3) * 32);
                    mma_bf16(d, smem_desc_sw128(sbase + Q_OFF + qoff), smem_desc_sw128(kbase + koff), id_s, k != 0);
                }
                mma_commit(bar(B_SF + sb));
                mma_commit(bar(B_KE + sb));
                return true;
            };
            if (ok) ok = issue_qk(0);
            if (ok && nkt > 1) ok = issue_qk(1);
            for (int j = 0; j < nkt && ok; j++) {
                const int sb = j & 1;
                if (!mbar_wait(bar(B_PF + sb), (uint32_t)((j >> 1) & 1), p.status, E2C_ERR_WAIT_MMA) ||
                    !mbar_wait(bar(B_VF + sb), (uint32_t)((j >> 1) & 1), p.status, E2C_ERR_WAIT_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t pa = tmem + (uint32_t)(sb * TKV);  // P(j): 32 columns of bf16 pairs
                const uint32_t vbase = sbase + V_OFF + sb * V_TILE;
#pragma unroll
                for (int k = 0; k < TKV / 16; k++)
                    mma_bf16_ts(tmem + 256, pa + 8 * k, smem_desc_sw128(vbase + (uint32_t)(k * 32)), id_o, (j | k) != 0);
                mma_commit(bar(B_PV + sb));
                mma_commit(bar(B_VE + sb));
                if (j + 2 < nkt && !(ok = issue_qk(j + 2))) break;
            }
            if (!ok) {
                // drain whatever was issued before TMEM is released
                mma_commit(bar(B_DRAIN));
                mbar_wait(bar(B_DRAIN), 0, nullptr, E2C_ERR_WAIT_DRAIN);
            }
        }
    } else {
        // ---------------------------------------------------------------- softmax / epilogue
        const int quad = warp & 3;
        const int kh = (warp - 3) >> 2;   // key half of every tile (and output-column half) this warp owns
        const int r = quad * 32 + lane;   // query row within the tile = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int qrow = q0 + r;
        const bool row_in = qrow < S;
        float *xch = reinterpret_cast<float *>(smem + X_OFF);  // [2][2][TQ]
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkt; j++) {
            const int sb = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_SF + sb), (uint32_t)((j >> 1) & 1), p.status, E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float s[32];
            {
                uint32_t rr[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(sb * TKV + 32 * kh), rr);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++) s[i] = __uint_as_float(rr[i]);
            }
            // masking only where a tile runs past the sequence or a valid mask is given
            const int k0 = j * TKV + 32 * kh;
            if (p.valid || k0 + 32 > S) {
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int key = k0 + i;
                    if (!(key < S && (!p.valid || p.valid[row0 + key]))) s[i] = -INFINITY;
                }
            }
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; i++) mx = fmaxf(mx, s[i]);
            // the row max over both key halves, through the partner warp
            xch[(sb * 2 + kh) * TQ + r] = mx;
            mbar_arrive(bar(B_PAIR + sb * 4 + quad));
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PAIR + sb * 4 + quad), (uint32_t)((j >> 1) & 1), p.status,
                                                   E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            mx = fmaxf(xch[(sb * 2) * TQ + r], xch[(sb * 2 + 1) * TQ + r]) * p.scale_log2;
            // Each row decides whether its running max moves; the O rescale is a warp-collective TMEM
            // round trip (tcgen05.ld/st are .sync.aligned), run when any row of the warp needs it.
            float alpha = 1.f;
            if (mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx > -INFINITY)) {
                alpha = m_used == -INFINITY ? 0.f : exp2f(m_used - mx);
                l *= alpha;
                m_used = mx;
            }
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                // O may be touched only once PV of tile j-1 completed
                if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PV + ((j - 1) & 1)), (uint32_t)(((j - 1) >> 1) & 1), p.status,
                                                       E2C_ERR_WAIT_ATTN))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < 4; c++) {
                    uint32_t o[32];
                    const uint32_t ta = tmem + lane_addr + (uint32_t)(256 + 128 * kh + c * 32);
                    tmem_ld32(ta, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(ta, o);
                }
                tmem_wait_st();
            }
            // probabilities -> bf16 pairs over this warp's S columns: P(j) occupies columns
            // [16 kh, 16 kh + 16) of the buffer (both halves already read S, through the exchange)
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
            {
                const uint32_t ta = tmem + lane_addr + (uint32_t)(sb * TKV + 16 * kh);
                asm volatile(
                    "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                    "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(ta),
                    "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3]), "r"(pk[4]), "r"(pk[5]), "r"(pk[6]), "r"(pk[7]),
                    "r"(pk[8]), "r"(pk[9]), "r"(pk[10]), "r"(pk[11]), "r"(pk[12]), "r"(pk[13]), "r"(pk[14]), "r"(pk[15])
                    : "memory");
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(B_PF + sb));
        }
        // ---------------------------------------------------------------- epilogue
        // PV of the last tile completes after every earlier product (tcgen05.commit tracks all prior MMAs)
        if (ok && __all_sync(0xffffffffu, mbar_wait(bar(B_PV + ((nkt - 1) & 1)), (uint32_t)(((nkt - 1) >> 1) & 1),
                                                    p.status, E2C_ERR_WAIT_ATTN))) {
            tc_fence_after();
            // the row sum over both key halves
            xch[kh * TQ + r] = l;  // buffer 0; its last use (the row max of an earlier tile) is fenced by B_PV
            mbar_arrive(bar(B_FIN + quad));
            if (__all_sync(0xffffffffu, mbar_wait(bar(B_FIN + quad), 0, p.status, E2C_ERR_WAIT_ATTN))) {
                const float lt = xch[r] + xch[TQ + r];
                const bool keep = row_in && (!p.valid || p.valid[row0 + qrow]) && lt > 0.f;
                const float inv = keep ? __fdiv_rn(1.0f, lt) : 0.f;
                float *out = p.ctx + ((size_t)row0 + qrow) * (size_t)(p.H * HD) + h * HD + 128 * kh;
                // Whole 32-row groups inside the sequence leave through a TMA store staged in the Q
                // tile (free: every QK product completed before the last PV); a group running past
                // the sequence end stores row by row so the next sequence's rows stay untouched.
                const bool tma = q0 + quad * 32 + 32 <= S;
                uint8_t *stg = smem + Q_OFF + (warp - 3) * 4096;
#pragma unroll
                for (int cp = 0; cp < 2; cp++) {
                    uint32_t o[2][32];
                    tmem_ld32(tmem + lane_addr + (uint32_t)(256 + 128 * kh + 64 * cp), o[0]);
                    tmem_ld32(tmem + lane_addr + (uint32_t)(256 + 128 * kh + 64 * cp + 32), o[1]);
                    tmem_wait_ld();
#pragma unroll
                    for (int h2 = 0; h2 < 2; h2++) {
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; i++) v[i] = __uint_as_float(o[h2][i]) * inv;
                        const int col = 64 * cp + 32 * h2;
                        if (tma) {
                            if (cp | h2) {
                                if (lane == 0) bulk_wait_read0();
                                __syncwarp();
                            }
                            uint8_t *rowp = stg + lane * 128;
#pragma unroll
                            for (int c = 0; c < 8; c++)
                                *reinterpret_cast<float4 *>(rowp + ((c ^ (lane & 7)) << 4)) =
                                    make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                tma_store_2d(&tmO, smem_u32(stg), h * HD + 128 * kh + col, row0 + q0 + quad * 32);
                                bulk_commit();
                            }
                        } else if (row_in) {
                            float4 *o4 = reinterpret_cast<float4 *>(out + col);
#pragma unroll
                            for (int i = 0; i < 8; i++) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                        }
                    }
                }
                if (lane == 0) bulk_wait0();
                __syncwarp();
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

extern "C" int e2c_attention(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                             int B, int S, int H, float scale, int *status, void *stream) {
    if (B <= 0 || S <= 0) return 0;
    if (H <= 0 || ldvt < S || ldvt % 8 || (((uintptr_t)q | (uintptr_t)k | (uintptr_t)vt) & 15)) {
        e2c_set_msg("attention: bad arguments (H=%d S=%d ldvt=%d; ldvt >= S, multiple of 8; 16-byte aligned)", H, S, ldvt);
        return -1;
    }
    if ((uintptr_t)ctx & 15) {
        e2c_set_msg("attention: ctx must be 16-byte aligned");
        return -1;
    }
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC) != cudaSuccess) {
            e2c_set_msg("attention: cannot reserve %d bytes of shared memory", SMEM_ALLOC);
            return -2;
        }
        attr = true;
    }
    CUtensorMap tq, tk, tv, to;
    const uint64_t rows = (uint64_t)B * S;
    if (e2c_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H * HD, rows, (uint64_t)H * HD * 2, 64, TQ) ||
        e2c_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, rows, HD * 2, 64, TKV) ||
        e2c_tmap_2d(&tv, vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)S, (uint64_t)B * HD, (uint64_t)ldvt * 2, 64, HD) ||
        e2c_tmap_2d(&to, ctx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)H * HD, rows, (uint64_t)H * HD * 4, 32, 32))
        return -3;
    AttnArgs a;
    a.valid = valid;
    a.ctx = ctx;
    a.S = S;
    a.H = H;
    a.nkt = (S + TKV - 1) / TKV;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.status = status;
    const dim3 grid((S + TQ - 1) / TQ, H, B);
    k_attention<<<grid, NTHREADS, SMEM_ALLOC, (cudaStream_t)stream>>>(tq, tk, tv, to, a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        e2c_set_msg("attention launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}
