// attention.cu — bidirectional GQA attention on the sm_100a tensor cores (tcgen05.mma kind::f16).
//
// One CTA per (sequence, query head, 128-query tile). Per 128-key tile j:
//   S_j = Q K_j^T        bf16 x bf16 -> fp32 in TMEM (two S buffers, so QK of tile j+1 overlaps the
//                        softmax of tile j)
//   P_j = exp2(S_j * scale * log2e - m)   online softmax in registers, one thread per query row,
//                        the running max only moved when it grows by more than 2^8 (then O is
//                        rescaled in TMEM), P written to shared memory as bf16 in the MMA's
//                        swizzled K-major layout
//   O  += P_j V_j        fp32 accumulator in TMEM (256 columns)
// and at the end ctx = O / rowsum in fp32. Keys past the sequence end or with valid == 0 get
// probability 0; query rows with valid == 0 get ctx 0 (the reference's masking, src/text.c:661-701).
//
// Operands: Q [B*S][H*256] and K [B*S][256] bf16 row-major (head dim contiguous, K-major for QK^T),
// V^T [B][256][ldvt] bf16 (keys contiguous, K-major for PV) — the QKV GEMM epilogue writes them so.
//
// Warps: 0 = TMA for Q and K, 1 = TMA for V^T, 2 = MMA issuer (+TMEM owner), 3..6 = softmax,
// rescale and epilogue (warp w owns TMEM lanes 32*(w%4) .. +31).
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
constexpr int TKV = 128;       // keys per tile
constexpr int NTHREADS = 224;  // 7 warps
constexpr float kRescaleLog2 = 8.0f;

// shared memory map (bytes, from a 1024-aligned base)
constexpr int Q_OFF = 0;                       // 4 x [128 q][64 d]   (16 KB each)
constexpr int K_OFF = Q_OFF + TQ * HD * 2;     // 4 x [128 k][64 d]
constexpr int V_OFF = K_OFF + TKV * HD * 2;    // 2 x [256 d][64 k]   (32 KB each)
constexpr int P_OFF = V_OFF + HD * TKV * 2;    // 2 x [128 q][64 k]   (16 KB each)
constexpr int BAR_OFF = P_OFF + TQ * TKV * 2;
enum { B_Q, B_KF, B_KE, B_VF, B_PV, B_SF0, B_SF1, B_SE0, B_SE1, B_PF, B_NUM };
constexpr int SMEM_BYTES = BAR_OFF + B_NUM * 8 + 16;
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;

struct AttnArgs {
    const uint8_t *valid;
    float *ctx;
    int S, H, nkt;
    float scale_log2;
    int *status;
};

__global__ void __launch_bounds__(NTHREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
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
        mbar_init(bar(B_KF), 1);
        mbar_init(bar(B_KE), 1);
        mbar_init(bar(B_VF), 1);
        mbar_init(bar(B_PV), 1);
        mbar_init(bar(B_SF0), 1);
        mbar_init(bar(B_SF1), 1);
        mbar_init(bar(B_SE0), 128);
        mbar_init(bar(B_SE1), 128);
        mbar_init(bar(B_PF), 128);
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
    const uint32_t tmem = *tmem_slot;  // S0: cols 0..127, S1: 128..255, O: 256..511

    if (warp == 0) {
        // ---------------------------------------------------------------- Q and K loads
        if (elect_one()) {
            mbar_arrive_expect_tx(bar(B_Q), TQ * HD * 2);
            for (int i = 0; i < 4; i++)
                tma_load_2d(sbase + Q_OFF + i * (TQ * 128), &tmQ, h * HD + 64 * i, row0 + q0, bar(B_Q));
            int issued = 0;
            for (int j = 0; j < nkt; j++) {
                if (!mbar_wait(bar(B_KE), (uint32_t)((j & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) break;
                mbar_arrive_expect_tx(bar(B_KF), TKV * HD * 2);
                for (int i = 0; i < 4; i++)
                    tma_load_2d(sbase + K_OFF + i * (TKV * 128), &tmK, 64 * i, row0 + j * TKV, bar(B_KF));
                issued = j + 1;
            }
            // the last K load (and Q) must have landed before the CTA may exit
            mbar_wait(bar(B_Q), 0, nullptr, E2C_ERR_WAIT_DRAIN);
            if (issued) mbar_wait(bar(B_KF), (uint32_t)((issued - 1) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- V^T loads
        if (elect_one()) {
            int issued = 0;
            for (int j = 0; j < nkt; j++) {
                // V buffer is free once PV of tile j-1 completed
                if (j > 0 && !mbar_wait(bar(B_PV), (uint32_t)((j - 1) & 1), p.status, E2C_ERR_WAIT_PRODUCER)) break;
                mbar_arrive_expect_tx(bar(B_VF), HD * TKV * 2);
                for (int i = 0; i < 2; i++)
                    tma_load_2d(sbase + V_OFF + i * (HD * 128), &tmV, j * TKV + 64 * i, b * HD, bar(B_VF));
                issued = j + 1;
            }
            if (issued) mbar_wait(bar(B_VF), (uint32_t)((issued - 1) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
        }
    } else if (warp == 2) {
        // ---------------------------------------------------------------- MMA issuer
        if (elect_one()) {
            constexpr uint32_t id_s = idesc_bf16(TKV), id_o = idesc_bf16(HD);
            bool ok = mbar_wait(bar(B_Q), 0, p.status, E2C_ERR_WAIT_MMA);
            auto issue_qk = [&](int j) -> bool {
                const int sb = j & 1;
                if (!mbar_wait(bar(B_KF), (uint32_t)(j & 1), p.status, E2C_ERR_WAIT_MMA)) return false;
                if (!mbar_wait(bar(sb ? B_SE1 : B_SE0), (uint32_t)(((j >> 1) & 1) ^ 1), p.status, E2C_ERR_WAIT_MMA))
                    return false;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(sb * TKV);
#pragma unroll
                for (int k = 0; k < HD / 16; k++) {
                    const uint32_t off = (uint32_t)((k >> 2) * (TQ * 128) + (k & 3) * 32);
                    mma_bf16(d, smem_desc_sw128(sbase + Q_OFF + off), smem_desc_sw128(sbase + K_OFF + off), id_s, k != 0);
                }
                mma_commit(bar(sb ? B_SF1 : B_SF0));
                mma_commit(bar(B_KE));
                return true;
            };
            if (ok) ok = issue_qk(0);
            for (int j = 0; j < nkt && ok; j++) {
                if (j + 1 < nkt && !(ok = issue_qk(j + 1))) break;
                if (!mbar_wait(bar(B_PF), (uint32_t)(j & 1), p.status, E2C_ERR_WAIT_MMA) ||
                    !mbar_wait(bar(B_VF), (uint32_t)(j & 1), p.status, E2C_ERR_WAIT_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < TKV / 16; k++) {
                    const uint32_t pa = sbase + P_OFF + (uint32_t)((k >> 2) * (TQ * 128) + (k & 3) * 32);
                    const uint32_t vb = sbase + V_OFF + (uint32_t)((k >> 2) * (HD * 128) + (k & 3) * 32);
                    mma_bf16(tmem + 2 * TKV, smem_desc_sw128(pa), smem_desc_sw128(vb), id_o, (j | k) != 0);
                }
                mma_commit(bar(B_PV));
            }
            if (!ok) {
                // drain whatever was issued before TMEM is released
                mma_commit(bar(B_SE0));
                mbar_wait(bar(B_SE0), 0, nullptr, E2C_ERR_WAIT_DRAIN);
            }
        }
    } else {
        // ---------------------------------------------------------------- softmax / epilogue
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // query row within the tile = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const int qrow = q0 + r;
        const bool row_in = qrow < S;
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkt; j++) {
            const int sb = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(bar(sb ? B_SF1 : B_SF0), (uint32_t)((j >> 1) & 1), p.status,
                                                   E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float s[TKV];
#pragma unroll
            for (int c = 0; c < TKV / 32; c++) {
                uint32_t rr[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(sb * TKV + c * 32), rr);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++) s[c * 32 + i] = __uint_as_float(rr[i]);
            }
            tc_fence_before();
            mbar_arrive(bar(sb ? B_SE1 : B_SE0));  // S buffer may be overwritten by QK of tile j+2
            // key mask and scaled logits (log2 units)
            const int k0 = j * TKV;
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < TKV; i++) {
                const int key = k0 + i;
                const bool kv = key < S && (!p.valid || p.valid[row0 + key]);
                s[i] = kv ? s[i] * p.scale_log2 : -INFINITY;
                mx = fmaxf(mx, s[i]);
            }
            // P and O may be touched only after PV of tile j-1 finished
            if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(bar(B_PV), (uint32_t)((j - 1) & 1), p.status, E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            tc_fence_after();
            // Each row (thread) decides whether its running max moves; the O rescale itself is a
            // warp-collective TMEM round trip (tcgen05.ld/st are .sync.aligned), so the warp runs it
            // whenever any of its rows needs it, rows that do not with alpha = 1.
            float alpha = 1.f;
            if (mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx > -INFINITY)) {
                alpha = m_used == -INFINITY ? 0.f : exp2f(m_used - mx);
                l *= alpha;
                m_used = mx;
            }
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                for (int c = 0; c < HD / 32; c++) {
                    uint32_t o[32];
                    const uint32_t ta = tmem + lane_addr + (uint32_t)(2 * TKV + c * 32);
                    tmem_ld32(ta, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(ta, o);
                }
                tmem_wait_st();
            }
            // probabilities -> bf16 P row (two 128-byte swizzled sub-tiles of 64 keys)
            float lsum = 0.f;
            uint8_t *prow = smem + P_OFF + r * 128;
#pragma unroll
            for (int c = 0; c < TKV / 8; c++) {
                float e[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float v = s[c * 8 + i];
                    e[i] = (v == -INFINITY || m_used == -INFINITY) ? 0.f : exp2f(v - m_used);
                }
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const __nv_bfloat162 hv = __floats2bfloat162_rn(e[2 * i], e[2 * i + 1]);
                    w[i] = *reinterpret_cast<const uint32_t *>(&hv);
                    const float2 back = __bfloat1622float2(hv);
                    lsum += back.x + back.y;  // the sum of what the MMA will actually weigh
                }
                const int sub = c >> 3, chunk = c & 7;
                *reinterpret_cast<uint4 *>(prow + sub * (TQ * 128) + ((chunk ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            l += lsum;
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar(B_PF));
        }
        // ---------------------------------------------------------------- epilogue
        if (ok && __all_sync(0xffffffffu, mbar_wait(bar(B_PV), (uint32_t)((nkt - 1) & 1), p.status, E2C_ERR_WAIT_ATTN))) {
            tc_fence_after();
            const bool keep = row_in && (!p.valid || p.valid[row0 + qrow]) && l > 0.f;
            const float inv = keep ? __fdiv_rn(1.0f, l) : 0.f;
            float *out = p.ctx + ((size_t)row0 + qrow) * (size_t)(p.H * HD) + h * HD;
#pragma unroll 1
            for (int c = 0; c < HD / 32; c++) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(2 * TKV + c * 32), o);
                tmem_wait_ld();
                if (row_in) {
                    float4 *o4 = reinterpret_cast<float4 *>(out + c * 32);
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

extern "C" int e2c_attention(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                             int B, int S, int H, float scale, int *status, void *stream) {
    if (B <= 0 || S <= 0) return 0;
    if (H <= 0 || ldvt < S || ldvt % 8 || (((uintptr_t)q | (uintptr_t)k | (uintptr_t)vt) & 15)) {
        e2c_set_msg("attention: bad arguments (H=%d S=%d ldvt=%d; ldvt >= S, multiple of 8; 16-byte aligned)", H, S, ldvt);
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
    CUtensorMap tq, tk, tv;
    const uint64_t rows = (uint64_t)B * S;
    if (e2c_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H * HD, rows, (uint64_t)H * HD * 2, 64, TQ) ||
        e2c_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, rows, HD * 2, 64, TKV) ||
        e2c_tmap_2d(&tv, vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)S, (uint64_t)B * HD, (uint64_t)ldvt * 2, 64, HD))
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
    k_attention<<<grid, NTHREADS, SMEM_ALLOC, (cudaStream_t)stream>>>(tq, tk, tv, a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        e2c_set_msg("attention launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}
