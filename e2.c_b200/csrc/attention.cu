// attention.cu — bidirectional GQA attention on the sm_100a tensor cores (tcgen05.mma kind::f16).
//
// Work unit: one (sequence, query head, 128-query tile). The kernel is persistent: one CTA per SM
// walks units u = blockIdx.x, + gridDim.x, ... so that the next unit's start (its Q and first K
// tiles, its first QK products) overlaps the current unit's end (softmax of the last tiles, the
// final normalisation and the ctx stores). Keys are swept in tiles of 64, K and V^T double-buffered
// in shared memory. Per key tile j:
//   S_j = Q K_j^T        bf16 x bf16 -> fp32 in TMEM (four S buffers: QK of tiles j+1, j+2 run while
//                        the softmax of tile j does, whatever the K loads' latency)
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
// Warps: 0 = TMA for Q and K, 1 = TMA for V^T, 2 = MMA issuer (+TMEM owner), 3..10 = softmax and
// rescale: warp w owns TMEM lanes 32*(w%4) .. +31 and, with its partner of the same quadrant, half
// of every key tile (keys 32*kh .. +31); 11..14 = epilogue, one per lane quadrant: ctx = O / rowsum
// for its 32 rows and all 256 columns, stored while the softmax warps run the next unit.
//
// Every per-tile barrier is indexed by a tile counter that runs across units (g): the S, P and PV
// barriers come four to a set (index g & 3, phase parity (g >> 2) & 1), the K and V buffers two to
// a set (g & 1, (g >> 1) & 1); per-unit barriers use the unit counter's parity. MMA issue order per
// tile j: QK(j+2), then PV(j). QK(j+2) writes S buffer (j+2) & 3, whose P(j-2) the PV issued in the
// previous-but-one step has read (tcgen05.mma from one thread executes in order).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "launch.h"
#include "devstate.cuh"
#include "pdl.h"
#include "ptx.cuh"
#include "tmap.h"

namespace {

constexpr int TQ = 128;        // queries per unit
constexpr int TKV = 64;        // keys per tile
constexpr int SM_WARPS = 8;    // softmax warps
constexpr int EP_WARPS = 4;    // epilogue warps
constexpr int NTHREADS = 96 + 32 * SM_WARPS + 32 * EP_WARPS;
constexpr float kRescaleLog2 = 8.0f;
// per epilogue warp, three 32-row x 16-column fp32 staging tiles for the ctx TMA stores (64-byte
// swizzle: 16-byte chunk c of row r at chunk c ^ ((r >> 1) & 3)), used in turn
constexpr int STG = 32 * 16 * 4;
constexpr int NSTG = 3;
// Q full / Q free / O free; K full x2, K empty x2, V full x2, V empty x2, PV done x4, S full x4,
// P full x4, pair [2][4], final [4], drain
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
    B_PAIR = B_PF + 4,
    B_FIN = B_PAIR + 8,
    B_DRAIN = B_FIN + 4,
    B_UD,  // [2 unit parities][4]: a unit's 1/rowsum of a lane quadrant is ready for its epilogue warp
    B_NUM = B_UD + 8
};

// shared memory map (bytes, from a 1024-aligned base) for head dim HD (64 or 256): Q as HD/64
// panels of [128 q][64 d], K as HD/64 panels of [64 k][64 d] per buffer, V^T as [HD d][64 k]
template <int HD>
struct AttnSmem {
    static_assert(HD == 64 || HD == 256, "head dim 64 or 256");
    static constexpr int Q_OFF = 0;
    static constexpr int K_TILE = TKV * HD * 2;
    static constexpr int V_TILE = HD * TKV * 2;
    static constexpr int K_OFF = Q_OFF + TQ * HD * 2;  // 2 buffers
    static constexpr int V_OFF = K_OFF + 2 * K_TILE;   // 2 buffers
    static constexpr int STG_OFF = V_OFF + 2 * V_TILE;
    static constexpr int X_OFF = STG_OFF + EP_WARPS * NSTG * STG;  // row-max exchange [2 tile parities][2 halves][128]
    static constexpr int INV_OFF = X_OFF + 2 * 2 * TQ * 4;        // 1 / rowsum of a unit's rows [2 unit parities][128]
    static constexpr int BAR_OFF = INV_OFF + 2 * TQ * 4;
    static constexpr int SMEM_BYTES = BAR_OFF + B_NUM * 8 + 16;
    // No alignment slack: the dynamic shared memory of a kernel without static shared variables
    // starts 1024-byte aligned, which the kernel checks before using it (the swizzled tiles need it).
    static constexpr int SMEM_ALLOC = SMEM_BYTES;
    static_assert(SMEM_ALLOC <= 232448, "shared memory");
};

struct AttnArgs {
    const uint8_t *valid;
    float *ctx;
    int S, H, KV, nkt, nqt, units;
    int window;  // keys j with |i - j| <= window attend to query i; < 0: every key
    float scale_log2;
    int *status;
};

E2C_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// unit u -> sequence, head, query tile (query tiles of one sequence and head are consecutive, so
// the units in flight at once share a few sequences' K and V^T in L2)
struct Unit {
    int b, h, qt;
};
E2C_DEV Unit unit_of(int u, const AttnArgs &p) {
    const int per_seq = p.H * p.nqt;
    const int b = u / per_seq, rem = u - b * per_seq;
    return {b, rem / p.nqt, rem % p.nqt};
}

// the key tiles a unit visits: all of them, or those a sliding window reaches from its queries
E2C_DEV void tile_range(const Unit &w, const AttnArgs &p, int &j0, int &nt) {
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

template <int HD>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const AttnArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    griddep_launch_dependents();
    if (smem_u32(smem_raw) & 1023) {  // never expected; refuse rather than misplace the swizzled tiles
        griddep_wait();
        if (threadIdx.x == 0) record_status(p.status, E2C_ERR_SMEM_ALIGN);
        return;
    }
    using L = AttnSmem<HD>;
    constexpr int Q_OFF = L::Q_OFF, K_OFF = L::K_OFF, V_OFF = L::V_OFF, K_TILE = L::K_TILE, V_TILE = L::V_TILE;
    constexpr int STG_OFF = L::STG_OFF, X_OFF = L::X_OFF, INV_OFF = L::INV_OFF, BAR_OFF = L::BAR_OFF;
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
        for (int i = 0; i < 8; i++) mbar_init(bar(B_PAIR + i), 64);
        for (int i = 0; i < 4; i++) mbar_init(bar(B_FIN + i), 64);
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
    griddep_wait();  // the previous kernel's Q, K, V (and its reads of ctx) are done
    const uint32_t tmem = *tmem_slot;  // S buffer i: cols 64 i .. +63 (i < 4), O: 256..511

    if (warp == 0) {
        // ---------------------------------------------------------------- Q and K loads
        if (elect_one()) {
            int g = 0, nu = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, nu++) {
                const Unit w = unit_of(u, p);
                const int row0 = w.b * S;
                const int kvh = w.h / (p.H / p.KV);
                int j0, nt;
                tile_range(w, p, j0, nt);
                // Q may be replaced once every QK product of the previous unit completed
                if (!mbar_wait(bar(B_QE), (uint32_t)((nu & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) break;
                mbar_arrive_expect_tx(bar(B_Q), TQ * HD * 2);
                for (int i = 0; i < HD / 64; i++)
                    tma_load_2d(sbase + Q_OFF + i * (TQ * 128), &tmQ, w.h * HD + 64 * i, row0 + w.qt * TQ, bar(B_Q));
                for (int j = j0; j < j0 + nt; j++, g++) {
                    const int kb = g & 1;
                    // buffer kb is free once QK of tile g-2 completed
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
            // the last loads must have landed before the CTA may exit
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
                int j0, nt;
                tile_range(w, p, j0, nt);
                for (int j = j0; j < j0 + nt; j++, g++) {
                    const int vb = g & 1;
                    // buffer vb is free once PV of tile g-2 completed
                    if (!mbar_wait(bar(B_VE + vb), (uint32_t)(((g >> 1) & 1) ^ 1), p.status, E2C_ERR_WAIT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(B_VF + vb), V_TILE);
                    tma_load_2d(sbase + V_OFF + vb * V_TILE, &tmV, j * TKV, (w.b * p.KV + w.h / (p.H / p.KV)) * HD,
                                bar(B_VF + vb));
                }
            }
            for (int i = g - 2 < 0 ? 0 : g - 2; i < g; i++)
                mbar_wait(bar(B_VF + (i & 1)), (uint32_t)((i >> 1) & 1), nullptr, E2C_ERR_WAIT_DRAIN);
        }
    } else if (warp == 2) {
        // ---------------------------------------------------------------- MMA issuer
        // Issue order per unit QK0, QK1, then per tile j: QK(j+2), PV(j).
        if (elect_one()) {
            constexpr uint32_t id_s = idesc_bf16(TKV), id_o = idesc_bf16(HD);
            int g0 = 0, nu = 0;  // first global tile of the unit, units done
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
                if (last) mma_commit(bar(B_QE));  // the unit's last read of Q
                return true;
            };
            int nt = 0;
            for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, nu++, g0 += nt) {
                int j0;
                tile_range(unit_of(u, p), p, j0, nt);
                if (!mbar_wait(bar(B_Q), (uint32_t)(nu & 1), p.status, E2C_ERR_WAIT_MMA)) {
                    ok = false;
                    break;
                }
                if (!issue_qk(g0, nt == 1) || (nt > 1 && !issue_qk(g0 + 1, nt == 2))) {
                    ok = false;
                    break;
                }
                for (int j = 0; j < nt; j++) {
                    const int g = g0 + j, vb = g & 1, s4 = g & 3;
                    if (j + 2 < nt && !(ok = issue_qk(g + 2, j + 2 == nt - 1))) break;
                    if (!mbar_wait(bar(B_PF + s4), (uint32_t)((g >> 2) & 1), p.status, E2C_ERR_WAIT_MMA) ||
                        !mbar_wait(bar(B_VF + vb), (uint32_t)((g >> 1) & 1), p.status, E2C_ERR_WAIT_MMA) ||
                        // the first PV of a unit overwrites O: the previous unit's epilogue has read it
                        (j == 0 && !mbar_wait(bar(B_OE), (uint32_t)((nu & 1) ^ 1), p.status, E2C_ERR_WAIT_MMA))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t pa = tmem + (uint32_t)(s4 * TKV);  // P(g): 32 columns of bf16 pairs
                    const uint32_t vbase = sbase + V_OFF + vb * V_TILE;
#pragma unroll
                    for (int k = 0; k < TKV / 16; k++)
                        mma_bf16_ts(tmem + 256, pa + 8 * k, smem_desc_sw128(vbase + (uint32_t)(k * 32)), id_o, (j | k) != 0);
                    mma_commit(bar(B_PV + s4));
                    mma_commit(bar(B_VE + vb));
                }
            }
            if (!ok) {
                // drain whatever was issued before TMEM is released
                mma_commit(bar(B_DRAIN));
                mbar_wait(bar(B_DRAIN), 0, nullptr, E2C_ERR_WAIT_DRAIN);
            }
        }
    } else if (warp < 3 + SM_WARPS) {
        // ---------------------------------------------------------------- softmax
        const int quad = warp & 3;
        const int kh = (warp - 3) >> 2;   // key half of every tile this warp owns
        const int r = quad * 32 + lane;   // query row within the tile = TMEM lane
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        float *xch = reinterpret_cast<float *>(smem + X_OFF);  // [2][2][TQ] row maxima
        float *invs = reinterpret_cast<float *>(smem + INV_OFF);  // [2][TQ]
        bool ok = true;
        int g0 = 0, nu = 0, nt = 0;
        for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, nu++, g0 += nt) {
            const Unit w = unit_of(u, p);
            const int row0 = w.b * S, q0 = w.qt * TQ;
            const int qrow = q0 + r;
            const bool row_in = qrow < S;
            int j0;
            tile_range(w, p, j0, nt);
            // the warp's 32 query rows start at wq0
            const int wq0 = q0 + quad * 32;
            float m_used = -INFINITY, l = 0.f;
            for (int jj = 0; jj < nt; jj++) {
                const int j = j0 + jj;
                const int g = g0 + jj, sb = g & 1, s4 = g & 3;
                if (!__all_sync(0xffffffffu, mbar_wait(bar(B_SF + s4), (uint32_t)((g >> 2) & 1), p.status, E2C_ERR_WAIT_ATTN))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float s[32];
                {
                    uint32_t rr[32];
                    tmem_ld32(tmem + lane_addr + (uint32_t)(s4 * TKV + 32 * kh), rr);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) s[i] = __uint_as_float(rr[i]);
                }
                // masking only where a tile runs past the sequence or a valid mask is given: lane i
                // reads key k0 + i's flag, a ballot gives every lane the 32 keys' bits
                const int k0 = j * TKV + 32 * kh;
                if (p.valid || k0 + 32 > S) {
                    const int key = k0 + lane;
                    const uint32_t keep = __ballot_sync(0xffffffffu, key < S && (!p.valid || p.valid[row0 + key]));
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (!((keep >> i) & 1u)) s[i] = -INFINITY;
                }
                // the window's edge runs through this warp's 32 x 32 block: per element
                if (p.window >= 0 && (k0 < wq0 + 31 - p.window || k0 + 31 > wq0 + p.window)) {
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (k0 + i < qrow - p.window || k0 + i > qrow + p.window) s[i] = -INFINITY;
                }
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < 32; i++) mx = fmaxf(mx, s[i]);
                // the row max over both key halves, through the partner warp
                xch[(sb * 2 + kh) * TQ + r] = mx;
                mbar_arrive(bar(B_PAIR + sb * 4 + quad));
                if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PAIR + sb * 4 + quad), (uint32_t)((g >> 1) & 1), p.status,
                                                       E2C_ERR_WAIT_ATTN))) {
                    ok = false;
                    break;
                }
                mx = fmaxf(xch[(sb * 2) * TQ + r], xch[(sb * 2 + 1) * TQ + r]) * p.scale_log2;
                // Each row decides whether its running max moves; the O rescale is a warp-collective
                // TMEM round trip (tcgen05.ld/st are .sync.aligned), run when any row of the warp needs it.
                float alpha = 1.f;
                if (mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx > -INFINITY)) {
                    alpha = m_used == -INFINITY ? 0.f : exp2f(m_used - mx);
                    l *= alpha;
                    m_used = mx;
                }
                if (jj > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                    // O may be touched only once PV of tile g-1 completed
                    if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PV + ((g - 1) & 3)), (uint32_t)(((g - 1) >> 2) & 1),
                                                           p.status, E2C_ERR_WAIT_ATTN))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < HD / 64; c++) {  // this warp's half of O's HD columns
                        uint32_t o[32];
                        const uint32_t ta = tmem + lane_addr + (uint32_t)(256 + (HD / 2) * kh + c * 32);
                        tmem_ld32(ta, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(ta, o);
                    }
                    tmem_wait_st();
                }
                // probabilities -> bf16 pairs over this warp's S columns: P(g) occupies columns
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
                    const uint32_t ta = tmem + lane_addr + (uint32_t)(s4 * TKV + 16 * kh);
                    asm volatile(
                        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(ta),
                        "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3]), "r"(pk[4]), "r"(pk[5]), "r"(pk[6]), "r"(pk[7]),
                        "r"(pk[8]), "r"(pk[9]), "r"(pk[10]), "r"(pk[11]), "r"(pk[12]), "r"(pk[13]), "r"(pk[14]), "r"(pk[15])
                        : "memory");
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(bar(B_PF + s4));
            }
            if (!ok) break;
            // ------------------------------------------------------------ end of the unit
            // The row sum over both key halves, exchanged in the row-max slots of the last tile's
            // parity: both warps of the pair have published P of that tile (so read its maxima) once
            // that tile's P-full barrier completed, and neither writes those slots again before both
            // have passed the next unit's first exchange, which follows the reads below.
            const int gl = g0 + nt - 1;
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PF + (gl & 3)), (uint32_t)((gl >> 2) & 1), p.status, E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            float *xfin = xch + (gl & 1) * 2 * TQ;
            xfin[kh * TQ + r] = l;
            mbar_arrive(bar(B_FIN + quad));
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_FIN + quad), (uint32_t)(nu & 1), p.status, E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            const float lt = xfin[r] + xfin[TQ + r];
            const bool keep = row_in && (!p.valid || p.valid[row0 + qrow]) && lt > 0.f;
            // ctx = O / rowsum is the epilogue warp's. Slot and barrier alternate by unit: both are
            // used again two units on, and unit nu+2's S tiles come from QK products the MMA issues
            // after unit nu+1's first PV, which waited for that warp to release O of unit nu+1, after
            // it had waited for and read unit nu's.
            if (kh == 0) {
                invs[(nu & 1) * TQ + r] = keep ? __fdiv_rn(1.0f, lt) : 0.f;
                mbar_arrive(bar(B_UD + (nu & 1) * 4 + quad));
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        // ctx = O / rowsum for this quadrant's 32 rows, 16 columns at a time through three staging
        // tiles and TMA stores that drain while the next unit runs. A 32-row group running past the
        // sequence end stores row by row instead, so the next sequence's rows stay untouched.
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const float *invs = reinterpret_cast<const float *>(smem + INV_OFF);
        uint8_t *stg = smem + STG_OFF + (warp - 3 - SM_WARPS) * NSTG * STG;
        int nst = 0;  // ctx stores this warp committed
        bool ok = true;
        int g0 = 0, nu = 0, nt = 0;
        for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, nu++, g0 += nt) {
            const Unit w = unit_of(u, p);
            const int row0 = w.b * S, q0 = w.qt * TQ;
            const int qrow = q0 + r;
            const bool row_in = qrow < S;
            int j0;
            tile_range(w, p, j0, nt);
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_UD + (nu & 1) * 4 + quad), (uint32_t)((nu >> 1) & 1), p.status,
                                                   E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            const float inv = invs[(nu & 1) * TQ + r];
            // PV of the last tile completes after every earlier product (tcgen05.commit tracks all
            // prior MMAs): O is final
            const int gl = g0 + nt - 1;
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_PV + (gl & 3)), (uint32_t)((gl >> 2) & 1), p.status, E2C_ERR_WAIT_ATTN))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int gq0 = q0 + quad * 32;  // first query row of this warp
            const bool tma = gq0 + 32 <= S;
            float *out = p.ctx + ((size_t)row0 + qrow) * (size_t)(p.H * HD) + w.h * HD;
#pragma unroll 1
            for (int cp = 0; cp < HD / 32; cp++) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(256 + 32 * cp), o);
                tmem_wait_ld();
                if (cp == HD / 32 - 1) {
                    // every O column this warp reads has been read: the next unit's PV may write O
                    tc_fence_before();
                    mbar_arrive(bar(B_OE));
                }
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    float v[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(o[16 * h + i]) * inv;
                    const int col = 32 * cp + 16 * h;
                    if (tma) {
                        uint8_t *buf = stg + (nst % NSTG) * STG;
                        if (nst >= NSTG) {  // the store that last read this tile has finished reading it
                            if (lane == 0) bulk_wait_read2();
                            __syncwarp();
                        }
                        uint8_t *rowp = buf + lane * 64;
#pragma unroll
                        for (int c = 0; c < 4; c++)
                            *reinterpret_cast<float4 *>(rowp + ((c ^ ((lane >> 1) & 3)) << 4)) =
                                make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tmO, smem_u32(buf), w.h * HD + col, row0 + gq0);
                            bulk_commit();
                        }
                        ++nst;
                    } else if (row_in) {
                        float4 *o4 = reinterpret_cast<float4 *>(out + col);
#pragma unroll
                        for (int i = 0; i < 4; i++) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    }
                }
            }
        }
        // the global writes of every store this warp issued complete before the kernel ends
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <int HD>
int launch_hd(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx, int B, int S,
              int H, int KV, float scale, int window, int *status, cudaStream_t st, int dev, int num_sms) {
    using L = AttnSmem<HD>;
    static E2cPerDev attr;  // the shared-memory opt-in, per device
    if (!attr.get(dev)) {
        if (cudaFuncSetAttribute(k_attention<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_ALLOC) != cudaSuccess) {
            cudaGetLastError();
            e2c_set_msg("attention: cannot reserve %d bytes of shared memory", L::SMEM_ALLOC);
            return -2;
        }
        attr.set(dev, 1);
    }
    CUtensorMap tq, tk, tv, to;
    const uint64_t rows = (uint64_t)B * S;
    if (e2c_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H * HD, rows, (uint64_t)H * HD * 2, 64, TQ) ||
        e2c_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)KV * HD, rows, (uint64_t)KV * HD * 2, 64, TKV) ||
        e2c_tmap_2d(&tv, vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)S, (uint64_t)B * KV * HD, (uint64_t)ldvt * 2, 64,
                    HD) ||
        e2c_tmap_2d_sw64(&to, ctx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)H * HD, rows, (uint64_t)H * HD * 4, 16, 32))
        return -3;
    AttnArgs a;
    a.valid = valid;
    a.ctx = ctx;
    a.S = S;
    a.H = H;
    a.KV = KV;
    a.nkt = (S + TKV - 1) / TKV;
    a.nqt = (S + TQ - 1) / TQ;
    a.units = B * H * a.nqt;
    a.window = window;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.status = status;
    const int grid = a.units < num_sms ? a.units : num_sms;
    e2c_launch(k_attention<HD>, dim3(grid), dim3(NTHREADS), L::SMEM_ALLOC, st, tq, tk, tv, to, a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        e2c_set_msg("attention launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}

}  // namespace

extern "C" int e2c_attention_win(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                                 int B, int S, int H, int KV, int D, float scale, int window, int *status, void *stream) {
    if (B <= 0 || S <= 0) return 0;
    if (H <= 0 || KV <= 0 || H % KV || (D != 64 && D != 256 && D != 512) || ldvt < S || ldvt % 8 ||
        (((uintptr_t)q | (uintptr_t)k | (uintptr_t)vt) & 15)) {
        e2c_set_msg("attention: bad arguments (H=%d KV=%d D=%d S=%d ldvt=%d; KV divides H, D 64, 256 or 512, ldvt >= S "
                    "and a multiple of 8, 16-byte aligned operands)", H, KV, D, S, ldvt);
        return -1;
    }
    if ((uintptr_t)ctx & 15) {
        e2c_set_msg("attention: ctx must be 16-byte aligned");
        return -1;
    }
    if (D == 512) return e2c_attention_wide(q, k, vt, ldvt, valid, ctx, B, S, H, KV, scale, window, status, stream);
    const int dev = e2c_device();
    const int num_sms = e2c_sm_count(dev);
    if (!num_sms) {
        e2c_set_msg("attention: no CUDA device");
        return -2;
    }
    cudaStream_t st = (cudaStream_t)stream;
    return D == 256 ? launch_hd<256>(q, k, vt, ldvt, valid, ctx, B, S, H, KV, scale, window, status, st, dev, num_sms)
                    : launch_hd<64>(q, k, vt, ldvt, valid, ctx, B, S, H, KV, scale, window, status, st, dev, num_sms);
}

extern "C" int e2c_attention_gqa(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                                 int B, int S, int H, int KV, int D, float scale, int *status, void *stream) {
    if (D == 512) {
        e2c_set_msg("attention: D=%d; head dim 512 runs through e2c_attention_win", D);
        return -1;
    }
    return e2c_attention_win(q, k, vt, ldvt, valid, ctx, B, S, H, KV, D, scale, -1, status, stream);
}

extern "C" int e2c_attention(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                             int B, int S, int H, float scale, int *status, void *stream) {
    return e2c_attention_gqa(q, k, vt, ldvt, valid, ctx, B, S, H, 1, 256, scale, status, stream);
}
