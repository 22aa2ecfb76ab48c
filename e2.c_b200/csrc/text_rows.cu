// text_rows.cu — the row passes of e2.c's own text tower (EmbeddingGemma-2, src/text.c:924-984)
// between its GEMMs, one warp per row (or per row and head / PLE slice):
//
//   token gather: bf16 table row * embed_scale      e2_embed_token, src/text.c:917-921
//     -> x (the residual stream), quantise(x) for the PLE projection, and
//        quantise(rmsnorm(x) * input_ln[0]) for layer 0's q|k|v        src/text.c:929,944
//   PLE gate: h = gelu_tanh(gate) * rmsnorm(ple slice * ple_scale) * ple_proj_norm, quantised: the
//     per-layer input's scale and norm (src/text.c:930-931) applied where each slice is read
//   q|k|v: per-head RMSNorm (q_norm, k_norm; v without a scale), RoPE on q and k, bf16 Q, K, V^T
//     for head dims 256 and 512 and any number of KV heads                src/text.c:842-857
//   x = (rmsnorm(t) * g1 + res) * layer_scalar, stored as the residual, then quantise either
//     rmsnorm(x) * g2 (the next norm_split) or x itself (the PLE gate's input)  src/text.c:947-960
//   h = gelu_tanh(gate) * up with up strided (the PLE slice), quantised  gate_quant, src/text.c:424-468
//
// The arithmetic is the reference's per element (x * inv * gamma, products and sums in fp32, the
// quantiser of src/int8.c:178-209); sums of squares run in warp order, so normed values agree to a
// few ulp.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "epi_math.cuh"
#include "launch.h"
#include "pdl.h"
#include "ptx.cuh"
#include "rowmath.cuh"

namespace {

__device__ __forceinline__ float4 bf16x4_to_f32(uint2 u) {
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
}

__device__ __forceinline__ float4 mul4(float4 a, float s) {
    return make_float4(__fmul_rn(a.x, s), __fmul_rn(a.y, s), __fmul_rn(a.z, s), __fmul_rn(a.w, s));
}

template <int NV>
__global__ void __launch_bounds__(256) k_tt_embed(const int32_t *__restrict__ ids, const uint16_t *__restrict__ table,
                                                  float escale, const float *__restrict__ gamma, float eps,
                                                  float *__restrict__ res, int8_t *__restrict__ qx, float *__restrict__ qxs,
                                                  int8_t *__restrict__ qn, float *__restrict__ qns, int M, int ablk, int vocab,
                                                  int *status) {
    griddep_launch_dependents();
    griddep_wait();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= M) return;
    constexpr int D = NV * 128;
    int id = __ldg(ids + row);
    if (id < 0 || id >= vocab) {  // never read outside the table: record and use row 0
        if (lane == 0 && status) atomicCAS(status, 0, 0x106);
        id = 0;
    }
    const uint2 *tr = reinterpret_cast<const uint2 *>(table + (size_t)id * D);
    float4 x[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
        x[i] = mul4(bf16x4_to_f32(__ldg(tr + lane + 32 * i)), escale);
        reinterpret_cast<float4 *>(res + (size_t)row * D)[lane + 32 * i] = x[i];
    }
    const int nb = D / ablk;
    quantize_row(x, ablk, D, qx + (size_t)row * D, qxs + (size_t)row * nb, lane);
    const float inv = rms_inv(sumsq(x), D, eps);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
#pragma unroll
    for (int i = 0; i < NV; i++) x[i] = norm4(x[i], inv, __ldg(g4 + lane + 32 * i));
    quantize_row(x, ablk, D, qn + (size_t)row * D, qns + (size_t)row * nb, lane);
}

// q|k|v fp32 [M][ldy] laid out [H q heads | KV k heads | KV v heads] of D = 256 NVH. One CTA per
// (sequence, tile of 32 positions); its 8 warps take (position, head) items in turn. Per item, lane l
// holds float4s l + 32 i of the head's first half (a) and their rotate-half partners in the second
// half (b): RMSNorm over the head, RoPE on q and k (the AVX-512 form of src/kernels_avx512.c:309-331, a' = fma(a, c, -(y s)), y' = fma(a, s, y c)); Q
// [M][H D] and K [M][KV D] are stored in bf16 straight from the warp, 512 contiguous bytes per
// instruction. V is staged in shared memory and leaves transposed, V^T [B][KV D][ldvt]: each of its
// rows gets the tile's 32 positions as 64 contiguous bytes (a position-major store would write one
// 2-byte element per 32-byte sector). The RoPE tables are position-major ([pos][ldrope], pair e of
// position p at p * ldrope + e: a lane's four pairs in one 16-byte load) or pair-major ([D/2][ldrope],
// at e * ldrope + p: the layout the fused QKV GEMM epilogue reads, where a warp's lanes are positions).
constexpr int QKV_TILE = 32;

template <int NVH>
__global__ void __launch_bounds__(256) k_tt_qkv_post(const float *__restrict__ y, int ldy, int H, int KV,
                                                     const float *__restrict__ qg, const float *__restrict__ kg, float eps,
                                                     const float *__restrict__ rcos, const float *__restrict__ rsin,
                                                     int ldrope, int pos_major, int S, int ntiles,
                                                     __nv_bfloat16 *__restrict__ Q,
                                                     __nv_bfloat16 *__restrict__ Kout, __nv_bfloat16 *__restrict__ Vt,
                                                     int ldvt) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr int D = 256 * NVH, HALF4 = D / 8;  // float4s in half a head
    extern __shared__ __nv_bfloat16 vs[];         // [QKV_TILE][KV D + 2]
    const int ldv = KV * D + 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x / ntiles, p0 = (blockIdx.x - b * ntiles) * QKV_TILE;
    const int npos = min(QKV_TILE, S - p0);
    const int nh = H + 2 * KV;
    for (int it = warp; it < npos * nh; it += 8) {
        const int r = it / nh, head = it - r * nh;
        const int pos = p0 + r;
        const size_t row = (size_t)b * S + pos;
        const int kind = head < H ? 0 : head < H + KV ? 1 : 2;  // q, k, v
        const float4 *src = reinterpret_cast<const float4 *>(y + row * ldy + (size_t)head * D);
        float4 a[NVH], bb[NVH];
#pragma unroll
        for (int i = 0; i < NVH; i++) {
            a[i] = src[lane + 32 * i];
            bb[i] = src[HALF4 + lane + 32 * i];
        }
        const float inv = rms_inv(__fadd_rn(sumsq(a), sumsq(bb)), D, eps);
        const float *g = kind == 0 ? qg : kind == 1 ? kg : nullptr;
#pragma unroll
        for (int i = 0; i < NVH; i++) {
            if (g) {
                a[i] = norm4(a[i], inv, __ldg(reinterpret_cast<const float4 *>(g) + lane + 32 * i));
                bb[i] = norm4(bb[i], inv, __ldg(reinterpret_cast<const float4 *>(g) + HALF4 + lane + 32 * i));
            } else {
                a[i] = mul4(a[i], inv);
                bb[i] = mul4(bb[i], inv);
            }
        }
        if (kind < 2) {
#pragma unroll
            for (int i = 0; i < NVH; i++) {
                float *pa = reinterpret_cast<float *>(&a[i]), *pb = reinterpret_cast<float *>(&bb[i]);
                const int e0 = 4 * (lane + 32 * i);
                float cc[4], ss[4];
                if (pos_major) {
                    const float4 c4 = __ldg(reinterpret_cast<const float4 *>(rcos + (size_t)pos * ldrope + e0));
                    const float4 s4 = __ldg(reinterpret_cast<const float4 *>(rsin + (size_t)pos * ldrope + e0));
                    cc[0] = c4.x, cc[1] = c4.y, cc[2] = c4.z, cc[3] = c4.w;
                    ss[0] = s4.x, ss[1] = s4.y, ss[2] = s4.z, ss[3] = s4.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        cc[j] = __ldg(rcos + (size_t)(e0 + j) * ldrope + pos);
                        ss[j] = __ldg(rsin + (size_t)(e0 + j) * ldrope + pos);
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float x = pa[j], z = pb[j];
                    pa[j] = __fmaf_rn(x, cc[j], -__fmul_rn(z, ss[j]));
                    pb[j] = __fmaf_rn(x, ss[j], __fmul_rn(z, cc[j]));
                }
            }
            __nv_bfloat16 *dst = kind == 0 ? Q + row * H * D + (size_t)head * D : Kout + row * KV * D + (size_t)(head - H) * D;
#pragma unroll
            for (int i = 0; i < NVH; i++) {
                const __nv_bfloat162 q0 = __floats2bfloat162_rn(a[i].x, a[i].y), q1 = __floats2bfloat162_rn(a[i].z, a[i].w);
                const __nv_bfloat162 q2 = __floats2bfloat162_rn(bb[i].x, bb[i].y), q3 = __floats2bfloat162_rn(bb[i].z, bb[i].w);
                *reinterpret_cast<uint2 *>(dst + 4 * (lane + 32 * i)) =
                    make_uint2(*reinterpret_cast<const uint32_t *>(&q0), *reinterpret_cast<const uint32_t *>(&q1));
                *reinterpret_cast<uint2 *>(dst + D / 2 + 4 * (lane + 32 * i)) =
                    make_uint2(*reinterpret_cast<const uint32_t *>(&q2), *reinterpret_cast<const uint32_t *>(&q3));
            }
        } else {
            __nv_bfloat16 *vr = vs + (size_t)r * ldv + (size_t)(head - H - KV) * D;
#pragma unroll
            for (int i = 0; i < NVH; i++) {
                const float *pa = reinterpret_cast<const float *>(&a[i]), *pb = reinterpret_cast<const float *>(&bb[i]);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int e = 4 * (lane + 32 * i) + j;
                    vr[e] = __float2bfloat16_rn(pa[j]);
                    vr[D / 2 + e] = __float2bfloat16_rn(pb[j]);
                }
            }
        }
    }
    __syncthreads();
    // V^T rows (kv head, dim) x the tile's positions, two positions per thread and word
    const int rows = KV * D;
    __nv_bfloat16 *vt = Vt + (size_t)b * rows * ldvt + p0;
    for (int w = threadIdx.x; w < rows * (QKV_TILE / 2); w += blockDim.x) {
        const int d = w / (QKV_TILE / 2), pp = 2 * (w - d * (QKV_TILE / 2));
        if (pp + 1 < npos) {
            __nv_bfloat162 v2;
            v2.x = vs[(size_t)pp * ldv + d];
            v2.y = vs[(size_t)(pp + 1) * ldv + d];
            *reinterpret_cast<__nv_bfloat162 *>(vt + (size_t)d * ldvt + pp) = v2;
        } else if (pp < npos) {
            vt[(size_t)d * ldvt + pp] = vs[(size_t)pp * ldv + d];
        }
    }
}

// x = (rmsnorm(t) * g1 + res) * ls -> res; then quantise rmsnorm(x) * g2 (g2 given) or x itself
template <int NV>
__global__ void __launch_bounds__(256) k_tt_norm_add(const float *__restrict__ t, float *__restrict__ res,
                                                     const float *__restrict__ g1, float ls, const float *__restrict__ g2,
                                                     float eps, int8_t *__restrict__ q, float *__restrict__ qs, int M,
                                                     int ablk) {
    griddep_launch_dependents();
    griddep_wait();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= M) return;
    constexpr int D = NV * 128;
    const float4 *t4 = reinterpret_cast<const float4 *>(t + (size_t)row * D);
    float4 *r4 = reinterpret_cast<float4 *>(res + (size_t)row * D);
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) v[i] = t4[lane + 32 * i];
    const float inv1 = rms_inv(sumsq(v), D, eps);
    const float4 *g14 = reinterpret_cast<const float4 *>(g1);
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float4 n = norm4(v[i], inv1, __ldg(g14 + lane + 32 * i));
        const float4 r = r4[lane + 32 * i];
        v[i] = mul4(make_float4(__fadd_rn(n.x, r.x), __fadd_rn(n.y, r.y), __fadd_rn(n.z, r.z), __fadd_rn(n.w, r.w)), ls);
        r4[lane + 32 * i] = v[i];
    }
    if (g2) {
        const float inv2 = rms_inv(sumsq(v), D, eps);
        const float4 *g24 = reinterpret_cast<const float4 *>(g2);
#pragma unroll
        for (int i = 0; i < NV; i++) v[i] = norm4(v[i], inv2, __ldg(g24 + lane + 32 * i));
    }
    quantize_row(v, ablk, D, q + (size_t)row * D, qs + (size_t)row * (D / ablk), lane);
}

// h = gelu_tanh(g) * u (u's rows ldu apart: the PLE slice of this layer), quantised per row. With
// ugamma given, u is first taken as rmsnorm(u * uscale) * ugamma over its I values: the PLE slice's
// scale and norm, the arithmetic of a separate pass over the slice (u * scale, then x * inv * gamma).
template <int NV>
__global__ void __launch_bounds__(256) k_tt_gate_quant(const float *__restrict__ g, int ldg, const float *__restrict__ u,
                                                       int ldu, float uscale, const float *__restrict__ ugamma, float eps,
                                                       int8_t *__restrict__ q, float *__restrict__ qs, int M, int ablk) {
    griddep_launch_dependents();
    griddep_wait();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= M) return;
    constexpr int I = NV * 128;
    const float4 *g4 = reinterpret_cast<const float4 *>(g + (size_t)row * ldg);
    const float4 *u4 = reinterpret_cast<const float4 *>(u + (size_t)row * ldu);
    float4 b[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) b[i] = u4[lane + 32 * i];
    if (ugamma) {
#pragma unroll
        for (int i = 0; i < NV; i++) b[i] = mul4(b[i], uscale);
        const float inv = rms_inv(sumsq(b), I, eps);
        const float4 *gm4 = reinterpret_cast<const float4 *>(ugamma);
#pragma unroll
        for (int i = 0; i < NV; i++) b[i] = norm4(b[i], inv, __ldg(gm4 + lane + 32 * i));
    }
    float4 h[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float4 a = g4[lane + 32 * i];
        h[i] = make_float4(__fmul_rn(gelu_tanh(a.x), b[i].x), __fmul_rn(gelu_tanh(a.y), b[i].y),
                           __fmul_rn(gelu_tanh(a.z), b[i].z), __fmul_rn(gelu_tanh(a.w), b[i].w));
    }
    quantize_row(h, ablk, I, q + (size_t)row * I, qs + (size_t)row * (I / ablk), lane);
}

int check(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        e2c_set_msg("%s launch: %s", what, cudaGetErrorString(e));
        return -2;
    }
    return 0;
}

bool ablk_ok(int ablk, int D) { return ablk == 128 || ablk == D; }

}  // namespace

#define E2C_TT_SWITCH(NV, CALL, WHAT)                                                              \
    switch (NV) {                                                                                  \
    case 1: { constexpr int V = 1; CALL; } break;                                                  \
    case 2: { constexpr int V = 2; CALL; } break;                                                  \
    case 4: { constexpr int V = 4; CALL; } break;                                                  \
    case 6: { constexpr int V = 6; CALL; } break;                                                  \
    case 8: { constexpr int V = 8; CALL; } break;                                                  \
    case 16: { constexpr int V = 16; CALL; } break;                                                \
    default: e2c_set_msg("%s: row width %d not supported (128 x 1, 2, 4, 6, 8, 16)", WHAT, 128 * (NV)); return -1; \
    }

extern "C" int e2c_tt_embed(const int32_t *ids, const uint16_t *table, float embed_scale, const float *gamma, float eps,
                            float *res, int8_t *qx, float *qxs, int8_t *qn, float *qns, int M, int D, int ablk, int vocab,
                            int *status, void *stream) {
    if (D % 128 || D > 1024 || !ablk_ok(ablk, D)) {
        e2c_set_msg("tt_embed: D=%d must be a multiple of 128 up to 1024, ablk 128 or D", D);
        return -1;
    }
    if (M <= 0) return 0;
    const dim3 grid((M + 7) / 8), block(256);
    cudaStream_t st = (cudaStream_t)stream;
    E2C_TT_SWITCH(D / 128, (e2c_launch(k_tt_embed<V>, grid, block, 0, st, ids, table, embed_scale, gamma, eps, res, qx, qxs,
                                       qn, qns, M, ablk, vocab, status)),
                  "tt_embed");
    return check("tt_embed");
}

extern "C" int e2c_tt_qkv_post(const float *y, int ldy, int H, int KV, int D, const float *q_gamma, const float *k_gamma,
                               float eps, const float *rope_cos, const float *rope_sin, int ldrope, int rope_pos_major,
                               int seq_len, void *q_out,
                               void *k_out, void *vt_out, int ldvt, int M, void *stream) {
    if ((D != 256 && D != 512) || H <= 0 || KV <= 0 || KV * D > 512 || ldy % 4 || ldy < D * (H + 2 * KV) || seq_len <= 0 ||
        M % seq_len || ldvt < seq_len || ldvt % 8 || (rope_pos_major ? ldrope < D / 2 || ldrope % 4 : ldrope < seq_len)) {
        e2c_set_msg("tt_qkv_post: bad geometry (D=%d H=%d KV=%d ldy=%d seq_len=%d ldrope=%d ldvt=%d M=%d; KV D <= 512, "
                    "ldvt a multiple of 8)", D, H, KV, ldy, seq_len, ldrope, ldvt, M);
        return -1;
    }
    if (M <= 0) return 0;
    const int ntiles = (seq_len + QKV_TILE - 1) / QKV_TILE;
    const dim3 grid((unsigned)((M / seq_len) * ntiles)), block(256);
    const size_t smem = (size_t)QKV_TILE * (KV * D + 2) * 2;
    cudaStream_t st = (cudaStream_t)stream;
    if (D == 256)
        e2c_launch(k_tt_qkv_post<1>, grid, block, smem, st, y, ldy, H, KV, q_gamma, k_gamma, eps, rope_cos, rope_sin, ldrope,
                   rope_pos_major, seq_len, ntiles, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)k_out, (__nv_bfloat16 *)vt_out, ldvt);
    else
        e2c_launch(k_tt_qkv_post<2>, grid, block, smem, st, y, ldy, H, KV, q_gamma, k_gamma, eps, rope_cos, rope_sin, ldrope,
                   rope_pos_major, seq_len, ntiles, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)k_out, (__nv_bfloat16 *)vt_out, ldvt);
    return check("tt_qkv_post");
}

extern "C" int e2c_tt_norm_add(const float *t, float *res, const float *g1, float layer_scalar, const float *g2, float eps,
                               int8_t *q, float *qs, int M, int D, int ablk, void *stream) {
    if (D % 128 || D > 1024 || !ablk_ok(ablk, D)) {
        e2c_set_msg("tt_norm_add: D=%d must be a multiple of 128 up to 1024, ablk 128 or D", D);
        return -1;
    }
    if (M <= 0) return 0;
    const dim3 grid((M + 7) / 8), block(256);
    cudaStream_t st = (cudaStream_t)stream;
    E2C_TT_SWITCH(D / 128, (e2c_launch(k_tt_norm_add<V>, grid, block, 0, st, t, res, g1, layer_scalar, g2, eps, q, qs, M, ablk)),
                  "tt_norm_add");
    return check("tt_norm_add");
}

extern "C" int e2c_tt_gate_quant(const float *g, int ldg, const float *u, int ldu, float uscale, const float *ugamma,
                                 float eps, int I, int8_t *q, float *qs, int M, int ablk, void *stream) {
    if (I % 128 || I > 2048 || ldg % 4 || ldu % 4 || ldg < I || !ablk_ok(ablk, I)) {
        e2c_set_msg("tt_gate_quant: I=%d must be a multiple of 128 up to 2048 (ldg %d, ldu %d), ablk 128 or I", I, ldg, ldu);
        return -1;
    }
    if (M <= 0) return 0;
    const dim3 grid((M + 7) / 8), block(256);
    cudaStream_t st = (cudaStream_t)stream;
    const int D = I;
    E2C_TT_SWITCH(D / 128, (e2c_launch(k_tt_gate_quant<V>, grid, block, 0, st, g, ldg, u, ldu, uscale, ugamma, eps, q, qs,
                                       M, ablk)),
                  "tt_gate_quant");
    return check("tt_gate_quant");
}
