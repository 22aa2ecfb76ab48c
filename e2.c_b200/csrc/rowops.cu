// rowops.cu — the encoder's row passes between GEMMs, each one warp per token row.
//
//   embed gather -> norm_split -> quantise           src/text.c:917-921, 944 (+ quant :321-339)
//   norm_add -> norm_split -> quantise              src/text.c:947,950 (o_proj / down tails)
//   masked mean pool, L2 normalise                   src/kernels.c:22-39, src/text.c:963-981
//   per-128-block activation mode (the reference engine's default recipe, src/int8.h:61-70), where
//   the GEMM epilogues that need whole-row per-token scales cannot run:
//     q|k|v fp32 -> per-head RMSNorm -> RoPE -> bf16 Q, K, V^T   src/text.c:835-856
//     gate|up fp32 -> GELU-tanh(gate) * up -> quantise           gate_quant, src/text.c:424-468
//
// RMSNorm is the reference's x * (1/sqrt(mean(x^2) + eps)) * gamma (src/kernels.c:76-87,144-171);
// the sum of squares runs in a different order than the reference's 16-lane AVX-512 sum, so normed
// values agree to a few ulp and the bytes quantised from them are compared teacher-forced.
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

template <int NV>
__global__ void __launch_bounds__(256) k_embed_norm_quant(const int32_t *__restrict__ ids, const int8_t *__restrict__ table,
                                                          const float *__restrict__ tscale, float escale,
                                                          const float *__restrict__ gamma, float eps, float *__restrict__ res,
                                                          int8_t *__restrict__ q, float *__restrict__ qs, int M, int ablk,
                                                          int vocab, int *status) {
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
    const float ts = __ldg(tscale + id);
    const char4 *tr = reinterpret_cast<const char4 *>(table + (size_t)id * D);
    float4 x[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const char4 c = __ldg(tr + lane + 32 * i);
        x[i] = make_float4(__fmul_rn(__fmul_rn((float)c.x, ts), escale), __fmul_rn(__fmul_rn((float)c.y, ts), escale),
                           __fmul_rn(__fmul_rn((float)c.z, ts), escale), __fmul_rn(__fmul_rn((float)c.w, ts), escale));
        reinterpret_cast<float4 *>(res + (size_t)row * D)[lane + 32 * i] = x[i];
    }
    const float inv = rms_inv(sumsq(x), D, eps);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
#pragma unroll
    for (int i = 0; i < NV; i++) x[i] = norm4(x[i], inv, __ldg(g4 + lane + 32 * i));
    quantize_row(x, ablk, D, q + (size_t)row * D, qs + (size_t)row * (D / ablk), lane);
}

template <int NV>
__global__ void __launch_bounds__(256) k_norm_add_norm_quant(const float *__restrict__ t, float *__restrict__ res,
                                                             const float *__restrict__ g1, const float *__restrict__ g2,
                                                             const float *__restrict__ gf, float eps, int8_t *__restrict__ q,
                                                             float *__restrict__ qs, int M, int ablk) {
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
        v[i] = make_float4(__fadd_rn(n.x, r.x), __fadd_rn(n.y, r.y), __fadd_rn(n.z, r.z), __fadd_rn(n.w, r.w));
    }
    const float inv2 = rms_inv(sumsq(v), D, eps);
    if (g2) {
        const float4 *g24 = reinterpret_cast<const float4 *>(g2);
#pragma unroll
        for (int i = 0; i < NV; i++) {
            r4[lane + 32 * i] = v[i];
            v[i] = norm4(v[i], inv2, __ldg(g24 + lane + 32 * i));
        }
        quantize_row(v, ablk, D, q + (size_t)row * D, qs + (size_t)row * (D / ablk), lane);
    } else {
        const float4 *gf4 = reinterpret_cast<const float4 *>(gf);
#pragma unroll
        for (int i = 0; i < NV; i++) r4[lane + 32 * i] = norm4(v[i], inv2, __ldg(gf4 + lane + 32 * i));
    }
}

template <int NV>
__global__ void __launch_bounds__(256) k_norm_quant(const float *__restrict__ x, const float *__restrict__ gamma, float eps,
                                                    int8_t *__restrict__ q, float *__restrict__ qs, int M, int ablk) {
    griddep_launch_dependents();
    griddep_wait();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= M) return;
    constexpr int D = NV * 128;
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)row * D);
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) v[i] = x4[lane + 32 * i];
    const float inv = rms_inv(sumsq(v), D, eps);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
#pragma unroll
    for (int i = 0; i < NV; i++) v[i] = norm4(v[i], inv, __ldg(g4 + lane + 32 * i));
    quantize_row(v, ablk, D, q + (size_t)row * D, qs + (size_t)row * (D / ablk), lane);
}

__global__ void k_meanpool(const float *__restrict__ x, const uint8_t *__restrict__ valid, float *__restrict__ out,
                           int S, int D) {
    griddep_launch_dependents();
    griddep_wait();
    const int b = blockIdx.y, d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= D) return;
    float s = 0.f;
    int cnt = 0;
    for (int i = 0; i < S; i++) {
        if (valid && !valid[(size_t)b * S + i]) continue;
        s = __fadd_rn(s, x[((size_t)b * S + i) * D + d]);
        cnt++;
    }
    out[(size_t)b * D + d] = cnt > 0 ? __fdiv_rn(s, (float)cnt) : 0.f;
}

__global__ void k_l2norm_rows(float *__restrict__ y, const uint8_t *__restrict__ valid, int B, int S, int D) {
    griddep_launch_dependents();
    griddep_wait();
    const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (b >= B) return;
    float *r = y + (size_t)b * D;
    int any = 1;
    if (valid) {
        any = 0;
        for (int i = lane; i < S; i += 32) any |= valid[(size_t)b * S + i] != 0;
        any = __any_sync(0xffffffffu, any);
    }
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s = __fmaf_rn(r[d], r[d], s);
    s = warp_sum(s);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(s));
    for (int d = lane; d < D; d += 32) r[d] = any ? __fmul_rn(r[d], inv) : 0.f;
}

// One warp per token row of the gate|up GEMM's fp32 output, columns interleaved per 128
// ([g 0..127 | u 0..127 | g 128..255 | ...]): h = gelu_tanh(g) * u with the GELU epilogue's element
// function, then the per-row quantiser of h (per 128-block or per token).
template <int NV>
__global__ void __launch_bounds__(256) k_gelu_mul_quant(const float *__restrict__ y, int ldy, int8_t *__restrict__ q,
                                                        float *__restrict__ qs, int M, int ablk) {
    griddep_launch_dependents();
    griddep_wait();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= M) return;
    constexpr int I = NV * 128;
    const float4 *src = reinterpret_cast<const float4 *>(y + (size_t)row * ldy);
    float4 h[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float4 g = src[64 * i + lane], u = src[64 * i + 32 + lane];
        h[i] = make_float4(__fmul_rn(gelu_tanh(g.x), u.x), __fmul_rn(gelu_tanh(g.y), u.y), __fmul_rn(gelu_tanh(g.z), u.z),
                           __fmul_rn(gelu_tanh(g.w), u.w));
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

}  // namespace

#define E2C_NV_SWITCH(NV, CALL)                                                            \
    switch (NV) {                                                                          \
    case 1: { constexpr int V = 1; CALL; } break;                                          \
    case 2: { constexpr int V = 2; CALL; } break;                                          \
    case 4: { constexpr int V = 4; CALL; } break;                                          \
    case 6: { constexpr int V = 6; CALL; } break;                                          \
    case 8: { constexpr int V = 8; CALL; } break;                                          \
    default: e2c_set_msg("row kernels: hidden size %d not supported (128, 256, 512, 768, 1024)", D); return -1; \
    }

extern "C" int e2c_embed_norm_quant(const int32_t *ids, const int8_t *table, const float *table_scale, float embed_scale,
                                    const float *gamma, float eps, float *res, int8_t *q, float *qs, int M, int D,
                                    int ablk, int vocab, int *status, void *stream) {
    if (D % 128 || (ablk != 128 && ablk != D)) {
        e2c_set_msg("embed_norm_quant: D=%d must be a multiple of 128, ablk 128 or D", D);
        return -1;
    }
    if (M <= 0) return 0;
    const dim3 grid((M + 7) / 8), block(256);
    cudaStream_t st = (cudaStream_t)stream;
    E2C_NV_SWITCH(D / 128, (e2c_launch(k_embed_norm_quant<V>, grid, block, 0, st, ids, table, table_scale, embed_scale, gamma, eps,
                                                      res, q, qs, M, ablk, vocab, status)));
    return check("embed_norm_quant");
}

extern "C" int e2c_norm_add_norm_quant(const float *t, float *res, const float *g1, const float *g2, const float *gfinal,
                                       float eps, int8_t *q, float *qs, int M, int D, int ablk, void *stream) {
    if (D % 128 || (ablk != 128 && ablk != D)) {
        e2c_set_msg("norm_add_norm_quant: D=%d must be a multiple of 128, ablk 128 or D", D);
        return -1;
    }
    if (M <= 0) return 0;
    const dim3 grid((M + 7) / 8), block(256);
    cudaStream_t st = (cudaStream_t)stream;
    E2C_NV_SWITCH(D / 128, (e2c_launch(k_norm_add_norm_quant<V>, grid, block, 0, st, t, res, g1, g2, gfinal, eps, q, qs, M, ablk)));
    return check("norm_add_norm_quant");
}

extern "C" int e2c_norm_quant(const float *x, const float *gamma, float eps, int8_t *q, float *qs, int M, int D,
                              int ablk, void *stream) {
    if (D % 128 || (ablk != 128 && ablk != D)) {
        e2c_set_msg("norm_quant: D=%d must be a multiple of 128, ablk 128 or D", D);
        return -1;
    }
    if (M <= 0) return 0;
    const dim3 grid((M + 7) / 8), block(256);
    cudaStream_t st = (cudaStream_t)stream;
    E2C_NV_SWITCH(D / 128, (e2c_launch(k_norm_quant<V>, grid, block, 0, st, x, gamma, eps, q, qs, M, ablk)));
    return check("norm_quant");
}

extern "C" int e2c_meanpool(const float *x, const uint8_t *valid, float *pooled, int B, int S, int D, void *stream) {
    if (B <= 0) return 0;
    const dim3 grid((D + 127) / 128, B), block(128);
    e2c_launch(k_meanpool, grid, block, 0, (cudaStream_t)stream, x, valid, pooled, S, D);
    return check("meanpool");
}

extern "C" int e2c_l2norm_rows(float *y, const uint8_t *valid, int B, int S, int D, void *stream) {
    if (B <= 0) return 0;
    e2c_launch(k_l2norm_rows, dim3((B + 7) / 8), dim3(256), 0, (cudaStream_t)stream, y, valid, B, S, D);
    return check("l2norm_rows");
}

extern "C" int e2c_qkv_post(const float *y, int ldy, int nq, const float *q_gamma, const float *k_gamma, float eps,
                            const float *rope_cos, const float *rope_sin, int ldrope, int seq_len, void *q_out,
                            void *k_out, void *vt_out, int ldvt, int M, void *stream) {
    // nq q heads, one k and one v head of 256: the text tower's finish with KV = 1 (text_rows.cu)
    return e2c_tt_qkv_post(y, ldy, nq, 1, 256, q_gamma, k_gamma, eps, rope_cos, rope_sin, ldrope, 0, seq_len, q_out,
                           k_out, vt_out, ldvt, M, stream);
}

extern "C" int e2c_gelu_mul_quant(const float *y, int ldy, int I, int8_t *q, float *qs, int M, int ablk, void *stream) {
    if (I % 128 || ldy % 4 || ldy < 2 * I || (ablk != 128 && ablk != I)) {
        e2c_set_msg("gelu_mul_quant: I=%d must be a multiple of 128 (ldy %d >= 2 I), ablk 128 or I", I, ldy);
        return -1;
    }
    if (M <= 0) return 0;
    const dim3 grid((M + 7) / 8), block(256);
    cudaStream_t st = (cudaStream_t)stream;
    switch (I / 128) {
#define E2C_GMQ(NV) case NV: e2c_launch(k_gelu_mul_quant<NV>, grid, block, 0, st, y, ldy, q, qs, M, ablk); break;
        E2C_GMQ(1) E2C_GMQ(2) E2C_GMQ(3) E2C_GMQ(4) E2C_GMQ(6) E2C_GMQ(8) E2C_GMQ(9) E2C_GMQ(12) E2C_GMQ(16)
#undef E2C_GMQ
    default: e2c_set_msg("gelu_mul_quant: I=%d not supported (128 x 1, 2, 3, 4, 6, 8, 9, 12, 16)", I); return -1;
    }
    return check("gelu_mul_quant");
}
