// rowops.cu — the encoder's row passes between GEMMs, each one warp per token row.
//
//   embed gather -> norm_split -> quantise           src/text.c:917-921, 944 (+ quant :321-339)
//   norm_add -> norm_split -> quantise              src/text.c:947,950 (o_proj / down tails)
//   masked mean pool, L2 normalise                   src/kernels.c:22-39, src/text.c:963-981
//
// RMSNorm is the reference's x * (1/sqrt(mean(x^2) + eps)) * gamma (src/kernels.c:76-87,144-171);
// the sum of squares runs in a different order than the reference's 16-lane AVX-512 sum, so normed
// values agree to a few ulp and the bytes quantised from them are compared teacher-forced.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "launch.h"
#include "pdl.h"
#include "ptx.cuh"

namespace {

constexpr float kInv127 = 0x1.020408p-7f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float rms_inv(float ss, int D, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
}
__device__ __forceinline__ int qround(float v, float inv) {
    int r = __float2int_rn(__fmul_rn(v, inv));
    return r > 127 ? 127 : (r < -127 ? -127 : r);
}

// Lane l holds float4 number l + 32 i of the row (i < NV): D = 128 * NV. With ablk == 128 the
// i-th float4 group of the warp is exactly activation block i.
template <int NV>
__device__ __forceinline__ void quantize_row(const float4 (&v)[NV], int ablk, int D, int8_t *q, float *qs, int lane) {
    float am[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) am[i] = fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w)));
    if (ablk == D) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) a = fmaxf(a, am[i]);
        a = warp_max(a);
#pragma unroll
        for (int i = 0; i < NV; i++) am[i] = a;
        if (lane == 0) qs[0] = a > 0.f ? __fmul_rn(a, kInv127) : 1.0f;
    } else {  // ablk == 128
#pragma unroll
        for (int i = 0; i < NV; i++) {
            am[i] = warp_max(am[i]);
            if (lane == 0) qs[i] = am[i] > 0.f ? __fmul_rn(am[i], kInv127) : 1.0f;
        }
    }
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float inv = am[i] > 0.f ? __fdiv_rn(127.0f, am[i]) : 1.0f;
        const int a = qround(v[i].x, inv), b = qround(v[i].y, inv), c = qround(v[i].z, inv), d = qround(v[i].w, inv);
        reinterpret_cast<uint32_t *>(q)[lane + 32 * i] =
            ((uint32_t)a & 0xffu) | (((uint32_t)b & 0xffu) << 8) | (((uint32_t)c & 0xffu) << 16) | (((uint32_t)d & 0xffu) << 24);
    }
}

template <int NV>
__device__ __forceinline__ float sumsq(const float4 (&v)[NV]) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        s = __fmaf_rn(v[i].x, v[i].x, s);
        s = __fmaf_rn(v[i].y, v[i].y, s);
        s = __fmaf_rn(v[i].z, v[i].z, s);
        s = __fmaf_rn(v[i].w, v[i].w, s);
    }
    return warp_sum(s);
}

__device__ __forceinline__ float4 norm4(float4 x, float inv, float4 g) {
    return make_float4(__fmul_rn(__fmul_rn(x.x, inv), g.x), __fmul_rn(__fmul_rn(x.y, inv), g.y),
                       __fmul_rn(__fmul_rn(x.z, inv), g.z), __fmul_rn(__fmul_rn(x.w, inv), g.w));
}

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
