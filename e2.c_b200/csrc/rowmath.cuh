// rowmath.cuh — warp-per-row arithmetic shared by the row kernels (rowops.cu, text_rows.cu): sums
// and maxima over a warp, the reference's RMSNorm factor, and the activation quantiser of one row
// held in registers (lane l holds float4 number l + 32 i of the row).
#pragma once
#include <stdint.h>

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

}  // namespace
