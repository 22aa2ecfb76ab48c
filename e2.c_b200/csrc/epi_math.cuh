// epi_math.cuh — element functions shared by the GEMM epilogues (one definition, so fused and
// unfused paths give the same bits).
#pragma once
#include <stdint.h>

// GELU-tanh, the reference's function (src/kernels_avx512.c:46-55,186-203):
//   0.5 v (1 + tanh(c (v + 0.044715 v^3))),  c = sqrt(2/pi).
// Evaluated through the identity 0.5 (1 + tanh z) = 1 / (1 + exp(-2z)):
//   gelu(v) = v / (1 + 2^(k v (1 + 0.044715 v^2))),  k = -2 c log2(e),
// with the SFU's ex2.approx (<= 2 ulp) and rcp.approx (<= 1 ulp): about 8 instructions, no range
// clamps (ex2 saturates to 0 or +inf, and v / inf = -0 matches tanh = -1 exactly), and no
// cancellation in 1 + tanh for negative v. Within ~1e-7 relative of the reference, whose own
// -ffast-math build divides with rcp14 plus a Newton step.
__device__ __forceinline__ float ex2_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_fast(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gelu_tanh(float v) {
    const float t = __fmaf_rn(0.044715f, __fmul_rn(v, v), 1.0f);
    const float e = ex2_fast(__fmul_rn(__fmul_rn(-2.302208198144325f, v), t));
    return __fmul_rn(v, rcp_fast(__fadd_rn(1.0f, e)));
}

// the per-token quantiser's byte: rint(v) for |v| < 2^22 as the low byte of v + 1.5 2^23 (the
// addition rounds to nearest even at integer spacing), equal to __float2int_rn(v) there
__device__ __forceinline__ uint32_t rint_low_byte(float v) { return __float_as_uint(__fadd_rn(v, 12582912.0f)); }
// four such words -> four int8 bytes in memory order
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
    return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

// Two fp32 lanes per instruction (sm_100's packed f32x2 FMA pipe): each lane is the IEEE
// round-to-nearest result of the scalar operation, so these give the same bits as two __fmul_rn /
// __fmaf_rn / __fadd_rn while issuing half the instructions. A mul2_rn whose result feeds an
// add2_rn has been seen to round like one fused operation (an exact .5 tie came out 1 ulp apart),
// so no kernel here feeds a packed product into a packed add where the bits matter.
__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
    return r;
}
__device__ __forceinline__ float2 f2_from(unsigned long long r) {
    float2 v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
    return v;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_from(d);
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return f2_from(d);
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return f2_from(d);
}
// gelu_tanh of two values: lane for lane the same operations, so the same bits, as gelu_tanh
__device__ __forceinline__ float2 gelu_tanh2(float2 v) {
    const float2 t = fma2_rn(make_float2(0.044715f, 0.044715f), mul2_rn(v, v), make_float2(1.0f, 1.0f));
    const float2 a = mul2_rn(mul2_rn(make_float2(-2.302208198144325f, -2.302208198144325f), v), t);
    const float2 d = add2_rn(make_float2(1.0f, 1.0f), make_float2(ex2_fast(a.x), ex2_fast(a.y)));
    return mul2_rn(v, make_float2(rcp_fast(d.x), rcp_fast(d.y)));
}
