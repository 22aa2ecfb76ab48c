// quant.cu — the activation quantiser on sm_100a: one warp per token row, warp-shuffle absmax,
// 16-byte stores.
//
// Semantics of the reference quantiser (src/int8.c:178-209, src/kernels_i8_avx512_vnni.c:312-366)
// as its -ffast-math build computes them: per block amax over |clamp(x)|, scale = amax * fl(1/127)
// (1 for an all-zero block), q = saturate_127(rint(x * fl(127 / amax))).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "launch.h"
#include "devstate.cuh"
#include "pdl.h"
#include "ptx.cuh"

namespace {

constexpr float kInv127 = 0x1.020408p-7f;  // fl(1/127)

__device__ __forceinline__ float clampv(float v, float lo, float hi, bool clamp) {
    return clamp ? (v < lo ? lo : (v > hi ? hi : v)) : v;
}
// |v| <= amax, so |v * fl(127/amax)| <= 127 (to within a rounding that rint absorbs): no saturation
__device__ __forceinline__ int qround(float v, float inv) { return __float2int_rn(__fmul_rn(v, inv)); }
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d, uint32_t bias) {
    return ((((uint32_t)a & 0xffu) | (((uint32_t)b & 0xffu) << 8) | (((uint32_t)c & 0xffu) << 16) |
             (((uint32_t)d & 0xffu) << 24)) ^
            bias);
}

// 16 consecutive elements of one lane -> one 16-byte store
__device__ __forceinline__ void quant16(const float (&v)[16], float inv, int8_t *dst, uint32_t bias) {
    int q[16];
#pragma unroll
    for (int i = 0; i < 16; i++) q[i] = qround(v[i], inv);
    uint4 o;
    o.x = pack4(q[0], q[1], q[2], q[3], bias);
    o.y = pack4(q[4], q[5], q[6], q[7], bias);
    o.z = pack4(q[8], q[9], q[10], q[11], bias);
    o.w = pack4(q[12], q[13], q[14], q[15], bias);
    *reinterpret_cast<uint4 *>(dst) = o;
}

__device__ __forceinline__ void load16(const float *src, float (&v)[16], float lo, float hi, bool clamp,
                                       float &amax) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 f = __ldg(s4 + i);
        v[4 * i + 0] = clampv(f.x, lo, hi, clamp);
        v[4 * i + 1] = clampv(f.y, lo, hi, clamp);
        v[4 * i + 2] = clampv(f.z, lo, hi, clamp);
        v[4 * i + 3] = clampv(f.w, lo, hi, clamp);
    }
#pragma unroll
    for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(v[i]));
}

// Blocks of G*16 elements (G a power of two <= 32 lanes): each warp pass covers 512 elements, one
// 16-element group per lane, G lanes per block reducing with xor-shuffles.
template <int G>
__global__ void __launch_bounds__(256) k_quant_small(const float *__restrict__ x, int ldx, int8_t *__restrict__ q,
                                                     int ldq, float *__restrict__ scales, int M, int K,
                                                     float lo, float hi, int clamp, uint32_t bias) {
    griddep_launch_dependents();
    griddep_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float *xr = x + (size_t)warp * ldx;
    int8_t *qr = q + (size_t)warp * ldq;
    const int nb = K / (G * 16);
    for (int k0 = 0; k0 < K; k0 += 512) {
        const int k = k0 + lane * 16;
        const bool active = k < K;  // K is a multiple of the block, so whole blocks are active
        float v[16];
        float amax = 0.f;
        if (active) load16(xr + k, v, lo, hi, clamp != 0, amax);
#pragma unroll
        for (int o = G / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (active) {
            const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 1.0f;
            quant16(v, inv, qr + k, bias);
            if ((lane & (G - 1)) == 0) scales[(size_t)warp * nb + k / (G * 16)] = amax > 0.f ? __fmul_rn(amax, kInv127) : 1.0f;
        }
    }
}

// Blocks of any multiple of 16 elements (per-row mode: the block is the whole row). Groups of 16
// are strided over the lanes; a lane holds at most REG groups (REG = ceil(groups / 32), so the whole
// block stays in registers and x is read once). |x * 127/amax| <= 127 for every x of the block, so
// the conversion needs no saturation.
template <int REG, bool CLAMP>
__global__ void __launch_bounds__(256) k_quant_wide(const float *__restrict__ x, int ldx, int8_t *__restrict__ q,
                                                    int ldq, float *__restrict__ scales, int M, int K, int ablk,
                                                    float lo, float hi, uint32_t bias) {
    griddep_launch_dependents();
    griddep_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float *xr = x + (size_t)warp * ldx;
    int8_t *qr = q + (size_t)warp * ldq;
    const int nb = K / ablk, ng = ablk / 16;
    for (int b = 0; b < nb; b++) {
        const int kb = b * ablk;
        float v[REG][16];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < REG; i++) {
            const int g = lane + 32 * i;
            if (g < ng) load16(xr + kb + 16 * g, v[i], lo, hi, CLAMP, amax);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 1.0f;
#pragma unroll
        for (int i = 0; i < REG; i++) {
            const int g = lane + 32 * i;
            if (g < ng) quant16(v[i], inv, qr + kb + 16 * g, bias);
        }
        if (lane == 0) scales[(size_t)warp * nb + b] = amax > 0.f ? __fmul_rn(amax, kInv127) : 1.0f;
    }
}

// Per-token mode, K = 128 NV: lane l holds the float4s l, l + 32, ... of a row (every lane busy, one
// coalesced 4-byte store per float4), and each warp walks rows with the next row's loads in flight
// while it quantises the current one. Bit-identical to k_quant_wide (the maximum does not depend on
// the order it is taken in; each element's arithmetic is the same).
template <int NV>
__global__ void __launch_bounds__(256) k_quant_rows(const float *__restrict__ x, int ldx, int8_t *__restrict__ q, int ldq,
                                                    float *__restrict__ scales, int M, uint32_t bias) {
    griddep_launch_dependents();
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int nw = (int)((gridDim.x * blockDim.x) >> 5);
    int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    float4 v[NV], nx[NV];
    auto load = [&](int row, float4 (&d)[NV]) {
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)row * ldx);
#pragma unroll
        for (int i = 0; i < NV; i++) d[i] = __ldcs(src + lane + 32 * i);
    };
    if (r < M) load(r, v);
    for (; r < M; r += nw) {
        if (r + nw < M) load(r + nw, nx);
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++)
            amax = fmaxf(fmaxf(fmaxf(amax, fabsf(v[i].x)), fmaxf(fabsf(v[i].y), fabsf(v[i].z))), fabsf(v[i].w));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 1.0f;
        uint32_t *dst = reinterpret_cast<uint32_t *>(q + (size_t)r * ldq);
#pragma unroll
        for (int i = 0; i < NV; i++)
            dst[lane + 32 * i] = pack4(qround(v[i].x, inv), qround(v[i].y, inv), qround(v[i].z, inv), qround(v[i].w, inv), bias);
        if (lane == 0) scales[r] = amax > 0.f ? __fmul_rn(amax, kInv127) : 1.0f;
#pragma unroll
        for (int i = 0; i < NV; i++) v[i] = nx[i];
    }
}

__global__ void k_flip_bias(uint32_t *q, size_t n4) {
    griddep_launch_dependents();
    griddep_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
        q[i] ^= 0x80808080u;
}

}  // namespace

extern "C" int e2c_flip_bias(int8_t *q, size_t n, void *stream) {
    if (((uintptr_t)q & 3) || (n & 3)) {
        e2c_set_msg("flip_bias: 4-byte aligned, length a multiple of 4");
        return -1;
    }
    if (!n) return 0;
    const size_t n4 = n / 4;
    const unsigned grid = (unsigned)((n4 + 255) / 256 < 4096 ? (n4 + 255) / 256 : 4096);
    e2c_launch(k_flip_bias, dim3(grid), dim3(256), 0, (cudaStream_t)stream, reinterpret_cast<uint32_t *>(q), n4);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        e2c_set_msg("flip_bias launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}

extern "C" int e2c_quantize(const float *x, int ldx, int8_t *q, int ldq, float *scales, int M, int K, int ablk,
                            float lo, float hi, int biased, void *stream) {
    if (M < 0 || K <= 0 || ablk <= 0 || K % ablk || ablk % 16) {
        e2c_set_msg("quantize: K=%d must be a multiple of ablk=%d, itself a multiple of 16", K, ablk);
        return -1;
    }
    if (((uintptr_t)x | (uintptr_t)q) & 15 || ldx % 4 || ldq % 16) {
        e2c_set_msg("quantize: x and q must be 16-byte aligned with 16-byte row strides");
        return -1;
    }
    if (M == 0) return 0;
    const int clamp = lo > -INFINITY || hi < INFINITY;
    const uint32_t bias = biased ? 0x80808080u : 0u;
    cudaStream_t st = (cudaStream_t)stream;
    const dim3 block(256), grid((unsigned)((M + 7) / 8));
    const int g = ablk / 16;
    if (ablk == K && K % 128 == 0 && K / 128 <= 9 && !clamp) {
        // per-token rows of 128 NV: persistent warps, as many CTAs as the SMs hold at once
        // blocks per SM depend only on the kernel's resources and the architecture (this library
        // holds sm_100a code only), so they are kept once; the SM count is the current device's
        static int resident[10] = { 0 };
        int sms = e2c_sm_count(e2c_device());
        if (sms <= 0) sms = 148;
        const int nv = K / 128;
        if (!resident[nv]) {
            const void *fn = nv == 1 ? (const void *)k_quant_rows<1> : nv == 2 ? (const void *)k_quant_rows<2>
                           : nv == 3 ? (const void *)k_quant_rows<3> : nv == 4 ? (const void *)k_quant_rows<4>
                           : nv == 5 ? (const void *)k_quant_rows<5> : nv == 6 ? (const void *)k_quant_rows<6>
                           : nv == 7 ? (const void *)k_quant_rows<7> : nv == 8 ? (const void *)k_quant_rows<8>
                                     : (const void *)k_quant_rows<9>;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident[nv], fn, 256, 0) != cudaSuccess || resident[nv] <= 0)
                resident[nv] = 1;
        }
        const long cap = (long)resident[nv] * sms;
        const unsigned rg = (unsigned)((M + 7) / 8 < cap ? (M + 7) / 8 : cap);
#define E2C_QR(NV) e2c_launch(k_quant_rows<NV>, dim3(rg), block, 0, st, x, ldx, q, ldq, scales, M, bias)
        switch (K / 128) {
        case 1: E2C_QR(1); break;
        case 2: E2C_QR(2); break;
        case 3: E2C_QR(3); break;
        case 4: E2C_QR(4); break;
        case 5: E2C_QR(5); break;
        case 6: E2C_QR(6); break;
        case 7: E2C_QR(7); break;
        case 8: E2C_QR(8); break;
        default: E2C_QR(9); break;
        }
#undef E2C_QR
    } else if (ablk <= 512 && (g & (g - 1)) == 0) {
        switch (g) {
        case 1: e2c_launch(k_quant_small<1>, grid, block, 0, st, x, ldx, q, ldq, scales, M, K, lo, hi, clamp, bias); break;
        case 2: e2c_launch(k_quant_small<2>, grid, block, 0, st, x, ldx, q, ldq, scales, M, K, lo, hi, clamp, bias); break;
        case 4: e2c_launch(k_quant_small<4>, grid, block, 0, st, x, ldx, q, ldq, scales, M, K, lo, hi, clamp, bias); break;
        case 8: e2c_launch(k_quant_small<8>, grid, block, 0, st, x, ldx, q, ldq, scales, M, K, lo, hi, clamp, bias); break;
        case 16: e2c_launch(k_quant_small<16>, grid, block, 0, st, x, ldx, q, ldq, scales, M, K, lo, hi, clamp, bias); break;
        default: e2c_launch(k_quant_small<32>, grid, block, 0, st, x, ldx, q, ldq, scales, M, K, lo, hi, clamp, bias); break;
        }
    } else {
        const int reg = (ablk / 16 + 31) / 32;  // groups of 16 per lane
        if (reg > 16) {
            e2c_set_msg("quantize: blocks longer than 8192 elements are not supported");
            return -1;
        }
#define E2C_QW(R)                                                                                            \
    (clamp ? e2c_launch(k_quant_wide<R, true>, grid, block, 0, st, x, ldx, q, ldq, scales, M, K, ablk, lo, hi, bias)   \
           : e2c_launch(k_quant_wide<R, false>, grid, block, 0, st, x, ldx, q, ldq, scales, M, K, ablk, lo, hi, bias))
        switch (reg) {
        case 1: E2C_QW(1); break;
        case 2: E2C_QW(2); break;
        case 3: E2C_QW(3); break;
        case 4: E2C_QW(4); break;
        case 5: case 6: E2C_QW(6); break;
        case 7: case 8: E2C_QW(8); break;
        case 9: case 10: case 11: case 12: E2C_QW(12); break;
        default: E2C_QW(16); break;  // up to 8192 per block
        }
#undef E2C_QW
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        e2c_set_msg("quantize launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}
