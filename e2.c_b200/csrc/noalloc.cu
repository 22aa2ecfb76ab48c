// noalloc.cu — e2cuda_i8_linear_noalloc: activation quantiser + W8A8 GEMM with no allocation.
//
// Some callers cannot let a library allocate device memory on their behalf:
//   - a serving process whose caching allocator (or its own arena) has already claimed the HBM it
//     will ever use, so a cudaMalloc from a library fails or fragments that pool;
//   - a latency-bound loop that must not meet cudaMalloc/cudaFree, which can block the calling
//     thread and synchronise the whole device;
//   - a host that budgets every byte of device memory up front and wants a fixed, known footprint.
// For them, the quantised activations that sit between the quantiser and the GEMM (and the status
// word the kernels report failures through) live in one file-scope __device__ array of fixed size,
// reserved with this library's device code on each GPU that loads it and held until the process
// exits. The caller passes the fp32 input, the weight and the fp32 output; nothing is allocated.
//
// Scratch layout (bytes from the array's start, which is 256-byte aligned):
//   [0, 4)                      status word of this entry point (0 = clean)
//   [256, 256 + M*K)            q, signed int8 [M][K] (row stride K, a multiple of 16)
//   [.. rounded to 256, + 4*M*K/ablk)  activation scales [M][K/ablk]
// Every byte of q and of the scales that the GEMM reads is written by the quantiser of the same
// call (rows past M and columns past K come from the tensor map's zero fill, never from the
// array), so only the status word has to start at zero: each call clears it first.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

extern "C" {
#include "internal.h"
}

namespace {

constexpr size_t kScratchBytes = E2CUDA_NOALLOC_SCRATCH_BYTES;
constexpr size_t kHeader = 256;
constexpr int kMaxDev = 64;

// the scratch itself: one copy per device, shared by every call on that device
__device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

// device address of g_noalloc_scratch per device, filled by the first call on that device (the host
// name of the array is only a stand-in for the runtime; its address is not a device address)
uint8_t *g_scratch_addr[kMaxDev];

size_t round_up(size_t x, size_t m) { return (x + m - 1) / m * m; }

// the current device's scratch address, looked up once per device with that device current
uint8_t *scratch_for_current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
        e2cu_err("i8_linear_noalloc: no CUDA device");
        return nullptr;
    }
    uint8_t *p = __atomic_load_n(&g_scratch_addr[dev], __ATOMIC_ACQUIRE);
    if (p) return p;
    const cudaError_t e = cudaGetSymbolAddress((void **)&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
        e2cu_err("i8_linear_noalloc: scratch lookup on device %d failed: %s", dev, cudaGetErrorString(e));
        return nullptr;
    }
    // racing first calls on one device look up the same address; either store is the answer
    __atomic_store_n(&g_scratch_addr[dev], p, __ATOMIC_RELEASE);
    return p;
}

}  // namespace

extern "C" int e2cuda_i8_linear_noalloc(const e2cuda_w8 *w, const float *x, int M, int ablk, float *y, int ldy,
                                        void *stream) {
    if (!w || !w->w || !w->scale || M < 0 || (M > 0 && (!x || !y)) || ldy < w->N) {
        e2cu_err("i8_linear_noalloc: bad arguments");
        return -1;
    }
    const int K = w->K;
    if (K % 16) {
        e2cu_err("i8_linear_noalloc: K (%d) must be a multiple of 16", K);
        return -1;
    }
    if (w->ld != K) {
        e2cu_err("i8_linear_noalloc: the weight's row stride (%d bytes) must equal K (%d)", w->ld, K);
        return -1;
    }
    if (ablk != K && (ablk <= 0 || ablk % 128 || K % ablk)) {
        e2cu_err("i8_linear_noalloc: ablk %d must be K (%d, per token) or a multiple of 128 dividing K", ablk, K);
        return -1;
    }
    const size_t q_bytes = (size_t)M * (size_t)K;
    const size_t s_off = round_up(kHeader + q_bytes, 256);
    const size_t need = s_off + sizeof(float) * (size_t)M * (size_t)(K / ablk);
    if (need > kScratchBytes) {
        e2cu_err("i8_linear_noalloc: M=%d K=%d ablk=%d needs %zu bytes of scratch; the maximum is %zu "
                 "(E2CUDA_NOALLOC_SCRATCH_BYTES): split the rows into smaller calls",
                 M, K, ablk, need, kScratchBytes);
        return -1;
    }
    uint8_t *scratch = scratch_for_current_device();
    if (!scratch) return -1;
    if (M == 0) return 0;

    cudaStream_t st = (cudaStream_t)stream;
    // The call ends by synchronising `stream` to read its status word. On a capturing stream that
    // would invalidate the caller's capture, so such a call is refused before anything is queued.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (e2cu_cuda(cudaStreamIsCapturing(st, &cap), "i8_linear_noalloc: capture query")) return -1;
    if (cap != cudaStreamCaptureStatusNone) {
        e2cu_err("i8_linear_noalloc: `stream` is being captured; this call synchronises its stream to read its "
                 "status, so it runs on a stream that is not capturing");
        return -1;
    }
    int *status = reinterpret_cast<int *>(scratch);
    int8_t *q = reinterpret_cast<int8_t *>(scratch + kHeader);
    float *qs = reinterpret_cast<float *>(scratch + s_off);
    if (e2cu_cuda(cudaMemsetAsync(status, 0, sizeof(int), st), "i8_linear_noalloc: status clear")) return -1;
    if (e2cu_launch(e2c_quantize(x, K, q, K, qs, M, K, ablk, -INFINITY, INFINITY, 0, stream),
                    "i8_linear_noalloc: quantize"))
        return -1;

    e2c_gemm_args a;
    memset(&a, 0, sizeof a);
    a.a = q;
    a.lda = K;
    a.a_scale = qs;
    a.w = w->w;
    a.ldw = w->ld;
    a.wrows = w->rows;
    a.w_scale = w->scale;
    a.M = M;
    a.K = K;
    a.ablk = ablk;
    a.n0 = 0;
    a.n1 = w->N;
    a.epi = E2C_EPI_F32;
    a.y = y;
    a.ldy = ldy;
    a.out_min = w->out_min;
    a.out_max = w->out_max;
    a.status = status;
    if (e2cu_launch(e2c_gemm(&a, stream), "i8_linear_noalloc: gemm")) return -1;

    // the call's own status word is in the scratch, so it is read here rather than by e2cuda_check
    int h = 0;
    if (e2cu_cuda(cudaMemcpyAsync(&h, status, sizeof h, cudaMemcpyDeviceToHost, st), "i8_linear_noalloc: status read") ||
        e2cu_cuda(cudaStreamSynchronize(st), "i8_linear_noalloc: synchronize"))
        return -1;
    if (h) {
        e2cu_err("i8_linear_noalloc: device kernel failure 0x%x", h);
        return -1;
    }
    return 0;
}
