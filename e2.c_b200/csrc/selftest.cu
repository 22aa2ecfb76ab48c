// selftest.cu — a launcher that exercises the bounded mbarrier wait every e2cuda kernel uses.
//
// One warp initialises an mbarrier that expects one arrival and waits on its first phase with
// mbar_wait, the same bounded wait (E2C_WAIT_NS, ~2 s) the GEMM, norm, GELU and attention kernels
// use. With `arrive` set, the warp's lane 0 arrives first and the wait completes at once; without,
// nothing ever arrives, the wait gives up after its bound, records `code` in the status word and the
// kernel returns. No fault, trap or endless loop is involved: the context stays usable, which is
// what lets a test make a wait run out and read the status back through e2cuda_check.
#include <cuda_runtime.h>
#include <stdint.h>

#include "launch.h"
#include "ptx.cuh"

namespace {

__global__ void k_wait_selftest(int *status, int code, int arrive, int *completed) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t b = smem_u32(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (arrive && threadIdx.x == 0) mbar_arrive(b);
    __syncwarp();
    if (threadIdx.x == 0) *completed = mbar_wait(b, 0, status, code) ? 1 : 0;
}

}  // namespace

extern "C" int e2c_wait_selftest(int *status, int code, int arrive, int *completed, void *stream) {
    if (!status || !completed || code < E2C_ERR_WAIT_PRODUCER || code > E2C_ERR_WAIT_DRAIN) {
        e2c_set_msg("wait_selftest: a status word, a result word and a wait code 0x101..0x105");
        return -1;
    }
    k_wait_selftest<<<1, 32, 0, (cudaStream_t)stream>>>(status, code, arrive, completed);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        e2c_set_msg("wait_selftest launch: %s", cudaGetErrorString(e));
        return -2;
    }
    return 0;
}
