// pdl.h — kernel launches with programmatic dependent launch (host side, C++).
//
// Every e2cuda kernel passes griddep_wait() (ptx.cuh) before it touches global memory that earlier
// kernels of its stream read or write, so each may be launched with the programmatic-serialization
// attribute: its CTAs are scheduled onto SMs the previous kernel's last CTAs leave, and its set-up
// (barriers, TMEM, tensor-map prefetch) overlaps that kernel's tail. Measured on the encoder's
// CUDA-graph pass it gained nothing (9.13 ms with, 9.02 ms without), so launches use plain stream
// order unless E2C_PDL=1 is set in the environment.
#pragma once
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <utility>

inline bool e2c_pdl_on() {
    static int on = -1;
    if (on < 0) {
        const char *v = getenv("E2C_PDL");
        on = v && v[0] == '1';
    }
    return on != 0;
}

// Appends the attribute to attrs[n] when enabled; returns the new count.
inline unsigned e2c_pdl_attr(cudaLaunchAttribute *attrs, unsigned n) {
    if (!e2c_pdl_on()) return n;
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    return n + 1;
}

// kern<<<grid, block, smem, st>>>(args...) with the attribute
template <typename... KArgs, typename... Args>
inline cudaError_t e2c_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attrs[1];
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attrs;
    cfg.numAttrs = e2c_pdl_attr(attrs, 0);
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
