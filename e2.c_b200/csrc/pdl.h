// pdl.h — kernel launches with programmatic dependent launch (host side, C++).
//
// Every e2cuda kernel passes griddep_wait() (ptx.cuh) before it touches global memory that earlier
// kernels of its stream read or write, so each may be launched with the programmatic-serialization
// attribute: its CTAs are scheduled onto SMs the previous kernel's last CTAs leave, and its set-up
// (barriers, TMEM, tensor-map prefetch) overlaps that kernel's tail. Measured on the encoder's
// CUDA-graph pass it gained nothing (9.13 ms with, 9.02 ms without), so launches use plain stream
// order unless E2C_PDL=1 is set in the environment. The GEMMs for a few rows against a short weight
// are the exception: there the attribute lets the next GEMM's CTAs become resident and fetch their
// weight while the previous one finishes, which a chain of such launches gains 20-25% from; they
// carry it unless E2C_PDL_SMALL=0.
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

// the co-resident small-row GEMMs launch with the attribute (E2C_PDL_SMALL=0: only with E2C_PDL=1)
inline bool e2c_pdl_small_on() {
    static int on = -1;
    if (on < 0) {
        const char *v = getenv("E2C_PDL_SMALL");
        on = !(v && v[0] == '0');
    }
    return on != 0 || e2c_pdl_on();
}

// Appends the attribute to attrs[n] when enabled (E2C_PDL=1, or `small` for the small-row GEMMs);
// returns the new count.
inline unsigned e2c_pdl_attr(cudaLaunchAttribute *attrs, unsigned n, bool small = false) {
    if (!(small ? e2c_pdl_small_on() : e2c_pdl_on())) return n;
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    return n + 1;
}

// kern<<<grid, block, smem, st>>>(args...) with the attribute (`small`: as a small-row GEMM)
template <typename... KArgs, typename... Args>
inline cudaError_t e2c_launch_as(bool small, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args &&...args) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attrs[1];
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attrs;
    cfg.numAttrs = e2c_pdl_attr(attrs, 0, small);
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
template <typename... KArgs, typename... Args>
inline cudaError_t e2c_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
    return e2c_launch_as(false, kern, grid, block, smem, st, std::forward<Args>(args)...);
}
