// devstate.cuh — launch state kept per CUDA device (host side, C++).
//
// A kernel's shared-memory opt-in (cudaFuncSetAttribute), an occupancy answer and the SM count all
// belong to one device: a process that drives two GPUs from one thread (cudaSetDevice between
// calls) must set the opt-in on each device before launching there. Launchers therefore keep such
// state in arrays indexed by the current device. Writes race only between threads that compute the
// same answer for the same device, so plain relaxed atomics suffice.
#pragma once
#include <cuda_runtime.h>

constexpr int E2C_MAX_DEV = 64;

// the current device, or -1 when there is none (or its index is past E2C_MAX_DEV)
inline int e2c_device() {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= E2C_MAX_DEV) return -1;
    return d;
}

// SM count of device `dev` (0 on failure), looked up once per device
inline int e2c_sm_count(int dev) {
    static int n[E2C_MAX_DEV];
    if (dev < 0 || dev >= E2C_MAX_DEV) return 0;
    int v = __atomic_load_n(&n[dev], __ATOMIC_RELAXED);
    if (v > 0) return v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
        cudaGetLastError();
        return 0;
    }
    __atomic_store_n(&n[dev], v, __ATOMIC_RELAXED);
    return v;
}

// a per-device flag or value: get(dev) / set(dev, v)
struct E2cPerDev {
    int v[E2C_MAX_DEV];
    int get(int dev) const { return __atomic_load_n(&v[dev], __ATOMIC_RELAXED); }
    void set(int dev, int x) { __atomic_store_n(&v[dev], x, __ATOMIC_RELAXED); }
};
