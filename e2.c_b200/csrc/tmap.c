/* tmap.c — TMA tensor maps and the launcher message buffer (C11 host code).
 *
 * cuTensorMapEncodeTiled lives in the driver; it is fetched once through the runtime's
 * cudaGetDriverEntryPoint so the library links only the CUDA runtime. */
#include "tmap.h"

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "launch.h"

static _Thread_local char g_msg[512];

const char *e2c_msg(void) { return g_msg; }

void e2c_set_msg(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof g_msg, fmt, ap);
    va_end(ap);
}

typedef CUresult (*encode_tiled_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                    CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                    CUtensorMapFloatOOBfill);

static encode_tiled_fn get_encode(void) {
    static encode_tiled_fn fn;
    if (!fn) {
        void *p = NULL;
        enum cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !p)
            return NULL;
        fn = (encode_tiled_fn)p;
    }
    return fn;
}

static int tmap_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                   uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer, uint32_t swz) {
    encode_tiled_fn enc = get_encode();
    if (!enc) {
        e2c_set_msg("tensor map: cuTensorMapEncodeTiled unavailable");
        return -1;
    }
    if ((swz ? box_inner * (uint32_t)elem_bytes != swz : (box_inner * (uint32_t)elem_bytes) % 16 != 0) ||
        ((uintptr_t)base & 15) || (row_stride & 15)) {
        e2c_set_msg("tensor map: %u-byte boxes, 16-byte aligned base and row stride required", swz ? swz : 16);
        return -1;
    }
    const cuuint64_t dims[2] = { inner, outer };
    const cuuint64_t strides[1] = { row_stride };
    const cuuint32_t box[2] = { box_inner, box_outer };
    const cuuint32_t estr[2] = { 1, 1 };
    memset(m, 0, sizeof *m);
    const CUresult r = enc(m, dt, 2, (void *)base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swz == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                           : swz == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                           : swz == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                       : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        e2c_set_msg("tensor map: encode failed (%d) for %llu x %llu, stride %llu, box %u x %u", (int)r,
                    (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)row_stride, box_inner,
                    box_outer);
        return -1;
    }
    return 0;
}

int e2c_tmap_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer) {
    return tmap_2d(m, base, dt, elem_bytes, inner, outer, row_stride, box_inner, box_outer, 128);
}

int e2c_tmap_2d_sw64(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                     uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer) {
    return tmap_2d(m, base, dt, elem_bytes, inner, outer, row_stride, box_inner, box_outer, 64);
}

int e2c_tmap_2d_sw32(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                     uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer) {
    return tmap_2d(m, base, dt, elem_bytes, inner, outer, row_stride, box_inner, box_outer, 32);
}

int e2c_tmap_2d_plain(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                      uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer) {
    return tmap_2d(m, base, dt, elem_bytes, inner, outer, row_stride, box_inner, box_outer, 0);
}
