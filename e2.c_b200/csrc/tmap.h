// tmap.h — TMA tensor-map construction (host side).
#pragma once
#include <cuda.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// 2D row-major tensor: `inner` elements per row (contiguous), `outer` rows `row_stride` bytes apart,
// copied in boxes of box_inner x box_outer elements with the 128-byte swizzle (box_inner * elem must
// be 128 bytes) and zero fill outside the tensor. Returns 0, or -1 with a message in e2c_msg().
int e2c_tmap_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer);
// The same with the 64-byte swizzle (box_inner * elem must be 64 bytes).
int e2c_tmap_2d_sw64(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                     uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer);
// The same with the 32-byte swizzle (box_inner * elem must be 32 bytes).
int e2c_tmap_2d_sw32(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                     uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer);
// Without swizzle: row-major boxes (box_inner * elem a multiple of 16 bytes).
int e2c_tmap_2d_plain(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                      uint64_t outer, uint64_t row_stride, uint32_t box_inner, uint32_t box_outer);

#ifdef __cplusplus
}
#endif
