// Host-side TMA tensor-map encoding.  The driver entry point is resolved at
// run time through the CUDA runtime, so the library has no link-time
// dependency on libcuda and loads on machines without a GPU.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace pmb {
namespace tma {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn();

// 3-D map (inner, mid, outer) over a 16-bit tensor with 128-byte swizzle.
// Strides are in bytes for the mid and outer dimensions.  Returns a status.
int make_map_3d(CUtensorMap& map, const void* base, int dtype, uint64_t inner, uint64_t mid, uint64_t outer,
                uint64_t stride_mid_bytes, uint64_t stride_outer_bytes, uint32_t box_inner, uint32_t box_mid,
                uint32_t box_outer, const char* name);

// 4-D map (d0 innermost .. d3) over a 16-bit tensor with 128-byte swizzle;
// strides in bytes for d1..d3; out-of-range boxes read zeros.
int make_map_4d(CUtensorMap& map, const void* base, int dtype, const uint64_t (&dims)[4],
                const uint64_t (&stride_bytes)[3], const uint32_t (&box)[4], const char* name);

// Output map for TMA tile stores: a 16-bit [rows, cols] matrix with a row
// pitch of ld_bytes (a multiple of 16), box {32 columns, 32 rows}, 64-byte
// swizzle (the layout ugemm::warp_tma_store writes).
int make_store_map_2d(CUtensorMap& map, const void* base, int dtype, uint64_t cols, uint64_t rows, uint64_t ld_bytes,
                      const char* name);

// 2-D map over an fp32 matrix [rows, cols] (row pitch in bytes, a multiple of
// 16), no swizzle, box {box_cols, 1}: one slice of one row per load.
int make_map_rows_f32(CUtensorMap& map, const void* base, uint64_t cols, uint64_t rows, uint64_t pitch_bytes,
                      uint32_t box_cols, const char* name);

}  // namespace tma
}  // namespace pmb
