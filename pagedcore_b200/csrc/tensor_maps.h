// TMA tensor maps (cuTensorMapEncodeTiled through the runtime's driver entry
// point, so the library links no libcuda): the KV pool's per-head block view,
// shared by the decode and prefill attention kernels, and plain FP16 matrices.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace pkv {

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled, or nullptr when the driver does not provide it.
EncodeTiled encode_fn();

// 3-D view of the pool [22][2][num_blocks][16][4][64] FP16 for per-head
// boxes: (dim 64, kv head 4, pool row), strides 128 B (head) and 512 B (row),
// box 64 x 1 x 16 (one head of one block, 2 KiB) with the 128-byte swizzle.
// Cached per (pool address, block count).  Returns a PKV_* status.
int pool_tensor_map(const void *pool, int32_t num_blocks, CUtensorMap *out);

// 2-D view of a row-major FP16 matrix [rows][cols] (rows `row_stride`
// elements apart; cols a multiple of 8, the base 16-byte aligned) with a box
// of box_rows x 64 columns and the 128-byte swizzle; rows past the end read
// as zeros.  Not cached.  Returns a PKV_* status.
int matrix_tensor_map(const void *base, uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_rows,
                      CUtensorMap *out);

}  // namespace pkv
