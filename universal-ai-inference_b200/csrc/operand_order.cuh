// operand_order.cuh -- where K element i of an activation (or h) row is stored
// in the f16 operand rows the expert GEMMs read.
//
// Both orders keep every dot product unchanged (the weight operand is built in
// the same order) and exist so that packed GGUF bytes unpack into operand
// registers with masks only.
#pragma once
#include <cstdint>

namespace uaii_b200 {

// Tensor-core (tcgen05) order: [0, 2, 1, 3] inside every group of four.
__host__ __device__ __forceinline__ int64_t tc_kpos(int64_t i) {
  return (i & ~int64_t(3)) | ((i & 1) << 1) | ((i >> 1) & 1);
}

// Warp-MMA (mma.sync m16n8k16) order, per block of 128: element 32t + 4s + j
// (t < 4, s < 8, j < 4) sits at 16s + 2t + 8*(j & 1) + (j >> 1), i.e. in the
// fragment slot of lane quarter t at k-step s.  One lane then holds one whole
// 32-element GGUF block (or K-quant sub-block) of its rows.  K % 128 == 0.
__host__ __device__ __forceinline__ int64_t wm_kpos(int64_t i) {
  const int64_t r = i & 127;
  return (i - r) + 16 * ((r & 31) >> 2) + 2 * (r >> 5) + 8 * (r & 1) + ((r >> 1) & 1);
}

}  // namespace uaii_b200
