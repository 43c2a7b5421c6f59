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

// Quad orders (the K-quant quad schedule, mma.sync m16n8k16 over whole 256-element
// super-blocks), per block of 256.  K-step s of a quad holds operand positions 16s ..
// 16s+15; lane quarter t owns positions 2t, 2t+1 (its first pair) and 2t+8, 2t+9 (its
// second pair) of every k-step, and a pair always holds bytes (0, 2) or (1, 3) of one
// 32-bit word of packed bytes, so a word unpacks with masks only.
//   Q4_K: lane quarter t decodes qs bytes [32t, 32t+32): sub-block 2t (low nibbles)
//         at k-steps 0-7 and sub-block 2t+1 (high nibbles) at k-steps 8-15; element
//         64t + 32b + 4w + u (b < 2, w < 8, u < 4) sits at k-step 8b + w.
//   Q6_K: lane quarter t = 2*hf + pp decodes positions [16pp, 16pp+16) of every quarter
//         c of half hf; element 128hf + 32c + 16pp + 4w + u (w < 4) sits at k-step 4c + w.
// In both, byte u of the word goes to position 16s + 2t + 8(u & 1) + (u >> 1).
__host__ __device__ __forceinline__ int64_t q4k_kpos(int64_t i) {
  const int64_t r = i & 255;
  const int64_t t = r >> 6, b = (r >> 5) & 1, w = (r >> 2) & 7, u = r & 3;
  return (i - r) + 16 * (8 * b + w) + 2 * t + 8 * (u & 1) + (u >> 1);
}
__host__ __device__ __forceinline__ int64_t q6k_kpos(int64_t i) {
  const int64_t r = i & 255;
  const int64_t hf = r >> 7, c = (r >> 5) & 3, pp = (r >> 4) & 1, w = (r >> 2) & 3, u = r & 3;
  return (i - r) + 16 * (4 * c + w) + 2 * (2 * hf + pp) + 8 * (u & 1) + (u >> 1);
}

// Which order an operand row is stored in.
enum OperandOrder : int { kOrderTc = 0, kOrderWm = 1, kOrderQ4K = 2, kOrderQ6K = 3, kOrderQ4KI8 = 4 };
// kOrderQ4KI8 is not an f16 order: route_gather writes 16-bit integer activations as int8 planes
// (see launch_gateup_umma); operand_pos does not apply to it.
__host__ __device__ __forceinline__ int64_t operand_pos(int order, int64_t i) {
  switch (order) {
    case kOrderWm: return wm_kpos(i);
    case kOrderQ4K: return q4k_kpos(i);
    case kOrderQ6K: return q6k_kpos(i);
    default: return tc_kpos(i);
  }
}

}  // namespace uaii_b200
