// dequant.cu -- GGUF rows -> f32 on the device, bitwise equal to the reference's
// quant::dequant_gguf_row (libs/uaii-quant/src/gguf_dequant.cpp:420-439).
// One thread decodes one 32-element sub-block.
#include "gguf_blocks.cuh"
#include "kernels.hpp"

namespace uaii_b200 {
namespace {

template <int F>
__global__ void dequant_rows_kernel(const uint8_t* __restrict__ packed, int64_t rows,
                                    int64_t cols, int64_t pitch, float* __restrict__ out) {
  const int64_t sub_per_row = cols / 32;
  const int64_t total = rows * sub_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / sub_per_row;
    const int sb = (int)(i - r * sub_per_row);
    int s;
    const uint8_t* blk = subblock_ptr<F>(packed + r * pitch, sb, s);
    float v[32];
    decode32<F>(blk, s, v);
    float4* o = reinterpret_cast<float4*>(out + r * cols + (int64_t)sb * 32);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

template <int F>
cudaError_t run(const void* packed, int64_t rows, int64_t cols, int64_t pitch, float* out,
                cudaStream_t st) {
  const int64_t total = rows * (cols / 32);
  if (total == 0) return cudaSuccess;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  dequant_rows_kernel<F><<<(unsigned)blocks, 256, 0, st>>>(
      static_cast<const uint8_t*>(packed), rows, cols, pitch, out);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_dequant_rows_f32(int fmt, const void* packed, int64_t rows, int64_t cols,
                                    int64_t pitch, float* out, cudaStream_t st) {
  switch (fmt) {
    case kF32: return run<kF32>(packed, rows, cols, pitch, out, st);
    case kF16: return run<kF16>(packed, rows, cols, pitch, out, st);
    case kQ4_0: return run<kQ4_0>(packed, rows, cols, pitch, out, st);
    case kQ4_1: return run<kQ4_1>(packed, rows, cols, pitch, out, st);
    case kQ5_0: return run<kQ5_0>(packed, rows, cols, pitch, out, st);
    case kQ5_1: return run<kQ5_1>(packed, rows, cols, pitch, out, st);
    case kQ8_0: return run<kQ8_0>(packed, rows, cols, pitch, out, st);
    case kQ2_K: return run<kQ2_K>(packed, rows, cols, pitch, out, st);
    case kQ3_K: return run<kQ3_K>(packed, rows, cols, pitch, out, st);
    case kQ4_K: return run<kQ4_K>(packed, rows, cols, pitch, out, st);
    case kQ5_K: return run<kQ5_K>(packed, rows, cols, pitch, out, st);
    case kQ6_K: return run<kQ6_K>(packed, rows, cols, pitch, out, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace uaii_b200
