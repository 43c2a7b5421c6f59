// experts_simt.cu -- grouped expert GEMV on CUDA cores, f32 end to end.
//
// This is the accuracy anchor of the device path and its small-batch schedule:
// weights are decoded with the exact f32 decoders of gguf_blocks.cuh and
// multiplied in f32, so it differs from the reference
// (kernels::moe_experts_swiglu_f32, libs/uaii-kernels/src/transformer.cpp:585-608)
// only in summation order.  One warp owns one weight row of one expert; lanes
// split the row into 32-element sub-blocks and the partial dot products of up
// to 8 slots are reduced with warp shuffles.  Dense f32/f16 expert weights (the
// reference op's own input type) are read element by element and may have any
// row length.
#include "gguf_blocks.cuh"
#include "kernels.hpp"

namespace uaii_b200 {
namespace {

constexpr int kNT = 8;            // slots per pass
constexpr int kWarps = 8;         // rows per block

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

template <int F>
__device__ __forceinline__ float dense_at(const uint8_t* row, int64_t i) {
  if constexpr (F == kF32) return reinterpret_cast<const float*>(row)[i];
  else return f16_bits_to_f32(ld_u16(row + 2 * i));
}

template <int F>
__global__ void __launch_bounds__(256) gateup_simt_kernel(
    const uint8_t* __restrict__ G, const uint8_t* __restrict__ U, int64_t I, int64_t D,
    int64_t gp, int64_t up, const float* __restrict__ xp, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ counts, float* __restrict__ h) {
  const int e = blockIdx.y;
  const int n_e = counts[e];
  if (n_e == 0) return;
  const int off = offsets[e];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nsb = (int)(D / 32);
  for (int64_t i = (int64_t)blockIdx.x * kWarps + wid; i < I; i += (int64_t)gridDim.x * kWarps) {
    const uint8_t* grow = G + ((int64_t)e * I + i) * gp;
    const uint8_t* urow = U + ((int64_t)e * I + i) * up;
    for (int n0 = 0; n0 < n_e; n0 += kNT) {
      const int nn = min(kNT, n_e - n0);
      float ag[kNT], au[kNT];
#pragma unroll
      for (int n = 0; n < kNT; ++n) { ag[n] = 0.f; au[n] = 0.f; }
      if constexpr (F == kF32 || F == kF16) {  // dense rows: any length
        for (int64_t d = lane; d < D; d += 32) {
          const float g1 = dense_at<F>(grow, d), u1 = dense_at<F>(urow, d);
#pragma unroll
          for (int n = 0; n < kNT; ++n) {
            if (n < nn) {
              const float xv = xp[(int64_t)(off + n0 + n) * D + d];
              ag[n] += g1 * xv;
              au[n] += u1 * xv;
            }
          }
        }
      } else {
      for (int sb = lane; sb < nsb; sb += 32) {
        float wg[32], wu[32];
        int s;
        decode32<F>(subblock_ptr<F>(grow, sb, s), s, wg);
        decode32<F>(subblock_ptr<F>(urow, sb, s), s, wu);
#pragma unroll
        for (int n = 0; n < kNT; ++n) {
          if (n < nn) {
            const float4* xr = reinterpret_cast<const float4*>(xp + (int64_t)(off + n0 + n) * D + sb * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 xv = xr[j];
              ag[n] += wg[4 * j] * xv.x + wg[4 * j + 1] * xv.y + wg[4 * j + 2] * xv.z + wg[4 * j + 3] * xv.w;
              au[n] += wu[4 * j] * xv.x + wu[4 * j + 1] * xv.y + wu[4 * j + 2] * xv.z + wu[4 * j + 3] * xv.w;
            }
          }
        }
      }
      }
#pragma unroll
      for (int n = 0; n < kNT; ++n) {
        const float g = warp_sum(ag[n]);
        const float u = warp_sum(au[n]);
        if (lane == n && n < nn) {
          const float sig = 1.0f / (1.0f + expf(-g));
          h[(int64_t)(off + n0 + n) * I + i] = (g * sig) * u;
        }
      }
    }
  }
}

template <int F>
__global__ void __launch_bounds__(256) down_simt_kernel(
    const uint8_t* __restrict__ Dn, int64_t D, int64_t I, int64_t dp,
    const float* __restrict__ h, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ counts, float* __restrict__ out) {
  const int e = blockIdx.y;
  const int n_e = counts[e];
  if (n_e == 0) return;
  const int off = offsets[e];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nsb = (int)(I / 32);
  for (int64_t o = (int64_t)blockIdx.x * kWarps + wid; o < D; o += (int64_t)gridDim.x * kWarps) {
    const uint8_t* row = Dn + ((int64_t)e * D + o) * dp;
    for (int n0 = 0; n0 < n_e; n0 += kNT) {
      const int nn = min(kNT, n_e - n0);
      float a[kNT];
#pragma unroll
      for (int n = 0; n < kNT; ++n) a[n] = 0.f;
      if constexpr (F == kF32 || F == kF16) {
        for (int64_t i = lane; i < I; i += 32) {
          const float w1 = dense_at<F>(row, i);
#pragma unroll
          for (int n = 0; n < kNT; ++n)
            if (n < nn) a[n] += w1 * h[(int64_t)(off + n0 + n) * I + i];
        }
      } else {
      for (int sb = lane; sb < nsb; sb += 32) {
        float w[32];
        int s;
        decode32<F>(subblock_ptr<F>(row, sb, s), s, w);
#pragma unroll
        for (int n = 0; n < kNT; ++n) {
          if (n < nn) {
            const float4* hr = reinterpret_cast<const float4*>(h + (int64_t)(off + n0 + n) * I + sb * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 hv = hr[j];
              a[n] += w[4 * j] * hv.x + w[4 * j + 1] * hv.y + w[4 * j + 2] * hv.z + w[4 * j + 3] * hv.w;
            }
          }
        }
      }
      }
#pragma unroll
      for (int n = 0; n < kNT; ++n) {
        const float v = warp_sum(a[n]);
        if (lane == n && n < nn) out[(int64_t)(off + n0 + n) * D + o] = v;
      }
    }
  }
}

unsigned row_blocks(int64_t rows) {
  int64_t b = (rows + kWarps - 1) / kWarps;
  if (b > 65535) b = 65535;
  return (unsigned)b;
}

template <int F>
cudaError_t gateup(const void* G, const void* U, int64_t E, int64_t I, int64_t D, int64_t gp,
                   int64_t up, const float* xp, const int32_t* offsets, const int32_t* counts,
                   float* h, cudaStream_t st) {
  dim3 grid(row_blocks(I), (unsigned)E);
  gateup_simt_kernel<F><<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(G),
                                              static_cast<const uint8_t*>(U), I, D, gp, up, xp,
                                              offsets, counts, h);
  return cudaGetLastError();
}

template <int F>
cudaError_t down(const void* Dn, int64_t E, int64_t D, int64_t I, int64_t dp, const float* h,
                 const int32_t* offsets, const int32_t* counts, float* out, cudaStream_t st) {
  dim3 grid(row_blocks(D), (unsigned)E);
  down_simt_kernel<F><<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(Dn), D, I, dp, h,
                                            offsets, counts, out);
  return cudaGetLastError();
}

// MoEExperts (legacy top-1 linear experts, libs/uaii-kernels/src/transformer.cpp:483-520):
// y[b, o] = sum_i x[b, i] * W[e, o, i], i ascending, products and sums rounded
// separately, e = (int)top[b] or expert 0 outside [0, E).  One block owns 128 outputs
// of one token; 32-column tiles of its 128 weight rows are staged through shared memory
// with coalesced loads (row pitch 33 floats: thread o reads row o without bank
// conflicts) and every thread walks its row's tile in order.
constexpr int kLinRows = 128, kLinCols = 32;

__global__ void __launch_bounds__(kLinRows) experts_linear_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ W,
                                                                  const float* __restrict__ top, int64_t D,
                                                                  int64_t E, float* __restrict__ y) {
  __shared__ float sw[kLinRows][kLinCols + 1];
  __shared__ float sx[kLinCols];
  const int64_t b = blockIdx.x;
  const int64_t o0 = (int64_t)blockIdx.y * kLinRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float v = top[b];
  const int64_t e = (v > -1.0f && v < (float)E) ? (int64_t)(int)v : 0;
  const float* We = W + e * D * D;
  float sum = 0.0f;
  for (int64_t i0 = 0; i0 < D; i0 += kLinCols) {
    const int64_t i = i0 + lane;
    for (int r = warp; r < kLinRows; r += kLinRows / 32)
      sw[r][lane] = (o0 + r < D && i < D) ? __ldg(We + (o0 + r) * D + i) : 0.0f;
    if (warp == 0) sx[lane] = i < D ? __ldg(x + b * D + i) : 0.0f;
    __syncthreads();
    const int n = D - i0 < kLinCols ? (int)(D - i0) : kLinCols;
    for (int j = 0; j < n; ++j) sum = __fadd_rn(sum, __fmul_rn(sx[j], sw[threadIdx.x][j]));
    __syncthreads();
  }
  if (o0 + threadIdx.x < D) y[b * D + o0 + threadIdx.x] = sum;
}

}  // namespace

cudaError_t launch_experts_linear(const float* x, const float* W, const float* top, int64_t B, int64_t D,
                                  int64_t E, float* y, cudaStream_t st) {
  if (B == 0) return cudaSuccess;
  if (B < 0 || D <= 0 || E <= 0 || B > INT32_MAX || (D + kLinRows - 1) / kLinRows > 65535)
    return cudaErrorInvalidValue;
  experts_linear_kernel<<<dim3((unsigned)B, (unsigned)((D + kLinRows - 1) / kLinRows)), kLinRows, 0, st>>>(
      x, W, top, D, E, y);
  return cudaGetLastError();
}

#define UAII_FMT_CASES(M)                                                          \
  M(kF32) M(kF16) M(kQ4_0) M(kQ4_1) M(kQ5_0) M(kQ5_1) M(kQ8_0) M(kQ2_K) M(kQ3_K)  \
  M(kQ4_K) M(kQ5_K) M(kQ6_K)

cudaError_t launch_gateup_simt(int gfmt, const void* G, int ufmt, const void* U, int64_t E,
                               int64_t I, int64_t D, int64_t g_pitch, int64_t u_pitch,
                               const float* xp, const int32_t* offsets, const int32_t* counts,
                               float* h, cudaStream_t st) {
  if (gfmt != ufmt || (fmt_is_gguf(gfmt) && D % 32 != 0)) return cudaErrorInvalidValue;
  switch (gfmt) {
#define M(F) case F: return gateup<F>(G, U, E, I, D, g_pitch, u_pitch, xp, offsets, counts, h, st);
    UAII_FMT_CASES(M)
#undef M
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_down_simt(int dfmt, const void* Dn, int64_t E, int64_t D, int64_t I,
                             int64_t d_pitch, const float* h, const int32_t* offsets,
                             const int32_t* counts, float* out, cudaStream_t st) {
  if (fmt_is_gguf(dfmt) && I % 32 != 0) return cudaErrorInvalidValue;
  switch (dfmt) {
#define M(F) case F: return down<F>(Dn, E, D, I, d_pitch, h, offsets, counts, out, st);
    UAII_FMT_CASES(M)
#undef M
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace uaii_b200
