// ep.cu -- expert parallelism: the device halves of the dispatch and combine
// exchange around the grouped expert GEMM.
//
// Rank r of R owns experts [r*epr, (r+1)*epr), epr = E / R.  For its own tokens a
// rank routes (router + top-k, identical to the single-GPU path), then sends each
// token ONCE to every rank that owns at least one of its k experts: one f16 row
// (tensor-core operand order) plus k (local expert, weight) entries, -1 where the
// k-th choice lives on another rank.  Rows are grouped by destination rank and,
// inside a group, follow token order (a stable scan), so every run lays out the
// exchange the same way.  The receiving rank runs its experts on the rows and
// sends back one f32 row per received row: the weighted sum of its experts'
// outputs in top-k rank order.  The source rank adds the returned rows of a
// token in rank order 0..R-1.
//
// The reference runs the layer in one host process (kernels::moe_experts_swiglu_f32,
// libs/uaii-kernels/src/transformer.cpp:564-609); across ranks the per-token sum
// is regrouped (per-rank partial sums first), which changes rounding only.
#include <cuda_fp16.h>

#include "kernels.hpp"

namespace uaii_b200 {
namespace {

// dmask[d*T + t] = d + 1 when token t has an expert on rank d (the stable scan
// then numbers each destination's tokens in token order).
__global__ void ep_plan_kernel(const int32_t* __restrict__ topk_ids, int64_t T, int k, int epr,
                               uint8_t* __restrict__ dmask) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= T) return;
  for (int r = 0; r < k; ++r) {
    const int d = topk_ids[t * k + r] / epr;
    dmask[(int64_t)d * T + t] = (uint8_t)(d + 1);
  }
}

// One warp per (token, destination).  Offsets of the destination groups come
// from a block-local scan of the R counts.
__global__ void ep_pack_kernel(const float* __restrict__ x, int64_t T, int64_t D, int k, int R, int epr,
                               const int32_t* __restrict__ topk_ids, const float* __restrict__ topk_w,
                               const uint8_t* __restrict__ dmask, const int32_t* __restrict__ rowpos,
                               const int32_t* __restrict__ dcounts, __half* __restrict__ send_x16, int64_t xs,
                               int32_t* __restrict__ send_ids, float* __restrict__ send_w, int64_t es,
                               int32_t* __restrict__ send_token, int32_t* __restrict__ row_of,
                               int32_t* __restrict__ send_counts, int32_t* __restrict__ send_entries) {
  extern __shared__ int offs[];  // [R]
  if (threadIdx.x == 0) {
    int run = 0;
    for (int d = 0; d < R; ++d) { offs[d] = run; run += dcounts[d]; }
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int d = threadIdx.x; d < R; d += blockDim.x) {
      send_counts[d] = dcounts[d];
      send_entries[d] = 0;
    }
  }
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t p = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; p < T * R; p += nw) {
    const int64_t t = p / R;
    const int d = (int)(p - t * R);
    if (dmask[(int64_t)d * T + t] == 0) {
      if (lane == 0) row_of[p] = -1;
      continue;
    }
    const int64_t row = offs[d] + rowpos[t * R + d];
    if (lane == 0) {
      row_of[p] = (int32_t)row;
      send_token[row] = (int32_t)t;
    }
    if (lane < k) {
      const int e = topk_ids[t * k + lane];
      const bool mine = e / epr == d;
      send_ids[row * es + lane] = mine ? e - d * epr : -1;
      send_w[row * es + lane] = mine ? topk_w[t * k + lane] : 0.0f;
    }
    if (D % 4 != 0) {
      for (int64_t i = lane; i < D; i += 32)
        send_x16[row * xs + ((i & ~3) | ((i & 1) << 1) | ((i >> 1) & 1))] = __float2half_rn(x[t * D + i]);
    } else {
      const float4* src = reinterpret_cast<const float4*>(x + t * D);
      for (int64_t i = lane; i < D / 4; i += 32) {
        const float4 v = src[i];
        __half2* d2 = reinterpret_cast<__half2*>(send_x16 + row * xs) + 2 * i;
        d2[0] = __floats2half2_rn(v.x, v.z);
        d2[1] = __floats2half2_rn(v.y, v.w);
      }
    }
  }
}

// Entries (valid (row, expert) pairs) per destination, for the receivers' plans.
__global__ void ep_entries_kernel(const int32_t* __restrict__ topk_ids, int64_t T, int k, int epr,
                                  int32_t* __restrict__ send_entries) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= T) return;
  for (int r = 0; r < k; ++r) atomicAdd(send_entries + topk_ids[t * k + r] / epr, 1);
}

// Receiving side: routing tables from the received entries (-1 = absent).
__global__ void ep_route_kernel(const int32_t* __restrict__ ids, const float* __restrict__ w, int64_t es,
                                int64_t N, int k, RouteBuffers rb) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= N) return;
  for (int r = 0; r < k; ++r) {
    const int e = ids[t * es + r];
    rb.topk_ids[t * k + r] = e;
    rb.topk_w[t * k + r] = w[t * es + r];
    if (e >= 0) rb.mask[(int64_t)e * N + t] = (uint8_t)(r + 1);
  }
}

// Gather received f16 rows (already in operand order) into expert-contiguous slots.
__global__ void route_gather16_kernel(const __half* __restrict__ rows, int64_t xs, int64_t N, int64_t D, int64_t E,
                                      int k, RouteBuffers rb, __half* __restrict__ xp16) {
  extern __shared__ int offs[];  // [E+1]
  if (threadIdx.x == 0) {
    int run = 0;
    for (int64_t e = 0; e < E; ++e) { offs[e] = run; run += rb.counts[e]; }
    offs[E] = run;
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int64_t e = threadIdx.x; e <= E; e += blockDim.x) rb.offsets[e] = offs[e];
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t p = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; p < N * k; p += nw) {
    const int e = rb.topk_ids[p];
    if (e < 0) continue;
    const int64_t t = p / k;
    const int slot = offs[e] + rb.slot_local[p];
    if (lane == 0) { rb.slot_of[p] = slot; rb.token_of[slot] = (int32_t)t; }
    if (D % 8 == 0 && xs % 8 == 0) {
      const uint4* src = reinterpret_cast<const uint4*>(rows + t * xs);
      uint4* dst = reinterpret_cast<uint4*>(xp16 + (int64_t)slot * D);
      for (int64_t i = lane; i < D / 8; i += 32) dst[i] = src[i];
    } else {
      for (int64_t i = lane; i < D; i += 32) xp16[(int64_t)slot * D + i] = rows[t * xs + i];
    }
  }
}

// y[t] = sum over ranks d = 0..R-1 holding a row of t of y_back[row] (fixed order).
__global__ void ep_combine_kernel(const float* __restrict__ y_back, const int32_t* __restrict__ row_of,
                                  int64_t T, int R, int64_t D, float* __restrict__ y) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * D) return;
  const int64_t t = i / D, c = i - t * D;
  float acc = 0.0f;
  for (int d = 0; d < R; ++d) {
    const int row = row_of[t * R + d];
    if (row >= 0) acc = __fadd_rn(acc, y_back[(int64_t)row * D + c]);
  }
  y[i] = acc;
}

// ep_combine_kernel on float4 columns for R <= RMAX: a token's row indices first, then
// all its row loads in flight together, then the same rank-ordered sum (bit-identical).
template <int RMAX>
__global__ void ep_combine4_kernel(const float* __restrict__ y_back, const int32_t* __restrict__ row_of,
                                   int64_t T, int R, int64_t D, float* __restrict__ y) {
  const int64_t d4 = D / 4;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * d4) return;
  const int64_t t = i / d4, c = i - t * d4;
  int row[RMAX];
#pragma unroll
  for (int d = 0; d < RMAX; ++d) row[d] = d < R ? row_of[t * R + d] : -1;
  float4 v[RMAX];
#pragma unroll
  for (int d = 0; d < RMAX; ++d)
    if (row[d] >= 0) v[d] = reinterpret_cast<const float4*>(y_back + (int64_t)row[d] * D)[c];
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int d = 0; d < RMAX; ++d) {
    if (row[d] < 0) continue;
    acc.x = __fadd_rn(acc.x, v[d].x);
    acc.y = __fadd_rn(acc.y, v[d].y);
    acc.z = __fadd_rn(acc.z, v[d].z);
    acc.w = __fadd_rn(acc.w, v[d].w);
  }
  reinterpret_cast<float4*>(y + t * D)[c] = acc;
}

// ep_combine_kernel on f16 returned rows (any rank count).
__global__ void ep_combine_h_kernel(const __half* __restrict__ y_back, const int32_t* __restrict__ row_of,
                                    int64_t T, int R, int64_t D, float* __restrict__ y) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * D) return;
  const int64_t t = i / D, c = i - t * D;
  float acc = 0.0f;
  for (int d = 0; d < R; ++d) {
    const int row = row_of[t * R + d];
    if (row >= 0) acc = __fadd_rn(acc, __half2float(y_back[(int64_t)row * D + c]));
  }
  y[i] = acc;
}

// ep_combine4_kernel on f16 returned rows: four halves per load, f32 sums in rank order.
template <int RMAX>
__global__ void ep_combine4h_kernel(const __half* __restrict__ y_back, const int32_t* __restrict__ row_of,
                                    int64_t T, int R, int64_t D, float* __restrict__ y) {
  const int64_t d4 = D / 4;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * d4) return;
  const int64_t t = i / d4, c = i - t * d4;
  int row[RMAX];
#pragma unroll
  for (int d = 0; d < RMAX; ++d) row[d] = d < R ? row_of[t * R + d] : -1;
  uint2 v[RMAX];
#pragma unroll
  for (int d = 0; d < RMAX; ++d)
    if (row[d] >= 0) v[d] = reinterpret_cast<const uint2*>(y_back + (int64_t)row[d] * D)[c];
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int d = 0; d < RMAX; ++d) {
    if (row[d] < 0) continue;
    __half2 a, b;
    memcpy(&a, &v[d].x, 4);
    memcpy(&b, &v[d].y, 4);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    acc.x = __fadd_rn(acc.x, fa.x);
    acc.y = __fadd_rn(acc.y, fa.y);
    acc.z = __fadd_rn(acc.z, fb.x);
    acc.w = __fadd_rn(acc.w, fb.y);
  }
  reinterpret_cast<float4*>(y + t * D)[c] = acc;
}

}  // namespace

cudaError_t launch_ep_plan(const int32_t* topk_ids, int64_t T, int k, int R, int epr, uint8_t* dmask,
                           int32_t* rowpos, int32_t* dcounts, cudaStream_t st) {
  if (R < 1 || R > 255 || epr < 1) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(dmask, 0, (size_t)(R * T), st);
  if (e != cudaSuccess || T == 0) return T == 0 ? cudaMemsetAsync(dcounts, 0, sizeof(int32_t) * R, st) : e;
  ep_plan_kernel<<<(unsigned)((T + 255) / 256), 256, 0, st>>>(topk_ids, T, k, epr, dmask);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  RouteBuffers rb{};
  rb.mask = dmask;
  rb.slot_local = rowpos;
  rb.counts = dcounts;
  return launch_route_scan(T, R, R, rb, st);
}

cudaError_t launch_ep_pack(const float* x, int64_t T, int64_t D, int k, int R, int epr, const int32_t* topk_ids,
                           const float* topk_w, const uint8_t* dmask, const int32_t* rowpos,
                           const int32_t* dcounts, void* send_x16, int32_t* send_ids, float* send_w,
                           int32_t* send_token, int32_t* row_of, int32_t* send_counts, int32_t* send_entries,
                           cudaStream_t st, int64_t x_pitch, int64_t e_pitch) {
  if (k > 32) return cudaErrorInvalidValue;
  if (x_pitch <= 0) x_pitch = D;
  if (e_pitch <= 0) e_pitch = k;
  if (x_pitch < D || e_pitch < k || (D % 4 == 0 && x_pitch % 2 != 0)) return cudaErrorInvalidValue;
  int64_t blocks = (T * R + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  ep_pack_kernel<<<(unsigned)blocks, 256, sizeof(int) * (size_t)R, st>>>(
      x, T, D, k, R, epr, topk_ids, topk_w, dmask, rowpos, dcounts, static_cast<__half*>(send_x16), x_pitch,
      send_ids, send_w, e_pitch, send_token, row_of, send_counts, send_entries);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || T == 0) return e;
  ep_entries_kernel<<<(unsigned)((T + 255) / 256), 256, 0, st>>>(topk_ids, T, k, epr, send_entries);
  return cudaGetLastError();
}

cudaError_t launch_ep_route(const int32_t* ids, const float* w, int64_t N, int64_t E, int k,
                            const RouteBuffers& rb, cudaStream_t st, int64_t e_pitch) {
  if (e_pitch <= 0) e_pitch = k;
  if (e_pitch < k) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(rb.mask, 0, (size_t)(E * N), st);
  if (e != cudaSuccess || N == 0) return e;
  ep_route_kernel<<<(unsigned)((N + 127) / 128), 128, 0, st>>>(ids, w, e_pitch, N, k, rb);
  return cudaGetLastError();
}

cudaError_t launch_route_gather16(const void* rows, int64_t N, int64_t D, int64_t E, int k, const RouteBuffers& rb,
                                  void* xp16, cudaStream_t st, int64_t x_pitch) {
  if (x_pitch <= 0) x_pitch = D;
  if (x_pitch < D) return cudaErrorInvalidValue;
  int64_t blocks = (N * k + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  route_gather16_kernel<<<(unsigned)blocks, 256, sizeof(int) * (size_t)(E + 1), st>>>(
      static_cast<const __half*>(rows), x_pitch, N, D, E, k, rb, static_cast<__half*>(xp16));
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const float* y_back, const int32_t* row_of, int64_t T, int R, int64_t D, float* y,
                              cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const bool vec = D % 4 == 0 && ((reinterpret_cast<uintptr_t>(y_back) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const unsigned blocks4 = (unsigned)((T * (D / 4) + 255) / 256);
  if (vec && R <= 2) ep_combine4_kernel<2><<<blocks4, 256, 0, st>>>(y_back, row_of, T, R, D, y);
  else if (vec && R <= 4) ep_combine4_kernel<4><<<blocks4, 256, 0, st>>>(y_back, row_of, T, R, D, y);
  else if (vec && R <= 8) ep_combine4_kernel<8><<<blocks4, 256, 0, st>>>(y_back, row_of, T, R, D, y);
  else ep_combine_kernel<<<(unsigned)((T * D + 255) / 256), 256, 0, st>>>(y_back, row_of, T, R, D, y);
  return cudaGetLastError();
}

cudaError_t launch_ep_combine_f16(const void* y_back16, const int32_t* row_of, int64_t T, int R, int64_t D, float* y,
                                  cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const __half* yb = static_cast<const __half*>(y_back16);
  if (D % 4 != 0 || R > 8 || ((reinterpret_cast<uintptr_t>(y_back16) & 7) | (reinterpret_cast<uintptr_t>(y) & 15))) {
    ep_combine_h_kernel<<<(unsigned)((T * D + 255) / 256), 256, 0, st>>>(yb, row_of, T, R, D, y);
    return cudaGetLastError();
  }
  const unsigned blocks4 = (unsigned)((T * (D / 4) + 255) / 256);
  if (R <= 2) ep_combine4h_kernel<2><<<blocks4, 256, 0, st>>>(yb, row_of, T, R, D, y);
  else if (R <= 4) ep_combine4h_kernel<4><<<blocks4, 256, 0, st>>>(yb, row_of, T, R, D, y);
  else ep_combine4h_kernel<8><<<blocks4, 256, 0, st>>>(yb, row_of, T, R, D, y);
  return cudaGetLastError();
}

}  // namespace uaii_b200
