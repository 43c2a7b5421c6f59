// route.cu -- token routing for the MoE FFN: top-k selection with renormalised
// weights, a stable token -> expert permutation, the gather of activation rows
// into expert-contiguous slots, and the weighted combine back to token order.
//
// Reference semantics (kernels::moe_experts_swiglu_f32,
// libs/uaii-kernels/src/transformer.cpp:564-609):
//   * experts ranked by probability descending with the reference's
//     std::partial_sort procedure (ties included, see route_topk_kernel);
//   * mass = sum of the k selected probabilities in rank order (1 if not > 0),
//     w = p / mass  (norm_topk = 1, the reference behaviour; 0 keeps w = p);
//   * y = 0, then y += w * expert_out in rank order.
// The permutation is deterministic: inside each expert, slots follow token
// order, so every run produces the same slot layout.
#include <cuda_fp16.h>

#include "kernels.hpp"
#include "operand_order.cuh"
#include "topk.cuh"

namespace uaii_b200 {
namespace {

// One warp per token, k <= 32, E <= 1024 (warp_topk, topk.cuh).
__global__ void route_topk_kernel(const float* __restrict__ scores, const float* __restrict__ probs,
                                  int64_t T, int64_t E, int k, int norm_topk, RouteBuffers rb) {
  __shared__ Pair sel[8][33];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  Pair* h = sel[wib];
  for (int64_t t = blockIdx.x * 8 + wib; t < T; t += (int64_t)gridDim.x * 8) {
    warp_topk(scores + t * E, E, k, h, lane);
    if (lane == 0) {
      float ps[32];
      for (int r = 0; r < k; ++r) ps[r] = (probs == scores) ? h[r].p : probs[t * E + h[r].e];
      float mass = 0.0f;
      for (int r = 0; r < k; ++r) mass = __fadd_rn(mass, ps[r]);
      if (!(mass > 0.0f)) mass = 1.0f;
      for (int r = 0; r < k; ++r) {
        rb.topk_ids[t * k + r] = h[r].e;
        rb.topk_w[t * k + r] = norm_topk ? __fdiv_rn(ps[r], mass) : ps[r];
        rb.mask[(int64_t)h[r].e * T + t] = (uint8_t)(r + 1);
      }
    }
    __syncwarp();
  }
}

// One block per expert: stable exclusive scan of its token mask.
__global__ void __launch_bounds__(1024) route_scan_kernel(int64_t T, int k, RouteBuffers rb) {
  __shared__ int warp_tot[32];
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const uint8_t* m = rb.mask + (int64_t)e * T;
  int running = 0;
  for (int64_t base = 0; base < T; base += 1024) {
    const int64_t t = base + threadIdx.x;
    const int mv = (t < T) ? m[t] : 0;
    const unsigned bal = __ballot_sync(0xffffffffu, mv != 0);
    const int in_warp = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) warp_tot[wid] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = warp_tot[w];
      before += (w < wid) ? c : 0;
      total += c;
    }
    if (mv != 0) rb.slot_local[t * k + (mv - 1)] = running + before + in_warp;
    running += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) rb.counts[e] = running;
}

// Offsets by a block-wide exclusive scan of counts; then one warp per (t, r).
__global__ void route_gather_kernel(const float* __restrict__ x, int64_t T, int64_t D,
                                    int64_t E, int k, RouteBuffers rb, float* xp32,
                                    __half* xp16, int order, TileTables tt) {
  extern __shared__ int offs[];  // [E+1]
  if (threadIdx.x == 0) {
    int run = 0;
    for (int64_t e = 0; e < E; ++e) { offs[e] = run; run += rb.counts[e]; }
    offs[E] = run;
    if (blockIdx.x == 0 && tt.gu) {  // the expert GEMMs' tile tables, from the same counts
      int tg = 0, td = 0;
      for (int64_t e = 0; e < E; ++e) {
        tt.gu[e] = tg;
        tt.dn[e] = td;
        const int c = rb.counts[e];
        tg += ((c + tt.bn - 1) / tt.bn) * tt.gu_mtiles;
        td += ((c + tt.bn - 1) / tt.bn) * tt.dn_mtiles * tt.dn_splits;
      }
      tt.gu[E] = tg;
      tt.dn[E] = td;
    }
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int64_t e = threadIdx.x; e <= E; e += blockDim.x) rb.offsets[e] = offs[e];
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t npairs = T * k;
  if (order == kOrderQ4KI8) {
    // 16-bit integer activations per 256-element quad: a = rint(x * 32767 / max|x|) as an s8 hi
    // and a u8 lo plane (256 bytes each) in the integer quad kernel's K order -- lane l holds
    // elements 8l .. 8l+7, sub-block l / 4 at K positions 4 (l % 4) + i and 16 + 4 (l % 4) + i --
    // with the sub-block sums of a / 1024 (f16 + f16 remainder, exact) and the scale max|x| / 32767.
    // One warp per (routed pair, quad), so all quads' loads are in flight together.  Non-finite
    // activations are not carried through (the f16 orders carry them).
    const int64_t nq = D / 256;
    const int sb = lane >> 2, u = lane & 3;
    for (int64_t wi = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; wi < npairs * nq; wi += nw) {
      const int64_t p = wi / nq, q = wi - p * nq;
      const int64_t t = p / k;
      const int slot = offs[rb.topk_ids[p]] + rb.slot_local[p];
      if (lane == 0 && q == 0) { rb.slot_of[p] = slot; rb.token_of[slot] = (int32_t)t; }
      uint8_t* row = reinterpret_cast<uint8_t*>(xp16) + (int64_t)slot * 2 * D;
      const float4* s4 = reinterpret_cast<const float4*>(x + t * D + 256 * q + 8 * lane);
      const float4 v0 = s4[0], v1 = s4[1];
      const float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(e[i]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float inv = m > 0.f ? 32767.f / m : 0.f;
      uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
      int sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int a = __float2int_rn(e[i] * inv);  // |e * inv| <= 32767 (+ rounding): no clamp
        sum += a;
        hw[i >> 2] |= ((uint32_t)(a >> 8) & 0xFFu) << (8 * (i & 3));
        lw[i >> 2] |= ((uint32_t)a & 0xFFu) << (8 * (i & 3));
      }
      uint8_t* qb = row + 512 * q + 32 * sb + 4 * u;
      *reinterpret_cast<uint32_t*>(qb) = hw[0];
      *reinterpret_cast<uint32_t*>(qb + 16) = hw[1];
      *reinterpret_cast<uint32_t*>(qb + 256) = lw[0];
      *reinterpret_cast<uint32_t*>(qb + 272) = lw[1];
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (u == 0) {
        __half* xs = static_cast<__half*>(tt.xsum) + ((int64_t)slot * nq + q) * 16;
        const float sf = (float)sum * (1.0f / 1024.0f);  // |sum| < 2^20: exact
        const __half hs = __float2half_rn(sf);
        xs[sb] = hs;
        xs[8 + sb] = __float2half_rn(sf - __half2float(hs));
      }
      if (lane == 0) tt.xscale[(int64_t)slot * nq + q] = m * (1.0f / 32767.0f);
    }
    return;
  }
  for (int64_t p = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; p < npairs; p += nw) {
    const int64_t t = p / k;
    const int e = rb.topk_ids[p];
    const int slot = offs[e] + rb.slot_local[p];
    if (lane == 0) { rb.slot_of[p] = slot; rb.token_of[slot] = (int32_t)t; }
    if (D % 4 != 0) {  // odd widths: element by element
      for (int64_t i = lane; i < D; i += 32) {
        const float v = x[t * D + i];
        if (xp32) xp32[(int64_t)slot * D + i] = v;
        if (xp16) xp16[(int64_t)slot * D + tc_kpos(i)] = __float2half_rn(v);  // D % 128 != 0: tc order only
      }
      continue;
    }
    const float4* src = reinterpret_cast<const float4*>(x + t * D);
    for (int64_t i = lane; i < D / 4; i += 32) {
      const float4 v = src[i];
      if (xp32) reinterpret_cast<float4*>(xp32 + (int64_t)slot * D)[i] = v;
      if (xp16) {  // elements (4i, 4i+2) and (4i+1, 4i+3) land on adjacent pairs in both orders
        __half* row = xp16 + (int64_t)slot * D;
        const __half2 lo = __floats2half2_rn(v.x, v.z), hi = __floats2half2_rn(v.y, v.w);
        if (order != kOrderTc) {  // warp-MMA and quad orders: the pairs sit at p0 and p0 + 8
          const int64_t p0 = operand_pos(order, 4 * i);
          *reinterpret_cast<__half2*>(row + p0) = lo;
          *reinterpret_cast<__half2*>(row + p0 + 8) = hi;
          if (tt.xsum) {  // sub-block (8 float4s, lanes 8m .. 8m+7) sums of the f16 values, f32
            const float2 a = __half22float2(lo), c = __half22float2(hi);
            float sum = (a.x + a.y) + (c.x + c.y);
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            if ((lane & 7) == 0) {
              const int64_t j = i >> 3;  // sub-block
              __half* xs = static_cast<__half*>(tt.xsum) + ((int64_t)slot * (D / 256) + (j >> 3)) * 16;
              const __half hs = __float2half_rn(sum);
              xs[j & 7] = hs;
              xs[8 + (j & 7)] = __float2half_rn(sum - __half2float(hs));
            }
          }
        } else {  // tc_kpos: the pairs sit at 4i and 4i + 2, one 8-byte store (D % 4 == 0)
          *reinterpret_cast<uint2*>(row + 4 * i) =
              make_uint2(reinterpret_cast<const uint32_t&>(lo), reinterpret_cast<const uint32_t&>(hi));
        }
      }
    }
  }
}

__device__ __forceinline__ float4 sum_planes(const float* base, int64_t off4, int splits, int64_t stride) {
  float4 o = reinterpret_cast<const float4*>(base)[off4];
  for (int s = 1; s < splits; ++s) {
    const float4 p = reinterpret_cast<const float4*>(base + s * stride)[off4];
    o.x = __fadd_rn(o.x, p.x);
    o.y = __fadd_rn(o.y, p.y);
    o.z = __fadd_rn(o.z, p.z);
    o.w = __fadd_rn(o.w, p.w);
  }
  return o;
}

// Four consecutive outputs: f32, or rounded to f16 (expert-parallel return rows).
__device__ __forceinline__ void store4(float* y, int64_t i4, const float4& v) { reinterpret_cast<float4*>(y)[i4] = v; }
__device__ __forceinline__ void store4(__half* y, int64_t i4, const float4& v) {
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  memcpy(&u.x, &a, 4);
  memcpy(&u.y, &b, 4);
  reinterpret_cast<uint2*>(y)[i4] = u;
}

template <typename OT>
__global__ void combine_kernel(const float* __restrict__ out, int64_t ld, int splits, int64_t stride,
                               int64_t T, int64_t D, int k, RouteBuffers rb, const float* __restrict__ sh,
                               int sh_splits, int64_t sh_stride, const float* __restrict__ gate,
                               OT* __restrict__ y) {
  const int64_t d4 = D / 4;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * d4) return;
  const int64_t t = i / d4, c = i - t * d4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < k; ++r) {
    if (rb.topk_ids[t * k + r] < 0) continue;  // absent entry (expert-parallel rows)
    const int slot = rb.slot_of[t * k + r];
    const float w = rb.topk_w[t * k + r];
    const float4 o = sum_planes(out, ((int64_t)slot * ld) / 4 + c, splits, stride);
    acc.x = __fadd_rn(acc.x, __fmul_rn(w, o.x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(w, o.y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(w, o.z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(w, o.w));
  }
  if (sh) {
    const float g = gate ? gate[t] : 1.0f;
    const float4 s = sum_planes(sh, t * d4 + c, sh_splits, sh_stride);
    acc.x = __fadd_rn(acc.x, __fmul_rn(g, s.x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(g, s.y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(g, s.z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(g, s.w));
  }
  store4(y, t * d4 + c, acc);
}

// combine_kernel for k <= KMAX: every entry's slot and weight first, then all k
// row loads in flight together, then the same ordered sum (bit-identical).
template <int KMAX, typename OT>
__global__ void combine_k_kernel(const float* __restrict__ out, int64_t ld, int splits, int64_t stride,
                                 int64_t T, int64_t D, int k, RouteBuffers rb, const float* __restrict__ sh,
                                 int sh_splits, int64_t sh_stride, const float* __restrict__ gate,
                                 OT* __restrict__ y) {
  const int64_t d4 = D / 4;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * d4) return;
  const int64_t t = i / d4, c = i - t * d4;
  int slot[KMAX];
  float w[KMAX];
#pragma unroll
  for (int r = 0; r < KMAX; ++r) {
    slot[r] = -1;
    w[r] = 0.f;
    if (r < k && rb.topk_ids[t * k + r] >= 0) {  // absent entries (expert-parallel rows) stay -1
      slot[r] = rb.slot_of[t * k + r];
      w[r] = rb.topk_w[t * k + r];
    }
  }
  float4 o[KMAX];
#pragma unroll
  for (int r = 0; r < KMAX; ++r)
    if (slot[r] >= 0) o[r] = sum_planes(out, ((int64_t)slot[r] * ld) / 4 + c, splits, stride);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < KMAX; ++r) {
    if (slot[r] < 0) continue;
    acc.x = __fadd_rn(acc.x, __fmul_rn(w[r], o[r].x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(w[r], o[r].y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(w[r], o[r].z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(w[r], o[r].w));
  }
  if (sh) {
    const float g = gate ? gate[t] : 1.0f;
    const float4 s = sum_planes(sh, t * d4 + c, sh_splits, sh_stride);
    acc.x = __fadd_rn(acc.x, __fmul_rn(g, s.x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(g, s.y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(g, s.z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(g, s.w));
  }
  store4(y, t * d4 + c, acc);
}

__global__ void combine1_kernel(const float* __restrict__ out, int64_t ld, int splits, int64_t stride,
                                int64_t T, int64_t D, int k, RouteBuffers rb, const float* __restrict__ sh,
                                int sh_splits, int64_t sh_stride, const float* __restrict__ gate,
                                float* __restrict__ y) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * D) return;
  const int64_t t = i / D, c = i - t * D;
  float acc = 0.f;
  for (int r = 0; r < k; ++r) {
    if (rb.topk_ids[t * k + r] < 0) continue;  // absent entry (expert-parallel rows)
    const int64_t at = (int64_t)rb.slot_of[t * k + r] * ld + c;
    float o = out[at];
    for (int s = 1; s < splits; ++s) o = __fadd_rn(o, out[at + s * stride]);
    acc = __fadd_rn(acc, __fmul_rn(rb.topk_w[t * k + r], o));
  }
  if (sh) {
    float o = sh[t * D + c];
    for (int s = 1; s < sh_splits; ++s) o = __fadd_rn(o, sh[t * D + c + s * sh_stride]);
    acc = __fadd_rn(acc, __fmul_rn(gate ? gate[t] : 1.0f, o));
  }
  y[i] = acc;
}

// f16 copy in an operand K order (tc_kpos: n % 4 == 0; wm_kpos: the row width
// and n are multiples of 128, so the order restarts with every row)
__global__ void to_f16_kernel(const float* __restrict__ x, int64_t n, __half* __restrict__ o, bool wm_order) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) o[wm_order ? wm_kpos(i) : tc_kpos(i)] = __float2half_rn(x[i]);
}

// gate[t] = 1 / (1 + exp(-(x[t] . w))), one warp per token.
__global__ void shared_gate_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                   int64_t T, int64_t D, float* __restrict__ gate) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  float s = 0.f;
  for (int64_t d = lane; d < D; d += 32) s += x[t * D + d] * w[d];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) gate[t] = 1.0f / (1.0f + expf(-s));
}

__global__ void identity_route_kernel(int32_t* buf, int64_t T) {
  buf[0] = 0;
  buf[1] = (int32_t)T;
  buf[2] = (int32_t)T;
}

// The packed MatMul's operand prep in one launch: x rows -> f16 operand order, the one-expert
// route (offsets {0, M}, counts {M}) and its tile table {0, tiles}.
__global__ void to_f16_route_kernel(const float* __restrict__ x, int64_t n, __half* __restrict__ o, bool wm_order,
                                    int32_t* route, int32_t* tile_base, int64_t M, int bn, int m_tiles, int splits) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i == 0) {
    route[0] = 0;
    route[1] = (int32_t)M;
    route[2] = (int32_t)M;
    tile_base[0] = 0;
    tile_base[1] = (int32_t)((M + bn - 1) / bn) * m_tiles * splits;
  }
  if (i < n) o[wm_order ? wm_kpos(i) : tc_kpos(i)] = __float2half_rn(x[i]);
}

}  // namespace

cudaError_t launch_to_f16_route(const float* x, int64_t M, int64_t K, void* out, bool wm_order, int32_t* route,
                                int32_t* tile_base, int bn, int m_tiles, int splits, cudaStream_t st) {
  if (wm_order && K % 128 != 0) return cudaErrorInvalidValue;
  const int64_t n = M * K;
  to_f16_route_kernel<<<(unsigned)((n + 255) / 256 > 0 ? (n + 255) / 256 : 1), 256, 0, st>>>(
      x, n, static_cast<__half*>(out), wm_order, route, tile_base, M, bn, m_tiles, splits);
  return cudaGetLastError();
}

cudaError_t launch_identity_route(int32_t* buf, int64_t T, cudaStream_t st) {
  identity_route_kernel<<<1, 1, 0, st>>>(buf, T);
  return cudaGetLastError();
}

cudaError_t launch_route_topk(const float* scores, const float* probs, int64_t T, int64_t E,
                              int k, int norm_topk, const RouteBuffers& rb, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (E > 1024 || k < 1 || k > 32 || k > E) return cudaErrorInvalidValue;
  cudaError_t err = cudaMemsetAsync(rb.mask, 0, (size_t)(E * T), st);
  if (err != cudaSuccess) return err;
  int64_t blocks = (T + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  route_topk_kernel<<<(unsigned)blocks, 256, 0, st>>>(scores, probs, T, E, k, norm_topk, rb);
  return cudaGetLastError();
}

cudaError_t launch_route_scan(int64_t T, int64_t E, int k, const RouteBuffers& rb,
                              cudaStream_t st) {
  if (T == 0) return cudaMemsetAsync(rb.counts, 0, sizeof(int32_t) * (size_t)E, st);
  route_scan_kernel<<<(unsigned)E, 1024, 0, st>>>(T, k, rb);
  return cudaGetLastError();
}

cudaError_t launch_route_gather(const float* x, int64_t T, int64_t D, int64_t E, int k,
                                const RouteBuffers& rb, float* xp_f32, void* xp_f16,
                                cudaStream_t st, int order, const TileTables* tables) {
  if ((order == kOrderWm && D % 128 != 0) ||
      ((order == kOrderQ4K || order == kOrderQ6K || order == kOrderQ4KI8) && D % 256 != 0))
    return cudaErrorInvalidValue;
  const TileTables tt = tables ? *tables : TileTables{};
  if (order == kOrderQ4KI8 && (tt.xsum == nullptr || tt.xscale == nullptr || xp_f16 == nullptr || xp_f32 != nullptr))
    return cudaErrorInvalidValue;
  int64_t blocks = (T * k * (order == kOrderQ4KI8 ? D / 256 : 1) + 7) / 8;  // 8 warps a block, one per work item
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  const size_t smem = sizeof(int) * (size_t)(E + 1);
  route_gather_kernel<<<(unsigned)blocks, 256, smem, st>>>(x, T, D, E, k, rb, xp_f32,
                                                           static_cast<__half*>(xp_f16), order, tt);
  return cudaGetLastError();
}

namespace {
// y[i] = planes[0][i] + planes[1][i] + ... (plane order, one rounding per add), then v > 0 ? v : 0 with relu
__global__ void sum_planes_kernel(const float* __restrict__ planes, int splits, int64_t stride, int64_t n,
                                  float* __restrict__ y, int relu) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = planes[i];
    for (int s = 1; s < splits; ++s) v = __fadd_rn(v, planes[s * stride + i]);
    y[i] = (!relu || v > 0.0f) ? v : 0.0f;  // the reference's relu: v > 0 ? v : 0 (-0 and NaN give 0)
  }
}
}  // namespace

cudaError_t launch_sum_planes(const float* planes, int splits, int64_t plane_stride, int64_t n, float* y, bool relu,
                              cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (splits < 1) return cudaErrorInvalidValue;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  sum_planes_kernel<<<(unsigned)blocks, 256, 0, st>>>(planes, splits, plane_stride, n, y, relu ? 1 : 0);
  return cudaGetLastError();
}

namespace {
template <typename OT>
cudaError_t combine_vec(const float* out, int64_t out_ld, int splits, int64_t split_stride, int64_t T, int64_t D,
                        int k, const RouteBuffers& rb, const float* shared_out, int sh_splits, int64_t sh_split_stride,
                        const float* shared_gate, OT* y, cudaStream_t st) {
  const int64_t n = T * (D / 4);
  const unsigned blocks = (unsigned)((n + 255) / 256);
#define UAII_COMBINE_K(KM)                                                                                      \
  combine_k_kernel<KM, OT><<<blocks, 256, 0, st>>>(out, out_ld, splits, split_stride, T, D, k, rb, shared_out, \
                                                   sh_splits, sh_split_stride, shared_gate, y)
  if (k <= 2) UAII_COMBINE_K(2);
  else if (k <= 4) UAII_COMBINE_K(4);
  else if (k <= 8) UAII_COMBINE_K(8);
  else
    combine_kernel<OT><<<blocks, 256, 0, st>>>(out, out_ld, splits, split_stride, T, D, k, rb, shared_out,
                                               sh_splits, sh_split_stride, shared_gate, y);
#undef UAII_COMBINE_K
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_combine(const float* out, int64_t out_ld, int splits, int64_t split_stride,
                           int64_t T, int64_t D, int k, const RouteBuffers& rb,
                           const float* shared_out, int sh_splits, int64_t sh_split_stride,
                           const float* shared_gate, void* y, cudaStream_t st, bool y_f16) {
  if (T == 0) return cudaSuccess;
  if (splits < 1) splits = 1;
  if (sh_splits < 1) sh_splits = 1;
  const bool vec = D % 4 == 0 && out_ld % 4 == 0 && split_stride % 4 == 0 && sh_split_stride % 4 == 0;
  if (y_f16) {
    if (!vec) return cudaErrorInvalidValue;
    return combine_vec(out, out_ld, splits, split_stride, T, D, k, rb, shared_out, sh_splits, sh_split_stride,
                       shared_gate, static_cast<__half*>(y), st);
  }
  if (!vec) {
    combine1_kernel<<<(unsigned)((T * D + 255) / 256), 256, 0, st>>>(out, out_ld, splits, split_stride, T, D, k,
                                                                     rb, shared_out, sh_splits, sh_split_stride,
                                                                     shared_gate, static_cast<float*>(y));
    return cudaGetLastError();
  }
  return combine_vec(out, out_ld, splits, split_stride, T, D, k, rb, shared_out, sh_splits, sh_split_stride,
                     shared_gate, static_cast<float*>(y), st);
}

cudaError_t launch_to_f16(const float* x, int64_t n, void* out, cudaStream_t st, bool wm_order) {
  if (n == 0) return cudaSuccess;
  if (wm_order && n % 128 != 0) return cudaErrorInvalidValue;
  to_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, n, static_cast<__half*>(out), wm_order);
  return cudaGetLastError();
}

cudaError_t launch_shared_gate(const float* x, const float* w, int64_t T, int64_t D, float* gate,
                               cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  shared_gate_kernel<<<(unsigned)((T * 32 + 255) / 256), 256, 0, st>>>(x, w, T, D, gate);
  return cudaGetLastError();
}

}  // namespace uaii_b200
