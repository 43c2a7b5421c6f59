// decode_model.cu -- device kernels of the batched greedy decode step around the
// MoE FFN layer: token embedding, residual add + RMSNorm, RoPE with the KV-cache
// append, grouped-query attention over the cache, greedy arg-max, and device-side
// synthetic inputs (normal draws, GGUF block quantizers, a random KV prefill).
//
// The step is the reference's seq-1 transformer graph (libs/uaii-loaders/src/gguf.cpp:
// 905-1210: Embedding -> per layer RMSNorm, Q/K/V MatMul, RoPE, Attention with KV
// cache, O MatMul, Add, RMSNorm, MoE, Add -> RMSNorm -> lm_head MatMul -> Softmax)
// applied to a batch of independent sequences at one position, the batched form of
// Session::generate (libs/uaii-runtime/src/session.cpp:910-1046).  The element-wise
// arithmetic follows the reference kernels (libs/uaii-kernels/src/norm.cpp:89-130,
// transformer.cpp:61-433) with explicit round-to-nearest intrinsics, so nvcc cannot
// contract a multiply and an add; reductions are tree-shaped (rounding-level
// differences from the reference's sequential sums).
#include <cuda_fp16.h>

#include <cfloat>
#include <cstdint>

#include "decode_kernels.hpp"
#include "gguf_blocks.cuh"

namespace uaii_b200 {
namespace {

// ---- embedding: x[b] = dequant(row tokens[b] of the table), bitwise the reference's
// embedding_f32 on packed weights (dequant_gguf_row) or f32 rows.
template <int F>
__global__ void embed_kernel(const int32_t* __restrict__ tokens, int64_t B, const uint8_t* __restrict__ table,
                             int64_t vocab, int64_t D, int64_t pitch, float* __restrict__ x, int* err) {
  const int64_t sub = D / 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < B * sub; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / sub;
    const int sb = (int)(i - b * sub);
    const int32_t tok = tokens[b];
    float v[32];
    if (tok < 0 || tok >= vocab) {  // out of range: the reference refuses the step; flag it, write zeros
      if (sb == 0) atomicExch(err, 16);
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
    } else {
      int s;
      const uint8_t* blk = subblock_ptr<F>(table + tok * pitch, sb, s);
      decode32<F>(blk, s, v);
    }
    float4* o = reinterpret_cast<float4*>(x + b * D + (int64_t)sb * 32);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];  // same order on every thread
  return s;
}

// ---- x += delta (the graph's residual Add, when delta is given); y = RMSNorm(x) * w:
// ms = sum(x^2) / D, inv = 1 / sqrt(ms + eps), y = (x * inv) * w (norm.cpp:114-128).
__global__ void add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta, const float* __restrict__ w,
                                   int64_t D, float eps, float* __restrict__ y) {
  __shared__ float red[32];
  float* xr = x + blockIdx.x * D;
  const float* dr = delta ? delta + blockIdx.x * D : nullptr;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    float v = xr[i];
    if (dr) {
      v = __fadd_rn(v, dr[i]);
      xr[i] = v;
    }
    ss = __fmaf_rn(v, v, ss);
  }
  const float ms = __fdiv_rn(block_sum(ss, red), (float)D);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  float* yr = y + blockIdx.x * D;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    const float v = __fmul_rn(xr[i], inv);
    yr[i] = w ? __fmul_rn(v, w[i]) : v;
  }
}

// ---- RoPE of q and k at position `pos` and the KV-cache append.  qkv [B, q_dim + 2 kv_dim]
// (the fused projection's output), freq[head_dim / 2] = 1 / theta^(2i / head_dim) made on the
// host exactly as rope_f32 does (transformer.cpp:197-225); mode 0 rotates pairs (2i, 2i + 1),
// mode 2 (NeoX) pairs (i, i + head_dim / 2).  q_out [B, q_dim] f32; K/V caches
// [B, kv_heads, max_seq, head_dim] f16.
__device__ __forceinline__ void rotate(float a, float b, float c, float s, float& oa, float& ob) {
  oa = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  ob = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

__global__ void rope_append_kernel(const float* __restrict__ qkv, int64_t H, int64_t Hkv, int64_t hd,
                                   const float* __restrict__ freq, int64_t pos, int mode, float* __restrict__ q_out,
                                   __half* __restrict__ kc, __half* __restrict__ vc, int64_t max_seq) {
  const int64_t b = blockIdx.x;
  const int64_t q_dim = H * hd, kv_dim = Hkv * hd, half = hd / 2;
  const float* row = qkv + b * (q_dim + 2 * kv_dim);
  const float fpos = (float)pos;
  // pairs: H * half of q, then Hkv * half of k
  for (int64_t p = threadIdx.x; p < (H + Hkv) * half; p += blockDim.x) {
    const bool is_q = p < H * half;
    const int64_t pp = is_q ? p : p - H * half;
    const int64_t h = pp / half, i = pp % half;
    const float angle = __fmul_rn(fpos, freq[i]);
    float s, c;
    sincosf(angle, &s, &c);
    const int64_t ia = mode == 2 ? i : 2 * i, ib = mode == 2 ? i + half : 2 * i + 1;
    const float* src = row + (is_q ? 0 : q_dim) + h * hd;
    float oa, ob;
    rotate(src[ia], src[ib], c, s, oa, ob);
    if (is_q) {
      q_out[b * q_dim + h * hd + ia] = oa;
      q_out[b * q_dim + h * hd + ib] = ob;
    } else {
      __half* dst = kc + ((b * Hkv + h) * max_seq + pos) * hd;
      dst[ia] = __float2half_rn(oa);
      dst[ib] = __float2half_rn(ob);
    }
  }
  for (int64_t j = threadIdx.x; j < kv_dim; j += blockDim.x) {
    const int64_t h = j / hd, d = j % hd;
    vc[((b * Hkv + h) * max_seq + pos) * hd + d] = __float2half_rn(row[q_dim + kv_dim + j]);
  }
}

// ---- attention of one new position over the cache (attention_kv_f32, transformer.cpp:227-345:
// scores q.k * scale, softmax over positions 0..len-1, sum of p * v), split over the
// positions: CTA (split, kv head, b) handles a chunk for the G = H / Hkv query heads that
// share the kv head and writes their unnormalised partial sums, maxima and denominators.
// Threads = head_dim (128): phase 1 has each thread score whole positions for all G heads
// (K rows read once), phase 3 has thread d accumulate dimension d for all G heads (V rows
// read coalesced).
constexpr int kAttnChunk = 256;   // positions per split

template <int HD, int G>
__global__ void __launch_bounds__(HD) attn_decode_kernel(const float* __restrict__ q, const __half* __restrict__ kc,
                                                         const __half* __restrict__ vc, int64_t H, int64_t Hkv,
                                                         int64_t len, int64_t max_seq, float scale,
                                                         float* __restrict__ po, float* __restrict__ pm,
                                                         float* __restrict__ pl) {
  static_assert(HD == 128, "head_dim 128: one thread per dimension");
  const int64_t split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int64_t nsplit = gridDim.x;
  const int64_t j0 = split * kAttnChunk, j1 = min(len, j0 + kAttnChunk);
  __shared__ __align__(16) float sq[G][HD];
  __shared__ __align__(16) float sp[G][kAttnChunk];
  __shared__ float red[G][HD / 32];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
#pragma unroll
  for (int g = 0; g < G; ++g) sq[g][t] = q[(b * H + kvh * G + g) * HD + t];
  __syncthreads();
  const __half* K = kc + (b * Hkv + kvh) * max_seq * HD;
  const __half* V = vc + (b * Hkv + kvh) * max_seq * HD;
  // phase 1: thread t scores positions j0 + t, j0 + t + HD, ... for all G heads (each K row read once)
  float mloc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) mloc[g] = -FLT_MAX;
  for (int64_t j = j0 + t; j < j1; j += HD) {
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.f;
    const uint4* kr = reinterpret_cast<const uint4*>(K + j * HD);
#pragma unroll 2
    for (int c = 0; c < HD / 8; ++c) {
      const uint4 u = kr[c];
      const __half2* h2 = reinterpret_cast<const __half2*>(&u);
      float kf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 kv = __half22float2(h2[e]);
        kf[2 * e] = kv.x;
        kf[2 * e + 1] = kv.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 qa = *reinterpret_cast<const float4*>(&sq[g][8 * c]);
        const float4 qb = *reinterpret_cast<const float4*>(&sq[g][8 * c + 4]);
        acc[g] = __fmaf_rn(qa.x, kf[0], acc[g]);
        acc[g] = __fmaf_rn(qa.y, kf[1], acc[g]);
        acc[g] = __fmaf_rn(qa.z, kf[2], acc[g]);
        acc[g] = __fmaf_rn(qa.w, kf[3], acc[g]);
        acc[g] = __fmaf_rn(qb.x, kf[4], acc[g]);
        acc[g] = __fmaf_rn(qb.y, kf[5], acc[g]);
        acc[g] = __fmaf_rn(qb.z, kf[6], acc[g]);
        acc[g] = __fmaf_rn(qb.w, kf[7], acc[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float s = __fmul_rn(acc[g], scale);
      sp[g][j - j0] = s;
      mloc[g] = fmaxf(mloc[g], s);
    }
  }
  // phase 2: chunk maximum, exponentials and their sum
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = mloc[g];
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[g][w] = m;
  }
  __syncthreads();
  float M[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = -FLT_MAX;
    for (int i = 0; i < HD / 32; ++i) m = fmaxf(m, red[g][i]);
    M[g] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float l = 0.f;
    for (int64_t j = j0 + t; j < j1; j += HD) {
      const float e = __expf(__fsub_rn(sp[g][j - j0], M[g]));
      sp[g][j - j0] = e;
      l = __fadd_rn(l, e);
    }
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) red[g][w] = l;
  }
  __syncthreads();
  // phase 3: o[g][t] = sum_j p[g][j] v[j][t]; V rows read coalesced, p four positions at a time
  float o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g] = 0.f;
  const int64_t n = j1 - j0;
  int64_t jj = 0;
  for (; jj + 4 <= n; jj += 4) {
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = __half2float(V[(j0 + jj + e) * HD + t]);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4 p = *reinterpret_cast<const float4*>(&sp[g][jj]);
      o[g] = __fmaf_rn(p.x, v[0], o[g]);
      o[g] = __fmaf_rn(p.y, v[1], o[g]);
      o[g] = __fmaf_rn(p.z, v[2], o[g]);
      o[g] = __fmaf_rn(p.w, v[3], o[g]);
    }
  }
  for (; jj < n; ++jj) {
    const float v = __half2float(V[(j0 + jj) * HD + t]);
#pragma unroll
    for (int g = 0; g < G; ++g) o[g] = __fmaf_rn(sp[g][jj], v, o[g]);
  }
  const int64_t base = (b * H + kvh * G) * nsplit + split;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    po[(base + g * nsplit) * HD + t] = o[g];
    if (t == 0) {
      float l = 0.f;
      for (int i = 0; i < HD / 32; ++i) l += red[g][i];
      pm[base + g * nsplit] = n > 0 ? M[g] : -FLT_MAX;
      pl[base + g * nsplit] = n > 0 ? l : 0.f;
    }
  }
}

// out[b, h] = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s
template <int HD>
__global__ void attn_combine_kernel(const float* __restrict__ po, const float* __restrict__ pm,
                                    const float* __restrict__ pl, int nsplit, float* __restrict__ out) {
  const int64_t bh = blockIdx.x;
  const int t = threadIdx.x;
  float M = -FLT_MAX;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, pm[bh * nsplit + s]);
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float l = pl[bh * nsplit + s];
    if (l == 0.f) continue;
    const float f = __expf(__fsub_rn(pm[bh * nsplit + s], M));
    L = __fmaf_rn(f, l, L);
    acc = __fmaf_rn(f, po[(bh * nsplit + s) * HD + t], acc);
  }
  out[bh * HD + t] = L > 0.f ? __fdiv_rn(acc, L) : 0.f;
}

// ---- greedy token: the first index of the largest value, as the reference's sampler scans
// (libs/uaii-runtime/src/sampling.cpp:38-50: strictly greater replaces; a NaN never does, and
// a NaN at index 0 is never replaced).
__global__ void argmax_kernel(const float* __restrict__ logits, int64_t V, int32_t* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const float* row = logits + blockIdx.x * V;
  float bv = -INFINITY;
  int bi = -1;
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = row[i];
    if (v > bv || (bi < 0 && !(v != v))) { bv = v; bi = (int)i; }  // first finite-or-inf value, then strictly greater
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
      if (si[i] >= 0 && (bi < 0 || sv[i] > bv || (sv[i] == bv && si[i] < bi))) { bv = sv[i]; bi = si[i]; }
    out[blockIdx.x] = row[0] != row[0] ? 0 : (bi < 0 ? 0 : bi);
  }
}

// ---- device-side synthetic inputs ------------------------------------------------------
// The counter-based normal generator of uaii_moe_fill_normal (splitmix64 finaliser keyed by
// (seed, stream), Box-Muller in double precision): the same draws up to the last bit of the
// device's double-precision log/sin/cos.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float normal_at(uint64_t key, int64_t i, float mean, float std) {
  const uint64_t p = (uint64_t)(i >> 1);
  const uint64_t a = mix64(key + 2 * p), b = mix64(key + 2 * p + 1);
  const double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
  const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
  const double r = sqrt(-2.0 * log(u1));
  const double two_pi = 6.283185307179586476925286766559;
  const double z = (i & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
  return (float)((double)mean + (double)std * z);
}

__global__ void fill_normal_kernel(float* __restrict__ out, int64_t n, uint64_t key, float mean, float std) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = normal_at(key, i, mean, std);
}

__global__ void fill_normal_f16_kernel(__half* __restrict__ out, int64_t n, uint64_t key, float mean, float std) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(normal_at(key, i, mean, std));
}

// GGUF block quantizers of uaii_moe_quantize_rows (round to nearest, per-block max-abs scales;
// Q4_K also per-sub-block minima), one thread per block, the same f32 arithmetic in the same
// order, so the packed bytes are identical to the host quantizer's.
__device__ __forceinline__ float signed_absmax(const float* x, int n) {
  float best = 0.f;
  for (int i = 0; i < n; ++i)
    if (fabsf(x[i]) > fabsf(best)) best = x[i];
  return best;
}
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
__device__ __forceinline__ int rnd(float v) { return (int)rintf(v); }
__device__ __forceinline__ uint16_t h_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ float h_val(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ void put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)(v & 0xff); p[1] = (uint8_t)(v >> 8); }

__device__ void q4_0_block(const float* x, uint8_t* b) {
  const float mx = signed_absmax(x, 32);
  const uint16_t dh = h_bits(__fdiv_rn(mx, -8.0f));
  const float d = h_val(dh);
  const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
  put16(b, dh);
  for (int j = 0; j < 16; ++j) {
    const int q0 = clampi(rnd(__fmul_rn(x[j], id)) + 8, 0, 15);
    const int q1 = clampi(rnd(__fmul_rn(x[j + 16], id)) + 8, 0, 15);
    b[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}

__device__ void q8_0_block(const float* x, uint8_t* b) {
  const float amax = fabsf(signed_absmax(x, 32));
  const uint16_t dh = h_bits(__fdiv_rn(amax, 127.0f));
  const float d = h_val(dh);
  const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
  put16(b, dh);
  for (int j = 0; j < 32; ++j) b[2 + j] = (uint8_t)(int8_t)clampi(rnd(__fmul_rn(x[j], id)), -127, 127);
}

__device__ void q4_k_block(const float* x, uint8_t* b) {
  float scale[8], negmin[8];
  for (int g = 0; g < 8; ++g) {
    float lo = 0.f, hi = x[32 * g];
    for (int l = 0; l < 32; ++l) {
      lo = fminf(lo, x[32 * g + l]);
      hi = fmaxf(hi, x[32 * g + l]);
    }
    hi = fmaxf(hi, lo);
    scale[g] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
    negmin[g] = -lo;
  }
  float smax = scale[0], mmax = negmin[0];
  for (int g = 1; g < 8; ++g) {
    smax = fmaxf(smax, scale[g]);
    mmax = fmaxf(mmax, negmin[g]);
  }
  const uint16_t dh = h_bits(__fdiv_rn(smax, 63.0f)), mh = h_bits(__fdiv_rn(mmax, 63.0f));
  const float d = h_val(dh), dm = h_val(mh);
  int sc[8], mn[8];
  for (int g = 0; g < 8; ++g) {
    sc[g] = d > 0.f ? clampi(rnd(__fdiv_rn(scale[g], d)), 0, 63) : 0;
    mn[g] = dm > 0.f ? clampi(rnd(__fdiv_rn(negmin[g], dm)), 0, 63) : 0;
  }
  put16(b, dh);
  put16(b + 2, mh);
  uint8_t* s12 = b + 4;
  for (int j = 0; j < 4; ++j) {
    s12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s12[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    s12[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
  }
  for (int c = 0; c < 4; ++c) {
    const float ed0 = __fmul_rn(d, (float)sc[2 * c]), em0 = __fmul_rn(dm, (float)mn[2 * c]);
    const float ed1 = __fmul_rn(d, (float)sc[2 * c + 1]), em1 = __fmul_rn(dm, (float)mn[2 * c + 1]);
    for (int l = 0; l < 32; ++l) {
      const int q0 = ed0 > 0.f ? clampi(rnd(__fdiv_rn(__fadd_rn(x[64 * c + l], em0), ed0)), 0, 15) : 0;
      const int q1 = ed1 > 0.f ? clampi(rnd(__fdiv_rn(__fadd_rn(x[64 * c + 32 + l], em1), ed1)), 0, 15) : 0;
      b[16 + 32 * c + l] = (uint8_t)(q0 | (q1 << 4));
    }
  }
}

__device__ void q6_k_block(const float* x, uint8_t* b) {
  float scale[16];
  float smax = 0.f;
  for (int j = 0; j < 16; ++j) {
    scale[j] = __fdiv_rn(signed_absmax(x + 16 * j, 16), -32.0f);
    smax = fmaxf(smax, fabsf(scale[j]));
  }
  const uint16_t dh = h_bits(__fdiv_rn(smax, 127.0f));
  const float d = h_val(dh);
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  int sc[16];
  for (int j = 0; j < 16; ++j) sc[j] = d > 0.f ? clampi(rnd(__fdiv_rn(scale[j], d)), -128, 127) : 0;
  for (int half = 0; half < 2; ++half)
    for (int l = 0; l < 32; ++l) {
      int q[4];
      for (int c = 0; c < 4; ++c) {
        const int idx = 128 * half + 32 * c + l;
        const float e = __fmul_rn(d, (float)sc[idx / 16]);
        q[c] = e != 0.f ? clampi(rnd(__fdiv_rn(x[idx], e)) + 32, 0, 63) : 32;
      }
      ql[64 * half + l] = (uint8_t)((q[0] & 15) | ((q[2] & 15) << 4));
      ql[64 * half + 32 + l] = (uint8_t)((q[1] & 15) | ((q[3] & 15) << 4));
      qh[32 * half + l] = (uint8_t)((q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) | ((q[3] >> 4) << 6));
    }
  for (int j = 0; j < 16; ++j) b[192 + j] = (uint8_t)(int8_t)sc[j];
  put16(b + 208, dh);
}

template <int F>
__global__ void quantize_kernel(const float* __restrict__ src, int64_t rows, int64_t cols, uint8_t* __restrict__ dst) {
  constexpr int QK = F == kQ4_0 || F == kQ8_0 ? 32 : 256;
  const int64_t nb = cols / QK, pitch = fmt_row_bytes(F, cols);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * nb; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nb, c = i - r * nb;
    const float* x = src + r * cols + c * QK;
    uint8_t* blk = dst + r * pitch + c * fmt_block_bytes(F);
    if constexpr (F == kQ4_0) q4_0_block(x, blk);
    else if constexpr (F == kQ8_0) q8_0_block(x, blk);
    else if constexpr (F == kQ4_K) q4_k_block(x, blk);
    else q6_k_block(x, blk);
  }
}

__global__ void to_half_rows_kernel(const float* __restrict__ src, int64_t rows, int64_t cols, __half* __restrict__ dst,
                                    int64_t dst_pitch) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * cols; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    dst[r * dst_pitch + c] = __float2half_rn(src[i]);
  }
}

unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 16) b = 148 * 16;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

uint64_t normal_key(uint64_t seed, uint64_t stream) {
  auto mix = [](uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  };
  return mix(seed ^ mix(stream * 0xD1B54A32D192ED03ull + 0x7F4A7C15ull));
}

cudaError_t launch_embed(int fmt, const void* table, int64_t vocab, int64_t D, const int32_t* tokens, int64_t B,
                         float* x, int* err, cudaStream_t st) {
  if (D % 32 != 0) return cudaErrorInvalidValue;
  const int64_t pitch = fmt == kF32 ? 4 * D : fmt_row_bytes(fmt, D);
  const unsigned g = grid_for(B * (D / 32), 128);
  const uint8_t* t = static_cast<const uint8_t*>(table);
  switch (fmt) {
    case kF32: embed_kernel<kF32><<<g, 128, 0, st>>>(tokens, B, t, vocab, D, pitch, x, err); break;
    case kF16: embed_kernel<kF16><<<g, 128, 0, st>>>(tokens, B, t, vocab, D, pitch, x, err); break;
    case kQ4_0: embed_kernel<kQ4_0><<<g, 128, 0, st>>>(tokens, B, t, vocab, D, pitch, x, err); break;
    case kQ8_0: embed_kernel<kQ8_0><<<g, 128, 0, st>>>(tokens, B, t, vocab, D, pitch, x, err); break;
    case kQ4_K: embed_kernel<kQ4_K><<<g, 128, 0, st>>>(tokens, B, t, vocab, D, pitch, x, err); break;
    case kQ6_K: embed_kernel<kQ6_K><<<g, 128, 0, st>>>(tokens, B, t, vocab, D, pitch, x, err); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_add_rmsnorm(float* x, const float* delta, const float* w, int64_t B, int64_t D, float eps, float* y,
                               cudaStream_t st) {
  if (B == 0) return cudaSuccess;
  add_rmsnorm_kernel<<<(unsigned)B, 256, 0, st>>>(x, delta, w, D, eps, y);
  return cudaGetLastError();
}

cudaError_t launch_rope_append(const float* qkv, int64_t B, int64_t H, int64_t Hkv, int64_t hd, const float* freq,
                               int64_t pos, int mode, float* q_out, void* kc, void* vc, int64_t max_seq,
                               cudaStream_t st) {
  if (hd % 2 || pos < 0 || pos >= max_seq) return cudaErrorInvalidValue;
  rope_append_kernel<<<(unsigned)B, 256, 0, st>>>(qkv, H, Hkv, hd, freq, pos, mode, q_out, static_cast<__half*>(kc),
                                                  static_cast<__half*>(vc), max_seq);
  return cudaGetLastError();
}

int attn_splits(int64_t len) { return (int)((len + kAttnChunk - 1) / kAttnChunk); }

cudaError_t launch_attn_decode(const float* q, const void* kc, const void* vc, int64_t B, int64_t H, int64_t Hkv,
                               int64_t hd, int64_t len, int64_t max_seq, float* po, float* pm, float* pl, float* out,
                               cudaStream_t st) {
  if (hd != 128 || Hkv <= 0 || H % Hkv || len <= 0 || len > max_seq) return cudaErrorInvalidValue;
  const int ns = attn_splits(len);
  const float scale = 1.0f / sqrtf((float)hd);  // attention_kv_f32's default scale
  const dim3 grid((unsigned)ns, (unsigned)Hkv, (unsigned)B);
  const __half* k = static_cast<const __half*>(kc);
  const __half* v = static_cast<const __half*>(vc);
  switch (H / Hkv) {
    case 1: attn_decode_kernel<128, 1><<<grid, 128, 0, st>>>(q, k, v, H, Hkv, len, max_seq, scale, po, pm, pl); break;
    case 2: attn_decode_kernel<128, 2><<<grid, 128, 0, st>>>(q, k, v, H, Hkv, len, max_seq, scale, po, pm, pl); break;
    case 4: attn_decode_kernel<128, 4><<<grid, 128, 0, st>>>(q, k, v, H, Hkv, len, max_seq, scale, po, pm, pl); break;
    case 8: attn_decode_kernel<128, 8><<<grid, 128, 0, st>>>(q, k, v, H, Hkv, len, max_seq, scale, po, pm, pl); break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_combine_kernel<128><<<(unsigned)(B * H), 128, 0, st>>>(po, pm, pl, ns, out);
  return cudaGetLastError();
}

cudaError_t launch_to_half_rows(const float* src, int64_t rows, int64_t cols, void* dst, int64_t dst_pitch,
                                cudaStream_t st) {
  if (rows * cols == 0) return cudaSuccess;
  to_half_rows_kernel<<<grid_for(rows * cols, 256), 256, 0, st>>>(src, rows, cols, static_cast<__half*>(dst), dst_pitch);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float* logits, int64_t B, int64_t V, int32_t* out, cudaStream_t st) {
  if (B == 0) return cudaSuccess;
  argmax_kernel<<<(unsigned)B, 1024, 0, st>>>(logits, V, out);
  return cudaGetLastError();
}

cudaError_t launch_fill_normal(float* out, int64_t n, uint64_t seed, uint64_t stream, float mean, float std,
                               cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  fill_normal_kernel<<<grid_for(n, 256), 256, 0, st>>>(out, n, normal_key(seed, stream), mean, std);
  return cudaGetLastError();
}

cudaError_t launch_fill_normal_f16(void* out, int64_t n, uint64_t seed, uint64_t stream, float mean, float std,
                                   cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  fill_normal_f16_kernel<<<grid_for(n, 256), 256, 0, st>>>(static_cast<__half*>(out), n, normal_key(seed, stream),
                                                           mean, std);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(int fmt, const float* src, int64_t rows, int64_t cols, void* dst, cudaStream_t st) {
  const int qk = fmt_block_elems(fmt);
  if (cols % qk != 0) return cudaErrorInvalidValue;
  const int64_t blocks = rows * (cols / qk);
  if (blocks == 0) return cudaSuccess;
  uint8_t* d = static_cast<uint8_t*>(dst);
  switch (fmt) {
    case kQ4_0: quantize_kernel<kQ4_0><<<grid_for(blocks, 128), 128, 0, st>>>(src, rows, cols, d); break;
    case kQ8_0: quantize_kernel<kQ8_0><<<grid_for(blocks, 128), 128, 0, st>>>(src, rows, cols, d); break;
    case kQ4_K: quantize_kernel<kQ4_K><<<grid_for(blocks, 128), 128, 0, st>>>(src, rows, cols, d); break;
    case kQ6_K: quantize_kernel<kQ6_K><<<grid_for(blocks, 128), 128, 0, st>>>(src, rows, cols, d); break;
    default: return cudaErrorNotSupported;
  }
  return cudaGetLastError();
}

}  // namespace uaii_b200
