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
#include <cuda.h>
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
// One block per row, float4 columns; a thread keeps its (at most kNormVec) float4s of x in
// registers between the two passes, so every load of a row is issued at once.
constexpr int kNormVec = 4;
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                                          const float* __restrict__ w, int D, float eps,
                                                          float* __restrict__ y) {
  __shared__ float red[32];
  float4* xr = reinterpret_cast<float4*>(x + (int64_t)blockIdx.x * D);
  const float4* dr = delta ? reinterpret_cast<const float4*>(delta + (int64_t)blockIdx.x * D) : nullptr;
  const int n4 = D / 4;
  float4 v[kNormVec];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormVec; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < n4) {
      v[k] = xr[i];
      if (dr) {
        const float4 d = dr[i];
        v[k].x = __fadd_rn(v[k].x, d.x);
        v[k].y = __fadd_rn(v[k].y, d.y);
        v[k].z = __fadd_rn(v[k].z, d.z);
        v[k].w = __fadd_rn(v[k].w, d.w);
        xr[i] = v[k];
      }
      ss = __fmaf_rn(v[k].x, v[k].x, ss);
      ss = __fmaf_rn(v[k].y, v[k].y, ss);
      ss = __fmaf_rn(v[k].z, v[k].z, ss);
      ss = __fmaf_rn(v[k].w, v[k].w, ss);
    }
  }
  const float ms = __fdiv_rn(block_sum(ss, red), (float)D);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  float4* yr = reinterpret_cast<float4*>(y + (int64_t)blockIdx.x * D);
  const float4* wr = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int k = 0; k < kNormVec; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < n4) {
      float4 o = make_float4(__fmul_rn(v[k].x, inv), __fmul_rn(v[k].y, inv), __fmul_rn(v[k].z, inv),
                             __fmul_rn(v[k].w, inv));
      if (wr) {
        const float4 g = wr[i];
        o = make_float4(__fmul_rn(o.x, g.x), __fmul_rn(o.y, g.y), __fmul_rn(o.z, g.z), __fmul_rn(o.w, g.w));
      }
      yr[i] = o;
    }
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
  const int q_dim = (int)(H * hd), kv_dim = (int)(Hkv * hd), half = (int)(hd / 2), nq = (int)H * half;
  const float* row = qkv + b * (q_dim + 2 * kv_dim);
  const float fpos = (float)pos;
  // pairs: H * half of q, then Hkv * half of k
  for (int p = threadIdx.x; p < nq + (int)Hkv * half; p += blockDim.x) {
    const bool is_q = p < nq;
    const int pp = is_q ? p : p - nq;
    const int h = pp / half, i = pp - h * half;
    const float angle = __fmul_rn(fpos, freq[i]);
    float s, c;
    sincosf(angle, &s, &c);
    const int ia = mode == 2 ? i : 2 * i, ib = mode == 2 ? i + half : 2 * i + 1;
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
  for (int j = threadIdx.x; j < kv_dim; j += blockDim.x) {
    const int h = j / (int)hd, d = j - h * (int)hd;
    vc[((b * Hkv + h) * max_seq + pos) * hd + d] = __float2half_rn(row[q_dim + kv_dim + j]);
  }
}

// ---- attention of one new position over the cache (attention_kv_f32, transformer.cpp:227-345:
// scores q.k * scale, softmax over positions 0..len-1, sum of p * v), on the tensor cores.
// CTA (split, kv head, b) handles kAttnChunk positions for the G = H / Hkv query heads that
// share the kv head (rows 0..G-1 of 16-row mma.sync tiles) and writes their unnormalised
// partial sums, maxima and denominators.  TMA brings the chunk's K and V rows (f16, 128 dims
// as two 64-column SWIZZLE_128B boxes each) into shared memory; warp w scores positions
// 32w .. 32w+31 (S = Q K^T, m16n8k16, K rows as the B operand through ldmatrix), the row
// maxima and sums meet across the warps in shared memory, and the same warp multiplies its
// probabilities (the S accumulators re-packed as the A operand) by its V rows (ldmatrix.trans).
// q and p enter the products rounded to f16; scores, exponentials and sums are f32.
constexpr int kAttnChunk = 128;   // positions per split
constexpr int kAttnWarps = 4;     // 32 positions each

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// byte offset of (row, 16-byte chunk c of 8) in a [rows][128 B] SWIZZLE_128B box
__device__ __forceinline__ uint32_t swz(int row, int c) { return (uint32_t)(row * 128 + ((c ^ (row & 7)) << 4)); }

template <int G>
__global__ void __launch_bounds__(32 * kAttnWarps) attn_mma_kernel(const __grid_constant__ CUtensorMap tk,
                                                                   const __grid_constant__ CUtensorMap tv,
                                                                   const float* __restrict__ q, int64_t H, int64_t Hkv,
                                                                   int64_t len, int64_t max_seq, float scale,
                                                                   float* __restrict__ po, float* __restrict__ pm,
                                                                   float* __restrict__ pl, int* err) {
  static_assert(G >= 1 && G <= 8, "query heads per kv head");
  constexpr int kBox = kAttnChunk * 128;  // bytes of one 64-column box
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sk = smem;             // K: box 0 (dims 0-63), box 1 (dims 64-127)
  uint8_t* sv = smem + 2 * kBox;  // V: the same
  float* red = reinterpret_cast<float*>(smem + 4 * kBox);  // [2][kAttnWarps][8]
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + 2 * kAttnWarps * 8);
  const int64_t split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int64_t nsplit = gridDim.x;
  const int64_t j0 = split * kAttnChunk;
  const int n = (int)min((int64_t)kAttnChunk, len - j0);
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, g = lane >> 2, tq = lane & 3;
  if (t == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (t == 0) {
    const int row0 = (int)((b * Hkv + kvh) * max_seq + j0);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(4 * kBox)
                 : "memory");
#pragma unroll
    for (int box = 0; box < 2; ++box) {
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
          ::"r"(smem_addr(sk + box * kBox)), "l"(&tk), "r"(smem_addr(bar)), "r"(64 * box), "r"(row0) : "memory");
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
          ::"r"(smem_addr(sv + box * kBox)), "l"(&tv), "r"(smem_addr(bar)), "r"(64 * box), "r"(row0) : "memory");
    }
  }
  // Q rows g < G as the A operand of the 8 k-steps: pairs (2tq, 2tq+1) and (2tq+8, 2tq+9)
  uint32_t qa[8][2];
  {
    const float* qr = q + (b * H + kvh * G + (g < G ? g : 0)) * 128;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const float2 lo = *reinterpret_cast<const float2*>(qr + 16 * ks + 2 * tq);
      const float2 hi = *reinterpret_cast<const float2*>(qr + 16 * ks + 2 * tq + 8);
      qa[ks][0] = g < G ? pack_h2(lo.x, lo.y) : 0u;
      qa[ks][1] = g < G ? pack_h2(hi.x, hi.y) : 0u;
    }
  }
  {  // bounded wait for the copies (about a second): a lost copy records an error instead of hanging
    uint32_t done = 0;
    const long long t0 = clock64();
    while (true) {
      asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0, 1000000;\n\t"
                   "selp.u32 %0, 1, 0, p;\n\t}\n" : "=r"(done) : "r"(smem_addr(bar)) : "memory");
      if (done || clock64() - t0 > 2000000000LL) break;
    }
    if (!done && t == 0) atomicExch(err, 17);
  }
  if (n < kAttnChunk) {  // the last chunk: V rows past the end (other sequences, or never written) become zeros,
    // so that the zero probabilities of masked positions cannot meet a non-finite value there
    for (int i = t; i < (kAttnChunk - n) * 16; i += 32 * kAttnWarps) {
      const int row = n + (i >> 4), c = i & 15;  // 16 chunks of 16 bytes per row: 8 per box
      *reinterpret_cast<uint4*>(sv + (c >> 3) * kBox + row * 128 + ((c & 7) << 4)) = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
  }
  // S = Q K^T for positions 32w + 8nt + (0..7); ldmatrix.x4: k-steps ks, ks+1, low and high 8 dims
  float sc[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[nt][i] = 0.f;
  const int mi = lane >> 3, r8 = lane & 7;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int pos = 32 * w + 8 * nt + r8;
#pragma unroll
    for (int ks = 0; ks < 8; ks += 2) {
      const int kstep = ks + (mi >> 1);  // matrices: (ks, lo), (ks, hi), (ks+1, lo), (ks+1, hi)
      const int chunk = 2 * (kstep & 3) + (mi & 1);
      const uint32_t addr = smem_addr(sk + (kstep >> 2) * kBox) + swz(pos, chunk);
      uint32_t b0, b1, b2, b3;
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                   : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(addr));
      mma16816(sc[nt], qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
      mma16816(sc[nt], qa[ks + 1][0], 0u, qa[ks + 1][1], 0u, b2, b3);
    }
  }
  // scale, mask positions past the end, row maxima (rows g: accumulators 0, 1; columns 2tq, 2tq+1)
  float m = -FLT_MAX;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int p = 32 * w + 8 * nt + 2 * tq + i;
      sc[nt][i] = p < n ? __fmul_rn(sc[nt][i], scale) : -FLT_MAX;
      m = fmaxf(m, sc[nt][i]);
    }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  if (tq == 0) red[w * 8 + g] = m;
  __syncthreads();
  float M = red[g];
#pragma unroll
  for (int i = 1; i < kAttnWarps; ++i) M = fmaxf(M, red[i * 8 + g]);
  float l = 0.f;
  uint32_t pa[2][2];  // P as the A operand of the two 16-position k-steps
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    float e[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      e[i] = sc[nt][i] > -FLT_MAX ? __expf(__fsub_rn(sc[nt][i], M)) : 0.f;
      l = __fadd_rn(l, e[i]);
    }
    pa[nt >> 1][nt & 1] = pack_h2(e[0], e[1]);
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  if (tq == 0) red[kAttnWarps * 8 + w * 8 + g] = l;
  // O = P V over this warp's 32 positions: 16 column tiles of 8 dims; ldmatrix.trans x4 gives
  // (positions lo, hi) x (dims tile dn, dn + 1)
  float o[16][4];
#pragma unroll
  for (int dn = 0; dn < 16; ++dn)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[dn][i] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
#pragma unroll
    for (int dn = 0; dn < 16; dn += 2) {
      const int pos = 32 * w + 16 * kk + 8 * (mi & 1) + r8;
      const int chunk = dn + (mi >> 1);  // 8-dim tile = 16-byte chunk; 8 chunks per box
      const uint32_t addr = smem_addr(sv + (chunk >> 3) * kBox) + swz(pos, chunk & 7);
      uint32_t b0, b1, b2, b3;
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                   : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(addr));
      mma16816(o[dn], pa[kk][0], 0u, pa[kk][1], 0u, b0, b1);
      mma16816(o[dn + 1], pa[kk][0], 0u, pa[kk][1], 0u, b2, b3);
    }
  }
  __syncthreads();  // every warp is done with K: its space holds the four warps' partial O rows
  float* ored = reinterpret_cast<float*>(sk);  // [kAttnWarps][8 rows][128 dims]
  if (g < G) {
#pragma unroll
    for (int dn = 0; dn < 16; ++dn) {
      float2* d = reinterpret_cast<float2*>(ored + (w * 8 + g) * 128 + 8 * dn + 2 * tq);
      *d = make_float2(o[dn][0], o[dn][1]);
    }
  }
  __syncthreads();
  const int64_t base = (b * H + kvh * G) * nsplit + split;
  for (int i = t; i < G * 128; i += 32 * kAttnWarps) {
    const int row = i >> 7, d = i & 127;
    float s = ored[row * 128 + d];
#pragma unroll
    for (int ww = 1; ww < kAttnWarps; ++ww) s = __fadd_rn(s, ored[(ww * 8 + row) * 128 + d]);
    po[(base + row * nsplit) * 128 + d] = s;
  }
  if (t < G) {
    float L = 0.f, MM = red[t];
    for (int ww = 0; ww < kAttnWarps; ++ww) {
      L = __fadd_rn(L, red[kAttnWarps * 8 + ww * 8 + t]);
      MM = fmaxf(MM, red[ww * 8 + t]);
    }
    pm[base + t * nsplit] = n > 0 ? MM : -FLT_MAX;
    pl[base + t * nsplit] = n > 0 ? L : 0.f;
  }
}

constexpr int kAttnSmem = 4 * kAttnChunk * 128 + 4 * 2 * kAttnWarps * 8 + 16 + 1024;

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

__device__ __forceinline__ uint64_t key_of(uint64_t seed, uint64_t stream) {
  return mix64(seed ^ mix64(stream * 0xD1B54A32D192ED03ull + 0x7F4A7C15ull));
}

// rows of `cols` f16 draws, `pitch` apart; row r is stream stream0 + r of the generator
__global__ void fill_normal_f16_rows_kernel(__half* __restrict__ out, int64_t rows, int64_t cols, int64_t pitch,
                                            uint64_t seed, uint64_t stream0, float mean, float std) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * cols; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    out[r * pitch + c] = __float2half_rn(normal_at(key_of(seed, stream0 + (uint64_t)r), c, mean, std));
  }
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
  if (D % 4 != 0 || D > 4 * 256 * kNormVec) return cudaErrorInvalidValue;
  add_rmsnorm_kernel<<<(unsigned)B, 256, 0, st>>>(x, delta, w, (int)D, eps, y);
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

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool make_kv_map(void* map, const void* cache, int64_t rows) {
  static EncodeTiledFn enc = nullptr;
  if (!enc) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess)
      return false;
    enc = reinterpret_cast<EncodeTiledFn>(p);
  }
  if (reinterpret_cast<uintptr_t>(cache) & 15) return false;
  const cuuint64_t dims[2] = {128, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {256};
  const cuuint32_t box[2] = {64, (cuuint32_t)kAttnChunk};
  const cuuint32_t es[2] = {1, 1};
  return enc(static_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(cache), dims,
             strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int attn_splits(int64_t len) { return (int)((len + kAttnChunk - 1) / kAttnChunk); }

cudaError_t launch_attn_decode(const void* kmap, const void* vmap, const float* q, int64_t B, int64_t H, int64_t Hkv,
                               int64_t hd, int64_t len, int64_t max_seq, float* po, float* pm, float* pl, float* out,
                               int* err, cudaStream_t st) {
  if (hd != 128 || Hkv <= 0 || H % Hkv || len <= 0 || len > max_seq || H / Hkv > 8) return cudaErrorInvalidValue;
  const int ns = attn_splits(len);
  const float scale = 1.0f / sqrtf((float)hd);  // attention_kv_f32's default scale
  const dim3 grid((unsigned)ns, (unsigned)Hkv, (unsigned)B);
  const CUtensorMap& tk = *static_cast<const CUtensorMap*>(kmap);
  const CUtensorMap& tv = *static_cast<const CUtensorMap*>(vmap);
  auto run = [&](auto kern, int gi) -> cudaError_t {
    static bool attr[9] = {};
    if (!attr[gi]) {
      const cudaError_t a = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
      if (a != cudaSuccess) return a;
      attr[gi] = true;
    }
    kern<<<grid, 32 * kAttnWarps, kAttnSmem, st>>>(tk, tv, q, H, Hkv, len, max_seq, scale, po, pm, pl, err);
    return cudaGetLastError();
  };
  cudaError_t e;
  switch (H / Hkv) {
    case 1: e = run(attn_mma_kernel<1>, 1); break;
    case 2: e = run(attn_mma_kernel<2>, 2); break;
    case 4: e = run(attn_mma_kernel<4>, 4); break;
    case 8: e = run(attn_mma_kernel<8>, 8); break;
    default: return cudaErrorInvalidValue;
  }
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

cudaError_t launch_fill_normal_f16_rows(void* out, int64_t rows, int64_t cols, int64_t pitch, uint64_t seed,
                                        uint64_t stream0, float mean, float std, cudaStream_t st) {
  if (rows * cols == 0) return cudaSuccess;
  fill_normal_f16_rows_kernel<<<grid_for(rows * cols, 256), 256, 0, st>>>(static_cast<__half*>(out), rows, cols, pitch,
                                                                          seed, stream0, mean, std);
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
