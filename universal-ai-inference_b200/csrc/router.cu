// router.cu -- MoERouter on the device (reference: kernels::moe_router_f32,
// libs/uaii-kernels/src/transformer.cpp:446-481).
//
// logits[t,e] reproduce the reference GEMM's summation order bit for bit
// (RefGemm::gemm_f32, libs/uaii-kernels/src/gemm_ref.cpp:45-75): for each
// 64-wide k tile, s = 0 then s += x*w sequentially; c (from 0) += s tile by
// tile.  Every multiply and add is a separate round-to-nearest operation.
// Four schedules compute the same values (the block schedule, for many experts,
// is described at router_block_kernel):
//   * token (small batches): one block per token, one thread per (k tile,
//     expert) partial, then one thread per expert adds the partials in order;
//   * chunk: a block owns 16 tokens and walks the row in chunks of 16 k tiles
//     staged in shared memory with coalesced loads (8 experts per pass),
//     folding each chunk's partials into running logits in tile order;
//   * tiled (very many experts): a block owns 16 tokens x 64 experts, stages
//     64-wide k tiles of x and w in shared memory, and each thread carries 2x2
//     dot products.
// softmax (softmax.cpp:55-75): max-subtract, exp, sequential sum over experts,
// multiply by 1/sum; exp is evaluated in double and rounded once to f32.
// top_expert is the first strict argmax of probs, stored as an f32 id.
#include "kernels.hpp"
#include "topk.cuh"

namespace uaii_b200 {
namespace {

constexpr int kTile = 64;

constexpr int kEC = 8;   // experts per pass
constexpr int kTB = 16;  // tokens per block (chunk schedule)
constexpr int kJC = 16;  // k tiles per chunk (chunk schedule)
constexpr int kTS = kTile + 1;         // staged tile stride: lanes on consecutive tiles hit distinct banks
constexpr int kXS = kJC * kTS;          // staged x chunk row (floats)

// Chunk schedule (256 threads): thread (t = tid / kJC, jj = tid % kJC) builds the
// partial of k tile (chunk + jj) for token t and kEC experts from staged x and
// w; then thread (t, e) folds the chunk's kJC partials, in tile order, into the
// running logit.  x is staged once per chunk, w once per (chunk, expert pass).
__global__ void __launch_bounds__(256) router_chunk_kernel(const float* __restrict__ x,
                                                           const float* __restrict__ w, int64_t T,
                                                           int64_t D, int64_t E,
                                                           float* __restrict__ logits) {
  extern __shared__ float sm[];
  float* xs = sm;                         // [kTB][kXS]
  float* ws = xs + kTB * kXS;             // [kEC][kJC * kTS]
  float* part = ws + kEC * kJC * kTS;     // [kTB][kEC][kJC]
  float* run = part + kTB * kEC * kJC;    // [kTB][E] running logits
  const int tid = threadIdx.x;
  const int64_t t0 = (int64_t)blockIdx.x * kTB;
  const int nkt = (int)((D + kTile - 1) / kTile);
  for (int i = tid; i < kTB * E; i += 256) run[i] = 0.f;
  const int lt = tid / kJC, jj = tid - lt * kJC;
  const bool vec = (D & 3) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
  for (int jc = 0; jc < nkt; jc += kJC) {
    const int64_t kc0 = (int64_t)jc * kTile;
    const int64_t kcn = (kc0 + kJC * kTile < D) ? kJC * kTile : D - kc0;  // valid k in this chunk
    __syncthreads();
    // coalesced x chunk; every load of a thread is issued before its stores
    if (vec && kcn == kJC * kTile && t0 + kTB <= T) {
      constexpr int kN = kTB * kJC * kTile / 4 / 256;
      float4 v[kN];
#pragma unroll
      for (int u = 0; u < kN; ++u) {
        const int i = tid + 256 * u, r = i / (kJC * kTile / 4), k4 = i - r * (kJC * kTile / 4);
        v[u] = __ldg(reinterpret_cast<const float4*>(x + (t0 + r) * D + kc0) + k4);
      }
#pragma unroll
      for (int u = 0; u < kN; ++u) {
        const int i = tid + 256 * u, r = i / (kJC * kTile / 4), k = 4 * (i - r * (kJC * kTile / 4));
        float* d = xs + r * kXS + (k / kTile) * kTS + (k % kTile);
        d[0] = v[u].x; d[1] = v[u].y; d[2] = v[u].z; d[3] = v[u].w;
      }
    } else {
      for (int i = tid; i < kTB * kJC * kTile; i += 256) {
        const int r = i / (kJC * kTile), k = i - r * (kJC * kTile);
        xs[r * kXS + (k / kTile) * kTS + (k % kTile)] = (t0 + r < T && k < kcn) ? __ldg(x + (t0 + r) * D + kc0 + k) : 0.f;
      }
    }
    for (int64_t e0 = 0; e0 < E; e0 += kEC) {
      const int ne = (int)((E - e0 < kEC) ? E - e0 : kEC);
      __syncthreads();
      if (vec && kcn == kJC * kTile && ne == kEC) {  // coalesced w chunk
        constexpr int kN = kEC * kJC * kTile / 4 / 256;
        float4 v[kN];
#pragma unroll
        for (int u = 0; u < kN; ++u) {
          const int i = tid + 256 * u, c = i / (kJC * kTile / 4), k4 = i - c * (kJC * kTile / 4);
          v[u] = __ldg(reinterpret_cast<const float4*>(w + (e0 + c) * D + kc0) + k4);
        }
#pragma unroll
        for (int u = 0; u < kN; ++u) {
          const int i = tid + 256 * u, c = i / (kJC * kTile / 4), k = 4 * (i - c * (kJC * kTile / 4));
          float* d = ws + c * kXS + (k / kTile) * kTS + (k % kTile);
          d[0] = v[u].x; d[1] = v[u].y; d[2] = v[u].z; d[3] = v[u].w;
        }
      } else {
        for (int i = tid; i < kEC * kJC * kTile; i += 256) {
          const int c = i / (kJC * kTile), k = i - c * (kJC * kTile);
          ws[c * kXS + (k / kTile) * kTS + (k % kTile)] = (c < ne && k < kcn) ? __ldg(w + (e0 + c) * D + kc0 + k) : 0.f;
        }
      }
      __syncthreads();
      const int64_t ktile0 = (int64_t)jj * kTile;
      const int kn = (int)((ktile0 + kTile <= kcn) ? kTile : (kcn > ktile0 ? kcn - ktile0 : 0));
      float sacc[kEC];
#pragma unroll
      for (int c = 0; c < kEC; ++c) sacc[c] = 0.f;
      const float* xr = xs + lt * kXS + jj * kTS;
      const float* wr = ws + jj * kTS;
      if (kn == kTile) {
#pragma unroll 8
        for (int k = 0; k < kTile; ++k) {
          const float xv = xr[k];
#pragma unroll
          for (int c = 0; c < kEC; ++c) sacc[c] = __fadd_rn(sacc[c], __fmul_rn(xv, wr[c * kXS + k]));
        }
      } else {
        for (int k = 0; k < kn; ++k) {
          const float xv = xr[k];
#pragma unroll
          for (int c = 0; c < kEC; ++c) sacc[c] = __fadd_rn(sacc[c], __fmul_rn(xv, wr[c * kXS + k]));
        }
      }
#pragma unroll
      for (int c = 0; c < kEC; ++c) part[(lt * kEC + c) * kJC + jj] = sacc[c];
      __syncthreads();
      const int ntiles = (int)((kcn + kTile - 1) / kTile);  // tiles of this chunk inside the row
      for (int idx = tid; idx < kTB * kEC; idx += 256) {
        const int l2 = idx / kEC, c = idx - l2 * kEC;
        if (c >= ne) continue;
        float acc = run[l2 * E + e0 + c];
        for (int q = 0; q < ntiles; ++q) acc = __fadd_rn(acc, __fmul_rn(1.0f, part[(l2 * kEC + c) * kJC + q]));
        run[l2 * E + e0 + c] = acc;
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < kTB * E; i += 256) {
    const int l2 = (int)(i / E);
    const int64_t t = t0 + l2;
    if (t < T) logits[t * E + (i - l2 * E)] = run[i];
  }
}

// Many experts (E >= 32): thread (token group, expert group) owns the logits of
// kRT tokens x kRE experts for the whole row.  Tile by tile (x and w of one 64-wide
// k tile staged in shared memory, k-major), it builds the tile's partials in k
// order and folds them into its running logits in tile order -- the reference
// order without any cross-thread combine.  Block: 256 threads = TG x EG groups.
constexpr int kRE = 8;  // experts per thread

// Small batches split the row across blockIdx.z: each block then covers k tiles
// [z*tpg, (z+1)*tpg) and writes the tile partials to `partials` (tile-major:
// [nkt][T*E]) for router_fold_kernel, which adds them in tile order.
// kRT: tokens per thread; EG: expert groups (4, 8 or 16, dividing the 256 threads).  Both are
// compile-time so that the staging index arithmetic is shifts and the k-step shared-memory
// offsets are immediates.  Block x owns tokens [x*T/gridDim.x, (x+1)*T/gridDim.x) (at most TB:
// the grid has at least ceil(T/TB) blocks), so a grid sized to whole waves of resident blocks
// spreads the tokens evenly; warps whose tokens all lie past the block's range skip the
// arithmetic.
template <int kRT, int EG>
__global__ void __launch_bounds__(256) router_block_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           int64_t T, int64_t D, int64_t E,
                                                           float* __restrict__ logits, float* __restrict__ partials,
                                                           int tpg) {
  extern __shared__ float sm[];
  constexpr int TG = 256 / EG, TB = TG * kRT, EB = EG * kRE;
  constexpr int XS = TB + 4, WS = EB + 4;  // padded k rows
  float* xs = sm;                      // [kTile][XS]
  float* ws = xs + kTile * XS;         // [kTile][WS]
  // Column of block expert r in a w row: experts 4..7 of every group after experts 0..3 of all
  // groups, so the 16-byte reads of one k step by all expert groups are contiguous.
  auto wcol = [](int r) { return ((r & 7) >> 2) * (EB / 2) + (r >> 3) * 4 + (r & 3); };
  const int tid = threadIdx.x, eg = tid % EG, tg = tid / EG;  // EG divides 256: every thread has a group
  const int64_t t0 = (int64_t)blockIdx.x * T / gridDim.x, e0 = (int64_t)blockIdx.y * EB;
  const int tn = (int)((int64_t)(blockIdx.x + 1) * T / gridDim.x - t0);  // tokens of this block (<= TB)
  const bool idle = (tid >> 5) * (32 / EG) * kRT >= tn;                  // warp-uniform
  float c[kRT][kRE];
#pragma unroll
  for (int a = 0; a < kRT; ++a)
#pragma unroll
    for (int b = 0; b < kRE; ++b) c[a][b] = 0.f;
  const bool vec = (D & 3) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
  const int nkt = (int)((D + kTile - 1) / kTile);
  const int j0 = partials ? (int)blockIdx.z * tpg : 0;
  const int j1 = partials ? min(nkt, j0 + tpg) : nkt;
  for (int j = j0; j < j1; ++j) {
    const int64_t k0 = (int64_t)j * kTile;
    const int kn = (int)((k0 + kTile < D) ? kTile : D - k0);
    __syncthreads();
    if (vec && kn == kTile) {  // float4 loads, transposed into k-major rows; lanes take consecutive rows
      for (int i = tid; i < TB * (kTile / 4); i += 256) {  // so that the transposed stores hit distinct banks
        const int k4 = i / TB, r = i - k4 * TB;
        const float4 v = r < tn ? __ldg(reinterpret_cast<const float4*>(x + (t0 + r) * D + k0) + k4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        xs[(4 * k4) * XS + r] = v.x; xs[(4 * k4 + 1) * XS + r] = v.y;
        xs[(4 * k4 + 2) * XS + r] = v.z; xs[(4 * k4 + 3) * XS + r] = v.w;
      }
      for (int i = tid; i < EB * (kTile / 4); i += 256) {
        const int k4 = i / EB, r = i - k4 * EB;
        const float4 v = (e0 + r < E) ? __ldg(reinterpret_cast<const float4*>(w + (e0 + r) * D + k0) + k4)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
        const int cr = wcol(r);
        ws[(4 * k4) * WS + cr] = v.x; ws[(4 * k4 + 1) * WS + cr] = v.y;
        ws[(4 * k4 + 2) * WS + cr] = v.z; ws[(4 * k4 + 3) * WS + cr] = v.w;
      }
    } else {
      for (int i = tid; i < TB * kTile; i += 256) {
        const int k = i / TB, r = i - k * TB;
        xs[k * XS + r] = (r < tn && k < kn) ? __ldg(x + (t0 + r) * D + k0 + k) : 0.f;
      }
      for (int i = tid; i < EB * kTile; i += 256) {
        const int k = i / EB, r = i - k * EB;
        ws[k * WS + wcol(r)] = (e0 + r < E && k < kn) ? __ldg(w + (e0 + r) * D + k0 + k) : 0.f;
      }
    }
    __syncthreads();
    float sacc[kRT][kRE];
#pragma unroll
    for (int a = 0; a < kRT; ++a)
#pragma unroll
      for (int b = 0; b < kRE; ++b) sacc[a][b] = 0.f;
    auto kstep = [&](int k) {
      float xa[kRT];
      if constexpr (kRT == 4) {
        const float4 xv = *reinterpret_cast<const float4*>(xs + k * XS + tg * kRT);
        xa[0] = xv.x; xa[1] = xv.y; xa[2] = xv.z; xa[3] = xv.w;
      } else if constexpr (kRT == 2) {
        const float2 xv = *reinterpret_cast<const float2*>(xs + k * XS + tg * kRT);
        xa[0] = xv.x; xa[1] = xv.y;
      } else {
        xa[0] = xs[k * XS + tg];
      }
      const float4 wa = *reinterpret_cast<const float4*>(ws + k * WS + eg * 4);
      const float4 wb = *reinterpret_cast<const float4*>(ws + k * WS + EB / 2 + eg * 4);
      const float wv[kRE] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int a = 0; a < kRT; ++a)
#pragma unroll
        for (int b = 0; b < kRE; ++b) sacc[a][b] = __fadd_rn(sacc[a][b], __fmul_rn(xa[a], wv[b]));
    };
    if (idle) {
    } else if (kn == kTile) {  // full tile: unrolled, shared-memory offsets become immediates
#pragma unroll 4
      for (int k = 0; k < kTile; ++k) kstep(k);
    } else {
      for (int k = 0; k < kn; ++k) kstep(k);
    }
    if (partials) {
#pragma unroll
      for (int a = 0; a < kRT; ++a) {
        const int64_t t = t0 + tg * kRT + a;
#pragma unroll
        for (int b = 0; b < kRE; ++b) {
          const int64_t e = e0 + eg * kRE + b;
          if (tg * kRT + a < tn && e < E) partials[(int64_t)j * T * E + t * E + e] = sacc[a][b];
        }
      }
      continue;
    }
#pragma unroll
    for (int a = 0; a < kRT; ++a)
#pragma unroll
      for (int b = 0; b < kRE; ++b) c[a][b] = __fadd_rn(c[a][b], __fmul_rn(1.0f, sacc[a][b]));
  }
  if (partials) return;
#pragma unroll
  for (int a = 0; a < kRT; ++a) {
    const int64_t t = t0 + tg * kRT + a;
    if (tg * kRT + a >= tn) continue;
#pragma unroll
    for (int b = 0; b < kRE; ++b) {
      const int64_t e = e0 + eg * kRE + b;
      if (e < E) logits[t * E + e] = c[a][b];
    }
  }
}

// logits[t][e] = tile partials added in tile order (the reference's c += 1 * s).
__global__ void router_fold_kernel(const float* __restrict__ partials, int64_t n, int nkt,
                                   float* __restrict__ logits) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float c = 0.0f;
  for (int j = 0; j < nkt; ++j) c = __fadd_rn(c, __fmul_rn(1.0f, partials[(int64_t)j * n + i]));
  logits[i] = c;
}

// One block, one token: thread (tile j, expert e) builds one partial from x staged in shared
// memory (xs [D]); thread e then adds its partials (part [E][nkt]) in tile order.  The logits go
// to out[e] (global or shared).
__device__ __forceinline__ void token_logits(const float* __restrict__ xrow, const float* __restrict__ w, int64_t D,
                                             int64_t E, float* xs, float* part, float* out) {
  const int nkt = (int)((D + kTile - 1) / kTile);
  for (int64_t k = threadIdx.x; k < D; k += blockDim.x) xs[k] = __ldg(xrow + k);
  __syncthreads();
  for (int64_t p = threadIdx.x; p < E * nkt; p += blockDim.x) {
    const int64_t e = p % E, j = p / E;
    const int64_t k0 = j * kTile;
    const int kn = (int)((k0 + kTile < D) ? kTile : D - k0);
    const float* wr = w + e * D + k0;
    float s = 0.f;
    if (kn == kTile && (((reinterpret_cast<uintptr_t>(wr)) & 15) == 0)) {
      const float4* w4 = reinterpret_cast<const float4*>(wr);
      float4 buf[kTile / 4];
#pragma unroll
      for (int i = 0; i < kTile / 4; ++i) buf[i] = __ldg(w4 + i);
#pragma unroll
      for (int i = 0; i < kTile / 4; ++i) {
        s = __fadd_rn(s, __fmul_rn(xs[k0 + 4 * i], buf[i].x));
        s = __fadd_rn(s, __fmul_rn(xs[k0 + 4 * i + 1], buf[i].y));
        s = __fadd_rn(s, __fmul_rn(xs[k0 + 4 * i + 2], buf[i].z));
        s = __fadd_rn(s, __fmul_rn(xs[k0 + 4 * i + 3], buf[i].w));
      }
    } else {
      for (int k = 0; k < kn; ++k) s = __fadd_rn(s, __fmul_rn(xs[k0 + k], __ldg(wr + k)));
    }
    part[e * nkt + j] = s;
  }
  __syncthreads();
  for (int64_t e = threadIdx.x; e < E; e += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < nkt; ++j) acc = __fadd_rn(acc, __fmul_rn(1.0f, part[e * nkt + j]));
    out[e] = acc;
  }
}

// Small batches: one block per token (token_logits).
__global__ void __launch_bounds__(1024) router_token_kernel(const float* __restrict__ x,
                                                            const float* __restrict__ w, int64_t D,
                                                            int64_t E, float* __restrict__ logits) {
  extern __shared__ float sm[];
  const int64_t t = blockIdx.x;
  token_logits(x + t * D, w, D, E, sm, sm + D, logits + t * E);
}

// 16 tokens x 64 experts per block, 256 threads, each 2 tokens x 2 experts.
__global__ void __launch_bounds__(256) router_tiled_kernel(const float* __restrict__ x,
                                                           const float* __restrict__ w,
                                                           int64_t T, int64_t D, int64_t E,
                                                           float* __restrict__ logits) {
  __shared__ float xs[16][kTile + 1];
  __shared__ float ws[64][kTile + 1];
  const int64_t t0 = (int64_t)blockIdx.x * 16;
  const int64_t e0 = (int64_t)blockIdx.y * 64;
  const int tid = threadIdx.x;
  const int te = tid & 31, tt = tid >> 5;  // experts te, te+32; tokens 2*tt, 2*tt+1
  float c[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  for (int64_t k0 = 0; k0 < D; k0 += kTile) {
    const int kn = (int)((k0 + kTile < D) ? kTile : D - k0);
    for (int i = tid; i < 16 * kTile; i += 256) {
      const int r = i / kTile, kk = i - r * kTile;
      xs[r][kk] = (t0 + r < T && kk < kn) ? x[(t0 + r) * D + k0 + kk] : 0.f;
    }
    for (int i = tid; i < 64 * kTile; i += 256) {
      const int r = i / kTile, kk = i - r * kTile;
      ws[r][kk] = (e0 + r < E && kk < kn) ? w[(e0 + r) * D + k0 + kk] : 0.f;
    }
    __syncthreads();
    float s[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    for (int kk = 0; kk < kn; ++kk) {
      const float x0 = xs[2 * tt][kk], x1 = xs[2 * tt + 1][kk];
      const float w0 = ws[te][kk], w1 = ws[te + 32][kk];
      s[0][0] = __fadd_rn(s[0][0], __fmul_rn(x0, w0));
      s[0][1] = __fadd_rn(s[0][1], __fmul_rn(x0, w1));
      s[1][0] = __fadd_rn(s[1][0], __fmul_rn(x1, w0));
      s[1][1] = __fadd_rn(s[1][1], __fmul_rn(x1, w1));
    }
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b) c[a][b] = __fadd_rn(c[a][b], __fmul_rn(1.0f, s[a][b]));
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    const int64_t t = t0 + 2 * tt + a;
    if (t >= T) continue;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int64_t e = e0 + te + 32 * b;
      if (e < E) logits[t * E + e] = c[a][b];
    }
  }
}

// One warp per token (8 per block).  The maximum and the final scaling are
// order-free and run across the lanes; the exponentials too.  The sum keeps the
// reference's order (index 0 up, one rounding per add), so one lane adds the
// warp's staged exponentials in sequence.  `top` = first index of the largest
// probability.
// One warp, one token: p[e] = softmax of l (max-subtract, exp in double rounded to f32, the
// denominator summed in index order on one lane, multiply by 1 / sum), sv [E] scratch; returns
// the first index of the largest probability on every lane.
__device__ __forceinline__ int warp_softmax(const float* __restrict__ l, int64_t E, float* __restrict__ p, float* sv,
                                            int lane) {
  {
    float mx = -__int_as_float(0x7f800000);
    for (int64_t e = lane; e < E; e += 32) mx = (mx < l[e]) ? l[e] : mx;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, mx, o);
      mx = (mx < m2) ? m2 : mx;
    }
    for (int64_t e = lane; e < E; e += 32) sv[e] = (float)exp((double)__fsub_rn(l[e], mx));
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0)
      for (int64_t e = 0; e < E; ++e) sum = __fadd_rn(sum, sv[e]);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    const float inv = (sum > 0.0f) ? __fdiv_rn(1.0f, sum) : 0.0f;
    float bp = 0.0f;
    int best = -1;
    for (int64_t e = lane; e < E; e += 32) {
      const float v = __fmul_rn(sv[e], inv);
      p[e] = v;
      if (best < 0 || v > bp) { bp = v; best = (int)e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {  // larger value wins; equal values: smaller index
      const float ov = __shfl_xor_sync(0xffffffffu, bp, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best, o);
      if (oe >= 0 && (best < 0 || ov > bp || (ov == bp && oe < best))) { bp = ov; best = oe; }
    }
    return best;
  }
}

// Decode widths (T <= kDecodeRouteMaxT): router (token_logits), softmax (warp_softmax) and the
// reference top-k (warp_topk on the logits, weights from the probabilities, renormalised) of
// token t in block t, then the stable per-expert slot numbering of route_scan_kernel by the
// block that finishes last (a counter in `done`, zero between launches; no block waits on
// another).  One launch instead of the router, the softmax, the mask clear, the top-k and the
// scan.
__global__ void __launch_bounds__(1024) route_decode_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            int64_t T, int64_t D, int64_t E, int k, int norm_topk,
                                                            float* __restrict__ logits, float* __restrict__ probs,
                                                            RouteBuffers rb, int* done) {
  extern __shared__ float sm[];
  const int nkt = (int)((D + kTile - 1) / kTile);
  float* xs = sm;                // [D]
  float* part = xs + D;          // [E][nkt]
  float* lg = part + E * nkt;    // [E] logits of this token
  float* sv = lg + E;            // [E] softmax scratch
  Pair* h = reinterpret_cast<Pair*>(sv + E);  // [33]
  const int64_t t = blockIdx.x;
  token_logits(x + t * D, w, D, E, xs, part, lg);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32) {
    for (int64_t e = lane; e < E; e += 32) logits[t * E + e] = lg[e];
    (void)warp_softmax(lg, E, probs + t * E, sv, lane);
    warp_topk(lg, E, k, h, lane);
    if (lane == 0) {
      float ps[32];
      for (int r = 0; r < k; ++r) ps[r] = probs[t * E + h[r].e];
      float mass = 0.0f;
      for (int r = 0; r < k; ++r) mass = __fadd_rn(mass, ps[r]);
      if (!(mass > 0.0f)) mass = 1.0f;
      for (int r = 0; r < k; ++r) {
        rb.topk_ids[t * k + r] = h[r].e;
        rb.topk_w[t * k + r] = norm_topk ? __fdiv_rn(ps[r], mass) : ps[r];
      }
      __threadfence();
    }
  }
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(done, 1) == (int)T - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int64_t S = T * k;
  for (int64_t s = threadIdx.x; s < S; s += blockDim.x) {  // earlier tokens' slots with the same expert
    const int e = __ldcg(rb.topk_ids + s);
    const int64_t first = (s / k) * k;
    int before = 0;
    for (int64_t s2 = 0; s2 < first; ++s2) before += __ldcg(rb.topk_ids + s2) == e;
    rb.slot_local[s] = before;
  }
  for (int64_t e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int64_t s2 = 0; s2 < S; ++s2) c += __ldcg(rb.topk_ids + s2) == (int)e;
    rb.counts[e] = c;
  }
  if (threadIdx.x == 0) *done = 0;  // ready for the next launch
}

__global__ void softmax_top_kernel(const float* __restrict__ logits, int64_t T, int64_t E,
                                   float* __restrict__ probs, float* __restrict__ top) {
  extern __shared__ float sv_all[];  // [8][E]
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  float* sv = sv_all + (int64_t)wib * E;
  for (int64_t t = blockIdx.x * 8 + wib; t < T; t += (int64_t)gridDim.x * 8) {
    const int best = warp_softmax(logits + t * E, E, probs + t * E, sv, lane);
    if (top && lane == 0) top[t] = (float)best;
    __syncwarp();  // sv is rewritten for the next token
  }
}

}  // namespace

namespace {
// Block schedule geometry for E >= 32: experts per block, tokens per thread and,
// for small batches, k-tile groups per row (0: one block walks the whole row).
struct BlockPlan {
  int eb, EG, rt, TB, groups, tpg;
  int64_t eblocks, tblocks;
};
BlockPlan block_plan(int64_t T, int64_t D, int64_t E) {
  BlockPlan p{};
  p.eb = E <= 32 ? 32 : E <= 64 ? 64 : 128;  // expert groups (4, 8, 16) divide the 256 threads
  p.EG = p.eb / kRE;
  p.eblocks = (E + p.eb - 1) / p.eb;
  p.rt = 4;
  p.TB = (256 / p.EG) * p.rt;
  p.tblocks = (T + p.TB - 1) / p.TB;
  const int nkt = (int)((D + kTile - 1) / kTile);
  p.groups = 0;
  if (p.tblocks * p.eblocks < 148 && nkt > 1) {  // under one wave of blocks: split the row, fold after
    // the group count whose busiest SM does the least work: ceil(blocks / SMs) blocks of
    // ceil(tiles / groups) tiles each (the smaller count on a tie: less to fold)
    const int64_t tb = p.tblocks * p.eblocks;
    int64_t best_g = 1, best = -1;
    for (int64_t g = 1; g <= nkt; ++g) {
      const int64_t tpg = (nkt + g - 1) / g, groups = (nkt + tpg - 1) / tpg;
      const int64_t cost = ((tb * groups + 147) / 148) * tpg;
      if (best < 0 || cost < best) {
        best = cost;
        best_g = groups;
      }
    }
    p.tpg = (int)((nkt + best_g - 1) / best_g);
    p.groups = (int)((nkt + p.tpg - 1) / p.tpg);
  }
  return p;
}
}  // namespace

size_t router_scratch_bytes(int64_t T, int64_t D, int64_t E) {
  if (E < 32 || T < 1) return 0;
  const BlockPlan p = block_plan(T, D, E);
  return p.groups ? sizeof(float) * (size_t)(T * E) * (size_t)((D + kTile - 1) / kTile) : 0;
}

cudaError_t launch_router(const float* x, const float* w, int64_t T, int64_t D, int64_t E,
                          float* logits, float* probs, float* top, cudaStream_t st, float* scratch,
                          size_t scratch_bytes) {
  if (T == 0) return cudaSuccess;
  if (logits == nullptr) return cudaErrorInvalidValue;
  const int64_t nkt = (D + kTile - 1) / kTile;
  const size_t token_smem = sizeof(float) * (size_t)(D + E * nkt);
  const size_t chunk_smem = sizeof(float) * (size_t)(kTB * kXS + kEC * kXS + kTB * kEC * kJC + kTB * E);
  static bool attrs = false;
  static int block_slots[3] = {0, 0, 0};  // resident block-schedule blocks on the GPU, per EG = 4, 8, 16
  if (!attrs) {  // first call: before any stream capture of a layer call
    attrs = true;
    (void)cudaFuncSetAttribute(router_token_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    (void)cudaFuncSetAttribute(router_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    (void)cudaFuncSetAttribute(router_block_kernel<4, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    (void)cudaFuncSetAttribute(router_block_kernel<4, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    (void)cudaFuncSetAttribute(router_block_kernel<4, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) {
      const void* fns[3] = {reinterpret_cast<const void*>(router_block_kernel<4, 4>),
                            reinterpret_cast<const void*>(router_block_kernel<4, 8>),
                            reinterpret_cast<const void*>(router_block_kernel<4, 16>)};
      for (int i = 0; i < 3; ++i) {
        const int eg = 4 << i, tb = (256 / eg) * 4, eb = eg * kRE;
        const size_t sm_bytes = sizeof(float) * (size_t)(kTile * (tb + 4) + kTile * (eb + 4));
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fns[i], 256, sm_bytes) == cudaSuccess)
          block_slots[i] = per_sm * sms;
      }
    }
    (void)cudaGetLastError();
  }
  const size_t need = router_scratch_bytes(T, D, E);
  if (E >= 32 && (T >= 128 || (need && scratch && scratch_bytes >= need))) {
    const BlockPlan p = block_plan(T, D, E);
    const bool split = p.groups > 0 && scratch && scratch_bytes >= need;
    const size_t smem = sizeof(float) * (size_t)(kTile * (p.TB + 4) + kTile * (p.eb + 4));
    // token blocks: whole waves of resident blocks, the tokens spread evenly over them
    int64_t bx = p.tblocks;
    const int64_t slots = block_slots[p.EG == 4 ? 0 : p.EG == 8 ? 1 : 2];
    if (!split && slots > 0) {
      const int64_t waves = (p.tblocks * p.eblocks + slots - 1) / slots;
      const int64_t want = (waves * slots + p.eblocks - 1) / p.eblocks;
      if (want > bx) bx = want < T ? want : T;
    }
    dim3 grid((unsigned)bx, (unsigned)p.eblocks, split ? (unsigned)p.groups : 1u);
    float* part = split ? scratch : nullptr;
    const int tpg = split ? p.tpg : 0;
    if (p.EG == 4) router_block_kernel<4, 4><<<grid, 256, smem, st>>>(x, w, T, D, E, logits, part, tpg);
    else if (p.EG == 8) router_block_kernel<4, 8><<<grid, 256, smem, st>>>(x, w, T, D, E, logits, part, tpg);
    else router_block_kernel<4, 16><<<grid, 256, smem, st>>>(x, w, T, D, E, logits, part, tpg);
    if (split) {
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return e;
      const int64_t n = T * E;
      router_fold_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(scratch, n, (int)((D + kTile - 1) / kTile),
                                                                       logits);
    }
  } else if (T < 128 && token_smem <= 200 * 1024) {
    router_token_kernel<<<(unsigned)T, 512, token_smem, st>>>(x, w, D, E, logits);
  } else if (chunk_smem <= 200 * 1024) {
    router_chunk_kernel<<<(unsigned)((T + kTB - 1) / kTB), 256, chunk_smem, st>>>(x, w, T, D, E, logits);
  } else {
    dim3 grid((unsigned)((T + 15) / 16), (unsigned)((E + 63) / 64));
    router_tiled_kernel<<<grid, 256, 0, st>>>(x, w, T, D, E, logits);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess || probs == nullptr) return err;
  int64_t blocks = (T + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  const size_t smem = sizeof(float) * 8 * (size_t)E;
  if (smem > 48 * 1024) {
    err = cudaFuncSetAttribute(softmax_top_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
  }
  softmax_top_kernel<<<(unsigned)blocks, 256, smem, st>>>(logits, T, E, probs, top);
  return cudaGetLastError();
}

namespace {
size_t route_decode_smem(int64_t D, int64_t E) {
  const int64_t nkt = (D + kTile - 1) / kTile;
  return sizeof(float) * (size_t)(D + E * nkt + 2 * E) + 33 * sizeof(Pair);
}
}  // namespace

bool route_decode_supported(int64_t T, int64_t D, int64_t E, int k) {
  return T >= 1 && T <= kDecodeRouteMaxT && D >= 1 && E >= 1 && E <= 1024 && k >= 1 && k <= 32 && k <= E &&
         route_decode_smem(D, E) <= 200 * 1024;
}

cudaError_t launch_route_decode(const float* x, const float* w, int64_t T, int64_t D, int64_t E, int k, int norm_topk,
                                float* logits, float* probs, const RouteBuffers& rb, int* done, cudaStream_t st) {
  const size_t smem = route_decode_smem(D, E);
  if (!route_decode_supported(T, D, E, k) || done == nullptr) return cudaErrorNotSupported;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(route_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               200 * 1024);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  route_decode_kernel<<<(unsigned)T, 1024, smem, st>>>(x, w, T, D, E, k, norm_topk, logits, probs, rb, done);
  return cudaGetLastError();
}

}  // namespace uaii_b200
