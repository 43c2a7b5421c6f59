// router.cu -- MoERouter on the device (reference: kernels::moe_router_f32,
// libs/uaii-kernels/src/transformer.cpp:446-481).
//
// logits[t,e] reproduce the reference GEMM's summation order bit for bit
// (RefGemm::gemm_f32, libs/uaii-kernels/src/gemm_ref.cpp:45-75): for each
// 64-wide k tile, s = 0 then s += x*w sequentially; c (from 0) += s tile by
// tile.  Every multiply and add is a separate round-to-nearest operation.
// Two schedules compute the same values:
//   * split: one thread per (token, expert, k-tile) partial, then one thread
//     per (token, expert) adds the partials in tile order -- enough
//     parallelism for decode-sized batches;
//   * tiled: a block owns 16 tokens x 64 experts, stages 64-wide k tiles of
//     x and w in shared memory, and each thread carries 2x2 dot products.
// softmax (softmax.cpp:55-75): max-subtract, exp, sequential sum over experts,
// multiply by 1/sum; exp is evaluated in double and rounded once to f32.
// top_expert is the first strict argmax of probs, stored as an f32 id.
#include "kernels.hpp"

namespace uaii_b200 {
namespace {

constexpr int kTile = 64;

__global__ void router_partials_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                       int64_t T, int64_t D, int64_t E, int nkt,
                                       int pairs_per_block, float* __restrict__ logits) {
  extern __shared__ float part[];  // [pairs_per_block][nkt]
  const int64_t p0 = (int64_t)blockIdx.x * pairs_per_block;
  const int64_t npairs = T * E;
  const int items = pairs_per_block * nkt;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int lp = it / nkt, j = it - lp * nkt;
    const int64_t p = p0 + lp;
    if (p >= npairs) continue;
    const int64_t t = p / E, e = p - t * E;
    const float* xr = x + t * D;
    const float* wr = w + e * D;
    const int64_t k0 = (int64_t)j * kTile;
    const int64_t k1 = (k0 + kTile < D) ? k0 + kTile : D;
    float s = 0.0f;
    for (int64_t k = k0; k < k1; ++k) s = __fadd_rn(s, __fmul_rn(xr[k], wr[k]));
    part[it] = s;
  }
  __syncthreads();
  for (int lp = threadIdx.x; lp < pairs_per_block; lp += blockDim.x) {
    const int64_t p = p0 + lp;
    if (p >= npairs) continue;
    float c = 0.0f;
    for (int j = 0; j < nkt; ++j) c = __fadd_rn(c, __fmul_rn(1.0f, part[lp * nkt + j]));
    logits[p] = c;
  }
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

__global__ void softmax_top_kernel(const float* __restrict__ logits, int64_t T, int64_t E,
                                   float* __restrict__ probs, float* __restrict__ top) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float* l = logits + t * E;
  float* p = probs + t * E;
  float mx = -__int_as_float(0x7f800000);
  for (int64_t e = 0; e < E; ++e) mx = (mx < l[e]) ? l[e] : mx;
  float sum = 0.0f;
  for (int64_t e = 0; e < E; ++e) {
    const float v = (float)exp((double)__fsub_rn(l[e], mx));
    p[e] = v;
    sum = __fadd_rn(sum, v);
  }
  const float inv = (sum > 0.0f) ? __fdiv_rn(1.0f, sum) : 0.0f;
  int best = 0;
  float bp = 0.0f;
  for (int64_t e = 0; e < E; ++e) {
    const float v = __fmul_rn(p[e], inv);
    p[e] = v;
    if (e == 0 || v > bp) { bp = v; best = (int)e; }
  }
  if (top) top[t] = (float)best;
}

}  // namespace

cudaError_t launch_router(const float* x, const float* w, int64_t T, int64_t D, int64_t E,
                          float* logits, float* probs, float* top, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (logits == nullptr) return cudaErrorInvalidValue;
  const int nkt = (int)((D + kTile - 1) / kTile);
  if (T * E <= 4096) {
    int ppb = 256 / nkt;
    if (ppb < 1) ppb = 1;
    const int64_t blocks = (T * E + ppb - 1) / ppb;
    const size_t smem = sizeof(float) * (size_t)ppb * nkt;
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    router_partials_kernel<<<(unsigned)blocks, 256, smem, st>>>(x, w, T, D, E, nkt, ppb, logits);
  } else {
    dim3 grid((unsigned)((T + 15) / 16), (unsigned)((E + 63) / 64));
    router_tiled_kernel<<<grid, 256, 0, st>>>(x, w, T, D, E, logits);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess || probs == nullptr) return err;
  softmax_top_kernel<<<(unsigned)((T + 127) / 128), 128, 0, st>>>(logits, T, E, probs, top);
  return cudaGetLastError();
}

}  // namespace uaii_b200
