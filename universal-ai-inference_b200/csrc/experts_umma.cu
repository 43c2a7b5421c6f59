// experts_umma.cu -- grouped expert GEMM on the 5th-generation tensor cores.
//
// One launch computes every (expert, weight-row tile, slot tile[, K split]) of
// one projection:  C[row, slot] = sum_k W_e[row, k] * X[slot, k]  with the
// weight rows as the MMA M dimension (128) and the expert's routed slots as N
// (16..256), so a decode step with one token per expert still fills the
// M = 128 tensor-core tile.
//
// Per CTA (persistent, one per SM, 10 warps):
//   warp 0   TMA producer: packed GGUF weight windows (2-D uint8 tensor map,
//            row pitch = packed row bytes, window start rounded down to 16 B)
//            and f16 activation tiles (SWIZZLE_128B) into shared-memory rings;
//   warp 1   TMEM allocation and the single MMA-issuing thread
//            (tcgen05.mma kind::f16, A and B from shared memory, D in TMEM);
//   warps 2-9 dequantize the packed window into the f16 A tile (K-major,
//            SWIZZLE_128B canonical layout; two warps per 32 rows, each half of
//            the 64-element K atom), then run the epilogue from TMEM, each
//            warp group on half of the slot columns: SwiGLU for gate/up (rows
//            0-63 gate, 64-127 up of the same 64 features) writing h in f16,
//            or f32 partial sums for down.  Consumer barriers take one elected
//            arrival per warp.
// The weights are never repacked: blocks stay byte-identical to GGUF.  Each
// dequantized operand is the GGUF value in f16: Q4_0 and Q8_0 exactly
// fp16(round(d*q)); K-quants scale by fp16(d*sc), fp16(dmin*m).
//
// Every mbarrier wait is bounded: on timeout the CTA records an error code in
// *err, waits (bounded) for its own copies and MMAs in flight, frees TMEM and
// exits.
#include <cuda.h>
#include <cuda_fp16.h>

#include "gguf_blocks.cuh"
#include "kernels.hpp"
#include "umma.cuh"

namespace uaii_b200 {
namespace {

using namespace umma;

// K chunk per packed-window load: one K-quant super-block (256) or two
// 32-element blocks (64).  kBytes = packed bytes of one chunk of one row.
template <int F> struct Fmt;
template <> struct Fmt<kQ4_0> { static constexpr int kChunk = 64, kAtoms = 1, kBytes = 36; };
template <> struct Fmt<kQ8_0> { static constexpr int kChunk = 64, kAtoms = 1, kBytes = 68; };
template <> struct Fmt<kQ4_K> { static constexpr int kChunk = 256, kAtoms = 4, kBytes = 144; };
template <> struct Fmt<kQ6_K> { static constexpr int kChunk = 256, kAtoms = 4, kBytes = 210; };

// Bytes of the 16-byte-aligned window that holds any chunk of a row, rounded
// up to an odd number of 16-byte units: rows of the packed stage then start in
// different 16-byte bank groups, so eight lanes reading eight rows with 16-byte
// loads never collide.
__host__ __device__ constexpr int window_bytes(int bytes) {
  int w = 0;
  for (int c = 0; c < 16; ++c) {
    const int x = ((((c * bytes) & 15) + bytes) + 15) & ~15;
    w = x > w ? x : w;
  }
  return ((w / 16) & 1) ? w : w + 16;
}

constexpr int kThreads = 352;  // warp 0 weight TMA, warp 1 MMA, warps 2-9 dequant + epilogue, warp 10 activation TMA
constexpr int kDqWarps = 8;
constexpr int kAtomBytes = 128 * 128;  // 128 rows x 64 f16

enum : int { kErrTimeoutProducer = 1, kErrTimeoutMma = 2, kErrTimeoutDequant = 3, kErrTimeoutEpilogue = 4 };

struct Args {
  const int32_t* counts;
  const int32_t* offsets;
  const int32_t* tile_base;  // [E+1]
  int E, m_tiles, splits, kchunks, rows_per_expert, gateup;
  __half* h_out;  // gate/up: [S, out_ld] f16
  float* out;     // down: [splits][S][out_ld] f32
  int64_t out_ld, split_stride;
  int* err;
};

__device__ __forceinline__ __half2 as_h2(uint32_t v) {
  __half2 h;
  memcpy(&h, &v, 4);
  return h;
}
__device__ __forceinline__ uint32_t as_u32(__half2 h) {
  uint32_t v;
  memcpy(&v, &h, 4);
  return v;
}

// NW consecutive 32-bit words starting at byte (16*q + OFF) of a 16-byte
// aligned row, read with 16-byte shared-memory loads; OFF (0..15) is a
// compile-time constant, q a runtime 16-byte index.
template <int OFF, int NW>
__device__ __forceinline__ void load_words(const uint8_t* row16, int q, uint32_t (&w)[NW]) {
  constexpr int kChunks = (OFF + 4 * NW + 15) / 16 + ((OFF % 4) ? 1 : 0);
  uint32_t u[4 * kChunks];
  const uint4* src = reinterpret_cast<const uint4*>(row16) + q;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const uint4 v = src[i];
    u[4 * i] = v.x; u[4 * i + 1] = v.y; u[4 * i + 2] = v.z; u[4 * i + 3] = v.w;
  }
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    constexpr int kShift = 8 * (OFF % 4);
    const int k = OFF / 4 + j;
    if constexpr (kShift == 0) w[j] = u[k];
    else w[j] = __funnelshift_r(u[k], u[k + 1], kShift);
  }
}

// Operand K order.  Inside every group of four consecutive K elements the
// tensor-core operands store elements in the order [0, 2, 1, 3] (both the
// weight tile built here and the activation rows written by the gather and
// the gate/up epilogue), which leaves every dot product unchanged and lets a
// 32-bit word of packed bytes unpack with one shift and one LOP3 per pair.
// the masked values (< 1024) of both 16-bit halves as f16 (1024 + v)
__device__ __forceinline__ uint32_t lo_pairs(uint32_t w, uint32_t mask) { return (w & mask) | 0x64006400u; }

// 8 elements (two words of four 4-bit values at bit offset s) -> one 16-byte chunk
__device__ __forceinline__ uint4 nib_chunk(uint32_t w0, uint32_t w1, int s, __half2 bias, __half2 d, __half2 nm,
                                          bool fma) {
  const uint32_t a[4] = {lo_pairs(w0 >> s, 0x000F000Fu), lo_pairs(w0 >> (s + 8), 0x000F000Fu),
                         lo_pairs(w1 >> s, 0x000F000Fu), lo_pairs(w1 >> (s + 8), 0x000F000Fu)};
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 q = __hsub2(as_h2(a[i]), bias);
    r[i] = as_u32(fma ? __hfma2(q, d, nm) : __hmul2(q, d));
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// 8 elements from two words of four byte values -> one 16-byte chunk
__device__ __forceinline__ uint4 byte_chunk(uint32_t w0, uint32_t w1, __half2 bias, __half2 d) {
  const uint32_t a[4] = {lo_pairs(w0, 0x00FF00FFu), lo_pairs(w0 >> 8, 0x00FF00FFu), lo_pairs(w1, 0x00FF00FFu),
                         lo_pairs(w1 >> 8, 0x00FF00FFu)};
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) r[i] = as_u32(__hmul2(__hsub2(as_h2(a[i]), bias), d));
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// Q4_0 / Q8_0: one thread makes half of the 64-element atom (block h of the
// two blocks in the chunk): four 16-byte chunks, chunks 4h..4h+3 of the atom.
template <int F, int OFF>
__device__ __forceinline__ void dequant_half(const uint8_t* row, int h, uint4 (&o)[4]);

// Q4_0 block: {f16 d; u8 qs[16]}, low nibbles -> elements 0..15, high -> 16..31, (q - 8) * d
template <int OFF, int H>
__device__ __forceinline__ void q4_0_block(const uint8_t* row, uint4 (&o)[4]) {
  constexpr int kB = OFF + 18 * H;
  uint32_t w[5];
  load_words<kB % 16, 5>(row, kB / 16, w);  // bytes kB .. kB+19
  const __half dh = __ushort_as_half((unsigned short)(w[0] & 0xFFFFu));
  const __half2 d = __halves2half2(dh, dh);
  const __half2 bias = __float2half2_rn(1032.f);  // 1024 + 8
  uint32_t q[4];  // qs bytes 0..15
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = __funnelshift_r(w[i], w[i + 1], 16);
  o[0] = nib_chunk(q[0], q[1], 0, bias, d, d, false);
  o[1] = nib_chunk(q[2], q[3], 0, bias, d, d, false);
  o[2] = nib_chunk(q[0], q[1], 4, bias, d, d, false);
  o[3] = nib_chunk(q[2], q[3], 4, bias, d, d, false);
}

// Q8_0 block: {f16 d; i8 qs[32]}, q * d
template <int OFF, int H>
__device__ __forceinline__ void q8_0_block(const uint8_t* row, uint4 (&o)[4]) {
  constexpr int kB = OFF + 34 * H;
  uint32_t w[9];
  load_words<kB % 16, 9>(row, kB / 16, w);  // bytes kB .. kB+35
  const __half dh = __ushort_as_half((unsigned short)(w[0] & 0xFFFFu));
  const __half2 d = __halves2half2(dh, dh);
  const __half2 bias = __float2half2_rn(1152.f);  // 1024 + 128
  uint32_t q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(w[i], w[i + 1], 16) ^ 0x80808080u;  // int8 -> q + 128
#pragma unroll
  for (int c = 0; c < 4; ++c) o[c] = byte_chunk(q[2 * c], q[2 * c + 1], bias, d);
}

#define UAII_HALF_OFF(F, FN, O)                                                                    \
  template <>                                                                                       \
  __device__ __forceinline__ void dequant_half<F, O>(const uint8_t* r, int h, uint4(&o)[4]) {       \
    h ? FN<O, 1>(r, o) : FN<O, 0>(r, o);                                                            \
  }
UAII_HALF_OFF(kQ4_0, q4_0_block, 0) UAII_HALF_OFF(kQ4_0, q4_0_block, 4)
UAII_HALF_OFF(kQ4_0, q4_0_block, 8) UAII_HALF_OFF(kQ4_0, q4_0_block, 12)
UAII_HALF_OFF(kQ8_0, q8_0_block, 0) UAII_HALF_OFF(kQ8_0, q8_0_block, 4)
UAII_HALF_OFF(kQ8_0, q8_0_block, 8) UAII_HALF_OFF(kQ8_0, q8_0_block, 12)
#undef UAII_HALF_OFF

// K-quants: one thread makes whole 64-element atoms of one super-block; the
// super-block header is decoded once per chunk into a Header.
struct Q4KHeader {
  uint32_t y, z, w;  // the 12 scale bytes
  float d, dmin;
};
__device__ __forceinline__ Q4KHeader q4_k_header(const uint8_t* blk) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(blk);  // d, dmin, scales[12]
  return Q4KHeader{hdr.y, hdr.z, hdr.w, f16_bits_to_f32(hdr.x & 0xFFFFu), f16_bits_to_f32(hdr.x >> 16)};
}
// (scale, min) pair j with the get_scale_min_k4 bit layout, from registers
__device__ __forceinline__ void q4_k_pair(const Q4KHeader& H, int j, __half2& d, __half2& nm) {
  const int sh = 8 * (j & 3);
  const uint32_t y = H.y >> sh, z = H.z >> sh, w4 = H.w >> sh;
  const int sc = j < 4 ? (int)(y & 63u) : (int)((w4 & 15u) | (((y >> 6) & 3u) << 4));
  const int m = j < 4 ? (int)(z & 63u) : (int)(((w4 >> 4) & 15u) | (((z >> 6) & 3u) << 4));
  d = __float2half2_rn(H.d * (float)sc);
  nm = __float2half2_rn(-(H.dmin * (float)m));
}
// atom `at` = qs[32*at .. +31]: low nibbles -> sub-block 2at, high -> 2at+1
__device__ __forceinline__ void q4_k_atom(const uint8_t* blk, const Q4KHeader& H, int at, uint4 (&o)[8]) {
  __half2 d0, n0, d1, n1;
  q4_k_pair(H, 2 * at, d0, n0);
  q4_k_pair(H, 2 * at + 1, d1, n1);
  const __half2 bias = __float2half2_rn(1024.f);
  const uint4* qp = reinterpret_cast<const uint4*>(blk + 16 + 32 * at);
  const uint4 qa = qp[0], qb = qp[1];
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    o[c] = nib_chunk(w[2 * c], w[2 * c + 1], 0, bias, d0, n0, true);
    o[4 + c] = nib_chunk(w[2 * c], w[2 * c + 1], 4, bias, d1, n1, true);
  }
}

// Q6_K super-block at even offset OFF: atom `at` covers quarters 2*(at&1) and
// 2*(at&1)+1 of half (at>>1)
template <int OFF>
__device__ __forceinline__ void q6_k_atom(const uint8_t* row, float d, int at, uint4 (&o)[8]) {
  const int n = at >> 1, hiq = at & 1;
  const int ns = hiq ? 4 : 0;
  uint32_t hw[8];
  load_words<OFF, 8>(row, 8 + 2 * n, hw);  // qh[32n .. +31]
  const int8_t* sc = reinterpret_cast<const int8_t*>(row + OFF + 192 + 8 * n);
  const __half2 bias = __float2half2_rn(1056.f);  // 1024 + 32
#pragma unroll
  for (int qq = 0; qq < 2; ++qq) {
    const int qt = 2 * hiq + qq;
    uint32_t lw[8];
    load_words<OFF, 8>(row, 4 * n + 2 * qq, lw);  // ql[64n + 32qq .. +31]
    const __half2 s_lo = __float2half2_rn(d * (float)sc[2 * qt]);
    const __half2 s_hi = __float2half2_rn(d * (float)sc[2 * qt + 1]);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t q6[2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
        q6[j] = ((lw[2 * c + j] >> ns) & 0x0F0F0F0Fu) | (((hw[2 * c + j] >> (2 * qt)) & 0x03030303u) << 4);
      o[4 * qq + c] = byte_chunk(q6[0], q6[1], bias, c < 2 ? s_lo : s_hi);
    }
  }
}

// Runtime (warp-uniform) chunk offset -> the specialised half decoder (Q4_0, Q8_0).
template <int F>
__device__ __forceinline__ void dequant_half_at(const uint8_t* row, int off, int h, uint4 (&o)[4]) {
  switch (off) {
    case 0: dequant_half<F, 0>(row, h, o); break;
    case 4: dequant_half<F, 4>(row, h, o); break;
    case 8: dequant_half<F, 8>(row, h, o); break;
    default: dequant_half<F, 12>(row, h, o); break;
  }
}

template <int F>
__device__ __forceinline__ void q6_k_atom_at(const uint8_t* row, int off, float d, int at, uint4 (&o)[8]) {
  switch (off) {
    case 0: q6_k_atom<0>(row, d, at, o); break;
    case 2: q6_k_atom<2>(row, d, at, o); break;
    case 4: q6_k_atom<4>(row, d, at, o); break;
    case 6: q6_k_atom<6>(row, d, at, o); break;
    case 8: q6_k_atom<8>(row, d, at, o); break;
    case 10: q6_k_atom<10>(row, d, at, o); break;
    case 12: q6_k_atom<12>(row, d, at, o); break;
    default: q6_k_atom<14>(row, d, at, o); break;
  }
}

// position of K element i in the operand order [0, 2, 1, 3] of every group of four
__device__ __forceinline__ int k_perm(int i) { return (i & ~3) | ((i & 1) << 1) | ((i >> 1) & 1); }

struct Tile {
  int e, m_tile, n_tile, split;
};

__device__ __forceinline__ Tile decode_tile(const Args& a, int tile, int bn) {
  int lo = 0, hi = a.E;  // largest e with tile_base[e] <= tile (always a non-empty expert)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(a.tile_base + mid) <= tile) lo = mid; else hi = mid;
  }
  Tile t;
  t.e = lo;
  int local = tile - __ldg(a.tile_base + lo);
  t.split = local % a.splits;
  local /= a.splits;
  const int nt = (__ldg(a.counts + lo) + bn - 1) / bn;
  t.n_tile = local % nt;
  t.m_tile = local / nt;
  return t;
}

#ifdef UAII_UMMA_STATS
// Diagnostic build only: cycles spent in each wait site, accumulated per
// thread and added to these grid-wide totals once at kernel exit.
__device__ unsigned long long g_wait_cycles[16];
__device__ unsigned long long g_wait_count[16];
struct WaitStats {
  unsigned long long cyc[12];
  unsigned int cnt[12];
};
#define UAII_WS_PARAM , WaitStats* ws
#define UAII_WS_ARG , &wstats
#else
#define UAII_WS_PARAM
#define UAII_WS_ARG
#endif

// Wait with abort: false when another role aborted or the clock budget ran out.
// `site` identifies the wait for the diagnostic build.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code,
                                         int site UAII_WS_PARAM) {
#ifdef UAII_UMMA_STATS
  struct Acc {
    WaitStats* ws;
    long long ts;
    int site;
    __device__ ~Acc() {
      ws->cyc[site] += (unsigned long long)(clock64() - ts);
      ws->cnt[site] += 1;
    }
  } acc{ws, clock64(), site};
#else
  (void)site;
#endif
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort = 1;
      atomicExch(err, code);
      return false;
    }
  }
  return true;
}

template <int F, int BN, int A_ST, int B_ST, int P_ST>
struct Cfg {
  static constexpr int kWB = window_bytes(Fmt<F>::kBytes);
  static constexpr int kPStage = 128 * kWB;
  static constexpr int kBStage = BN * 128;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + A_ST * kAtomBytes;
  static constexpr int kOffP = kOffB + B_ST * kBStage;
  static constexpr int kOffBar = kOffP + P_ST * kPStage;
  static constexpr int kNumBars = 2 * (P_ST + A_ST + B_ST) + 2 + 1;
  static constexpr int kSmem = kOffBar + kNumBars * 8 + 16 + 1024;  // + alignment slack
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
};

template <int F, int BN, int A_ST, int B_ST, int P_ST>
__global__ void __launch_bounds__(kThreads, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_x, const Args args) {
  using C = Cfg<F, BN, A_ST, B_ST, P_ST>;
  constexpr int kAtoms = Fmt<F>::kAtoms;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + C::kOffA;
  uint8_t* sB = smem + C::kOffB;
  uint8_t* sP = smem + C::kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* pk_full = bars;
  uint64_t* pk_empty = pk_full + P_ST;
  uint64_t* a_full = pk_empty + P_ST;
  uint64_t* a_empty = a_full + A_ST;
  uint64_t* b_full = a_empty + A_ST;
  uint64_t* b_empty = b_full + B_ST;
  uint64_t* acc_full = b_empty + B_ST;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* mma_done = acc_empty + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifdef UAII_UMMA_STATS
  WaitStats wstats{};
  const long long t_kernel = clock64();
#endif
  if (threadIdx.x == 0) {
    // consumer-side barriers count one elected lane per dequant warp
    for (int i = 0; i < P_ST; ++i) { mbar_init(pk_full + i, 1); mbar_init(pk_empty + i, kDqWarps); }
    // K-quant atoms are written whole by one warp group (4 warps), 32-element-block
    // atoms in halves by both groups (8 warps)
    for (int i = 0; i < A_ST; ++i) { mbar_init(a_full + i, kAtoms == 4 ? 4 : kDqWarps); mbar_init(a_empty + i, 1); }
    for (int i = 0; i < B_ST; ++i) { mbar_init(b_full + i, 1); mbar_init(b_empty + i, 1); }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kDqWarps);
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w0);
    prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_x);
  }
  if (warp == 1) tmem_alloc(s_tmem, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int total = __ldg(args.tile_base + args.E);
  int* err = args.err;

  if (warp == 0) {
    // ------------------------------------------------------------ weight TMA producer
    if (lane == 0) {
      uint32_t pi = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const Tile t = decode_tile(args, tile, BN);
        const int row0 = t.e * args.rows_per_expert + t.m_tile * (args.gateup ? 64 : 128);
        const int c0 = t.split * args.kchunks / args.splits, c1 = (t.split + 1) * args.kchunks / args.splits;
        for (int c = c0; c < c1 && ok; ++c) {
          const int ps = pi % P_ST;
          if (!(ok = wait_bar(pk_empty + ps, ((pi / P_ST) & 1) ^ 1, s_abort, err, kErrTimeoutProducer, 0 UAII_WS_ARG))) break;
          mbar_arrive_expect_tx(pk_full + ps, C::kPStage);
          const int x = (c * Fmt<F>::kBytes) & ~15;
          uint8_t* dst = sP + ps * C::kPStage;
          if (args.gateup) {
            tma_load_2d(dst, &tm_w0, pk_full + ps, x, row0);
            tma_load_2d(dst + 64 * C::kWB, &tm_w1, pk_full + ps, x, row0);
          } else {
            tma_load_2d(dst, &tm_w0, pk_full + ps, x, row0);
            tma_load_2d(dst + 64 * C::kWB, &tm_w0, pk_full + ps, x, row0 + 64);
          }
          ++pi;
        }
      }
      // never leave with copies in flight: wait (bounded) for the last load of every stage
      for (uint32_t j = (pi > (uint32_t)P_ST ? pi - P_ST : 0); j < pi; ++j)
        (void)mbar_wait(pk_full + j % P_ST, (j / P_ST) & 1);
    }
    __syncwarp();
  } else if (warp == 10) {
    // ------------------------------------------------------------ activation TMA producer
    if (lane == 0) {
      uint32_t bi = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const Tile t = decode_tile(args, tile, BN);
        const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
        const int c0 = t.split * args.kchunks / args.splits, c1 = (t.split + 1) * args.kchunks / args.splits;
        for (int c = c0; c < c1 && ok; ++c) {
          for (int at = 0; at < kAtoms && ok; ++at) {
            const int bs = bi % B_ST;
            if (!(ok = wait_bar(b_empty + bs, ((bi / B_ST) & 1) ^ 1, s_abort, err, kErrTimeoutProducer, 1 UAII_WS_ARG))) break;
            mbar_arrive_expect_tx(b_full + bs, C::kBStage);
            tma_load_2d(sB + bs * C::kBStage, &tm_x, b_full + bs, c * Fmt<F>::kChunk + at * 64, slot0);
            ++bi;
          }
        }
      }
      for (uint32_t j = (bi > (uint32_t)B_ST ? bi - B_ST : 0); j < bi; ++j)
        (void)mbar_wait(b_full + j % B_ST, (j / B_ST) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      uint32_t ai = 0, bi = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
        const Tile t = decode_tile(args, tile, BN);
        const int c0 = t.split * args.kchunks / args.splits, c1 = (t.split + 1) * args.kchunks / args.splits;
        if (!(ok = wait_bar(acc_empty, (it & 1) ^ 1, s_abort, err, kErrTimeoutMma, 2 UAII_WS_ARG))) break;
        tc_fence_after();
        uint32_t acc = 0;
        for (int c = c0; c < c1 && ok; ++c) {
          for (int at = 0; at < kAtoms; ++at) {
            const int as = ai % A_ST, bs = bi % B_ST;
            if (!(ok = wait_bar(a_full + as, (ai / A_ST) & 1, s_abort, err, kErrTimeoutMma, 3 UAII_WS_ARG))) break;
            if (!(ok = wait_bar(b_full + bs, (bi / B_ST) & 1, s_abort, err, kErrTimeoutMma, 4 UAII_WS_ARG))) break;
            tc_fence_after();
            const uint64_t ad = sw128_desc(smem_u32(sA + as * kAtomBytes));
            const uint64_t bd = sw128_desc(smem_u32(sB + bs * C::kBStage));
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              mma_f16(tmem, ad + 2 * ks, bd + 2 * ks, idesc, acc);
              acc = 1;
            }
            mma_commit(a_empty + as);
            mma_commit(b_empty + bs);
            ++ai;
            ++bi;
          }
        }
        if (ok) mma_commit(acc_full);
      }
      // the tensor core must be idle before TMEM is freed
      mma_commit(mma_done);
      (void)mbar_wait(mma_done, 0);
    }
    __syncwarp();
  } else if (warp >= 2 && warp < 10) {
    // ------------------------------------------------------------ dequant + epilogue (256 threads)
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int row = 32 * q + lane;     // A-tile row == accumulator lane
    const int grp = (warp - 2) >> 2;   // 0: warps 2-5, 1: warps 6-9 (each row has one of each)
    // Gate/up tiles hold 64 features: in every 32-row block (one TMEM lane
    // quarter) lanes 0-15 are gate rows and lanes 16-31 the up rows of the same
    // 16 features, so the SwiGLU epilogue pairs them with one lane shuffle.
    // The packed stage keeps the TMA layout: gate rows 0-63, up rows 64-127.
    const int src_row = args.gateup ? (lane < 16 ? 16 * q + lane : 64 + 16 * q + (lane - 16)) : row;
    uint32_t pi = 0, ai = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
      const Tile t = decode_tile(args, tile, BN);
      const int c0 = t.split * args.kchunks / args.splits, c1 = (t.split + 1) * args.kchunks / args.splits;
      for (int c = c0; c < c1 && ok; ++c) {
        const int ps = pi % P_ST;
        if (!(ok = wait_bar(pk_full + ps, (pi / P_ST) & 1, s_abort, err, kErrTimeoutDequant, 5 UAII_WS_ARG))) break;
        const uint8_t* rowp = sP + ps * C::kPStage + src_row * C::kWB;
        const int off = (c * Fmt<F>::kBytes) & 15;
        if constexpr (kAtoms == 4) {
          // this warp group makes atoms grp and grp + 2 of the super-block
          Q4KHeader h4{};
          float d6 = 0.f;
          if constexpr (F == kQ4_K) h4 = q4_k_header(rowp);
          else d6 = f16_bits_to_f32(ld_u16(rowp + off + 208));
          for (int k = 0; k < 2 && ok; ++k) {
            const int at = grp + 2 * k;
            const uint32_t aidx = ai + at;
            const int as = aidx % A_ST;
            if (!(ok = wait_bar(a_empty + as, ((aidx / A_ST) & 1) ^ 1, s_abort, err, kErrTimeoutDequant, 6 UAII_WS_ARG)))
              break;
            uint4 o[8];
#ifdef UAII_UMMA_STATS
            const long long tq = clock64();
#endif
            if constexpr (F == kQ4_K) q4_k_atom(rowp, h4, at, o);
            else q6_k_atom_at<F>(rowp, off, d6, at, o);
#ifdef UAII_UMMA_STATS
            asm volatile("" ::"r"(o[0].x), "r"(o[3].y), "r"(o[5].z), "r"(o[7].w));
            wstats.cyc[10] += (unsigned long long)(clock64() - tq);
            wstats.cnt[10] += 1;
#endif
            uint8_t* arow = sA + as * kAtomBytes + row * 128;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) *reinterpret_cast<uint4*>(arow + ((cc ^ (row & 7)) << 4)) = o[cc];
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(a_full + as);
          }
          ai += kAtoms;
        } else {
          const int as = ai % A_ST;
          if (!(ok = wait_bar(a_empty + as, ((ai / A_ST) & 1) ^ 1, s_abort, err, kErrTimeoutDequant, 6 UAII_WS_ARG)))
            break;
          uint4 o[4];
#ifdef UAII_UMMA_STATS
          const long long tq = clock64();
#endif
          dequant_half_at<F>(rowp, off, grp, o);
#ifdef UAII_UMMA_STATS
          asm volatile("" ::"r"(o[0].x), "r"(o[1].y), "r"(o[2].z), "r"(o[3].w));
          wstats.cyc[10] += (unsigned long long)(clock64() - tq);
          wstats.cnt[10] += 1;
#endif
          uint8_t* arow = sA + as * kAtomBytes + row * 128;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc)
            *reinterpret_cast<uint4*>(arow + (((4 * grp + cc) ^ (row & 7)) << 4)) = o[cc];
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(a_full + as);
          ++ai;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(pk_empty + ps);
        ++pi;
      }
      if (!ok) break;
      // ---- epilogue: group `grp` owns accumulator columns [grp*BN/2, (grp+1)*BN/2)
      if (!(ok = wait_bar(acc_full, it & 1, s_abort, err, kErrTimeoutEpilogue, 7 UAII_WS_ARG))) break;
      tc_fence_after();
      const int n_valid = min(BN, __ldg(args.counts + t.e) - t.n_tile * BN);
      const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
      constexpr int kHalf = BN / 2;
      if (args.gateup) {
        // lane l < 16 holds gate, lane l + 16 up of feature i0 + 16q + (l & 15); each
        // column pair (n, n+1) is split: the gate lane finishes n, the up lane n + 1
        const int feat = k_perm(t.m_tile * 64 + 16 * q + (lane & 15));
        const bool gate_lane = lane < 16;
        for (int cb = grp * kHalf; cb < (grp + 1) * kHalf; cb += 8) {
          uint32_t r[8];
          tmem_ld8(taddr + cb, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const float mine0 = __uint_as_float(r[j]), mine1 = __uint_as_float(r[j + 1]);
            const float other = __shfl_xor_sync(0xffffffffu, gate_lane ? mine1 : mine0, 16);
            const float g = gate_lane ? mine0 : other;  // column n (gate lane) or n + 1 (up lane)
            const float u = gate_lane ? other : mine1;
            const int n = cb + j + (gate_lane ? 0 : 1);
            const float sig = 1.0f / (1.0f + __expf(-g));
            if (n < n_valid) args.h_out[(int64_t)(slot0 + n) * args.out_ld + feat] = __float2half_rn((g * sig) * u);
          }
        }
      } else {
        const int o0 = t.m_tile * 128;
        float* out = args.out + (int64_t)t.split * args.split_stride;
        for (int cb = grp * kHalf; cb < (grp + 1) * kHalf; cb += 8) {
          uint32_t r[8];
          tmem_ld8(taddr + cb, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int n = cb + j;
            if (n < n_valid) out[(int64_t)(slot0 + n) * args.out_ld + o0 + row] = __uint_as_float(r[j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
    }
  }
#ifdef UAII_UMMA_STATS
  wstats.cyc[11] = (unsigned long long)(clock64() - t_kernel);
  wstats.cnt[11] = 1;
  for (int i = 0; i < 12; ++i)
    if (wstats.cnt[i]) {
      atomicAdd(&g_wait_cycles[i], wstats.cyc[i]);
      atomicAdd(&g_wait_count[i], (unsigned long long)wstats.cnt[i]);
    }

#endif
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

__global__ void tile_table_kernel(const int32_t* counts, int E, int bn, int m_tiles, int splits,
                                  int32_t* tile_base) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int run = 0;
  for (int e = 0; e < E; ++e) {
    tile_base[e] = run;
    run += ((counts[e] + bn - 1) / bn) * m_tiles * splits;
  }
  tile_base[E] = run;
}

// ---- host side ----------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                 CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

// packed weights: [rows_total, pitch] bytes, box = window x 64 rows
bool make_weight_map(CUtensorMap* m, const void* base, int64_t pitch, int64_t rows_total, int window) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)pitch, (cuuint64_t)rows_total};
  const cuuint64_t strides[1] = {(cuuint64_t)pitch};
  const cuuint32_t box[2] = {(cuuint32_t)window, 64};
  const cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// f16 activations: [rows, K], box = 64 x bn, SWIZZLE_128B
bool make_act_map(CUtensorMap* m, const void* base, int64_t K, int64_t rows, int bn) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
  const cuuint32_t box[2] = {64, (cuuint32_t)bn};
  const cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int F, int BN, int A_ST, int B_ST, int P_ST>
cudaError_t run_gemm(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x, const Args& a,
                     cudaStream_t st) {
  using C = Cfg<F, BN, A_ST, B_ST, P_ST>;
  static_assert(C::kSmem <= 227 * 1024, "shared memory budget");
  auto kern = expert_gemm_kernel<F, BN, A_ST, B_ST, P_ST>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  kern<<<num_sms(), kThreads, C::kSmem, st>>>(w0, w1, x, a);
  return cudaGetLastError();
}

template <int F>
cudaError_t dispatch_bn(int bn, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
                        const Args& a, cudaStream_t st) {
  switch (bn) {
    case 16: return run_gemm<F, 16, 4, 8, 4>(w0, w1, x, a, st);
    case 32: return run_gemm<F, 32, 4, 8, 4>(w0, w1, x, a, st);
    case 64: return run_gemm<F, 64, 4, 4, 3>(w0, w1, x, a, st);
    case 128: return run_gemm<F, 128, 4, 4, 2>(w0, w1, x, a, st);
    case 256: return run_gemm<F, 256, 3, 3, 2>(w0, w1, x, a, st);
    default: return cudaErrorInvalidValue;
  }
}

int chunk_elems(int fmt) {
  switch (fmt) {
    case kQ4_0: return Fmt<kQ4_0>::kChunk;
    case kQ8_0: return Fmt<kQ8_0>::kChunk;
    case kQ4_K: return Fmt<kQ4_K>::kChunk;
    case kQ6_K: return Fmt<kQ6_K>::kChunk;
    default: return 0;
  }
}
int chunk_bytes(int fmt) {
  switch (fmt) {
    case kQ4_0: return Fmt<kQ4_0>::kBytes;
    case kQ8_0: return Fmt<kQ8_0>::kBytes;
    case kQ4_K: return Fmt<kQ4_K>::kBytes;
    case kQ6_K: return Fmt<kQ6_K>::kBytes;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

cudaError_t launch_common(int fmt, bool gateup, const void* W0, const void* W1, int64_t E, int64_t rows,
                          int64_t K, const void* act16, int64_t S_rows, const int32_t* counts,
                          const int32_t* offsets, int32_t* tile_base, int bn, int splits, void* h16,
                          float* out, int64_t out_ld, int64_t split_stride, int* err, cudaStream_t st) {
  const int ce = chunk_elems(fmt);
  if (!ce || K % ce != 0) return cudaErrorNotSupported;
  const int64_t pitch = fmt_row_bytes(fmt, K);
  const int m_rows = gateup ? 64 : 128;
  if (rows % m_rows != 0 || pitch % 16 != 0) return cudaErrorNotSupported;
  if (!aligned16(W0) || !aligned16(W1) || !aligned16(act16) || K % 8 != 0) return cudaErrorNotSupported;
  const int kchunks = (int)(K / ce);
  if (splits < 1) splits = 1;
  if (splits > kchunks) splits = kchunks;
  const int window = window_bytes(chunk_bytes(fmt));
  CUtensorMap m0, m1, mx;
  if (!make_weight_map(&m0, W0, pitch, E * rows, window) || !make_weight_map(&m1, W1, pitch, E * rows, window) ||
      !make_act_map(&mx, act16, K, S_rows, bn))
    return cudaErrorNotSupported;
  const int m_tiles = (int)(rows / m_rows);
  tile_table_kernel<<<1, 32, 0, st>>>(counts, (int)E, bn, m_tiles, splits, tile_base);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  Args a{};
  a.counts = counts;
  a.offsets = offsets;
  a.tile_base = tile_base;
  a.E = (int)E;
  a.m_tiles = m_tiles;
  a.splits = splits;
  a.kchunks = kchunks;
  a.rows_per_expert = (int)rows;
  a.gateup = gateup ? 1 : 0;
  a.h_out = static_cast<__half*>(h16);
  a.out = out;
  a.out_ld = out_ld;
  a.split_stride = split_stride;
  a.err = err;
  switch (fmt) {
    case kQ4_0: return dispatch_bn<kQ4_0>(bn, m0, m1, mx, a, st);
    case kQ8_0: return dispatch_bn<kQ8_0>(bn, m0, m1, mx, a, st);
    case kQ4_K: return dispatch_bn<kQ4_K>(bn, m0, m1, mx, a, st);
    case kQ6_K: return dispatch_bn<kQ6_K>(bn, m0, m1, mx, a, st);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace

#ifdef UAII_UMMA_STATS
extern "C" __attribute__((visibility("default"))) int uaii_moe_debug_wait_stats(unsigned long long* cycles,
                                                                                unsigned long long* counts,
                                                                                int reset) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(cycles, g_wait_cycles, sizeof(g_wait_cycles));
  cudaMemcpyFromSymbol(counts, g_wait_count, sizeof(g_wait_count));
  if (reset) {
    unsigned long long z[16] = {};
    cudaMemcpyToSymbol(g_wait_cycles, z, sizeof(z));
    cudaMemcpyToSymbol(g_wait_count, z, sizeof(z));
  }
  return 0;
}
#endif

bool umma_format_supported(int fmt) { return chunk_elems(fmt) != 0; }

bool umma_shapes_supported(int gfmt, int dfmt, int64_t D, int64_t I) {
  if (!umma_format_supported(gfmt) || !umma_format_supported(dfmt)) return false;
  if (D % chunk_elems(gfmt) || I % chunk_elems(dfmt) || I % 64 || D % 128) return false;
  return fmt_row_bytes(gfmt, D) % 16 == 0 && fmt_row_bytes(dfmt, I) % 16 == 0 && D % 8 == 0 && I % 8 == 0;
}

cudaError_t launch_gateup_umma(int fmt, const void* G, const void* U, int64_t E, int64_t I, int64_t D,
                               const void* xp16, int64_t S_rows, const int32_t* counts, const int32_t* offsets,
                               int32_t* tile_base, int bn, void* h16, int* err, cudaStream_t st) {
  return launch_common(fmt, true, G, U, E, I, D, xp16, S_rows, counts, offsets, tile_base, bn, 1, h16, nullptr,
                       I, 0, err, st);
}

cudaError_t launch_down_umma(int fmt, const void* Dn, int64_t E, int64_t D, int64_t I, const void* h16,
                             int64_t S_rows, const int32_t* counts, const int32_t* offsets, int32_t* tile_base,
                             int bn, int splits, float* out, int* err, cudaStream_t st) {
  return launch_common(fmt, false, Dn, Dn, E, D, I, h16, S_rows, counts, offsets, tile_base, bn, splits, nullptr,
                       out, D, S_rows * D, err, st);
}

int umma_kchunks(int fmt, int64_t K) {
  const int ce = chunk_elems(fmt);
  return ce ? (int)(K / ce) : 0;
}

}  // namespace uaii_b200
