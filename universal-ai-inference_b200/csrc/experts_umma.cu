// experts_umma.cu -- grouped expert GEMM on the 5th-generation tensor cores.
//
// One launch computes every (expert, weight-row tile, slot tile[, K split]) of
// one projection:  C[row, slot] = sum_k W_e[row, k] * X[slot, k]  with the
// weight rows as the MMA M dimension (128) and the expert's routed slots as N
// (16..128), so a decode step with one token per expert still fills the
// M = 128 tensor-core tile.
//
// The K loop runs in quads of 256 elements (one K-quant super-block, eight
// 32-element blocks): one packed-window stage, one activation stage and one
// A stage per quad, so the single MMA-issuing thread waits on two barriers and
// commits once per 16 MMAs.  Narrow MMAs are bound by how fast one thread can
// issue them, and every barrier wait on that thread's path costs as much as
// several MMAs.
//
// Per CTA (persistent, one per SM, 19 warps):
//   warp 0   TMA producer of packed GGUF weight windows (2-D uint8 tensor map,
//            row pitch = packed row bytes, window start rounded down to 16 B);
//   warp 1   TMEM allocation and the MMA-issuing thread (tcgen05.mma kind::f16,
//            A from tensor memory, B from shared memory, D in tensor memory);
//   warps 2-17 (four groups of four warps, each group covering all 128 rows)
//            dequantize: group g turns 64-element atom g of every quad into f16
//            and stores it into the quad's A stage in tensor memory; then they
//            run the epilogue from TMEM, each group on a quarter of the slot
//            columns: SwiGLU for gate/up writing h in f16, or f32 partial sums
//            for down.  Consumer barriers take one elected arrival per warp;
//   warp 18  TMA producer of the f16 activation tiles (SWIZZLE_128B).
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
#include "operand_order.cuh"
#include "umma.cuh"

namespace uaii_b200 {
namespace {

using namespace umma;

constexpr int kQuadK = 256;  // K elements per quad = 4 atoms of 64

// Packed bytes of one quad of one row (kBytes), and the TMA boxes that carry a
// quad's window: kBoxes boxes of kBoxBytes (<= 256, the TMA box limit), box j
// starting 128 * j bytes after the 16-byte-aligned window start.  kBoxBytes
// is an odd number of 16-byte units, so rows of a packed stage start in
// different 16-byte bank groups and eight lanes reading eight rows with
// 16-byte loads never collide.  Q4_0 / Q8_0 rows may end in a partial quad
// (K a multiple of 64); K-quant rows hold whole super-blocks.
template <int F> struct Fmt;
template <> struct Fmt<kQ4_0> { static constexpr int kBytes = 144, kBoxes = 1, kBoxBytes = 144, kMinK = 64; };
template <> struct Fmt<kQ8_0> { static constexpr int kBytes = 272, kBoxes = 2, kBoxBytes = 144, kMinK = 64; };
template <> struct Fmt<kQ4_K> { static constexpr int kBytes = 144, kBoxes = 1, kBoxBytes = 144, kMinK = 256; };
template <> struct Fmt<kQ6_K> { static constexpr int kBytes = 210, kBoxes = 1, kBoxBytes = 240, kMinK = 256; };

constexpr int kGroups = 4;                // dequant warp groups (4 warps = 128 rows each)
constexpr int kDqWarps = 4 * kGroups;     // warps 2 .. 2+kDqWarps-1
constexpr int kBWarp = 2 + kDqWarps;      // activation TMA producer warp
constexpr int kMma1Warp = kBWarp + 1;     // second MMA-issuing warp (slot tiles up to 64 wide)
constexpr int kThreads = 32 * (kMma1Warp + 1);

enum : int { kErrTimeoutProducer = 1, kErrTimeoutMma = 2, kErrTimeoutDequant = 3, kErrTimeoutEpilogue = 4 };

struct Args {
  const int32_t* counts;
  const int32_t* offsets;
  const int32_t* tile_base;  // [E+1]
  int E, m_tiles, splits;
  int kquads;   // quads per row: ceil(K / 256)
  int k_atoms;  // 64-element atoms per row: K / 64
  int rows_per_expert, gateup;
  int band_m;  // weight-row tiles per band of the tile order (see decode_tile)
  __half* h_out;  // gate/up: [S, out_ld] f16 in K order h_order (tcgen05 and quad; the per-unit warp schedule: wm_kpos)
  int h_order;
  float* out;     // down: [splits][S][out_ld] f32
  int64_t out_ld, split_stride;
  int* err;
  // Quad schedule, Q4_K activations: per slot and quad, the f32 sums of the eight 32-element
  // sub-blocks of the f16 activations as f16 (hi) and f16 (remainder) pairs, [S_rows][kquads][16];
  // null: the minima go through one MMA per k-step instead.
  const __half* xsum;
  // Integer variant: per slot and quad the activations' dequant scale, [S_rows][kquads] f32 (the
  // activations are the int8 hi / lo planes of route_gather's kOrderQ4KI8 and xsum holds their
  // integer sub-block sums / 1024); null: f16 activations.
  const float* xscale;
  int64_t S_rows;
  // Quad schedule, gate/up: when the last wave of tiles fills at most half of the grid, its
  // tiles are cut into K ranges run by different CTAs; tail_part [tiles][ranges][128][BN] f32
  // holds the ranges' sums and tail_cnt [tiles] (zero between launches) counts finished ranges.
  // Null: no tail split.
  float* tail_part;
  int* tail_cnt;
  // Quad schedule, down: balanced ranges over the tile-major quad sequence (tail_part holds two
  // pieces per CTA, tail_cnt one counter per CTA); 0: whole units
  int ranges;
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
// 32-bit word of packed bytes unpack with masks only: for a word w and
// w8 = w >> 8, (w & 0x000F000F) holds the low nibbles of bytes (0, 2), (w8 & ...)
// those of bytes (1, 3), and (w & 0x00F000F0) the high nibbles times 16.
// OR-ing 0x6400 into a 16-bit half gives the f16 value 1024 + v exactly.
constexpr uint32_t kMagic = 0x64006400u;
__device__ __forceinline__ __half2 magic_pair(uint32_t w, uint32_t mask) { return as_h2((w & mask) | kMagic); }

// An atom is 64 K elements = 32 words of two f16; word 4c + j belongs to the
// 16-byte chunk c (elements 8c .. 8c+7).
using AtomWords = uint32_t[32];

// Q4_0: one 32-element block {f16 d; u8 qs[16]}: low nibbles -> elements 0..15,
// high -> 16..31, value (q - 8) * d; writes words 16h .. 16h+15 of the atom.
template <int OFF, int H>
__device__ __forceinline__ void q4_0_block(const uint8_t* row, uint32_t* out) {
  constexpr int kB = OFF + 18 * H;
  uint32_t w[5];
  load_words<kB % 16, 5>(row, kB / 16, w);  // bytes kB .. kB+19
  const __half dh = __ushort_as_half((unsigned short)(w[0] & 0xFFFFu));
  const __half2 d = __halves2half2(dh, dh);
  const __half2 lo_bias = __float2half2_rn(1032.f);  // 1024 + 8
  const __half2 k16 = __float2half2_rn(0.0625f), hi_bias = __float2half2_rn(-72.f);  // (1024 + 16q)/16 - 72 = q - 8
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t q = __funnelshift_r(w[i], w[i + 1], 16), q8 = q >> 8;  // qs bytes 4i .. 4i+3
    uint32_t* lo = out + 16 * H + 4 * (i >> 1) + 2 * (i & 1);
    uint32_t* hi = lo + 8;
    lo[0] = as_u32(__hmul2(__hsub2(magic_pair(q, 0x000F000Fu), lo_bias), d));
    lo[1] = as_u32(__hmul2(__hsub2(magic_pair(q8, 0x000F000Fu), lo_bias), d));
    hi[0] = as_u32(__hmul2(__hfma2(magic_pair(q, 0x00F000F0u), k16, hi_bias), d));
    hi[1] = as_u32(__hmul2(__hfma2(magic_pair(q8, 0x00F000F0u), k16, hi_bias), d));
  }
}

// Q8_0: one 32-element block {f16 d; i8 qs[32]}: value q * d; words 16h .. 16h+15.
template <int OFF, int H>
__device__ __forceinline__ void q8_0_block(const uint8_t* row, uint32_t* out) {
  constexpr int kB = OFF + 34 * H;
  uint32_t w[9];
  load_words<kB % 16, 9>(row, kB / 16, w);  // bytes kB .. kB+35
  const __half dh = __ushort_as_half((unsigned short)(w[0] & 0xFFFFu));
  const __half2 d = __halves2half2(dh, dh);
  const __half2 bias = __float2half2_rn(1152.f);  // 1024 + 128
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t q = __funnelshift_r(w[i], w[i + 1], 16) ^ 0x80808080u;  // int8 -> q + 128
    out[16 * H + 2 * i] = as_u32(__hmul2(__hsub2(magic_pair(q, 0x00FF00FFu), bias), d));
    out[16 * H + 2 * i + 1] = as_u32(__hmul2(__hsub2(magic_pair(q >> 8, 0x00FF00FFu), bias), d));
  }
}

template <int F, int OFF>
__device__ __forceinline__ void dequant_block32_atom(const uint8_t* row, uint32_t* out) {
  if constexpr (F == kQ4_0) {
    q4_0_block<OFF, 0>(row, out);
    q4_0_block<OFF, 1>(row, out);
  } else {
    q8_0_block<OFF, 0>(row, out);
    q8_0_block<OFF, 1>(row, out);
  }
}

// K-quants: the super-block header is decoded per atom from one 16-byte load.
// K-quant scale products in f16 arithmetic.  A small integer becomes an exact f16 through the
// magic exponent (1024 + v, minus 1024); the f16 product of an f16 scale and such an integer
// (at most 8 bits) is its exact product rounded once to f16 -- the same value as rounding the
// exact f32 product -- at a fraction of the instructions of the f32 route.
// Q4_K: dm = (d, dmin) f16 bits, sc and m 6-bit -> dd = (d*sc, d*sc), nm = -(dmin*m) twice.
__device__ __forceinline__ void q4k_scales(uint32_t dm, uint32_t sc, uint32_t m, __half2& dd, __half2& nm) {
  const __half2 v = __hsub2(as_h2(sc | (m << 16) | kMagic), __float2half2_rn(1024.f));  // (sc, m)
  const __half2 p = __hmul2(as_h2(dm), v);                                                 // (d*sc, dmin*m)
  dd = __low2half2(p);
  nm = __hneg2(__high2half2(p));
}
// Q6_K: d f16 bits, two int8 scales in bits 0-7 and 8-15 -> (d*sc0, d*sc1)
__device__ __forceinline__ __half2 q6k_scales(uint32_t d, uint32_t sc2) {
  const uint32_t u = (sc2 ^ 0x8080u) & 0xFFFFu;  // sc + 128 as unsigned bytes
  const __half2 v = __hsub2(as_h2((u & 0xFFu) | ((u & 0xFF00u) << 8) | kMagic), __float2half2_rn(1152.f));
  return __hmul2(as_h2(d | (d << 16)), v);
}

// Q4_K atom AT = qs[32*AT .. +31]: low nibbles -> sub-block 2AT (words 0..15),
// high nibbles -> sub-block 2AT+1 (words 16..31); value d*sc*q - dmin*m
template <int AT>
__device__ __forceinline__ void q4_k_atom(const uint8_t* blk, uint32_t* out) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(blk);  // d, dmin, scales[12]
  __half2 dd[2], nm[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {  // (scale, min) pair j with the get_scale_min_k4 bit layout
    const int j = 2 * AT + h, sh = 8 * (j & 3);
    const uint32_t y = hdr.y >> sh, z = hdr.z >> sh, w4 = hdr.w >> sh;
    const uint32_t sc = j < 4 ? (y & 63u) : ((w4 & 15u) | (((y >> 6) & 3u) << 4));
    const uint32_t m = j < 4 ? (z & 63u) : (((w4 >> 4) & 15u) | (((z >> 6) & 3u) << 4));
    q4k_scales(hdr.x, sc, m, dd[h], nm[h]);
  }
  const __half2 k1024 = __float2half2_rn(1024.f);
  const __half2 k16 = __float2half2_rn(0.0625f), km64 = __float2half2_rn(-64.f);  // (1024 + 16q)/16 - 64 = q
  const uint4* qp = reinterpret_cast<const uint4*>(blk + 16 + 32 * AT);
  const uint4 qa = qp[0], qb = qp[1];
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t q = w[i], q8 = q >> 8;
    out[2 * i] = as_u32(__hfma2(__hsub2(magic_pair(q, 0x000F000Fu), k1024), dd[0], nm[0]));
    out[2 * i + 1] = as_u32(__hfma2(__hsub2(magic_pair(q8, 0x000F000Fu), k1024), dd[0], nm[0]));
    out[16 + 2 * i] = as_u32(__hfma2(__hfma2(magic_pair(q, 0x00F000F0u), k16, km64), dd[1], nm[1]));
    out[16 + 2 * i + 1] = as_u32(__hfma2(__hfma2(magic_pair(q8, 0x00F000F0u), k16, km64), dd[1], nm[1]));
  }
}

// Q6_K super-block at even byte offset OFF of the row: atom `at` covers
// quarters 2*(at&1) and 2*(at&1)+1 of half (at>>1); value d*sc*(q - 32).
// Specialised on OFF (16-byte loads, compile-time word alignment); the atom
// index stays a runtime value so that only eight decoder copies exist.
template <int OFF>
__device__ __forceinline__ void q6_k_atom(const uint8_t* row, int at, uint32_t* out) {
  const int n = at >> 1, hiq = at & 1;
  const int ns = hiq ? 4 : 0;
  uint32_t hw[8];
  load_words<OFF, 8>(row, 8 + 2 * n, hw);  // qh[32n .. +31]
  const uint8_t* sc = row + OFF + 192 + 8 * n;
  const uint32_t d = ld_u16(row + OFF + 208);
  const __half2 bias = __float2half2_rn(1056.f);  // 1024 + 32
#pragma unroll
  for (int qq = 0; qq < 2; ++qq) {
    const int qt = 2 * hiq + qq;
    uint32_t lw[8];
    load_words<OFF, 8>(row, 4 * n + 2 * qq, lw);  // ql[64n + 32qq .. +31]
    const __half2 s2 = q6k_scales(d, ld_u16(sc + 2 * qt));  // (d*sc[2qt], d*sc[2qt+1])
    const __half2 s_lo = __low2half2(s2), s_hi = __high2half2(s2);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // the 2-bit fields of quarter qt moved to bits 4-5 of every byte; bits 6-7
      // take neighbouring fields and are cleared together with the magic OR
      // rotate so bits 2qt..2qt+1 of every byte land on bits 4-5 (one funnel shift; wrapped
      // bits reach only bits 0-3, cleared below, and bits 6-7, dropped by the magic mask)
      const uint32_t hs = __funnelshift_r(hw[i], hw[i], (uint32_t)(2 * qt + 28) & 31u);
      const uint32_t lo = lw[i] >> ns;
      const uint32_t q6 = (lo & 0x0F0F0F0Fu) | (hs & 0xF0F0F0F0u);  // one LOP3; bits 6-7 junk
      const __half2 s = i < 4 ? s_lo : s_hi;
      out[16 * qq + 2 * i] = as_u32(__hmul2(__hsub2(magic_pair(q6, 0x003F003Fu), bias), s));
      out[16 * qq + 2 * i + 1] = as_u32(__hmul2(__hsub2(magic_pair(q6 >> 8, 0x003F003Fu), bias), s));
    }
  }
}

// Atom g (elements 64g .. 64g+63) of a quad, from the packed row `row` of the
// stage (box 0; box 1 follows 128 rows later) whose window starts `off` bytes
// before the quad; g is warp-uniform.
template <int F, int kRowsStride, int G>
__device__ __forceinline__ void dequant_atom_g(const uint8_t* row, int off, uint32_t* out) {
  if constexpr (F == kQ4_K) {
    q4_k_atom<G>(row, out);
  } else if constexpr (F == kQ4_0) {  // atom G = blocks 2G, 2G+1 at byte 36G
    dequant_block32_atom<F, 4 * G>(row + 32 * G, out);
  } else {  // Q8_0: atom G = blocks 2G, 2G+1 at byte 68G; bytes 128.. come from box 1
    dequant_block32_atom<F, 4 * G>(row + (G >= 2 ? kRowsStride : 0) + 64 * (G & 1), out);
  }
}

// The warp-uniform atom index selects a decoder specialised for it (Q6_K:
// the window offset does, the atom index stays a runtime value).
template <int F, int kRowsStride>
__device__ __forceinline__ void dequant_atom(const uint8_t* row, int off, int g, uint32_t* out) {
  if constexpr (F == kQ6_K) {
    switch (off) {
      case 0: q6_k_atom<0>(row, g, out); return;
      case 2: q6_k_atom<2>(row, g, out); return;
      case 4: q6_k_atom<4>(row, g, out); return;
      case 6: q6_k_atom<6>(row, g, out); return;
      case 8: q6_k_atom<8>(row, g, out); return;
      case 10: q6_k_atom<10>(row, g, out); return;
      case 12: q6_k_atom<12>(row, g, out); return;
      default: q6_k_atom<14>(row, g, out); return;
    }
  } else {
    switch (g) {
      case 0: dequant_atom_g<F, kRowsStride, 0>(row, off, out); break;
      case 1: dequant_atom_g<F, kRowsStride, 1>(row, off, out); break;
      case 2: dequant_atom_g<F, kRowsStride, 2>(row, off, out); break;
      default: dequant_atom_g<F, kRowsStride, 3>(row, off, out); break;
    }
  }
}

struct Tile {
  int e, m_tile, n_tile, split;
};

// Tile order inside an expert: K splits fastest, then bands of band_m weight-row
// tiles -- the row tiles of a band fastest, then the slot tiles.  The tiles in
// flight at once (one per SM) then share band_m weight tiles and about
// SMs / band_m activation tiles, so an expert with many slot tiles re-reads
// neither its weights nor its activations once per wave from HBM.  An expert whose
// tiles straddle two waves is read in both: with wide bands its weights (every
// slot tile needs all rows), with one-tile bands its activations.  Gate/up uses
// bands of kBandM (its activations are the small operand either way); the down
// projection uses one-tile bands, where the f16 hidden rows are smaller than the
// expert's down weights (Mixtral: 29 MB against 48 MB).
constexpr int kBandM = 32;
constexpr int kDownBandM = 1;

__device__ __forceinline__ Tile decode_tile(const Args& a, int tile, int bn) {
  int lo = 0, hi = a.E;  // largest e with tile_base[e] <= tile (always a non-empty expert)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(a.tile_base + mid) <= tile) lo = mid; else hi = mid;
  }
  Tile t;
  t.e = lo;
  int local = tile - __ldg(a.tile_base + lo);
  t.split = 0;
  if (a.splits > 1) {
    t.split = local % a.splits;
    local /= a.splits;
  }
  const int nt = (__ldg(a.counts + lo) + bn - 1) / bn;
  if (nt == 1) {  // one slot tile (decode): the band order is the row-tile order
    t.n_tile = 0;
    t.m_tile = local;
    return t;
  }
  const int band = local / (a.band_m * nt);
  const int m0 = band * a.band_m;
  const int bm = min(a.band_m, a.m_tiles - m0);  // the last band may be narrower
  const int r = local - band * a.band_m * nt;
  t.n_tile = r / bm;
  t.m_tile = m0 + r % bm;
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
  return bounded_wait(bar, parity, abort, err, code);
}

// Tensor memory: two accumulator buffers per issuing thread, then the A ring
// (one 128-column stage per quad: 32 columns per atom, two f16 K elements per
// column).  Slot tiles up to 64 wide have two issuing threads: narrow MMAs are
// bound by how fast one thread issues them, so the two take alternate quads of
// every tile into their own accumulators and the epilogue adds the two.
// 256-slot tiles: one accumulator (the epilogue of a tile runs once the next
// tile's first A stages are made) and activation stages of one 64-K atom
// (a whole quad of 256 activation rows does not fit twice in shared memory).
template <int F, int BN, int A_Q, int B_Q, int P_ST>
struct Cfg {
  static constexpr int kIssuers = BN <= 64 ? 2 : 1;
  static constexpr bool kWide = BN == 256;
  static constexpr int kAccBufs = kWide ? 1 : 2;
  using Fm = Fmt<F>;
  static constexpr int kWB = Fm::kBoxBytes;            // packed stage row stride
  static constexpr int kPStage = Fm::kBoxes * 128 * kWB;
  static constexpr int kBAtom = BN * 128;               // one 64-K box of BN activation rows
  static constexpr int kBQuad = 4 * kBAtom;
  static constexpr int kOffB = 0;
  static constexpr int kBStage = kWide ? kBAtom : kBQuad;  // B_Q stages of this size
  static constexpr int kOffP = kOffB + B_Q * kBStage;
  static constexpr int kOffBar = kOffP + P_ST * kPStage;
  // Stage release: one commit per quad arrives on rel[quad % kRelBars] and
  // frees that quad's A and B stages.  The producer of quad n waits for quad
  // n - depth; kRelBars >= depth keeps the barrier from moving on by a whole
  // phase before that producer has seen it.
  static constexpr int kRelBars = kWide ? A_Q : (A_Q > B_Q ? A_Q : B_Q);  // wide: A stages only
  static constexpr int kNumBars = 2 * P_ST + A_Q + 2 * B_Q + kRelBars + 4 + 2;
  static constexpr int kSmem = kOffBar + kNumBars * 8 + 16 + 1024;  // + alignment slack
  static constexpr uint32_t kAccCols = BN < 32 ? 32 : BN;  // one accumulator
  static constexpr uint32_t kACol0 = kAccBufs * kIssuers * kAccCols;  // first A column
  static constexpr uint32_t kUsedCols = kACol0 + A_Q * 128;
  static constexpr uint32_t kTmemCols = kUsedCols <= 256 ? 256 : 512;
  static_assert(kUsedCols <= 512, "tensor memory budget");
  static_assert(kOffP % 1024 == 0 && kBAtom % 1024 == 0, "SWIZZLE_128B stages must be 1024-byte aligned");
  static_assert((64 * kWB) % 128 == 0, "TMA destinations must be 128-byte aligned");
};

template <int F, int BN, int A_Q, int B_Q, int P_ST>
__global__ void __launch_bounds__(kThreads, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_x, const Args args) {
  using C = Cfg<F, BN, A_Q, B_Q, P_ST>;
  using Fm = Fmt<F>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem + C::kOffB;
  uint8_t* sP = smem + C::kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* pk_full = bars;
  uint64_t* pk_empty = pk_full + P_ST;
  uint64_t* a_full = pk_empty + P_ST;
  uint64_t* b_full = a_full + A_Q;
  uint64_t* rel = b_full + B_Q;               // [kRelBars]
  uint64_t* b_empty = rel + C::kRelBars;      // [B_Q], wide tiles: activation atoms released per atom
  uint64_t* acc_full = b_empty + B_Q;         // [2]
  uint64_t* acc_empty = acc_full + 2;         // [2]
  uint64_t* mma_done = acc_empty + 2;        // [2], one per issuer
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifdef UAII_UMMA_STATS
  WaitStats wstats{};
  const long long t_kernel = clock64();
#endif
  if (threadIdx.x == 0) {
    // every packed stage and every A stage is read / written by all 16 dequant warps
    for (int i = 0; i < P_ST; ++i) { mbar_init(pk_full + i, 1); mbar_init(pk_empty + i, kDqWarps); }
    for (int i = 0; i < A_Q; ++i) mbar_init(a_full + i, kDqWarps);
    for (int i = 0; i < B_Q; ++i) { mbar_init(b_full + i, 1); mbar_init(b_empty + i, 1); }
    for (int i = 0; i < C::kRelBars; ++i) mbar_init(rel + i, 1);
    for (int b = 0; b < 2; ++b) { mbar_init(acc_full + b, C::kIssuers); mbar_init(acc_empty + b, kDqWarps); }
    mbar_init(mma_done, 1);
    mbar_init(mma_done + 1, 1);
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
  // Wait until the stages that quad n takes over from quad n - depth are free.
  auto stage_free = [&](uint32_t n, uint32_t depth, int code, int site) -> bool {
    if (n < depth) return true;
    const uint32_t g = n - depth;
    return wait_bar(rel + g % C::kRelBars, (g / C::kRelBars) & 1, s_abort, err, code, site UAII_WS_ARG);
  };
  auto quad_range = [&](const Tile& t, int& q0, int& q1) {
    q0 = t.split * args.kquads / args.splits;
    q1 = (t.split + 1) * args.kquads / args.splits;
  };
  // 64-element atoms of quad q (4, or fewer in the last quad of a Q4_0 / Q8_0 row)
  auto quad_atoms = [&](int q) { return min(4, args.k_atoms - 4 * q); };

  if (warp == 0) {
    // ------------------------------------------------------------ weight TMA producer
    // (converged warp, one elected lane issues the copies; as for the MMA issuer)
    {
      uint32_t pi = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const Tile t = decode_tile(args, tile, BN);
        const int row0 = t.e * args.rows_per_expert + t.m_tile * (args.gateup ? 64 : 128);
        int q0, q1;
        quad_range(t, q0, q1);
        for (int q = q0; q < q1 && ok; ++q) {
          const int ps = pi % P_ST;
          if (!(ok = wait_bar(pk_empty + ps, ((pi / P_ST) & 1) ^ 1, s_abort, err, kErrTimeoutProducer, 0 UAII_WS_ARG))) break;
          const int x = (q * Fm::kBytes) & ~15;
          uint8_t* dst = sP + ps * C::kPStage;
          if (elect_one()) {
            mbar_arrive_expect_tx(pk_full + ps, C::kPStage);
#pragma unroll
            for (int j = 0; j < Fm::kBoxes; ++j) {
              uint8_t* d = dst + j * 128 * C::kWB;
              if (args.gateup) {
                tma_load_2d(d, &tm_w0, pk_full + ps, x + 128 * j, row0);
                tma_load_2d(d + 64 * C::kWB, &tm_w1, pk_full + ps, x + 128 * j, row0);
              } else {
                tma_load_2d(d, &tm_w0, pk_full + ps, x + 128 * j, row0);
                tma_load_2d(d + 64 * C::kWB, &tm_w0, pk_full + ps, x + 128 * j, row0 + 64);
              }
            }
          }
          __syncwarp();
          ++pi;
        }
      }
      // never leave with copies in flight: wait (bounded) for the last load of every stage
      for (uint32_t j = (pi > (uint32_t)P_ST ? pi - P_ST : 0); j < pi; ++j)
        (void)mbar_wait(pk_full + j % P_ST, (j / P_ST) & 1);
    }
    __syncwarp();
  } else if (warp == kBWarp) {
    // ------------------------------------------------------------ activation TMA producer
    {
      uint32_t bi = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const Tile t = decode_tile(args, tile, BN);
        const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
        int q0, q1;
        quad_range(t, q0, q1);
        for (int q = q0; q < q1 && ok; ++q) {
          const int na = quad_atoms(q);
          if constexpr (C::kWide) {  // one stage per atom
            for (int j = 0; j < na && ok; ++j) {
              const int bs = bi % B_Q;
              if (!(ok = wait_bar(b_empty + bs, ((bi / B_Q) & 1) ^ 1, s_abort, err, kErrTimeoutProducer, 1 UAII_WS_ARG))) break;
              if (elect_one()) {
                mbar_arrive_expect_tx(b_full + bs, C::kBAtom);
                tma_load_2d(sB + bs * C::kBStage, &tm_x, b_full + bs, q * kQuadK + 64 * j, slot0);
              }
              __syncwarp();
              ++bi;
            }
          } else {  // one stage per quad
            const int bs = bi % B_Q;
            if (!(ok = stage_free(bi, B_Q, kErrTimeoutProducer, 1))) break;
            if (elect_one()) {
              mbar_arrive_expect_tx(b_full + bs, na * C::kBAtom);
              for (int j = 0; j < na; ++j)
                tma_load_2d(sB + bs * C::kBStage + j * C::kBAtom, &tm_x, b_full + bs, q * kQuadK + 64 * j, slot0);
            }
            __syncwarp();
            ++bi;
          }
        }
      }
      for (uint32_t j = (bi > (uint32_t)B_Q ? bi - B_Q : 0); j < bi; ++j)
        (void)mbar_wait(b_full + j % B_Q, (j / B_Q) & 1);
    }
    __syncwarp();
  } else if (warp == 1 || (warp == kMma1Warp && C::kIssuers == 2)) {
    // ------------------------------------------------------------ MMA issuer(s)
    // The whole warp runs the loop (waits, stage bookkeeping) in step and one
    // elected lane issues the MMAs and commits: converged code issues narrow
    // MMAs several times faster than a loop run by a single lane.
    {
      const int me = warp == 1 ? 0 : 1;  // takes the quads of every tile with local index % kIssuers == me
      uint32_t sa = 0, pa = 0;  // A stage and its phase
      uint32_t sb = 0, pb = 0;  // B stage and its phase
      uint32_t sr = 0;          // release barrier
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
        const Tile t = decode_tile(args, tile, BN);
        int q0, q1;
        quad_range(t, q0, q1);
        // MMA width: the tile's valid slots rounded up to 16 (the M = 128 minimum
        // step), so an expert's last, partly filled slot tile costs only its columns.
        // The epilogue stores only the valid slots; the columns left out are never read.
        const int n_valid = min(BN, __ldg(args.counts + t.e) - t.n_tile * BN);
        const uint32_t idesc = idesc_f16_f32(128, min(BN, max(16, (n_valid + 15) & ~15)));
        const uint32_t ab = it % C::kAccBufs;  // accumulator buffer of this tile
        if (!(ok = wait_bar(acc_empty + ab, ((it / C::kAccBufs) & 1) ^ 1, s_abort, err, kErrTimeoutMma, 2 UAII_WS_ARG)))
          break;
        tc_fence_after();
        const uint32_t dacc = tmem + (ab * C::kIssuers + me) * C::kAccCols;
        uint32_t acc = 0;
        for (int q = q0; q < q1; ++q) {
          if ((q - q0) % C::kIssuers != me) {  // the other issuer's quad
            sa = sa + 1 == A_Q ? (pa ^= 1, 0) : sa + 1;
            sb = sb + 1 == B_Q ? (pb ^= 1, 0) : sb + 1;
            sr = sr + 1 == C::kRelBars ? 0 : sr + 1;
            continue;
          }
          if (!(ok = wait_bar(a_full + sa, pa, s_abort, err, kErrTimeoutMma, 3 UAII_WS_ARG))) break;
          if constexpr (C::kWide) {
            tc_fence_after();
            const int na = quad_atoms(q);
            const uint32_t at = tmem + C::kACol0 + sa * 128;
            for (int j = 0; j < na && ok; ++j) {
              if (!(ok = wait_bar(b_full + sb, pb, s_abort, err, kErrTimeoutMma, 4 UAII_WS_ARG))) break;
              tc_fence_after();
              const uint64_t bd = sw128_desc(smem_u32(sB + sb * C::kBStage));
              if (elect_one()) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                  mma_f16_ts(dacc, at + 32 * j + 8 * ks, bd + 2 * ks, idesc, acc);
                  acc = 1;
                }
                mma_commit(b_empty + sb);
              }
              __syncwarp();
              acc = 1;
              sb = sb + 1 == B_Q ? (pb ^= 1, 0) : sb + 1;
            }
            if (!ok) break;
            if (elect_one()) mma_commit(rel + sr);
            __syncwarp();
            sa = sa + 1 == A_Q ? (pa ^= 1, 0) : sa + 1;
            sr = sr + 1 == C::kRelBars ? 0 : sr + 1;
            continue;
          }
          if (!(ok = wait_bar(b_full + sb, pb, s_abort, err, kErrTimeoutMma, 4 UAII_WS_ARG))) break;
          tc_fence_after();
#ifdef UAII_UMMA_STATS
          const long long t_issue = clock64();
#endif
          const int na = quad_atoms(q);
          const uint64_t bd = sw128_desc(smem_u32(sB + sb * C::kBQuad));
          const uint32_t at = tmem + C::kACol0 + sa * 128;
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (j < na) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                  mma_f16_ts(dacc, at + 32 * j + 8 * ks, bd + (uint64_t)((j * C::kBAtom) >> 4) + 2 * ks, idesc, acc);
                  acc = 1;
                }
              }
            }
            mma_commit(rel + sr);
          }
          __syncwarp();
          acc = 1;
#ifdef UAII_UMMA_STATS
          wstats.cyc[8] += (unsigned long long)(clock64() - t_issue);
          wstats.cnt[8] += 1;
#endif
          sa = sa + 1 == A_Q ? (pa ^= 1, 0) : sa + 1;
          sb = sb + 1 == B_Q ? (pb ^= 1, 0) : sb + 1;
          sr = sr + 1 == C::kRelBars ? 0 : sr + 1;
        }
        if (ok) {
          if (elect_one()) mma_commit(acc_full + ab);
          __syncwarp();
        }
      }
      // the tensor core must be idle before TMEM is freed
      if (elect_one()) mma_commit(mma_done + me);
      __syncwarp();
      (void)mbar_wait(mma_done + me, 0);
    }
    __syncwarp();
  } else if (warp >= 2 && warp < kBWarp) {
    // ------------------------------------------------------------ dequant + epilogue (kDqWarps warps)
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int row = 32 * q + lane;     // A-tile row == accumulator lane
    const int grp = (warp - 2) >> 2;   // warp group 0..kGroups-1 == atom of every quad it makes
    // Gate/up tiles hold 64 features: in every 32-row block (one TMEM lane
    // quarter) lanes 0-15 are gate rows and lanes 16-31 the up rows of the same
    // 16 features, so the SwiGLU epilogue pairs them with one lane shuffle.
    // The packed stage keeps the TMA layout: gate rows 0-63, up rows 64-127.
    const int src_row = args.gateup ? (lane < 16 ? 16 * q + lane : 64 + 16 * q + (lane - 16)) : row;
    uint32_t pi = 0, qi = 0, it = 0;
    bool ok = true;
    // Epilogue of tile number `e_it` (accumulator buffer e_it & 1), run after the
    // next tile's dequantization has been issued so that the tensor core keeps
    // working while the accumulator is drained.
    constexpr int kCols = BN / kGroups;          // columns per group (>= 4)
    constexpr int kW = kCols >= 8 ? 8 : 4;       // columns per TMEM load
    auto epilogue = [&](const Tile& t, uint32_t e_it) -> bool {
      const uint32_t eb = e_it % C::kAccBufs;
      if (!wait_bar(acc_full + eb, (e_it / C::kAccBufs) & 1, s_abort, err, kErrTimeoutEpilogue, 7 UAII_WS_ARG))
        return false;
      tc_fence_after();
      const int n_valid = min(BN, __ldg(args.counts + t.e) - t.n_tile * BN);
      const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
      const uint32_t taddr = tmem + eb * C::kIssuers * C::kAccCols + ((uint32_t)(32 * q) << 16);
      int q0, q1;
      quad_range(t, q0, q1);
      const bool two = C::kIssuers == 2 && q1 - q0 >= 2;  // the second issuer's accumulator holds quads too
      // kW accumulator columns at `a` (+ the second issuer's at a + kAccCols)
      auto load_acc = [&](uint32_t a, uint32_t (&r)[8]) {
        if constexpr (kW == 8) tmem_ld8(a, r);
        else tmem_ld4(a, r);
        tmem_ld_wait();
        if (two) {
          uint32_t v[8];
          if constexpr (kW == 8) tmem_ld8(a + C::kAccCols, v);
          else tmem_ld4(a + C::kAccCols, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < kW; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(v[j]));
        }
      };
      if (args.gateup) {
        // lane l < 16 holds gate, lane l + 16 up of feature i0 + 16q + (l & 15); each
        // column pair (n, n+1) is split: the gate lane finishes n, the up lane n + 1
        const int feat = (int)operand_pos(args.h_order, t.m_tile * 64 + 16 * q + (lane & 15));
        const bool gate_lane = lane < 16;
        for (int cb = grp * kCols; cb < (grp + 1) * kCols; cb += kW) {
          uint32_t r[8];
          load_acc(taddr + cb, r);
#pragma unroll
          for (int j = 0; j < kW; j += 2) {
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
        for (int cb = grp * kCols; cb < (grp + 1) * kCols; cb += kW) {
          uint32_t r[8];
          load_acc(taddr + cb, r);
#pragma unroll
          for (int j = 0; j < kW; ++j) {
            const int n = cb + j;
            if (n < n_valid) out[(int64_t)(slot0 + n) * args.out_ld + o0 + row] = __uint_as_float(r[j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + eb);
      return true;
    };
    Tile prev{};
    bool have_prev = false;
    uint32_t sa = 0;
    // The A stage of a quad is handed to the MMA issuers one quad late: its
    // TMEM store stays in flight while the next quad is decoded (registers
    // only), and is waited for and announced just before the next store.
    bool pending = false;
    uint32_t pending_sa = 0;
    auto announce = [&]() {
      if (!pending) return;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(a_full + pending_sa);
      pending = false;
    };
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
      const Tile t = decode_tile(args, tile, BN);
      int q0, q1;
      quad_range(t, q0, q1);
      for (int qq = q0; qq < q1 && ok; ++qq, ++pi, ++qi) {
        const int ps = pi % P_ST;
        const bool active = grp < quad_atoms(qq);
        if (!(ok = wait_bar(pk_full + ps, (pi / P_ST) & 1, s_abort, err, kErrTimeoutDequant, 5 UAII_WS_ARG))) break;
        uint32_t o[32];
        if (active) {
#ifdef UAII_UMMA_STATS
          const long long tq = clock64();
#endif
          dequant_atom<F, 128 * C::kWB>(sP + ps * C::kPStage + src_row * C::kWB, (qq * Fm::kBytes) & 15, grp, o);
#ifdef UAII_UMMA_STATS
          asm volatile("" ::"r"(o[0]), "r"(o[13]), "r"(o[22]), "r"(o[31]));
          wstats.cyc[10] += (unsigned long long)(clock64() - tq);
          wstats.cnt[10] += 1;
#endif
        }
#ifdef UAII_UMMA_STATS
        const long long t_post = clock64();
#endif
        __syncwarp();
        if (lane == 0) mbar_arrive(pk_empty + ps);  // the window has been read
        announce();                                 // the previous quad's A stage
        if (!(ok = stage_free(qi, A_Q, kErrTimeoutDequant, 6))) break;
        if (active) {
          tc_fence_after();  // after the MMAs that last read this stage (stage_free)
          tmem_st32(tmem + C::kACol0 + sa * 128 + grp * 32 + ((uint32_t)(32 * q) << 16), o);
        }
        pending = true;
        pending_sa = sa;
        // one accumulator: drain the previous tile as soon as the MMAs of this
        // tile have A stages to start on (they wait for the drain)
        if (C::kAccBufs == 1 && have_prev && qq - q0 + 1 == min(A_Q, q1 - q0)) {
          announce();
          if (!(ok = epilogue(prev, it - 1))) break;
          have_prev = false;
        }
#ifdef UAII_UMMA_STATS
        wstats.cyc[9] += (unsigned long long)(clock64() - t_post);
        wstats.cnt[9] += 1;
#endif
        sa = sa + 1 == A_Q ? 0 : sa + 1;
      }
      if (!ok) break;
      announce();  // the MMAs of this tile must be able to finish before any epilogue wait
      if (C::kAccBufs == 2 && have_prev && !(ok = epilogue(prev, it - 1))) break;
      prev = t;
      have_prev = true;
    }
    if (ok) announce();
    if (ok && have_prev) (void)epilogue(prev, it - 1);
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

// ======================================================================
// Warp-MMA schedule for narrow slot tiles (8 or 16 routed slots: decode).
//
// At N <= 16 the tcgen05 schedule spends most of each quad moving the
// dequantized A tile into tensor memory and handing it to the issuing thread.
// Here every compute warp keeps its dequantized A fragments in registers and
// multiplies them with mma.sync.m16n8k16 (f16 x f16 -> f32): no A store, no
// issuing thread, no A barriers.  Warp w of the 16 compute warps owns weight
// rows 16*(w%8) .. +15 of the 128-row tile and K half w/8 of every quad; its
// lane (g = lane/4, t = lane%4) decodes rows g and g+8 of that block for the
// 32 K elements [32t, 32t+32) of the half -- one Q4_0 / Q8_0 block or one
// K-quant sub-block, so one scale per row.  The activation and h rows are
// stored in the matching order (wm_kpos).  The two K halves are added in
// shared memory after each tile.  Warp 16 is the TMA producer of the packed
// weight windows and of the activation tiles (SWIZZLE_128B, read with
// ldmatrix).  Each dequantized operand equals the tcgen05 schedule's.
constexpr int kWmWarps = 16;                   // compute warps
constexpr int kWmThreads = 32 * (kWmWarps + 1);

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Integer products m16n8k32: u8 weights times s8 (hi) or u8 (lo) activation bytes, exact int32
// sums, no accumulator input (the products of one sub-block are scaled before they are added).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_u8u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// Named barrier over `n` threads that also ORs a predicate across them.
__device__ __forceinline__ bool bar_any(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Split-work arrival of a CTA whose compute threads 0 .. n-1 have stored their partial sums: after
// the barrier one thread makes the CTA's stores visible device-wide (a fence is cumulative over
// what the barrier ordered before it), counts the arrival, and on the last of `parts` arrivals
// fences again so that the whole CTA then reads the other CTAs' partials.  True on the last.
__device__ __forceinline__ bool arrive_last(int id, int n, int* cnt, int parts) {
  bar_sync(id, n);
  bool last = false;
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(cnt, 1) == parts - 1;
    if (last) __threadfence();
  }
  return bar_any(id, n, last);
}

// NW 32-bit words starting at an even byte offset `off` of shared memory row
// `p` (4-byte aligned): 4-byte loads joined by a funnel shift of 0 or 16 bits.
template <int NW>
__device__ __forceinline__ void words_at(const uint8_t* p, int off, uint32_t (&w)[NW]) {
  const uint32_t* src = reinterpret_cast<const uint32_t*>(p + (off & ~3));
  const uint32_t sh = (uint32_t)(off & 2) * 8u;
  uint32_t u[NW + 1];
#pragma unroll
  for (int j = 0; j <= NW; ++j) u[j] = src[j];
#pragma unroll
  for (int j = 0; j < NW; ++j) w[j] = __funnelshift_r(u[j], u[j + 1], sh);
}

// One row's unit t of half h (32 K elements): loaded and scaled once per quad,
// then unpacked two f16 pairs per k-step: pair(ks) gives lo = elements
// (4ks, 4ks+2) and hi = (4ks+1, 4ks+3) of the unit -- the fragment registers of
// positions (2t, 2t+1) and (2t+8, 2t+9) of k-step ks.  Unpacking per k-step
// lets the MMA of one k-step run while the next one is unpacked.  `row` is the
// row in box 0 of the packed stage, `row1` the same row in box 1 (Q8_0), `off`
// the quad's offset in its window (Q6_K; 0 for the others).
template <int F> struct WmUnit;

// Q4_K: sub-block sb = 4h + t = nibble (t & 1) of qs[32 * (sb / 2) ..]; value
// d*sc*q - dmin*m.  Low nibble: (1024 + q) - 1024; high nibble: (1024 + 16q) / 16 - 64
// (both exact), so one code path serves both with per-lane mask and constants.
template <> struct WmUnit<kQ4_K> {
  struct Lane {
    int sb, sh;
    uint32_t mask;
    __half2 c1, c0;
    __device__ Lane(int h, int t)
        : sb(4 * h + t), sh(8 * (t & 3)), mask((t & 1) ? 0x00F000F0u : 0x000F000Fu),
          c1(__float2half2_rn((t & 1) ? 0.0625f : 1.0f)), c0(__float2half2_rn((t & 1) ? -64.f : -1024.f)) {}
  };
  uint32_t w[8];
  __half2 dd, nm;
  __device__ __forceinline__ void load(const uint8_t* row, const uint8_t*, int, const Lane& L) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(row);  // d, dmin, scales[12]
    const uint32_t y = hdr.y >> L.sh, z = hdr.z >> L.sh, w4 = hdr.w >> L.sh;
    const uint32_t sc = L.sb < 4 ? (y & 63u) : ((w4 & 15u) | (((y >> 6) & 3u) << 4));
    const uint32_t m = L.sb < 4 ? (z & 63u) : (((w4 >> 4) & 15u) | (((z >> 6) & 3u) << 4));
    q4k_scales(hdr.x, sc, m, dd, nm);
    const uint4* qp = reinterpret_cast<const uint4*>(row + 16 + 32 * (L.sb >> 1));
    const uint4 qa = qp[0], qb = qp[1];
    w[0] = qa.x; w[1] = qa.y; w[2] = qa.z; w[3] = qa.w;
    w[4] = qb.x; w[5] = qb.y; w[6] = qb.z; w[7] = qb.w;
  }
  __device__ __forceinline__ void pair(int ks, const Lane& L, uint32_t& lo, uint32_t& hi) const {
    lo = as_u32(__hfma2(__hfma2(magic_pair(w[ks], L.mask), L.c1, L.c0), dd, nm));
    hi = as_u32(__hfma2(__hfma2(magic_pair(w[ks] >> 8, L.mask), L.c1, L.c0), dd, nm));
  }
};

// Q4_0: block b = 4h + t at byte 18b {f16 d; u8 qs[16]}: low nibbles -> elements
// 0..15 (k-steps 0-3), high -> 16..31 (k-steps 4-7); value (q - 8) * d.
template <> struct WmUnit<kQ4_0> {
  struct Lane {
    int b;
    __device__ Lane(int h, int t) : b(4 * h + t) {}
  };
  uint32_t w[4];
  __half2 d;
  __device__ __forceinline__ void load(const uint8_t* row, const uint8_t*, int, const Lane& L) {
    const __half dh = __ushort_as_half((unsigned short)ld_u16(row + 18 * L.b));
    d = __halves2half2(dh, dh);
    words_at<4>(row, 18 * L.b + 2, w);
  }
  __device__ __forceinline__ void pair(int ks, const Lane&, uint32_t& lo, uint32_t& hi) const {
    const uint32_t q = w[ks & 3];
    if (ks < 4) {
      const __half2 bias = __float2half2_rn(1032.f);
      lo = as_u32(__hmul2(__hsub2(magic_pair(q, 0x000F000Fu), bias), d));
      hi = as_u32(__hmul2(__hsub2(magic_pair(q >> 8, 0x000F000Fu), bias), d));
    } else {
      const __half2 k16 = __float2half2_rn(0.0625f), bias = __float2half2_rn(-72.f);
      lo = as_u32(__hmul2(__hfma2(magic_pair(q, 0x00F000F0u), k16, bias), d));
      hi = as_u32(__hmul2(__hfma2(magic_pair(q >> 8, 0x00F000F0u), k16, bias), d));
    }
  }
};

// Q8_0: block b = 4h + t at byte 34b {f16 d; i8 qs[32]}; blocks 4..7 are read from
// box 1 (window byte 128 on).  q ^ 0x80 = q + 128 as an unsigned byte.
template <> struct WmUnit<kQ8_0> {
  struct Lane {
    int b;
    __device__ Lane(int h, int t) : b(4 * h + t) {}
  };
  uint32_t w[8];
  __half2 d;
  __device__ __forceinline__ void load(const uint8_t* row, const uint8_t* row1, int, const Lane& L) {
    const uint8_t* base = L.b < 4 ? row : row1 - 128;
    const __half dh = __ushort_as_half((unsigned short)ld_u16(base + 34 * L.b));
    d = __halves2half2(dh, dh);
    words_at<8>(base, 34 * L.b + 2, w);
  }
  __device__ __forceinline__ void pair(int ks, const Lane&, uint32_t& lo, uint32_t& hi) const {
    const __half2 bias = __float2half2_rn(1152.f);
    const uint32_t q = w[ks] ^ 0x80808080u;
    lo = as_u32(__hmul2(__hsub2(magic_pair(q, 0x00FF00FFu), bias), d));
    hi = as_u32(__hmul2(__hsub2(magic_pair(q >> 8, 0x00FF00FFu), bias), d));
  }
};

// Q6_K half h, quarter t: ql nibble (t >> 1) of ql[64h + 32(t & 1) ..], bits 2t of
// qh[32h ..], scales sc[8h + 2t] (k-steps 0-3) and sc[8h + 2t + 1]; value d*sc*(q - 32).
template <> struct WmUnit<kQ6_K> {
  struct Lane {
    int h, t;
    uint32_t ns, hrot;  // hrot: rotation taking bits 2t..2t+1 of every byte to bits 4-5
    __device__ Lane(int h_, int t_)
        : h(h_), t(t_), ns(4u * (uint32_t)(t_ >> 1)), hrot((2u * (uint32_t)t_ + 28u) & 31u) {}
  };
  uint32_t q6[8];  // 6-bit values in the low bits of each byte (bits 6-7: junk)
  __half2 s0, s1;
  // OFF = the super-block's offset in its 16-byte aligned window (even, 0..14)
  template <int OFF>
  __device__ __forceinline__ void load_off(const uint8_t* row, const Lane& L) {
    uint32_t w[8];
    load_words<OFF, 8>(row, 4 * L.h + 2 * (L.t & 1), w);  // ql bytes 64h + 32(t & 1) ..
#pragma unroll
    for (int i = 0; i < 8; ++i) q6[i] = (w[i] >> L.ns) & 0x0F0F0F0Fu;
    load_words<OFF, 8>(row, 8 + 2 * L.h, w);  // qh bytes 128 + 32h ..
    // bits 6-7 of every byte carry junk from the neighbouring 2-bit fields; the 0x3F mask in pair() drops them
#pragma unroll
    for (int i = 0; i < 8; ++i) q6[i] |= __funnelshift_r(w[i], w[i], L.hrot) & 0xF0F0F0F0u;
    const __half2 s2 = q6k_scales(ld_u16(row + OFF + 208), ld_u16(row + OFF + 192 + 8 * L.h + 2 * L.t));
    s0 = __low2half2(s2);
    s1 = __high2half2(s2);
  }
  __device__ __forceinline__ void pair(int ks, const Lane&, uint32_t& lo, uint32_t& hi) const {
    const __half2 s = ks < 4 ? s0 : s1;
    const __half2 bias = __float2half2_rn(1056.f);
    lo = as_u32(__hmul2(__hsub2(magic_pair(q6[ks], 0x003F003Fu), bias), s));
    hi = as_u32(__hmul2(__hsub2(magic_pair(q6[ks] >> 8, 0x003F003Fu), bias), s));
  }
};

template <int F, int NT, int ST>
struct WmCfg {
  using Fm = Fmt<F>;
  static constexpr int BN = 8 * NT;
  static constexpr int kWB = Fm::kBoxBytes;
  static constexpr int kPStage = Fm::kBoxes * 128 * kWB;
  static constexpr int kBAtom = BN * 128;  // one 64-K SWIZZLE_128B box of BN activation rows
  static constexpr int kBQuad = 4 * kBAtom;
  static constexpr int kOffB = 0;
  static constexpr int kOffP = kOffB + ST * kBQuad;
  // warp-MMA schedule: [8 row blocks][32 lanes][4 NT] f32; quad schedule: [2 halves][128 rows][BN] f32
  static constexpr int kRedBytes = 2 * 128 * BN * 4;
  static constexpr int kOffR = kOffP + ST * kPStage;
  static constexpr int kOffBar = kOffR + kRedBytes;
  static constexpr int kNumBars = 2 * ST;
  static constexpr int kSmem = kOffBar + kNumBars * 8 + 16 + 1024;
  static_assert(kOffP % 1024 == 0 && kBAtom % 1024 == 0, "SWIZZLE_128B stages must be 1024-byte aligned");
};

template <int F, int NT, int ST>
__global__ void __launch_bounds__(kWmThreads, 1)
    expert_warp_mma_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                           const __grid_constant__ CUtensorMap tm_x, const Args args) {
  using C = WmCfg<F, NT, ST>;
  using Fm = Fmt<F>;
  constexpr int BN = C::BN;
  constexpr int kCompute = kWmWarps * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem + C::kOffB;
  uint8_t* sP = smem + C::kOffP;
  float* sR = reinterpret_cast<float*>(smem + C::kOffR);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* full = bars;        // weight window + activation tile of a quad landed
  uint64_t* empty = full + ST;  // every compute warp is done with the stage
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + C::kNumBars);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kWmWarps);
    }
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == kWmWarps && lane == 0) {
    prefetch_tmap(&tm_w0);
    prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_x);
  }
  __syncthreads();
  const int total = __ldg(args.tile_base + args.E);
  int* err = args.err;
  auto quad_range = [&](const Tile& t, int& q0, int& q1) {
    q0 = t.split * args.kquads / args.splits;
    q1 = (t.split + 1) * args.kquads / args.splits;
  };
  auto quad_atoms = [&](int q) { return min(4, args.k_atoms - 4 * q); };

  if (warp == kWmWarps) {
    // ------------------------------------------------------------ TMA producer
    uint32_t n = 0;  // stages issued
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      const Tile t = decode_tile(args, tile, BN);
      const int row0 = t.e * args.rows_per_expert + t.m_tile * (args.gateup ? 64 : 128);
      const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
      int q0, q1;
      quad_range(t, q0, q1);
      for (int q = q0; q < q1; ++q) {
        const int s = n % ST;
        if (!(ok = bounded_wait(empty + s, ((n / ST) & 1) ^ 1, s_abort, err, kErrTimeoutProducer))) break;
        const int x = (q * Fm::kBytes) & ~15;
        const int na = quad_atoms(q);
        uint8_t* dst = sP + s * C::kPStage;
        if (elect_one()) {
          mbar_arrive_expect_tx(full + s, C::kPStage + na * C::kBAtom);
#pragma unroll
          for (int j = 0; j < Fm::kBoxes; ++j) {
            uint8_t* d = dst + j * 128 * C::kWB;
            tma_load_2d(d, &tm_w0, full + s, x + 128 * j, row0);
            if (args.gateup) tma_load_2d(d + 64 * C::kWB, &tm_w1, full + s, x + 128 * j, row0);
            else tma_load_2d(d + 64 * C::kWB, &tm_w0, full + s, x + 128 * j, row0 + 64);
          }
          for (int j = 0; j < na; ++j)
            tma_load_2d(sB + s * C::kBQuad + j * C::kBAtom, &tm_x, full + s, q * kQuadK + 64 * j, slot0);
        }
        __syncwarp();
        ++n;
      }
    }
    // never leave with copies in flight: the last ST stages
    for (uint32_t j = n > (uint32_t)ST ? n - ST : 0; j < n; ++j) (void)mbar_wait(full + j % ST, (j / ST) & 1);
  } else {
    // ------------------------------------------------------------ compute warps
    const int mw = warp & 7, h = warp >> 3;   // 16-row block, K half of every quad
    const int g = lane >> 2, tq = lane & 3;   // fragment row group, K unit
    const int r0 = 16 * mw + g, r1 = r0 + 8;  // packed stage rows (gate/up: gate 0-63, up 64-127)
    // ldmatrix: lanes 8i .. 8i+7 address the rows of matrix i = (slot octet i/2, k octet i%2)
    const int ld_mi = lane >> 3, ld_n = 8 * (ld_mi >> 1) + (lane & 7), ld_kh = ld_mi & 1;
    float* red = sR + (mw * 32 + lane) * 4 * NT;
    const typename WmUnit<F>::Lane ul(h, tq);
    uint32_t pi = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      const Tile t = decode_tile(args, tile, BN);
      int q0, q1;
      quad_range(t, q0, q1);
      float acc[2][4];  // NT accumulators; for NT == 1 the even / odd k-step halves of one
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
      WmUnit<F> u0, u1;
      auto fetch = [&](WmUnit<F>& x0, WmUnit<F>& x1, int q, uint32_t p) -> bool {
        if (!bounded_wait(full + p % ST, (p / ST) & 1, s_abort, err, kErrTimeoutDequant)) return false;
        if (2 * h < quad_atoms(q)) {  // this half of the quad exists (K % 256 == 128 leaves it out)
          const int off = (q * Fm::kBytes) & 15;
          const uint8_t* stage = sP + (p % ST) * C::kPStage;
          if constexpr (F == kQ6_K) {  // 16-byte loads with the window offset as a constant
            switch (off) {
#define UAII_WM_Q6(O)                                              \
  case O:                                                          \
    x0.template load_off<O>(stage + r0 * C::kWB, ul);              \
    x1.template load_off<O>(stage + r1 * C::kWB, ul);              \
    break;
              UAII_WM_Q6(0) UAII_WM_Q6(2) UAII_WM_Q6(4) UAII_WM_Q6(6)
              UAII_WM_Q6(8) UAII_WM_Q6(10) UAII_WM_Q6(12) UAII_WM_Q6(14)
#undef UAII_WM_Q6
              default: break;
            }
          } else {
            x0.load(stage + r0 * C::kWB, stage + (128 + r0) * C::kWB, off, ul);
            x1.load(stage + r1 * C::kWB, stage + (128 + r1) * C::kWB, off, ul);
          }
        }
        return true;
      };
      auto multiply = [&](const WmUnit<F>& x0, const WmUnit<F>& x1, int q, uint32_t p) {
        if (2 * h < quad_atoms(q)) {
          const uint8_t* bq = sB + (p % ST) * C::kBQuad;
          __syncwarp();  // ldmatrix / mma.sync below need the whole warp converged
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            uint32_t a[4];  // rows g, g + 8 at positions (2tq, 2tq+1); the same at (2tq+8, 2tq+9)
            x0.pair(ks, ul, a[0], a[2]);
            x1.pair(ks, ul, a[1], a[3]);
            // k-step ks of half h = operand positions 128h + 16ks .. +15: atom 2h + ks/4, 16-byte chunk
            // 2(ks % 4) + k octet, stored at chunk ^ (row % 8) (SWIZZLE_128B)
            const int chunk = 2 * (ks & 3) + ld_kh;
            const uint32_t addr =
                smem_u32(bq + (2 * h + (ks >> 2)) * C::kBAtom + ld_n * 128 + ((chunk ^ (ld_n & 7)) << 4));
            if constexpr (NT == 2) {
              uint32_t b[4];
              asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                           : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                           : "r"(addr));
              mma_16816(acc[0], a, b[0], b[1]);
              mma_16816(acc[NT - 1], a, b[2], b[3]);
            } else {  // even and odd k-steps in two accumulators: two independent MMA chains
              uint32_t b[2];
              asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
                           : "=r"(b[0]), "=r"(b[1])
                           : "r"(addr));
              mma_16816(acc[ks & 1], a, b[0], b[1]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + p % ST);
      };
      for (int q = q0; q < q1 && ok; ++q) {
        if (!(ok = fetch(u0, u1, q, pi))) break;
        multiply(u0, u1, q, pi++);
      }
      if constexpr (NT == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[0][i] += acc[1][i];
      }
      // every compute warp reaches this barrier once per tile; a wait that gave up stops all of them
      if (bar_any(1, kCompute, !ok)) break;
      if (h == 1) {  // K half 1 hands its sums to half 0
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) red[4 * n + i] = acc[n][i];
      }
      bar_sync(1, kCompute);
      if (h == 1) continue;
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[n][i] += red[4 * n + i];
      // accumulator (n, i): row g + 8(i / 2) of the block, slot 8n + 2tq + i % 2
      const int n_valid = min(BN, __ldg(args.counts + t.e) - t.n_tile * BN);
      const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
      if (args.gateup) {  // up rows (blocks 4-7) meet the gate rows (blocks 0-3) of the same features
        if (mw >= 4) {
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[4 * n + i] = acc[n][i];
        }
        bar_sync(2, kCompute / 2);
        if (mw < 4) {
          const float* up = sR + ((mw + 4) * 32 + lane) * 4 * NT;
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int feat = t.m_tile * 64 + 16 * mw + g + 8 * (i >> 1);
              const int sl = 8 * n + 2 * tq + (i & 1);
              const float gv = acc[n][i], uv = up[4 * n + i];
              const float sig = 1.0f / (1.0f + __expf(-gv));
              if (sl < n_valid)
                args.h_out[(int64_t)(slot0 + sl) * args.out_ld + wm_kpos(feat)] = __float2half_rn((gv * sig) * uv);
            }
        }
      } else {
        float* out = args.out + (int64_t)t.split * args.split_stride;
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int o = t.m_tile * 128 + 16 * mw + g + 8 * (i >> 1);
            const int sl = 8 * n + 2 * tq + (i & 1);
            if (sl < n_valid) out[(int64_t)(slot0 + sl) * args.out_ld + o] = acc[n][i];
          }
      }
    }
  }
  __syncthreads();
}

// ---- Quad schedule: mma.sync over whole K-quant super-blocks (decode widths) ----
//
// The warp-MMA schedule above gives each lane one 32-element unit of each of
// its two rows per quad, so a lane decodes a super-block header for every 32
// elements, and its Q4_K operands carry d*sc and dmin*m in every element.  Here
// warp w owns rows 16*(w%8) .. +15 of the 128-row tile and every other quad of
// the tile (half h = w/8 takes the quads q0 + h, q0 + h + 2, ...): a lane decodes
// 64 elements of each of its two rows per header (K order q4k_kpos / q6k_kpos,
// operand_order.cuh).
//   Q4_K: the operand is q*sc, exact in f16 (at most 945): one f16 FMA per pair,
//         fma(1024 + q, sc, -1024 sc) for low nibbles and fma(1024 + 16q, sc/16,
//         -64 sc) for high ones; a second MMA per k-step multiplies the
//         activations by the sub-block minima m (exact in f16); d and dmin are
//         applied once per quad in f32: acc += d * M1 - dmin * M2.  The weights
//         enter the products unrounded, unlike the other schedules' fp16(d*sc*q -
//         dmin*m).
//   Q6_K: quarters are assembled with one select-LOP3 per word from the low or
//         high nibbles and the 2-bit fields; the operand is fp16((q - 32) *
//         fp16(d*sc)), the same value as the other schedules.
// Warp 16 is the TMA producer of the packed weight windows and activation tiles,
// as in the warp-MMA schedule; the two halves' sums meet in shared memory after
// each tile and gate/up rows of the same features meet there for SwiGLU.
template <int F> struct QuadUnit;

template <> struct QuadUnit<kQ4_K> {
  uint32_t w[8];                   // qs bytes [32t, 32t + 32)
  __half2 f_lo, b_lo, f_hi, b_hi;  // fold constants of sub-blocks 2t and 2t + 1
  uint32_t m_lo, m_hi;             // (m, m) of the two sub-blocks, f16
  uint32_t mf;                     // (m of sub-block 2t, m of 2t + 1), f16
  float d, dmin;
  __device__ __forceinline__ void load(const uint8_t* row, int t) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(row);  // d, dmin, scales[12]
    const uint4 qa = *reinterpret_cast<const uint4*>(row + 16 + 32 * t);
    const uint4 qb = *reinterpret_cast<const uint4*>(row + 32 + 32 * t);
    w[0] = qa.x; w[1] = qa.y; w[2] = qa.z; w[3] = qa.w;
    w[4] = qb.x; w[5] = qb.y; w[6] = qb.z; w[7] = qb.w;
    // (scale, min) of sub-blocks j = 2t, 2t + 1 in the get_scale_min_k4 bit layout, as byte pairs
    const uint32_t sh = 16u * (uint32_t)(t & 1);
    const uint32_t y2 = hdr.y >> sh, z2 = hdr.z >> sh, w2 = hdr.w >> sh;
    uint32_t sc2, m2;
    if (t < 2) {
      sc2 = y2 & 0x3F3Fu;
      m2 = z2 & 0x3F3Fu;
    } else {
      sc2 = (w2 & 0x0F0Fu) | ((y2 >> 2) & 0x3030u);
      m2 = ((w2 >> 4) & 0x0F0Fu) | ((z2 >> 2) & 0x3030u);
    }
    const __half2 k1024 = __float2half2_rn(1024.f);
    const __half2 scf = __hsub2(as_h2(__byte_perm(sc2, 0, 0x4140) | kMagic), k1024);  // (sc_a, sc_b)
    const __half2 mf = __hsub2(as_h2(__byte_perm(m2, 0, 0x4140) | kMagic), k1024);   // (m_a, m_b)
    const __half2 fb = __hmul2(scf, __floats2half2_rn(1.0f, 0.0625f));
    const __half2 bb = __hmul2(scf, __floats2half2_rn(-1024.0f, -64.0f));
    f_lo = __low2half2(fb);
    f_hi = __high2half2(fb);
    b_lo = __low2half2(bb);
    b_hi = __high2half2(bb);
    m_lo = as_u32(__low2half2(mf));
    m_hi = as_u32(__high2half2(mf));
    this->mf = as_u32(mf);
    const __half2 dm = as_h2(hdr.x);
    d = __low2float(dm);
    dmin = __high2float(dm);
  }
  // k-step s: the pair at positions (2t, 2t+1) (bytes 0, 2 of word s % 8) and at
  // (2t+8, 2t+9) (bytes 1, 3), low nibbles for s < 8, high nibbles after.  The caller
  // runs k-steps s and s + 8 back to back, so the shifted word is formed once for both.
  __device__ __forceinline__ void pair(int s, uint32_t& lo, uint32_t& hi) const {
    const uint32_t q = w[s & 7], q8 = w[s & 7] >> 8;
    if (s < 8) {
      lo = as_u32(__hfma2(magic_pair(q, 0x000F000Fu), f_lo, b_lo));
      hi = as_u32(__hfma2(magic_pair(q8, 0x000F000Fu), f_lo, b_lo));
    } else {
      lo = as_u32(__hfma2(magic_pair(q, 0x00F000F0u), f_hi, b_hi));
      hi = as_u32(__hfma2(magic_pair(q8, 0x00F000F0u), f_hi, b_hi));
    }
  }
};

template <> struct QuadUnit<kQ6_K> {
  uint32_t q6[16];  // [4c + w]: 6-bit values of quarter c, positions 16pp + 4w .. +3 (bits 6-7 junk)
  __half2 s[4];     // (d*sc, d*sc) of sub-block 8hf + pp + 2c
  // OFF: the super-block's offset in its 16-byte aligned window (even, 0..14)
  template <int OFF>
  __device__ __forceinline__ void load(const uint8_t* row, int t) {
    const int hf = t >> 1, pp = t & 1;
    uint32_t l0[4], l1[4], qh[4];
    load_words<OFF, 4>(row, 4 * hf + pp, l0);      // ql[64hf + 16pp .. +15]
    load_words<OFF, 4>(row, 4 * hf + 2 + pp, l1);  // ql[64hf + 32 + 16pp .. +15]
    load_words<OFF, 4>(row, 8 + 2 * hf + pp, qh);  // qh[32hf + 16pp .. +15]
    constexpr uint32_t kHi = 0xF0F0F0F0u;  // bits 4-7 from the 2-bit fields, 0-3 from a nibble
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q6[i] = (l0[i] & ~kHi) | ((qh[i] << 4) & kHi);
      q6[4 + i] = (l1[i] & ~kHi) | ((qh[i] << 2) & kHi);
      q6[8 + i] = ((l0[i] >> 4) & ~kHi) | (qh[i] & kHi);
      q6[12 + i] = ((l1[i] >> 4) & ~kHi) | ((qh[i] >> 2) & kHi);
    }
    uint32_t sw[2];
    words_at<2>(row, OFF + 192 + 8 * hf, sw);  // scales[8hf .. 8hf + 7]
    const uint32_t dd = ld_u16(row + OFF + 208);
    const __half2 bias = __float2half2_rn(1152.f);  // 1024 + 128
    const __half2 d2 = as_h2(dd | (dd << 16));
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {  // scales pp + 4*h2 + {0, 2}: bytes pp and pp + 2 of word h2
      const uint32_t v = ((sw[h2] >> (8 * pp)) & 0x00FF00FFu) ^ 0x00800080u;  // sc + 128 as unsigned
      const __half2 p = __hmul2(d2, __hsub2(as_h2(v | kMagic), bias));      // (d*sc, d*sc')
      s[2 * h2] = __low2half2(p);
      s[2 * h2 + 1] = __high2half2(p);
    }
  }
  // k-step s = 4c + w: bytes (0, 2) and (1, 3) of quarter c's word w, value d*sc*(q - 32)
  __device__ __forceinline__ void pair(int k, uint32_t& lo, uint32_t& hi) const {
    const __half2 bias = __float2half2_rn(1056.f);  // 1024 + 32
    const uint32_t q = q6[k];
    lo = as_u32(__hmul2(__hsub2(magic_pair(q, 0x003F003Fu), bias), s[k >> 2]));
    hi = as_u32(__hmul2(__hsub2(magic_pair(q >> 8, 0x003F003Fu), bias), s[k >> 2]));
  }
};

// Integer variant (Q4_K gate/up, 8-slot tiles).  The activations arrive as 16-bit integers per
// (slot, quad): x ~ s * a, s = max|x| / 32767 over the quad's 256 elements, a = 256 * hi + lo
// split into an s8 byte plane (hi) and a u8 plane (lo) (route_gather, kOrderQ4KI8).  One k-step
// of m16n8k32 is one 32-element sub-block: the operands are the raw nibbles as bytes -- q for
// the low-nibble sub-blocks (one AND per 4 elements), 16 q for the high-nibble ones -- and the
// exact int32 products of each plane are scaled by the sub-block's 6-bit scale and added in
// int32 (no overflow: at most 9.9e8 per quad).  The minima use the activations' integer
// sub-block sums (f16 hi + lo, divided by 1024) in one f16 MMA per sum word, as above.  Per quad
// and output: acc += s * (d / 16 * (256 * main_hi + main_lo) - 1024 * dmin * sum_m).  Within a
// sub-block, K position 4t + i holds element 8t + i and 16 + 4t + i holds 8t + 4 + i (t = lane
// quarter, i < 4), so a lane's operand words are qs words 8p + 2t and 8p + 2t + 1.
struct QuadI8 {
  uint32_t sc[2];  // 6-bit scales of sub-blocks 0-3 and 4-7, one per byte
  uint32_t mf;     // (m of sub-block 2t, m of 2t + 1), f16: A operand of the minima MMA
  float d16, dm1024;
  // qs words 8p + 2t and 8p + 2t + 1 of sub-block pair p (loaded where they are used)
  __device__ __forceinline__ static uint2 words(const uint8_t* row, int p, int t) {
    return *reinterpret_cast<const uint2*>(row + 16 + 32 * p + 8 * t);
  }
  __device__ __forceinline__ void load(const uint8_t* row, int t) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(row);  // d, dmin, scales[12]
    // get_scale_min_k4 for all eight sub-blocks at once, one byte each
    sc[0] = hdr.y & 0x3F3F3F3Fu;
    sc[1] = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t m_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    const uint32_t mw = (t < 2 ? m_lo : m_hi) >> (16u * (uint32_t)(t & 1));  // bytes m(2t), m(2t + 1)
    mf = as_u32(__hsub2(as_h2(__byte_perm(mw, 0, 0x4140) | kMagic), __float2half2_rn(1024.f)));
    const float2 dm = __half22float2(as_h2(hdr.x));
    d16 = dm.x * 0.0625f;
    dm1024 = dm.y * 1024.f;
  }
  // scale of sub-block j (compile-time) as an integer
  __device__ __forceinline__ int scale(int j) const { return (int)__byte_perm(sc[j >> 2], 0, 0x4440 | (j & 3)); }
};

template <int F, int NT, int ST, bool kXSum, bool kI8 = false>
__global__ void __launch_bounds__(kWmThreads, 1)
    expert_quad_mma_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                           const __grid_constant__ CUtensorMap tm_x, const Args args) {
  static_assert(F == kQ4_K || F == kQ6_K, "quad schedule: K-quants only");
  static_assert(!kXSum || F == kQ4_K, "activation sub-block sums serve the Q4_K minima");
  static_assert(!kI8 || (F == kQ4_K && kXSum), "integer activations: Q4_K gate/up");  // launched with NT == 1
  using C = WmCfg<F, NT, ST>;
  using Fm = Fmt<F>;
  constexpr int BN = C::BN;
  constexpr int kCompute = kWmWarps * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem + C::kOffB;
  uint8_t* sP = smem + C::kOffP;
  float* sR = reinterpret_cast<float*>(smem + C::kOffR);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* full = bars;        // weight window + activation tile of a quad landed
  uint64_t* empty = full + ST;  // the half that used the stage is done with it
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + C::kNumBars);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kWmWarps / 2);
    }
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == kWmWarps && lane == 0) {
    prefetch_tmap(&tm_w0);
    prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_x);
  }
  __syncthreads();
  const int tiles = __ldg(args.tile_base + args.E);
  int* err = args.err;
  // Tail split (gate/up): `rem` tiles of a last wave that fills at most half of the grid each
  // become `ts` units of consecutive quads (at least two, one per half); the CTA that finishes
  // a tile's last unit adds the units' sums in unit order and runs the epilogue.
  int tail_base = tiles, ts = 1;
  if (args.tail_part != nullptr && args.gateup) {
    const int G = (int)gridDim.x, rem = tiles % G, smax = args.kquads / 2;
    if (rem > 0 && 2 * rem <= G && smax >= 2) {
      ts = min(smax, G / rem);
      tail_base = tiles - rem;
    }
  }
  const int total = tail_base + (tiles - tail_base) * ts;
  // Balanced ranges (down): CTA c takes quads [W c / G, W (c + 1) / G) of the tile-major sequence
  // of all W = tiles x kquads quads, so every CTA streams the same number of weight bytes; a tile
  // cut between CTAs is finished by whichever CTA completes its last piece.
  // With fewer quads than CTAs only the first W CTAs take ranges (one quad or more each), so every
  // CTA between a cut tile's first and last holds a piece of it.
  const bool ranges = args.ranges != 0 && !args.gateup && args.tail_part != nullptr;
  const int64_t wq = (int64_t)tiles * args.kquads;
  const int64_t gr = min((int64_t)gridDim.x, wq);
  const bool has_range = ranges && (int64_t)blockIdx.x < gr;
  const int64_t rw0 = has_range ? wq * blockIdx.x / gr : 0;
  const int64_t rw1 = has_range ? wq * (blockIdx.x + 1) / gr : 0;
  const int rt0 = ranges ? (int)(rw0 / args.kquads) : 0;
  // the CTA whose range holds quad x of the sequence
  auto cta_of = [&](int64_t x) { return (int)(((x + 1) * gr + wq - 1) / wq) - 1; };
  // unit -> tile, quad range, and (tail units) the tail tile index and the unit's rank in it
  auto unit_tile = [&](int unit, Tile& t, int& q0, int& q1, int& tail, int& tsp) {
    int tile = unit;
    tail = -1;
    tsp = 0;
    if (unit >= tail_base) {
      const int u = unit - tail_base;
      tail = u / ts;
      tsp = u - tail * ts;
      tile = tail_base + tail;
    }
    t = decode_tile(args, tile, BN);
    q0 = t.split * args.kquads / args.splits;
    q1 = (t.split + 1) * args.kquads / args.splits;
    if (tail >= 0) {
      const int a0 = q0, nq = q1 - q0;
      q0 = a0 + tsp * nq / ts;
      q1 = a0 + (tsp + 1) * nq / ts;
    }
  };
  // this CTA's u-th unit (false past the last); rt: its tile index (ranges)
  auto unit_at = [&](int u, Tile& t, int& q0, int& q1, int& tail, int& tsp, int& rt) -> bool {
    if (ranges) {
      rt = rt0 + u;
      const int64_t base = (int64_t)rt * args.kquads;
      if (rw0 >= rw1 || base >= rw1) return false;
      t = decode_tile(args, rt, BN);  // splits == 1
      q0 = (int)(max(rw0, base) - base);
      q1 = (int)(min(rw1, base + args.kquads) - base);
      tail = -1;
      tsp = 0;
      return true;
    }
    const int unit = (int)blockIdx.x + u * (int)gridDim.x;
    if (unit >= total) return false;
    rt = unit;
    unit_tile(unit, t, q0, q1, tail, tsp);
    return true;
  };

  if (warp == kWmWarps) {
    // ------------------------------------------------------------ TMA producer
    uint32_t n = 0;  // stages issued
    bool ok = true;
    Tile t;
    int q0, q1, tail, tsp, rt;
    for (int u = 0; ok && unit_at(u, t, q0, q1, tail, tsp, rt); ++u) {
      const int row0 = t.e * args.rows_per_expert + t.m_tile * (args.gateup ? 64 : 128);
      const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
      for (int q = q0; q < q1; ++q) {
        const int s = n % ST;
        if (!(ok = bounded_wait(empty + s, ((n / ST) & 1) ^ 1, s_abort, err, kErrTimeoutProducer))) break;
        const int x = (q * Fm::kBytes) & ~15;
        uint8_t* dst = sP + s * C::kPStage;
        if (elect_one()) {
          mbar_arrive_expect_tx(full + s, C::kPStage + 4 * C::kBAtom);
          tma_load_2d(dst, &tm_w0, full + s, x, row0);
          if (args.gateup) tma_load_2d(dst + 64 * C::kWB, &tm_w1, full + s, x, row0);
          else tma_load_2d(dst + 64 * C::kWB, &tm_w0, full + s, x, row0 + 64);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tma_load_2d(sB + s * C::kBQuad + j * C::kBAtom, &tm_x, full + s, q * kQuadK + 64 * j, slot0);
        }
        __syncwarp();
        ++n;
      }
    }
    // never leave with copies in flight: the last ST stages
    for (uint32_t j = n > (uint32_t)ST ? n - ST : 0; j < n; ++j) (void)mbar_wait(full + j % ST, (j / ST) & 1);
  } else {
    // ------------------------------------------------------------ compute warps
    const int mw = warp & 7, h = warp >> 3;   // 16-row block, quad parity of the tile
    const int g = lane >> 2, tq = lane & 3;   // fragment row group, lane quarter
    const int r0 = 16 * mw + g, r1 = r0 + 8;  // packed stage rows (gate/up: gate 0-63, up 64-127)
    // ldmatrix: lanes 8i .. 8i+7 address the rows of matrix i = (slot octet i/2, k octet i%2);
    // k-step s reads 16-byte chunk 2(s%4) + (k octet) of atom s/4, stored at chunk ^ (row % 8)
    const int ld_mi = lane >> 3, ld_n = 8 * (ld_mi >> 1) + (lane & 7);
    const uint32_t cx = (uint32_t)((ld_mi & 1) ^ (lane & 7));
    uint32_t boff[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) boff[j] = (uint32_t)(ld_n * 128) + (((uint32_t)(2 * j) ^ cx) << 4);
    // integer variant: matrices (hi, K 0-15), (hi, K 16-31), (lo, K 0-15), (lo, K 16-31) of a sub-block;
    // sub-block j sits in atom 2 * plane + j / 4 at chunks 2 (j % 4) and 2 (j % 4) + 1
    uint32_t i8off[4];
    if constexpr (kI8) {
      const uint32_t r8 = (uint32_t)(lane & 7), half = (uint32_t)(ld_mi & 1), plane = (uint32_t)(ld_mi >> 1);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        i8off[j] = plane * 2u * (uint32_t)C::kBAtom + r8 * 128u + ((((uint32_t)(2 * j) + half) ^ r8) << 4);
    }
    const uint32_t sB0 = smem_u32(sB);
    uint32_t pi = 0;
    bool ok = true;
    Tile t;
    int q0, q1, tail, tsp, rt;
    for (int u = 0; unit_at(u, t, q0, q1, tail, tsp, rt); ++u) {
      float acc[NT][4], acc2[NT][4];  // acc2: Q6_K odd k-steps with one slot octet
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[n][i] = acc2[n][i] = 0.f;
      // per-tile bases of the slot-side records: sub-block sums of slots g (+ 8n), read as
      // (S[2tq], S[2tq+1]) words, and (integer variant) the scales of accumulator columns 2tq, 2tq+1
      const uint32_t* xs_row[NT];
      const float* xsc_row[NT][2];
      if constexpr (kXSum) {
        const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const int64_t slot = min((int64_t)(slot0 + 8 * n + g), args.S_rows - 1);
          xs_row[n] = reinterpret_cast<const uint32_t*>(args.xsum + slot * args.kquads * 16) + tq;
          if constexpr (kI8) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
              xsc_row[n][c] =
                  args.xscale + min((int64_t)(slot0 + 8 * n + 2 * tq + c), args.S_rows - 1) * args.kquads;
          }
        }
      }
      // this half's quads q0 + h, q0 + h + 2, ...; quad q sits in stage (pi + q - q0) % ST
      const uint32_t pi0 = pi;
      pi += (uint32_t)(q1 - q0);
      for (int q = q0 + h; q < q1; q += 2) {
        const uint32_t ps = pi0 + (uint32_t)(q - q0);
        if (!(ok = bounded_wait(full + ps % ST, (ps / ST) & 1, s_abort, err, kErrTimeoutDequant))) break;
        const uint8_t* stage = sP + (ps % ST) * C::kPStage;
        // Q4_K with activation sums: this quad's sub-block sums of slots g (and g + 8), issued
        // first so that their latency hides behind the decode below
        uint32_t xs[NT][2];
        if constexpr (kXSum) {
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            xs[n][0] = __ldg(xs_row[n] + 8 * q);      // (S[2tq], S[2tq+1]) rounded to f16
            xs[n][1] = __ldg(xs_row[n] + 8 * q + 4);  // their remainders
          }
        }
        if constexpr (kI8) {
          float xsc[NT][2];  // dequant scales of accumulator columns 8n + 2tq, 8n + 2tq + 1
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            xsc[n][0] = __ldg(xsc_row[n][0] + q);
            xsc[n][1] = __ldg(xsc_row[n][1] + q);
          }
          const uint8_t* row0 = stage + r0 * C::kWB;
          const uint8_t* row1 = stage + r1 * C::kWB;
          QuadI8 v0, v1;
          v0.load(row0, tq);
          v1.load(row1, tq);
          const uint32_t bq = sB0 + (ps % ST) * C::kBQuad;
          int ah[NT][4], al[NT][4];  // per accumulator: 16 x sum_j sc_j sum_k q_k (hi and lo plane bytes)
          __syncwarp();              // ldmatrix / mma.sync below need the whole warp converged
          uint2 w0 = QuadI8::words(row0, 0, tq), w1 = QuadI8::words(row1, 0, tq);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t M = (j & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;  // 16 q (high nibbles) or q
            const int nb = j & 1;
            if (j > 0 && nb == 0) {
              w0 = QuadI8::words(row0, j >> 1, tq);
              w1 = QuadI8::words(row1, j >> 1, tq);
            }
            const uint32_t a[4] = {w0.x & M, w1.x & M, w0.y & M, w1.y & M};
            // scales of rows g (accumulators 0, 1) and g + 8 (2, 3); x16 where the operand is q, not 16 q
            const int s0 = v0.scale(j) << (nb ? 0 : 4), s1 = v1.scale(j) << (nb ? 0 : 4);
#pragma unroll
            for (int n = 0; n < NT; ++n) {  // slot octet n: activation rows 8n .. 8n + 7 of the atoms
              uint32_t b[4];
              asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                           : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                           : "r"(bq + i8off[j & 3] + (uint32_t)((j >> 2) * C::kBAtom + n * 1024)));
              int ph[4], pl[4];
              mma_u8s8(ph, a, b[0], b[1]);
              mma_u8u8(pl, a, b[2], b[3]);
              if (j == 0) {
                ah[n][0] = s0 * ph[0]; ah[n][1] = s0 * ph[1]; ah[n][2] = s1 * ph[2]; ah[n][3] = s1 * ph[3];
                al[n][0] = s0 * pl[0]; al[n][1] = s0 * pl[1]; al[n][2] = s1 * pl[2]; al[n][3] = s1 * pl[3];
              } else {
                ah[n][0] += s0 * ph[0]; ah[n][1] += s0 * ph[1]; ah[n][2] += s1 * ph[2]; ah[n][3] += s1 * ph[3];
                al[n][0] += s0 * pl[0]; al[n][1] += s0 * pl[1]; al[n][2] += s1 * pl[2]; al[n][3] += s1 * pl[3];
              }
            }
          }
          const uint32_t amf[4] = {v0.mf, v1.mf, 0u, 0u};
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            float m2[4] = {0.f, 0.f, 0.f, 0.f};  // sum_k m(row, k) S(slot, k) / 1024
            mma_16816(m2, amf, xs[n][0], 0u);
            mma_16816(m2, amf, xs[n][1], 0u);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float d16 = i < 2 ? v0.d16 : v1.d16, dm = i < 2 ? v0.dm1024 : v1.dm1024;
              const float main = fmaf(256.f, (float)ah[n][i], (float)al[n][i]);  // 16 x sum_j sc_j sum_k q_k a_k
              acc[n][i] = fmaf(xsc[n][i & 1], fmaf(d16, main, -dm * m2[i]), acc[n][i]);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(empty + ps % ST);
          continue;
        }
        QuadUnit<F> u0, u1;
        if constexpr (F == kQ6_K) {  // 16-byte loads with the window offset as a constant
          switch ((q * Fm::kBytes) & 15) {
#define UAII_QM_Q6(O)                                  \
  case O:                                              \
    u0.template load<O>(stage + r0 * C::kWB, tq);      \
    u1.template load<O>(stage + r1 * C::kWB, tq);      \
    break;
            UAII_QM_Q6(0) UAII_QM_Q6(2) UAII_QM_Q6(4) UAII_QM_Q6(6)
            UAII_QM_Q6(8) UAII_QM_Q6(10) UAII_QM_Q6(12) UAII_QM_Q6(14)
#undef UAII_QM_Q6
            default: break;
          }
        } else {
          u0.load(stage + r0 * C::kWB, tq);
          u1.load(stage + r1 * C::kWB, tq);
        }
        // the four lane addresses of the stage's k-step columns; atoms are constant offsets from them
        const uint32_t bq = sB0 + (ps % ST) * C::kBQuad;
        const uint32_t bqa[4] = {bq + boff[0], bq + boff[1], bq + boff[2], bq + boff[3]};
        uint32_t am_lo[4], am_hi[4];  // Q4_K min operands: rows g, g + 8 of sub-block 2t, then 2t + 1
        if constexpr (F == kQ4_K && !kXSum) {
          am_lo[0] = am_lo[2] = u0.m_lo;
          am_lo[1] = am_lo[3] = u1.m_lo;
          am_hi[0] = am_hi[2] = u0.m_hi;
          am_hi[1] = am_hi[3] = u1.m_hi;
        }
        // Q4_K: this quad's sums of q*sc*x and of m*x.  With one slot octet (NT == 1) the odd
        // k-steps accumulate into a second register set (m1o, and acc2 for Q6_K), so the warp's
        // MMAs form two dependency chains instead of one.
        constexpr int kChains = NT == 1 ? 2 : 1;
        float m1[NT][4], m2[NT][4], m1o[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) m1[n][i] = m2[n][i] = m1o[n][i] = 0.f;
        __syncwarp();  // ldmatrix / mma.sync below need the whole warp converged
#pragma unroll
        for (int idx = 0; idx < 16; ++idx) {
          // Q4_K: k-steps j and j + 8 (the low and high nibbles of packed word j) back to back
          const int s = F == kQ4_K ? (idx >> 1) + 8 * (idx & 1) : idx;
          uint32_t a[4];  // rows g, g + 8 at positions (2tq, 2tq+1); the same at (2tq+8, 2tq+9)
          u0.pair(s, a[0], a[2]);
          u1.pair(s, a[1], a[3]);
          const uint32_t addr = bqa[s & 3] + (s >> 2) * C::kBAtom;
          uint32_t b[2 * NT];
          if constexpr (NT == 2) {
            asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                         : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                         : "r"(addr));
          } else {
            asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
                         : "=r"(b[0]), "=r"(b[1])
                         : "r"(addr));
          }
          const bool odd = kChains == 2 && (idx & 1);
          if constexpr (F == kQ4_K) {
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              mma_16816(odd ? m1o[n] : m1[n], a, b[2 * n], b[2 * n + 1]);
              if constexpr (!kXSum) mma_16816(m2[n], s < 8 ? am_lo : am_hi, b[2 * n], b[2 * n + 1]);
            }
          } else {
#pragma unroll
            for (int n = 0; n < NT; ++n) mma_16816(odd ? acc2[n] : acc[n], a, b[2 * n], b[2 * n + 1]);
          }
        }
        if constexpr (kXSum) {  // sum_k m(row, sub-block k) S(slot, k): one k-step of 8 sub-blocks (+ 8 zeros), twice
          const uint32_t amf[4] = {u0.mf, u1.mf, 0u, 0u};
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            mma_16816(m2[n], amf, xs[n][0], 0u);
            mma_16816(m2[n], amf, xs[n][1], 0u);
          }
        }
        if constexpr (F == kQ4_K) {  // accumulator (n, i): row g + 8(i / 2)
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float dv = i < 2 ? u0.d : u1.d, mv = i < 2 ? u0.dmin : u1.dmin;
              const float p = kChains == 2 ? m1[n][i] + m1o[n][i] : m1[n][i];
              acc[n][i] = fmaf(-mv, m2[n][i], fmaf(dv, p, acc[n][i]));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + ps % ST);
      }
      if constexpr (F == kQ6_K && NT == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[0][i] += acc2[0][i];
      }
      // every compute warp reaches this barrier once per tile; a wait that gave up stops all of them.
      // It also puts every thread's reads of the previous tile's sums before this tile's writes.
      if (bar_any(1, kCompute, !ok)) break;
      {  // both halves' sums: sR[h][slot][row], row 16 mw + g + 8 (i / 2), slot 8 n + 2 tq + i % 2
        float* rs = sR + h * (128 * BN);
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) rs[(8 * n + 2 * tq + (i & 1)) * 128 + 16 * mw + g + 8 * (i >> 1)] = acc[n][i];
      }
      bar_sync(1, kCompute);
      // The tile's outputs, spread over all compute threads with the row fastest (coalesced
      // stores): each the even half's sum plus the odd half's.
      const int ct = threadIdx.x;
      const int n_valid = min(BN, __ldg(args.counts + t.e) - t.n_tile * BN);
      const int slot0 = __ldg(args.offsets + t.e) + t.n_tile * BN;
      if (args.gateup) {  // feature f: gate row f and up row 64 + f
        constexpr int kPer = 64 * BN / kCompute;
        float gv[kPer], uv[kPer];
#pragma unroll
        for (int r = 0; r < kPer; ++r) {
          const int o = ct + r * kCompute, f = o % 64, sl = o / 64;
          gv[r] = sR[sl * 128 + f] + sR[128 * BN + sl * 128 + f];
          uv[r] = sR[sl * 128 + 64 + f] + sR[128 * BN + sl * 128 + 64 + f];
        }
        if (tail >= 0) {  // a tail unit: publish this range's sums; the tile's last unit adds them all
          float* part = args.tail_part + (int64_t)tail * ts * (128 * BN);
#pragma unroll
          for (int r = 0; r < kPer; ++r) {
            const int o = ct + r * kCompute, f = o % 64, sl = o / 64;
            part[(int64_t)tsp * (128 * BN) + sl * 128 + f] = gv[r];
            part[(int64_t)tsp * (128 * BN) + sl * 128 + 64 + f] = uv[r];
          }
          if (!arrive_last(1, kCompute, args.tail_cnt + tail, ts)) continue;
#pragma unroll
          for (int r = 0; r < kPer; ++r) {
            const int o = ct + r * kCompute, f = o % 64, sl = o / 64;
            float a = 0.f, b = 0.f;
            for (int u = 0; u < ts; ++u) {
              a += __ldcg(part + (int64_t)u * (128 * BN) + sl * 128 + f);
              b += __ldcg(part + (int64_t)u * (128 * BN) + sl * 128 + 64 + f);
            }
            gv[r] = a;
            uv[r] = b;
          }
          if (ct == 0) args.tail_cnt[tail] = 0;  // zero again for the next launch
        }
#pragma unroll
        for (int r = 0; r < kPer; ++r) {
          const int o = ct + r * kCompute, f = o % 64, sl = o / 64;
          const float sig = 1.0f / (1.0f + __expf(-gv[r]));
          if (sl < n_valid)
            args.h_out[(int64_t)(slot0 + sl) * args.out_ld + operand_pos(args.h_order, t.m_tile * 64 + f)] =
                __float2half_rn((gv[r] * sig) * uv[r]);
        }
      } else {
        constexpr int kPer = 128 * BN / kCompute;
        float v[kPer];  // output o = ct + r * kCompute: row o % 128, slot o / 128
#pragma unroll
        for (int r = 0; r < kPer; ++r) {
          const int o = ct + r * kCompute;
          v[r] = sR[o] + sR[128 * BN + o];
        }
        if (ranges && (q0 != 0 || q1 != args.kquads)) {
          // a piece of a tile cut between CTAs cf .. cl: piece p = this CTA - cf goes to slot 1 of
          // CTA cf (its last piece) or slot 0 of this CTA (its first piece); the CTA that completes
          // the last piece adds pieces 0 .. np - 1 in order
          const int cf = cta_of((int64_t)rt * args.kquads), cl = cta_of((int64_t)(rt + 1) * args.kquads - 1);
          const int np = cl - cf + 1, p = (int)blockIdx.x - cf;
          float* mine = args.tail_part + (int64_t)(2 * (int)blockIdx.x + (p == 0 ? 1 : 0)) * (128 * BN);
#pragma unroll
          for (int r = 0; r < kPer; ++r) mine[ct + r * kCompute] = v[r];
          if (!arrive_last(1, kCompute, args.tail_cnt + cf, np)) continue;
#pragma unroll
          for (int r = 0; r < kPer; ++r) {
            float a = 0.f;
            for (int u2 = 0; u2 < np; ++u2)
              a += __ldcg(args.tail_part + (int64_t)(2 * (cf + u2) + (u2 == 0 ? 1 : 0)) * (128 * BN) + ct +
                          r * kCompute);
            v[r] = a;
          }
          if (ct == 0) args.tail_cnt[cf] = 0;  // zero again for the next launch
        }
        float* out = args.out + (int64_t)t.split * args.split_stride;
#pragma unroll
        for (int r = 0; r < kPer; ++r) {
          const int o = ct + r * kCompute, row = o % 128, sl = o / 128;
          if (sl < n_valid) out[(int64_t)(slot0 + sl) * args.out_ld + t.m_tile * 128 + row] = v[r];
        }
      }
    }
  }
  __syncthreads();
}

// tile_base[e] = tiles of the experts before e (an exclusive scan over one warp, 32 experts
// per round), tile_base[E] = all tiles.
__global__ void tile_table_kernel(const int32_t* counts, int E, int bn, int m_tiles, int splits,
                                  int32_t* tile_base) {
  const int lane = threadIdx.x;
  int run = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int n = e < E ? ((counts[e] + bn - 1) / bn) * m_tiles * splits : 0;
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (e < E) tile_base[e] = run + incl - n;
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) tile_base[E] = run;
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

template <int F, int BN, int A_Q, int B_Q, int P_ST>
cudaError_t run_gemm(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x, const Args& a,
                     cudaStream_t st) {
  using C = Cfg<F, BN, A_Q, B_Q, P_ST>;
  static_assert(C::kSmem <= 227 * 1024, "shared memory budget");
  auto kern = expert_gemm_kernel<F, BN, A_Q, B_Q, P_ST>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  kern<<<num_sms(), kThreads, C::kSmem, st>>>(w0, w1, x, a);
  return cudaGetLastError();
}

// Ring depths per (format, slot tile), in quads.  A stages: as many 128-column
// stages as tensor memory leaves next to the two accumulators.  Activation
// stages: 4 for narrow tiles, fewer as they grow.  Packed windows: the rest of
// shared memory, up to 8 (decode widths are bound by HBM latency).
template <int F, int BN>
struct Stages {
  static constexpr int kBudget = 224 * 1024;  // stage bytes; barriers and alignment slack come on top
  static constexpr int A = BN <= 32 ? 3 : 2;
  static constexpr int kPStage = Fmt<F>::kBoxes * 128 * Fmt<F>::kBoxBytes;
  // 256-slot tiles: 3 packed stages (2 above 30 KB), the rest for 32 KB activation atoms
  static constexpr int P_wide = kPStage <= 30 * 1024 ? 3 : 2;
  static constexpr int B_wide_fit = (kBudget - P_wide * kPStage) / (256 * 128);
  static constexpr int B = BN == 256 ? (B_wide_fit > 6 ? 6 : B_wide_fit) : BN <= 32 ? 4 : (BN == 64 ? 3 : 2);
  static constexpr int kBBytes = BN == 256 ? B * 256 * 128 : B * BN * 512;
  static constexpr int P_fit = (kBudget - kBBytes) / kPStage;
  static constexpr int P = BN == 256 ? P_wide : (P_fit > 8 ? 8 : P_fit);
  static_assert(P >= 2 && B >= 2, "shared-memory budget");
};

template <int F, int BN>
cudaError_t run_cfg(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x, const Args& a,
                    cudaStream_t st) {
  using S = Stages<F, BN>;
  return run_gemm<F, BN, S::A, S::B, S::P>(w0, w1, x, a, st);
}

template <int F>
cudaError_t dispatch_bn(int bn, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
                        const Args& a, cudaStream_t st) {
  switch (bn) {
    case 16: return run_cfg<F, 16>(w0, w1, x, a, st);
    case 32: return run_cfg<F, 32>(w0, w1, x, a, st);
    case 64: return run_cfg<F, 64>(w0, w1, x, a, st);
    case 128: return run_cfg<F, 128>(w0, w1, x, a, st);
    case 256: return run_cfg<F, 256>(w0, w1, x, a, st);
    default: return cudaErrorInvalidValue;
  }
}

// Warp-MMA schedule: ST (packed window + activation) stage pairs, as many as
// fit next to the K-half exchange area, up to 8.
template <int F, int NT>
struct WmStages {
  static constexpr int kBudget = 220 * 1024;
  static constexpr int kPair = Fmt<F>::kBoxes * 128 * Fmt<F>::kBoxBytes + 4 * 8 * NT * 128;
  static constexpr int kFit = (kBudget - 2 * 128 * 8 * NT * 4) / kPair;
  static constexpr int ST = kFit > 8 ? 8 : kFit;
  static_assert(ST >= 2, "shared-memory budget");
};

template <int F, int NT>
cudaError_t run_warp_mma(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x, const Args& a,
                         cudaStream_t st) {
  constexpr int ST = WmStages<F, NT>::ST;
  using C = WmCfg<F, NT, ST>;
  static_assert(C::kSmem <= 227 * 1024, "shared memory budget");
  auto kern = expert_warp_mma_kernel<F, NT, ST>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  kern<<<num_sms(), kWmThreads, C::kSmem, st>>>(w0, w1, x, a);
  return cudaGetLastError();
}

template <int F, int NT, bool kXSum = false, bool kI8 = false>
cudaError_t run_quad_mma(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x, const Args& a,
                         cudaStream_t st) {
  constexpr int ST = WmStages<F, NT>::ST;
  using C = WmCfg<F, NT, ST>;
  static_assert(C::kSmem <= 227 * 1024, "shared memory budget");
  auto kern = expert_quad_mma_kernel<F, NT, ST, kXSum, kI8>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  kern<<<num_sms(), kWmThreads, C::kSmem, st>>>(w0, w1, x, a);
  return cudaGetLastError();
}

template <int F>
cudaError_t dispatch_quad(int bn, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
                          const Args& a, cudaStream_t st) {
  if constexpr (F == kQ4_K) {
    if (a.xscale) return bn == 8 && a.xsum ? run_quad_mma<F, 1, true, true>(w0, w1, x, a, st) : cudaErrorInvalidValue;
    if (a.xsum) {
      switch (bn) {
        case 8: return run_quad_mma<F, 1, true>(w0, w1, x, a, st);
        case 16: return run_quad_mma<F, 2, true>(w0, w1, x, a, st);
        default: return cudaErrorInvalidValue;
      }
    }
  }
  switch (bn) {
    case 8: return run_quad_mma<F, 1>(w0, w1, x, a, st);
    case 16: return run_quad_mma<F, 2>(w0, w1, x, a, st);
    default: return cudaErrorInvalidValue;
  }
}

template <int F>
cudaError_t dispatch_warp(int bn, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
                          const Args& a, cudaStream_t st) {
  switch (bn) {
    case 8: return run_warp_mma<F, 1>(w0, w1, x, a, st);
    case 16: return run_warp_mma<F, 2>(w0, w1, x, a, st);
    default: return cudaErrorInvalidValue;
  }
}

// K granularity a row of this format must have (64 or 256), 0 if unsupported.
int min_k(int fmt) {
  switch (fmt) {
    case kQ4_0: return Fmt<kQ4_0>::kMinK;
    case kQ8_0: return Fmt<kQ8_0>::kMinK;
    case kQ4_K: return Fmt<kQ4_K>::kMinK;
    case kQ6_K: return Fmt<kQ6_K>::kMinK;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int F>
bool make_weight_maps(CUtensorMap* m0, CUtensorMap* m1, const void* W0, const void* W1, int64_t pitch,
                      int64_t rows_total) {
  return make_weight_map(m0, W0, pitch, rows_total, Fmt<F>::kBoxBytes) &&
         make_weight_map(m1, W1, pitch, rows_total, Fmt<F>::kBoxBytes);
}

// sched: kSchedWarpMma, the mma.sync schedule (slot tiles of 8 or 16, K % 128 == 0,
// operand rows in wm_kpos order); kSchedQuadMma, mma.sync over whole K-quant
// super-blocks (slot tiles of 8 or 16, Q4_K / Q6_K, operand rows in q4k_kpos /
// q6k_kpos order); else tcgen05 (slot tiles 16..256, tc_kpos order).  h_order: the
// order the quad schedule's gate/up epilogue writes h in.
cudaError_t launch_common(int sched, int fmt, bool gateup, const void* W0, const void* W1, int64_t pitch,
                          int64_t E, int64_t rows, int64_t K, const void* act16, int64_t S_rows,
                          const int32_t* counts, const int32_t* offsets, int32_t* tile_base, int bn, int splits,
                          void* h16, float* out, int64_t out_ld, int64_t split_stride, int* err, cudaStream_t st,
                          int h_order, bool table_ready, const void* xsum, const TailSplit* tail,
                          const float* xscale) {
  const int mk = min_k(fmt);
  const bool warp_mma = sched == kSchedWarpMma, quad = sched == kSchedQuadMma;
  if (!mk || K % mk != 0 || K <= 0) return cudaErrorNotSupported;
  if ((warp_mma || quad) && (K % 128 != 0 || (bn != 8 && bn != 16))) return cudaErrorNotSupported;
  if (quad && fmt != kQ4_K && fmt != kQ6_K) return cudaErrorNotSupported;
  const int m_rows = gateup ? 64 : 128;
  if (rows % m_rows != 0 || pitch % 16 != 0 || pitch < fmt_row_bytes(fmt, K)) return cudaErrorNotSupported;
  if (!aligned16(W0) || !aligned16(W1) || !aligned16(act16) || K % 8 != 0) return cudaErrorNotSupported;
  const int kquads = (int)((K + kQuadK - 1) / kQuadK);
  if (splits < 1) splits = 1;
  if (splits > kquads) splits = kquads;
  CUtensorMap m0, m1, mx;
  bool maps = make_act_map(&mx, act16, K, S_rows, bn);
  switch (fmt) {
    case kQ4_0: maps = maps && make_weight_maps<kQ4_0>(&m0, &m1, W0, W1, pitch, E * rows); break;
    case kQ8_0: maps = maps && make_weight_maps<kQ8_0>(&m0, &m1, W0, W1, pitch, E * rows); break;
    case kQ4_K: maps = maps && make_weight_maps<kQ4_K>(&m0, &m1, W0, W1, pitch, E * rows); break;
    default: maps = maps && make_weight_maps<kQ6_K>(&m0, &m1, W0, W1, pitch, E * rows); break;
  }
  if (!maps) return cudaErrorNotSupported;
  const int m_tiles = (int)(rows / m_rows);
  if (!table_ready) {
    tile_table_kernel<<<1, 32, 0, st>>>(counts, (int)E, bn, m_tiles, splits, tile_base);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  Args a{};
  a.counts = counts;
  a.offsets = offsets;
  a.tile_base = tile_base;
  a.E = (int)E;
  a.m_tiles = m_tiles;
  a.splits = splits;
  a.kquads = kquads;
  a.k_atoms = (int)(K / 64);
  a.rows_per_expert = (int)rows;
  a.gateup = gateup ? 1 : 0;
  a.band_m = gateup ? kBandM : kDownBandM;
  a.h_out = static_cast<__half*>(h16);
  a.h_order = h_order;
  a.xsum = quad && fmt == kQ4_K ? static_cast<const __half*>(xsum) : nullptr;
  a.xscale = quad && fmt == kQ4_K && gateup ? xscale : nullptr;
  if (xscale != nullptr && a.xscale == nullptr) return cudaErrorInvalidValue;
  a.S_rows = S_rows;
  if (quad && gateup && tail != nullptr && tail->part != nullptr && tail->cnt != nullptr && bn <= kTailMaxBn &&
      num_sms() <= kTailMaxUnits) {
    a.tail_part = tail->part;
    a.tail_cnt = tail->cnt;
  }
  if (quad && !gateup && tail != nullptr && tail->part != nullptr && tail->cnt != nullptr && splits == 1 &&
      bn <= kTailMaxBn && 2 * num_sms() * bn <= kTailMaxUnits * kTailMaxBn && num_sms() <= kTailMaxUnits) {
    a.tail_part = tail->part;
    a.tail_cnt = tail->cnt;
    a.ranges = 1;
  }
  a.out = out;
  a.out_ld = out_ld;
  a.split_stride = split_stride;
  a.err = err;
  if (quad) return fmt == kQ4_K ? dispatch_quad<kQ4_K>(bn, m0, m1, mx, a, st)
                                : dispatch_quad<kQ6_K>(bn, m0, m1, mx, a, st);
  if (warp_mma) {
    switch (fmt) {
      case kQ4_0: return dispatch_warp<kQ4_0>(bn, m0, m1, mx, a, st);
      case kQ8_0: return dispatch_warp<kQ8_0>(bn, m0, m1, mx, a, st);
      case kQ4_K: return dispatch_warp<kQ4_K>(bn, m0, m1, mx, a, st);
      case kQ6_K: return dispatch_warp<kQ6_K>(bn, m0, m1, mx, a, st);
      default: return cudaErrorNotSupported;
    }
  }
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

bool umma_format_supported(int fmt) { return min_k(fmt) != 0; }

bool umma_shapes_supported(int gfmt, int dfmt, int64_t D, int64_t I) {
  if (!umma_format_supported(gfmt) || !umma_format_supported(dfmt)) return false;
  if (D % min_k(gfmt) || I % min_k(dfmt) || I % 64 || D % 128) return false;
  return D % 8 == 0 && I % 8 == 0;
}

int64_t umma_pitch(int fmt, int64_t K) { return (fmt_row_bytes(fmt, K) + 15) / 16 * 16; }

bool umma_down_supported(int fmt, int64_t N, int64_t K, bool warp_mma) {
  const int mk = min_k(fmt);
  return mk != 0 && K % mk == 0 && K % 64 == 0 && N % 128 == 0 && (!warp_mma || K % 128 == 0);
}

bool warp_mma_shapes_supported(int gfmt, int dfmt, int64_t D, int64_t I) {
  return umma_shapes_supported(gfmt, dfmt, D, I) && D % 128 == 0 && I % 128 == 0;
}

cudaError_t launch_gateup_umma(int fmt, const void* G, const void* U, int64_t pitch, int64_t E, int64_t I, int64_t D,
                               const void* xp16, int64_t S_rows, const int32_t* counts, const int32_t* offsets,
                               int32_t* tile_base, int bn, void* h16, int* err, cudaStream_t st, int sched,
                               int h_order, bool table_ready, const void* xsum, const TailSplit* tail,
                               const float* xscale) {
  return launch_common(sched, fmt, true, G, U, pitch, E, I, D, xp16, S_rows, counts, offsets, tile_base, bn, 1,
                       h16, nullptr, I, 0, err, st, h_order, table_ready, xsum, tail, xscale);
}

cudaError_t launch_down_umma(int fmt, const void* Dn, int64_t pitch, int64_t E, int64_t D, int64_t I, const void* h16,
                             int64_t S_rows, const int32_t* counts, const int32_t* offsets, int32_t* tile_base,
                             int bn, int splits, float* out, int* err, cudaStream_t st, int sched,
                             bool table_ready, const TailSplit* ranges) {
  return launch_common(sched, fmt, false, Dn, Dn, pitch, E, D, I, h16, S_rows, counts, offsets, tile_base, bn,
                       splits, nullptr, out, D, S_rows * D, err, st, kOrderTc, table_ready, nullptr, ranges,
                       nullptr);
}

namespace {
// One thread per 16-bit unit of the padded destination (row bytes are even for every GGUF format).
__global__ void pad_rows_kernel(const uint16_t* __restrict__ src, int64_t src_pitch2, int64_t rows, int64_t row2,
                                uint16_t* __restrict__ dst, int64_t dst_pitch2) {
  const int64_t n = rows * dst_pitch2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / dst_pitch2, c = i - r * dst_pitch2;
    dst[i] = c < row2 ? src[r * src_pitch2 + c] : (uint16_t)0;
  }
}
}  // namespace

cudaError_t launch_pad_rows(const void* src, int64_t src_pitch, int64_t rows, int64_t row_bytes, void* dst,
                            int64_t dst_pitch, cudaStream_t st) {
  if ((src_pitch | row_bytes | dst_pitch) & 1 || (reinterpret_cast<uintptr_t>(src) & 1) || dst_pitch % 16 ||
      row_bytes > dst_pitch || row_bytes > src_pitch)
    return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int64_t n = rows * (dst_pitch / 2);
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  pad_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const uint16_t*>(src), src_pitch / 2, rows,
                                                     row_bytes / 2, static_cast<uint16_t*>(dst), dst_pitch / 2);
  return cudaGetLastError();
}

int umma_kchunks(int fmt, int64_t K) {
  return umma_format_supported(fmt) ? (int)((K + kQuadK - 1) / kQuadK) : 0;
}

}  // namespace uaii_b200
