// gguf_blocks.cuh -- GGUF block layouts on the device, byte-identical to the
// host format, and an exact f32 decoder per 32-element sub-block.
//
// The decoders reproduce the reference arithmetic of
// libs/uaii-quant/src/gguf_dequant.cpp (dequant_gguf_row, :117-439) operation
// for operation, with explicit round-to-nearest intrinsics so that nvcc cannot
// contract a multiply and an add into one fused operation.  Their f32 outputs
// are therefore bitwise equal to the reference's for every finite input.
//
// A "sub-block" is 32 consecutive elements of a row.  For the 32-element
// formats it is one block; for the 256-element K-quant super-blocks it is one
// of the eight 32-element groups.  Element order is the ggml order.
#pragma once

#include <cstdint>

#include "gguf_format.hpp"

namespace uaii_b200 {

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
}

// Exact f16 -> f32 on bits, subnormals normalised, inf/NaN payload kept
// (gguf_dequant.cpp:79-105).  Integer-only, so no conversion mode applies.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t ex = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (ex == 0) {
    if (mant == 0) {
      bits = sign;
    } else {
      const int shift = __clz(mant) - 21;  // moves the leading one to bit 10
      bits = sign | ((uint32_t)(113 - shift) << 23) | (((mant << shift) & 0x3ffu) << 13);
    }
  } else if (ex == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((ex + 112u) << 23) | (mant << 13);
  }
  return __uint_as_float(bits);
}

__device__ __forceinline__ void k4_scale_min(int j, const uint8_t* q, int& sc, int& mn) {
  if (j < 4) {
    sc = q[j] & 63;
    mn = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4);
    mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Decode sub-block `s` (32 elements) of the block starting at `blk`.
// For 32-element formats s must be 0; for K-quants s is 0..7.
template <int F>
__device__ __forceinline__ void decode32(const uint8_t* blk, int s, float* o) {
  if constexpr (F == kQ4_0) {
    const float d = f16_bits_to_f32(ld_u16(blk));
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint8_t b = blk[2 + j];
      o[j] = __fmul_rn((float)((b & 15) - 8), d);
      o[j + 16] = __fmul_rn((float)((b >> 4) - 8), d);
    }
  } else if constexpr (F == kQ4_1) {
    const float d = f16_bits_to_f32(ld_u16(blk));
    const float m = f16_bits_to_f32(ld_u16(blk + 2));
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint8_t b = blk[4 + j];
      o[j] = __fadd_rn(__fmul_rn((float)(b & 15), d), m);
      o[j + 16] = __fadd_rn(__fmul_rn((float)(b >> 4), d), m);
    }
  } else if constexpr (F == kQ5_0) {
    const float d = f16_bits_to_f32(ld_u16(blk));
    const uint32_t qh = ld_u16(blk + 2) | (ld_u16(blk + 4) << 16);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint8_t b = blk[6 + j];
      const int h0 = (int)((qh >> j) & 1u) << 4, h1 = (int)((qh >> (j + 16)) & 1u) << 4;
      o[j] = __fmul_rn((float)(((b & 15) | h0) - 16), d);
      o[j + 16] = __fmul_rn((float)(((b >> 4) | h1) - 16), d);
    }
  } else if constexpr (F == kQ5_1) {
    const float d = f16_bits_to_f32(ld_u16(blk));
    const float m = f16_bits_to_f32(ld_u16(blk + 2));
    const uint32_t qh = ld_u16(blk + 4) | (ld_u16(blk + 6) << 16);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint8_t b = blk[8 + j];
      const int h0 = (int)((qh >> j) & 1u) << 4, h1 = (int)((qh >> (j + 16)) & 1u) << 4;
      o[j] = __fadd_rn(__fmul_rn((float)((b & 15) | h0), d), m);
      o[j + 16] = __fadd_rn(__fmul_rn((float)((b >> 4) | h1), d), m);
    }
  } else if constexpr (F == kQ8_0) {
    const float d = f16_bits_to_f32(ld_u16(blk));
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = __fmul_rn((float)(int8_t)blk[2 + j], d);
  } else if constexpr (F == kQ2_K) {
    // {u8 scales[16]; u8 qs[64]; f16 d; f16 dmin}; sub-block s = (half, j)
    const int half = s >> 2, j = s & 3;
    const float d = f16_bits_to_f32(ld_u16(blk + 80));
    const float mn = f16_bits_to_f32(ld_u16(blk + 82));
    const uint8_t* q = blk + 16 + 32 * half;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const uint8_t sc = blk[8 * half + 2 * j + part];
      const float dl = __fmul_rn(d, (float)(sc & 15));
      const float ml = __fmul_rn(mn, (float)(sc >> 4));
#pragma unroll
      for (int l = 0; l < 16; ++l) {
        const int v = (q[16 * part + l] >> (2 * j)) & 3;
        o[16 * part + l] = __fsub_rn(__fmul_rn(dl, (float)v), ml);
      }
    }
  } else if constexpr (F == kQ3_K) {
    // {u8 hmask[32]; u8 qs[64]; u8 scales[12]; f16 d}
    const int half = s >> 2, j = s & 3;
    const float dall = f16_bits_to_f32(ld_u16(blk + 108));
    const uint8_t* s12 = blk + 96;
    const uint8_t mbit = (uint8_t)(1u << (4 * half + j));
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const int i = 8 * half + 2 * j + part;
      const int lo = (i < 8) ? (s12[i] & 15) : (s12[i - 8] >> 4);
      const int hi = (s12[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
      const float dl = __fmul_rn(dall, (float)((lo | (hi << 4)) - 32));
#pragma unroll
      for (int l = 0; l < 16; ++l) {
        const int idx = 16 * part + l;
        const int v = ((blk[32 + 32 * half + idx] >> (2 * j)) & 3) - ((blk[idx] & mbit) ? 0 : 4);
        o[idx] = __fmul_rn(dl, (float)v);
      }
    }
  } else if constexpr (F == kQ4_K) {
    // {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]}; sub-block s = (group g, high half)
    const int g = s >> 1, hiq = s & 1;
    const float d = f16_bits_to_f32(ld_u16(blk));
    const float mn = f16_bits_to_f32(ld_u16(blk + 2));
    int sc, m;
    k4_scale_min(s, blk + 4, sc, m);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(mn, (float)m);
    const uint8_t* q = blk + 16 + 32 * g;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int v = hiq ? (q[l] >> 4) : (q[l] & 15);
      o[l] = __fsub_rn(__fmul_rn(d1, (float)v), m1);
    }
  } else if constexpr (F == kQ5_K) {
    // {f16 d; f16 dmin; u8 scales[12]; u8 qh[32]; u8 qs[128]}
    const int g = s >> 1, hiq = s & 1;
    const float d = f16_bits_to_f32(ld_u16(blk));
    const float mn = f16_bits_to_f32(ld_u16(blk + 2));
    int sc, m;
    k4_scale_min(s, blk + 4, sc, m);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(mn, (float)m);
    const uint8_t* qh = blk + 16;
    const uint8_t* q = blk + 48 + 32 * g;
    const uint8_t u = (uint8_t)((hiq ? 2u : 1u) << (2 * g));
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int v = (hiq ? (q[l] >> 4) : (q[l] & 15)) + ((qh[l] & u) ? 16 : 0);
      o[l] = __fsub_rn(__fmul_rn(d1, (float)v), m1);
    }
  } else if constexpr (F == kQ6_K) {
    // {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d}; sub-block s = (half, quarter)
    const int half = s >> 2, qt = s & 3;
    const float d = f16_bits_to_f32(ld_u16(blk + 208));
    const uint8_t* ql = blk + 64 * half + ((qt & 1) ? 32 : 0);
    const uint8_t* qh = blk + 128 + 32 * half;
    const int8_t* sc = (const int8_t*)(blk + 192 + 8 * half);
    const int nshift = (qt >> 1) ? 4 : 0;  // quarters 2,3 use the high nibbles
    const int hshift = 2 * qt;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int v = (((ql[l] >> nshift) & 15) | (((qh[l] >> hshift) & 3) << 4)) - 32;
      o[l] = __fmul_rn(__fmul_rn(d, (float)sc[(l >> 4) + 2 * qt]), (float)v);
    }
  } else if constexpr (F == kF16) {
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = f16_bits_to_f32(ld_u16(blk + 2 * j));
  } else if constexpr (F == kF32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = reinterpret_cast<const float*>(blk)[j];
  }
}

// Address of the block that holds sub-block `sb` (32-element index along the
// row) and the sub-block number inside it.
template <int F>
__device__ __forceinline__ const uint8_t* subblock_ptr(const uint8_t* row, int sb, int& s) {
  if constexpr (F == kF32) { s = 0; return row + (size_t)sb * 128; }
  else if constexpr (F == kF16) { s = 0; return row + (size_t)sb * 64; }
  else if constexpr (fmt_block_elems(F) == 256) {
    s = sb & 7;
    return row + (size_t)(sb >> 3) * fmt_block_bytes(F);
  } else {
    s = 0;
    return row + (size_t)sb * fmt_block_bytes(F);
  }
}

}  // namespace uaii_b200
