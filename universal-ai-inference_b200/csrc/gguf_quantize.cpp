// gguf_quantize.cpp -- synthetic-input utilities: a GGUF block quantizer and a
// counter-based normal generator.  The reference has no GGUF block quantizer
// (its codec returns NotImplemented for Q* packing, libs/uaii-quant/src/codec.cpp:81-179),
// so seeded synthetic weights are produced here.  Any deterministic scheme is
// valid because parity is checked on the packed bytes themselves; this one is
// round-to-nearest with per-block max-abs (and, for Q4_K, min) scales.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/uaii_moe.h"
#include "gguf_format.hpp"

namespace uaii_b200 {
namespace {

uint32_t fbits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

// f32 -> f16 bits, round to nearest even, overflow to inf.
uint16_t f32_to_f16(float f) {
  const uint32_t x = fbits(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (ax < 0x38800000u) {  // below the smallest f16 normal: multiples of 2^-24
    const float v = std::fabs(f) * 16777216.0f;
    return (uint16_t)(sign | (uint32_t)std::nearbyint(v));
  }
  uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13);
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t ex = (h >> 10) & 0x1fu, mant = h & 0x3ffu, bits;
  if (ex == 0) {
    if (mant == 0) bits = sign;
    else {
      uint32_t e = 113;
      while ((mant & 0x400u) == 0) { mant <<= 1; --e; }
      bits = sign | (e << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (ex == 31) bits = sign | 0x7f800000u | (mant << 13);
  else bits = sign | ((ex + 112u) << 23) | (mant << 13);
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

void put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)(v & 0xff); p[1] = (uint8_t)(v >> 8); }
int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
int rnd(float v) { return (int)std::nearbyint(v); }

// value of largest magnitude (first on ties), keeping its sign
float signed_absmax(const float* x, int n) {
  float best = 0.f;
  for (int i = 0; i < n; ++i) if (std::fabs(x[i]) > std::fabs(best)) best = x[i];
  return best;
}

void q4_0_block(const float* x, uint8_t* b) {
  const float mx = signed_absmax(x, 32);
  const uint16_t dh = f32_to_f16(mx / -8.0f);
  const float d = f16_to_f32(dh);
  const float id = d != 0.f ? 1.0f / d : 0.f;
  put16(b, dh);
  for (int j = 0; j < 16; ++j) {
    const int q0 = clampi(rnd(x[j] * id) + 8, 0, 15);
    const int q1 = clampi(rnd(x[j + 16] * id) + 8, 0, 15);
    b[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}

void q8_0_block(const float* x, uint8_t* b) {
  const float amax = std::fabs(signed_absmax(x, 32));
  const uint16_t dh = f32_to_f16(amax / 127.0f);
  const float d = f16_to_f32(dh);
  const float id = d != 0.f ? 1.0f / d : 0.f;
  put16(b, dh);
  for (int j = 0; j < 32; ++j) b[2 + j] = (uint8_t)(int8_t)clampi(rnd(x[j] * id), -127, 127);
}

void q4_k_block(const float* x, uint8_t* b) {
  float scale[8], negmin[8];
  for (int g = 0; g < 8; ++g) {
    float lo = 0.f, hi = x[32 * g];
    for (int l = 0; l < 32; ++l) { lo = std::min(lo, x[32 * g + l]); hi = std::max(hi, x[32 * g + l]); }
    hi = std::max(hi, lo);
    scale[g] = (hi - lo) / 15.0f;
    negmin[g] = -lo;
  }
  const float smax = *std::max_element(scale, scale + 8);
  const float mmax = *std::max_element(negmin, negmin + 8);
  const uint16_t dh = f32_to_f16(smax / 63.0f), mh = f32_to_f16(mmax / 63.0f);
  const float d = f16_to_f32(dh), dm = f16_to_f32(mh);
  int sc[8], mn[8];
  for (int g = 0; g < 8; ++g) {
    sc[g] = d > 0.f ? clampi(rnd(scale[g] / d), 0, 63) : 0;
    mn[g] = dm > 0.f ? clampi(rnd(negmin[g] / dm), 0, 63) : 0;
  }
  put16(b, dh);
  put16(b + 2, mh);
  uint8_t* s12 = b + 4;
  for (int j = 0; j < 4; ++j) {
    s12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s12[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    s12[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
  }
  uint8_t q[256];
  for (int g = 0; g < 8; ++g) {
    const float ed = d * (float)sc[g], em = dm * (float)mn[g];
    for (int l = 0; l < 32; ++l)
      q[32 * g + l] = (uint8_t)(ed > 0.f ? clampi(rnd((x[32 * g + l] + em) / ed), 0, 15) : 0);
  }
  for (int c = 0; c < 4; ++c)
    for (int l = 0; l < 32; ++l) b[16 + 32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

void q6_k_block(const float* x, uint8_t* b) {
  float scale[16];
  float smax = 0.f;
  for (int j = 0; j < 16; ++j) {
    scale[j] = signed_absmax(x + 16 * j, 16) / -32.0f;
    smax = std::max(smax, std::fabs(scale[j]));
  }
  const uint16_t dh = f32_to_f16(smax / 127.0f);
  const float d = f16_to_f32(dh);
  int sc[16];
  uint8_t q[256];
  for (int j = 0; j < 16; ++j) {
    sc[j] = d > 0.f ? clampi(rnd(scale[j] / d), -128, 127) : 0;
    const float e = d * (float)sc[j];
    for (int l = 0; l < 16; ++l)
      q[16 * j + l] = (uint8_t)(e != 0.f ? clampi(rnd(x[16 * j + l] / e) + 32, 0, 63) : 32);
  }
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  for (int half = 0; half < 2; ++half) {
    for (int l = 0; l < 32; ++l) {
      const int q1 = q[128 * half + l], q2 = q[128 * half + 32 + l];
      const int q3 = q[128 * half + 64 + l], q4 = q[128 * half + 96 + l];
      ql[64 * half + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
      ql[64 * half + 32 + l] = (uint8_t)((q2 & 15) | ((q4 & 15) << 4));
      qh[32 * half + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  for (int j = 0; j < 16; ++j) b[192 + j] = (uint8_t)(int8_t)sc[j];
  put16(b + 208, dh);
}

template <class F>
void parallel_chunks(int64_t n, int64_t chunk, F fn) {
  const int64_t nchunks = (n + chunk - 1) / chunk;
  unsigned hw = std::thread::hardware_concurrency();
  int64_t nt = std::min<int64_t>(nchunks, hw == 0 ? 1 : std::min(hw, 32u));
  if (nt <= 1) { for (int64_t c = 0; c < nchunks; ++c) fn(c); return; }
  std::vector<std::thread> pool;
  for (int64_t t = 0; t < nt; ++t)
    pool.emplace_back([=]() { for (int64_t c = t; c < nchunks; c += nt) fn(c); });
  for (auto& th : pool) th.join();
}

uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace
}  // namespace uaii_b200

extern "C" int uaii_moe_quantize_rows(int fmt, const float* src, int64_t rows, int64_t cols,
                                      void* dst) {
  using namespace uaii_b200;
  if (!src || !dst || rows < 0 || cols <= 0) return UAII_MOE_INVALID_ARGUMENT;
  const int qk = fmt_block_elems(fmt);
  if (!(fmt == kQ4_0 || fmt == kQ8_0 || fmt == kQ4_K || fmt == kQ6_K)) return UAII_MOE_NOT_IMPLEMENTED;
  if (cols % qk != 0) return UAII_MOE_INVALID_ARGUMENT;
  const int64_t pitch = fmt_row_bytes(fmt, cols);
  const int64_t nb = cols / qk;
  uint8_t* out = static_cast<uint8_t*>(dst);
  parallel_chunks(rows, 64, [&](int64_t c) {
    const int64_t r1 = std::min(rows, (c + 1) * 64);
    for (int64_t r = c * 64; r < r1; ++r) {
      for (int64_t b = 0; b < nb; ++b) {
        const float* x = src + r * cols + b * qk;
        uint8_t* blk = out + r * pitch + b * fmt_block_bytes(fmt);
        switch (fmt) {
          case kQ4_0: q4_0_block(x, blk); break;
          case kQ8_0: q8_0_block(x, blk); break;
          case kQ4_K: q4_k_block(x, blk); break;
          default: q6_k_block(x, blk); break;
        }
      }
    }
  });
  return UAII_MOE_OK;
}

extern "C" int uaii_moe_fill_normal(float* out, int64_t n, uint64_t seed, uint64_t stream,
                                    float mean, float std) {
  using namespace uaii_b200;
  if (!out || n < 0) return UAII_MOE_INVALID_ARGUMENT;
  const uint64_t key = mix64(seed ^ mix64(stream * 0xD1B54A32D192ED03ull + 0x7F4A7C15ull));
  const double two_pi = 6.283185307179586476925286766559;
  parallel_chunks(n, 1 << 20, [&](int64_t c) {
    const int64_t i1 = std::min(n, (c + 1) << 20);
    for (int64_t i = c << 20; i < i1; ++i) {
      const uint64_t p = (uint64_t)(i >> 1);
      const uint64_t a = mix64(key + 2 * p), b = mix64(key + 2 * p + 1);
      const double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
      const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double z = (i & 1) ? r * std::sin(two_pi * u2) : r * std::cos(two_pi * u2);
      out[i] = (float)((double)mean + (double)std * z);
    }
  });
  return UAII_MOE_OK;
}

extern "C" uint64_t uaii_moe_packed_nbytes(int fmt, int64_t n) {
  using namespace uaii_b200;
  if (fmt == kF32) return (uint64_t)n * 4;
  if (fmt == kF16 || fmt == kBF16) return (uint64_t)n * 2;
  if (!fmt_is_gguf(fmt)) return 0;
  return (uint64_t)fmt_row_bytes(fmt, n);
}
