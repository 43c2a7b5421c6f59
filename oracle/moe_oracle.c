/*
 * moe_oracle.c -- CPU restatement of the UAII GGUF mixture-of-experts FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path: it is
 * loaded by tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline
 * leg, and by nothing else.  The product library never links, loads or calls
 * it, and it must never be used as a fallback for the device path.
 *
 * Parity is pinned: tests/test_oracle.py checks every function here against
 * the reference's own compiled code (oracle/_ref, built from the reference
 * sources by oracle/Makefile) and against the committed golden fixtures under
 * tests/golden/, which were produced by that same reference build.
 *
 * Every function follows the reference arithmetic order exactly (plain f32
 * multiply then add, no fused multiply-add; build with -ffp-contract=off).
 * Citations are paths inside the reference project (arjun988/Universal-AI-Inference).
 *
 * Format codes are the values of uaii::quant::QuantFormat
 * (include/uaii/quant/formats.hpp:10-29): F32=0, F16=1, ..., Q4_0=7, Q4_1=8,
 * Q5_0=9, Q5_1=10, Q8_0=11, Q2_K=12, Q3_K=13, Q4_K=14, Q5_K=15, Q6_K=16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum {
  UO_F32 = 0, UO_F16 = 1, UO_BF16 = 2,
  UO_Q4_0 = 7, UO_Q4_1 = 8, UO_Q5_0 = 9, UO_Q5_1 = 10, UO_Q8_0 = 11,
  UO_Q2_K = 12, UO_Q3_K = 13, UO_Q4_K = 14, UO_Q5_K = 15, UO_Q6_K = 16,
};

/* Status codes mirror uaii::ErrorCode (include/uaii/core/error.hpp:12-22). */
enum { UO_OK = 0, UO_INVALID_ARGUMENT = 1, UO_NOT_IMPLEMENTED = 7 };

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Exact f16 -> f32 including subnormals, inf and NaN payloads
 * (libs/uaii-quant/src/gguf_dequant.cpp:79-105). */
float uo_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
  uint32_t ex = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (ex == 0) {
    if (mant == 0) {
      bits = sign;
    } else {
      /* normalise: shift the mantissa up until its leading one reaches bit 10 */
      uint32_t e = 113; /* 127 - 15 + 1 */
      while ((mant & 0x400u) == 0) { mant <<= 1; --e; }
      bits = sign | (e << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (ex == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((ex + 112u) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Bytes per row of n elements (include/uaii/quant/formats.hpp:81-102). */
size_t uo_packed_nbytes(int fmt, int64_t n) {
  switch (fmt) {
    case UO_F32: return (size_t)n * 4;
    case UO_F16: case UO_BF16: return (size_t)n * 2;
    case UO_Q4_0: return (size_t)(n / 32) * 18;
    case UO_Q4_1: return (size_t)(n / 32) * 20;
    case UO_Q5_0: return (size_t)(n / 32) * 22;
    case UO_Q5_1: return (size_t)(n / 32) * 24;
    case UO_Q8_0: return (size_t)(n / 32) * 34;
    case UO_Q2_K: return (size_t)(n / 256) * 84;
    case UO_Q3_K: return (size_t)(n / 256) * 110;
    case UO_Q4_K: return (size_t)(n / 256) * 144;
    case UO_Q5_K: return (size_t)(n / 256) * 176;
    case UO_Q6_K: return (size_t)(n / 256) * 210;
    default: return 0;
  }
}

/* 6-bit (scale, min) pair j of a Q4_K/Q5_K super-block
 * (libs/uaii-quant/src/gguf_dequant.cpp:107-115). */
static void scale_min_k4(int j, const uint8_t* q, int* sc, int* mn) {
  if (j < 4) {
    *sc = q[j] & 63;
    *mn = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
    *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

/* One GGUF row -> f32 in ggml element order
 * (libs/uaii-quant/src/gguf_dequant.cpp:117-439). */
int uo_dequant_row(int fmt, const uint8_t* p, int64_t cols, float* y) {
  if (!p || !y) return UO_INVALID_ARGUMENT;
  if (fmt == UO_F32) { memcpy(y, p, (size_t)cols * 4); return UO_OK; }
  if (fmt == UO_F16) {
    for (int64_t i = 0; i < cols; ++i) y[i] = uo_f16_to_f32(rd16(p + 2 * i));
    return UO_OK;
  }
  const int is_k = fmt >= UO_Q2_K && fmt <= UO_Q6_K;
  const int64_t qk = is_k ? 256 : 32;
  if (fmt < UO_Q4_0 || fmt > UO_Q6_K) return UO_NOT_IMPLEMENTED;
  if (cols % qk != 0) return UO_INVALID_ARGUMENT;
  const int64_t nb = cols / qk;
  const size_t bsz = uo_packed_nbytes(fmt, qk);
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = p + (size_t)b * bsz;
    float* o = y + b * qk;
    switch (fmt) {
      case UO_Q4_0: { /* :117-134  {f16 d; u8 qs[16]} lo nibble -> j, hi -> j+16 */
        const float d = uo_f16_to_f32(rd16(blk));
        for (int j = 0; j < 16; ++j) {
          o[j] = (float)((blk[2 + j] & 15) - 8) * d;
          o[j + 16] = (float)((blk[2 + j] >> 4) - 8) * d;
        }
      } break;
      case UO_Q4_1: { /* :136-154  {f16 d, m; u8 qs[16]} */
        const float d = uo_f16_to_f32(rd16(blk));
        const float m = uo_f16_to_f32(rd16(blk + 2));
        for (int j = 0; j < 16; ++j) {
          o[j] = (float)(blk[4 + j] & 15) * d + m;
          o[j + 16] = (float)(blk[4 + j] >> 4) * d + m;
        }
      } break;
      case UO_Q5_0: { /* :156-177  {f16 d; u8 qh[4]; u8 qs[16]} */
        const float d = uo_f16_to_f32(rd16(blk));
        uint32_t qh;
        memcpy(&qh, blk + 2, 4);
        for (int j = 0; j < 16; ++j) {
          const int hb0 = (int)((qh >> j) & 1u) << 4;
          const int hb1 = (int)((qh >> (j + 16)) & 1u) << 4;
          o[j] = (float)(((blk[6 + j] & 15) | hb0) - 16) * d;
          o[j + 16] = (float)(((blk[6 + j] >> 4) | hb1) - 16) * d;
        }
      } break;
      case UO_Q5_1: { /* :179-201  {f16 d, m; u8 qh[4]; u8 qs[16]} */
        const float d = uo_f16_to_f32(rd16(blk));
        const float m = uo_f16_to_f32(rd16(blk + 2));
        uint32_t qh;
        memcpy(&qh, blk + 4, 4);
        for (int j = 0; j < 16; ++j) {
          const int hb0 = (int)((qh >> j) & 1u) << 4;
          const int hb1 = (int)((qh >> (j + 16)) & 1u) << 4;
          o[j] = (float)((blk[8 + j] & 15) | hb0) * d + m;
          o[j + 16] = (float)((blk[8 + j] >> 4) | hb1) * d + m;
        }
      } break;
      case UO_Q8_0: { /* :203-217  {f16 d; i8 qs[32]} */
        const float d = uo_f16_to_f32(rd16(blk));
        for (int j = 0; j < 32; ++j) o[j] = (float)(int8_t)blk[2 + j] * d;
      } break;
      case UO_Q2_K: { /* :219-253  {u8 scales[16]; u8 qs[64]; f16 d, dmin} */
        const uint8_t* sc = blk;
        const uint8_t* q = blk + 16;
        const float d = uo_f16_to_f32(rd16(blk + 80));
        const float mn = uo_f16_to_f32(rd16(blk + 82));
        for (int half = 0; half < 2; ++half) {
          for (int j = 0; j < 4; ++j) {
            for (int part = 0; part < 2; ++part) {
              const uint8_t s = sc[8 * half + 2 * j + part];
              const float dl = d * (float)(s & 15);
              const float ml = mn * (float)(s >> 4);
              for (int l = 0; l < 16; ++l) {
                const int v = (q[32 * half + 16 * part + l] >> (2 * j)) & 3;
                o[128 * half + 32 * j + 16 * part + l] = dl * (float)v - ml;
              }
            }
          }
        }
      } break;
      case UO_Q3_K: { /* :255-306  {u8 hmask[32]; u8 qs[64]; u8 scales[12]; f16 d} */
        const uint8_t* hm = blk;
        const uint8_t* q = blk + 32;
        const uint8_t* s12 = blk + 96;
        const float dall = uo_f16_to_f32(rd16(blk + 108));
        int scl[16];
        for (int i = 0; i < 16; ++i) {
          /* low 4 bits: nibble i of bytes 0..7; high 2 bits: 2-bit field of bytes 8..11 */
          const int lo = (i < 8) ? (s12[i] & 15) : (s12[i - 8] >> 4);
          const int hi = (s12[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
          scl[i] = (lo | (hi << 4)) - 32;
        }
        for (int half = 0; half < 2; ++half) {
          for (int j = 0; j < 4; ++j) {
            const uint8_t mbit = (uint8_t)(1u << (4 * half + j));
            for (int part = 0; part < 2; ++part) {
              const float dl = dall * (float)scl[8 * half + 2 * j + part];
              for (int l = 0; l < 16; ++l) {
                const int idx = 16 * part + l;
                const int v = ((q[32 * half + idx] >> (2 * j)) & 3) - ((hm[idx] & mbit) ? 0 : 4);
                o[128 * half + 32 * j + idx] = dl * (float)v;
              }
            }
          }
        }
      } break;
      case UO_Q4_K: { /* :308-340  {f16 d, dmin; u8 scales[12]; u8 qs[128]} */
        const float d = uo_f16_to_f32(rd16(blk));
        const float mn = uo_f16_to_f32(rd16(blk + 2));
        const uint8_t* s12 = blk + 4;
        const uint8_t* q = blk + 16;
        for (int g = 0; g < 4; ++g) {
          int sc, m;
          scale_min_k4(2 * g, s12, &sc, &m);
          const float d1 = d * (float)sc, m1 = mn * (float)m;
          scale_min_k4(2 * g + 1, s12, &sc, &m);
          const float d2 = d * (float)sc, m2 = mn * (float)m;
          for (int l = 0; l < 32; ++l) o[64 * g + l] = d1 * (float)(q[32 * g + l] & 15) - m1;
          for (int l = 0; l < 32; ++l) o[64 * g + 32 + l] = d2 * (float)(q[32 * g + l] >> 4) - m2;
        }
      } break;
      case UO_Q5_K: { /* :342-379  {f16 d, dmin; u8 scales[12]; u8 qh[32]; u8 qs[128]} */
        const float d = uo_f16_to_f32(rd16(blk));
        const float mn = uo_f16_to_f32(rd16(blk + 2));
        const uint8_t* s12 = blk + 4;
        const uint8_t* qh = blk + 16;
        const uint8_t* q = blk + 48;
        for (int g = 0; g < 4; ++g) {
          int sc, m;
          scale_min_k4(2 * g, s12, &sc, &m);
          const float d1 = d * (float)sc, m1 = mn * (float)m;
          scale_min_k4(2 * g + 1, s12, &sc, &m);
          const float d2 = d * (float)sc, m2 = mn * (float)m;
          const uint8_t u1 = (uint8_t)(1u << (2 * g)), u2 = (uint8_t)(2u << (2 * g));
          for (int l = 0; l < 32; ++l)
            o[64 * g + l] = d1 * (float)((q[32 * g + l] & 15) + ((qh[l] & u1) ? 16 : 0)) - m1;
          for (int l = 0; l < 32; ++l)
            o[64 * g + 32 + l] = d2 * (float)((q[32 * g + l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
        }
      } break;
      case UO_Q6_K: { /* :381-416  {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d} */
        const float d = uo_f16_to_f32(rd16(blk + 208));
        for (int half = 0; half < 2; ++half) {
          const uint8_t* ql = blk + 64 * half;
          const uint8_t* qh = blk + 128 + 32 * half;
          const int8_t* sc = (const int8_t*)(blk + 192 + 8 * half);
          float* oh = o + 128 * half;
          for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q1 = ((ql[l] & 15) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q2 = ((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            oh[l] = d * (float)sc[is] * (float)q1;
            oh[l + 32] = d * (float)sc[is + 2] * (float)q2;
            oh[l + 64] = d * (float)sc[is + 4] * (float)q3;
            oh[l + 96] = d * (float)sc[is + 6] * (float)q4;
          }
        }
      } break;
      default: return UO_NOT_IMPLEMENTED;
    }
  }
  return UO_OK;
}

/* `rows` consecutive rows of `cols` elements, row pitch `pitch` bytes
 * (0 means packed_nbytes(fmt, cols)). */
int uo_dequant_rows(int fmt, const uint8_t* p, int64_t rows, int64_t cols, int64_t pitch,
                    float* y) {
  if (pitch == 0) pitch = (int64_t)uo_packed_nbytes(fmt, cols);
  for (int64_t r = 0; r < rows; ++r) {
    int st = uo_dequant_row(fmt, p + r * pitch, cols, y + r * cols);
    if (st != UO_OK) return st;
  }
  return UO_OK;
}

/* Dense projection with a packed B, restating kernels::quant_gemm_f32
 * (libs/uaii-kernels/src/quant_gemm.cpp:22-70): for every output column j the
 * packed row B[j] is dequantized (dequant_gguf_row), then for every row i
 * c[i][j] = sum over k of a[i][k] * row[k], one rounding per multiply and per
 * add, k ascending from 0.  relu != 0 then maps every value v to v > 0 ? v : 0
 * (MatMulRelu, libs/uaii-kernels/src/dispatch.cpp:82-100). */
int uo_quant_gemm(const float* a, int64_t M, int64_t K, const uint8_t* b, int fmt, int64_t N, int relu, float* c) {
  const int64_t stride = (int64_t)uo_packed_nbytes(fmt, K);
  float* row = (float*)malloc(sizeof(float) * (size_t)K);
  if (!row) return UO_INVALID_ARGUMENT;
  for (int64_t j = 0; j < N; ++j) {
    int st = uo_dequant_row(fmt, b + j * stride, K, row);
    if (st != UO_OK) {
      free(row);
      return st;
    }
    for (int64_t i = 0; i < M; ++i) {
      float sum = 0.0f;
      for (int64_t k = 0; k < K; ++k) sum += a[i * K + k] * row[k];
      c[i * N + j] = (!relu || sum > 0.0f) ? sum : 0.0f; /* relu_f32: x > 0 ? x : 0 (elementwise.cpp:44-52) */
    }
  }
  free(row);
  return UO_OK;
}

/* Router logits in the Ref tiled GEMM order: per element, 64-wide k tiles summed
 * sequentially from 0, and each tile partial added in order to c (initialised 0)
 * (libs/uaii-kernels/src/gemm_ref.cpp:45-75, via matmul.cpp:22-56 with
 * transpose_b=true).  Row tiling does not change per-element arithmetic. */
void uo_router_logits(const float* x, const float* w, int64_t T, int64_t D, int64_t E,
                      float* logits) {
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t e = 0; e < E; ++e) {
      float c = 0.0f;
      for (int64_t k0 = 0; k0 < D; k0 += 64) {
        const int64_t k1 = (k0 + 64 < D) ? k0 + 64 : D;
        float s = 0.0f;
        for (int64_t k = k0; k < k1; ++k) s += x[t * D + k] * w[e * D + k];
        c += 1.0f * s;
      }
      logits[t * E + e] = c;
    }
  }
}

/* Row softmax: max-subtract, expf, sequential sum, multiply by 1/sum
 * (libs/uaii-kernels/src/softmax.cpp:55-75). */
void uo_softmax_rows(const float* in, int64_t T, int64_t E, float* out) {
  for (int64_t t = 0; t < T; ++t) {
    const float* x = in + t * E;
    float* y = out + t * E;
    float mx = -INFINITY;
    for (int64_t e = 0; e < E; ++e) mx = (mx < x[e]) ? x[e] : mx;
    float sum = 0.0f;
    for (int64_t e = 0; e < E; ++e) {
      const float v = expf(x[e] - mx);
      y[e] = v;
      sum += v;
    }
    const float inv = (sum > 0.0f) ? (1.0f / sum) : 0.0f;
    for (int64_t e = 0; e < E; ++e) y[e] *= inv;
  }
}

/* MoERouter: logits -> softmax -> first strict argmax as an f32 id
 * (libs/uaii-kernels/src/transformer.cpp:446-481).  `logits` may be NULL. */
int uo_moe_router(const float* x, const float* w, int64_t T, int64_t D, int64_t E,
                  float* logits, float* probs, float* top) {
  if (!x || !w || !probs || !top || T < 0 || D <= 0 || E <= 0) return UO_INVALID_ARGUMENT;
  float* lg = logits ? logits : (float*)malloc(sizeof(float) * (size_t)(T * E + 1));
  uo_router_logits(x, w, T, D, E, lg);
  uo_softmax_rows(lg, T, E, probs);
  for (int64_t t = 0; t < T; ++t) {
    int best = 0;
    float bp = probs[t * E];
    for (int64_t e = 1; e < E; ++e) {
      if (probs[t * E + e] > bp) { bp = probs[t * E + e]; best = (int)e; }
    }
    top[t] = (float)best;
  }
  if (!logits) free(lg);
  return UO_OK;
}

/* The reference ranks experts with std::partial_sort over (prob, index) pairs
 * and the comparator a.prob > b.prob (transformer.cpp:564-570).  The standard
 * leaves the order of equal probabilities open, so the exact procedure of the
 * reference's toolchain (GNU libstdc++) is restated here: a binary heap over
 * the first k pairs ("greater" on top means the smallest probability sits at
 * the root), each later pair replaces the root only if strictly greater, then
 * the heap is sorted.  With distinct probabilities this is plain "largest k,
 * descending"; with ties it selects and orders exactly as the reference does
 * (pinned in tests/test_oracle.py against the reference build). */
typedef struct { float p; int32_t e; } uo_pair;

static int uo_before(uo_pair a, uo_pair b) { return a.p > b.p; } /* the comparator */

static void uo_push_heap(uo_pair* h, int64_t hole, int64_t top, uo_pair v) {
  int64_t parent = (hole - 1) / 2;
  while (hole > top && uo_before(h[parent], v)) {
    h[hole] = h[parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  h[hole] = v;
}

static void uo_adjust_heap(uo_pair* h, int64_t hole, int64_t len, uo_pair v) {
  const int64_t top = hole;
  int64_t child = hole;
  while (child < (len - 1) / 2) {
    child = 2 * (child + 1);
    if (uo_before(h[child], h[child - 1])) child--;
    h[hole] = h[child];
    hole = child;
  }
  if ((len & 1) == 0 && child == (len - 2) / 2) {
    child = 2 * (child + 1);
    h[hole] = h[child - 1];
    hole = child - 1;
  }
  uo_push_heap(h, hole, top, v);
}

/* ranked[0..E) in index order -> ranked[0..k) = the reference's top-k order */
void uo_partial_sort(uo_pair* a, int64_t E, int k) {
  if (k >= 2) { /* make_heap over [0, k) */
    for (int64_t parent = (k - 2) / 2;; --parent) {
      uo_adjust_heap(a, parent, k, a[parent]);
      if (parent == 0) break;
    }
  }
  for (int64_t i = k; i < E; ++i) { /* heap select */
    if (uo_before(a[i], a[0])) {
      const uo_pair v = a[i];
      a[i] = a[0];
      uo_adjust_heap(a, 0, k, v);
    }
  }
  for (int64_t last = k; last > 1;) { /* sort_heap */
    --last;
    const uo_pair v = a[last];
    a[last] = a[0];
    uo_adjust_heap(a, 0, last, v);
  }
}

/* Top-k of one probability row in the reference's order, then
 * mass = sum of the selected probabilities in rank order (1 if not > 0) and
 * w = p / mass when `norm_topk` (transformer.cpp:571-580); w = p otherwise
 * (no reference counterpart: restatement only). */
void uo_topk_row(const float* p, int64_t E, int k, int norm_topk, int32_t* ids, float* w) {
  uo_pair* a = (uo_pair*)malloc(sizeof(uo_pair) * (size_t)E);
  for (int64_t e = 0; e < E; ++e) { a[e].p = p[e]; a[e].e = (int32_t)e; }
  uo_partial_sort(a, E, k);
  for (int r = 0; r < k; ++r) ids[r] = a[r].e;
  free(a);
  float mass = 0.0f;
  for (int r = 0; r < k; ++r) mass += p[ids[r]];
  if (!(mass > 0.0f)) mass = 1.0f;
  for (int r = 0; r < k; ++r) w[r] = norm_topk ? p[ids[r]] / mass : p[ids[r]];
}

/* Weight source for the expert loop: either dense f32 [E,rows,cols] or packed
 * GGUF rows dequantized on the fly (identical values to a load-time dequant). */
typedef struct {
  int fmt;            /* UO_F32 for dense */
  const void* data;
  int64_t rows, cols; /* per expert */
  int64_t pitch;      /* bytes per row for packed */
} uo_wsrc;

static const float* uo_row(const uo_wsrc* s, int64_t e, int64_t r, float* scratch) {
  if (s->fmt == UO_F32) return (const float*)s->data + (e * s->rows + r) * s->cols;
  const uint8_t* p = (const uint8_t*)s->data + (size_t)((e * s->rows + r) * s->pitch);
  uo_dequant_row(s->fmt, p, s->cols, scratch);
  return scratch;
}

/* MoEExpertsSwiGLU for a list of tokens (transformer.cpp:522-612):
 * per token, top-k from probs; y = 0; for each selected expert in rank order:
 * g_i = sum_d x_d*G[e,i,d], u_i = sum_d x_d*U[e,i,d] (sequential over d),
 * h_i = (g * (1/(1+exp(-g)))) * u, y_o += w * sum_i h_i*Dn[e,o,i].
 * Optional `ids_out`/`w_out` receive the selection ([T,k]). */
static int uo_experts_impl(const float* x, const uo_wsrc* G, const uo_wsrc* U,
                           const uo_wsrc* Dn, const float* probs, int64_t T, int64_t D,
                           int64_t E, int64_t I, int top_k, int norm_topk, float* y,
                           int32_t* ids_out, float* w_out) {
  int k = top_k > 0 ? top_k : 1;
  if (k > E) k = (int)E;
  float* h = (float*)malloc(sizeof(float) * (size_t)I);
  float* sg = (float*)malloc(sizeof(float) * (size_t)D);
  float* su = (float*)malloc(sizeof(float) * (size_t)D);
  float* sd = (float*)malloc(sizeof(float) * (size_t)I);
  int32_t ids[256];
  float wts[256];
  if (!h || !sg || !su || !sd || k > 256) { free(h); free(sg); free(su); free(sd); return UO_INVALID_ARGUMENT; }
  for (int64_t b = 0; b < T; ++b) {
    uo_topk_row(probs + b * E, E, k, norm_topk, ids, wts);
    if (ids_out) for (int r = 0; r < k; ++r) ids_out[b * k + r] = ids[r];
    if (w_out) for (int r = 0; r < k; ++r) w_out[b * k + r] = wts[r];
    float* yb = y + b * D;
    for (int64_t o = 0; o < D; ++o) yb[o] = 0.0f;
    const float* xb = x + b * D;
    for (int r = 0; r < k; ++r) {
      const int64_t e = ids[r];
      const float w = wts[r];
      for (int64_t i = 0; i < I; ++i) {
        const float* gr = uo_row(G, e, i, sg);
        const float* ur = uo_row(U, e, i, su);
        float gs = 0.0f, us = 0.0f;
        for (int64_t d = 0; d < D; ++d) {
          gs += xb[d] * gr[d];
          us += xb[d] * ur[d];
        }
        const float sig = 1.0f / (1.0f + expf(-gs));
        h[i] = (gs * sig) * us;
      }
      for (int64_t o = 0; o < D; ++o) {
        const float* dr = uo_row(Dn, e, o, sd);
        float s = 0.0f;
        for (int64_t i = 0; i < I; ++i) s += h[i] * dr[i];
        yb[o] += w * s;
      }
    }
  }
  free(h); free(sg); free(su); free(sd);
  return UO_OK;
}

/* MoEExperts (legacy top-1 linear experts): y[b] = x[b] . W[e]^T with W [E, D, D] f32,
 * e = (int)top_expert[b], expert 0 when that is outside [0, E); per output a sequential
 * f32 sum over i of x*w (libs/uaii-kernels/src/transformer.cpp:483-520).  The range test
 * is written on the float so that NaN and huge ids also select expert 0, as the
 * reference's truncating conversion followed by its range check does on x86. */
int uo_moe_experts_linear(const float* x, const float* W, const float* top, int64_t B, int64_t D,
                          int64_t E, float* y) {
  if (!x || !W || !top || !y || B < 0 || D <= 0 || E <= 0) return UO_INVALID_ARGUMENT;
  for (int64_t b = 0; b < B; ++b) {
    const float v = top[b];
    const int64_t e = (v > -1.0f && v < (float)E) ? (int64_t)(int)v : 0;
    const float* We = W + e * D * D;
    for (int64_t o = 0; o < D; ++o) {
      float sum = 0.0f;
      for (int64_t i = 0; i < D; ++i) sum += x[b * D + i] * We[o * D + i];
      y[b * D + o] = sum;
    }
  }
  return UO_OK;
}

/* Dense f32 expert weights: gate/up [E,I,D], down [E,D,I] (kernels.hpp:104-114). */
int uo_moe_experts_swiglu(const float* x, const float* G, const float* U, const float* Dn,
                          const float* probs, int64_t T, int64_t D, int64_t E, int64_t I,
                          int top_k, int norm_topk, float* y, int32_t* ids_out,
                          float* w_out) {
  if (!x || !G || !U || !Dn || !probs || !y || D <= 0 || E <= 0 || I <= 0)
    return UO_INVALID_ARGUMENT;
  uo_wsrc g = {UO_F32, G, I, D, 0}, u = {UO_F32, U, I, D, 0}, dn = {UO_F32, Dn, D, I, 0};
  return uo_experts_impl(x, &g, &u, &dn, probs, T, D, E, I, top_k, norm_topk, y, ids_out, w_out);
}

/* Packed GGUF expert weights; rows dequantized on the fly with uo_dequant_row,
 * which is value-identical to dequantizing the whole tensor first. */
int uo_moe_experts_swiglu_packed(const float* x, const void* G, int gfmt, const void* U,
                                 int ufmt, const void* Dn, int dfmt, const float* probs,
                                 int64_t T, int64_t D, int64_t E, int64_t I, int top_k,
                                 int norm_topk, float* y, int32_t* ids_out, float* w_out) {
  if (!x || !G || !U || !Dn || !probs || !y || D <= 0 || E <= 0 || I <= 0)
    return UO_INVALID_ARGUMENT;
  uo_wsrc g = {gfmt, G, I, D, (int64_t)uo_packed_nbytes(gfmt, D)};
  uo_wsrc u = {ufmt, U, I, D, (int64_t)uo_packed_nbytes(ufmt, D)};
  uo_wsrc dn = {dfmt, Dn, D, I, (int64_t)uo_packed_nbytes(dfmt, I)};
  return uo_experts_impl(x, &g, &u, &dn, probs, T, D, E, I, top_k, norm_topk, y, ids_out, w_out);
}

/* Shared expert added after the routed experts.  The reference graph
 * (libs/uaii-loaders/src/gguf.cpp:1107-1128) is MatMul(x,Wg_sh) -> Silu ->
 * Mul(.,x·Wu_sh) -> MatMul(.,Wd_sh) -> Add with no gate; Silu there is
 * v/(1+exp(-v)) (libs/uaii-kernels/src/elementwise.cpp:73-82).  The optional
 * sigmoid gate y += sigmoid(x·w_sg) * shared(x) has no reference counterpart
 * (parity unpinned; restatement only).  `wsg` may be NULL for the ungated form.
 * Weights are packed GGUF rows: gate/up [I_sh, D], down [D, I_sh]. */
int uo_shared_expert_packed(const float* x, const void* G, int gfmt, const void* U, int ufmt,
                            const void* Dn, int dfmt, const float* wsg, int64_t T, int64_t D,
                            int64_t Ish, float* y) {
  uo_wsrc g = {gfmt, G, Ish, D, (int64_t)uo_packed_nbytes(gfmt, D)};
  uo_wsrc u = {ufmt, U, Ish, D, (int64_t)uo_packed_nbytes(ufmt, D)};
  uo_wsrc dn = {dfmt, Dn, D, Ish, (int64_t)uo_packed_nbytes(dfmt, Ish)};
  float* h = (float*)malloc(sizeof(float) * (size_t)Ish);
  float* s1 = (float*)malloc(sizeof(float) * (size_t)(D > Ish ? D : Ish));
  float* s2 = (float*)malloc(sizeof(float) * (size_t)(D > Ish ? D : Ish));
  if (!h || !s1 || !s2) { free(h); free(s1); free(s2); return UO_INVALID_ARGUMENT; }
  for (int64_t b = 0; b < T; ++b) {
    const float* xb = x + b * D;
    for (int64_t i = 0; i < Ish; ++i) {
      const float* gr = uo_row(&g, 0, i, s1);
      const float* ur = uo_row(&u, 0, i, s2);
      float gs = 0.0f, us = 0.0f;
      for (int64_t d = 0; d < D; ++d) { gs += xb[d] * gr[d]; us += xb[d] * ur[d]; }
      h[i] = (gs / (1.0f + expf(-gs))) * us;
    }
    float gate = 1.0f;
    if (wsg) {
      float z = 0.0f;
      for (int64_t d = 0; d < D; ++d) z += xb[d] * wsg[d];
      gate = 1.0f / (1.0f + expf(-z));
    }
    for (int64_t o = 0; o < D; ++o) {
      const float* dr = uo_row(&dn, 0, o, s1);
      float s = 0.0f;
      for (int64_t i = 0; i < Ish; ++i) s += h[i] * dr[i];
      y[b * D + o] += gate * s;
    }
  }
  free(h); free(s1); free(s2);
  return UO_OK;
}
