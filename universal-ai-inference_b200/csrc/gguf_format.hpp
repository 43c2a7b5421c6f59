// gguf_format.hpp -- GGUF block geometry shared by host and device code.
// Values follow uaii::quant::QuantFormat and quant::packed_nbytes
// (include/uaii/quant/formats.hpp:10-29, :81-102).
#pragma once

#ifdef __CUDACC__
#define UAII_HD __host__ __device__
#else
#define UAII_HD
#endif

namespace uaii_b200 {

// uaii::quant::QuantFormat values (include/uaii/quant/formats.hpp:10-29).
enum Fmt : int {
  kF32 = 0, kF16 = 1, kBF16 = 2,
  kQ4_0 = 7, kQ4_1 = 8, kQ5_0 = 9, kQ5_1 = 10, kQ8_0 = 11,
  kQ2_K = 12, kQ3_K = 13, kQ4_K = 14, kQ5_K = 15, kQ6_K = 16,
};

UAII_HD constexpr int fmt_block_elems(int f) {
  return (f >= kQ2_K && f <= kQ6_K) ? 256 : ((f >= kQ4_0 && f <= kQ8_0) ? 32 : 1);
}
UAII_HD constexpr int fmt_block_bytes(int f) {
  return f == kF32 ? 4 : f == kF16 ? 2 : f == kBF16 ? 2 : f == kQ4_0 ? 18 : f == kQ4_1 ? 20
       : f == kQ5_0 ? 22 : f == kQ5_1 ? 24 : f == kQ8_0 ? 34 : f == kQ2_K ? 84
       : f == kQ3_K ? 110 : f == kQ4_K ? 144 : f == kQ5_K ? 176 : f == kQ6_K ? 210 : 0;
}
// packed bytes of a row of n elements (include/uaii/quant/formats.hpp:81-102)
UAII_HD constexpr long long fmt_row_bytes(int f, long long n) {
  return (n / fmt_block_elems(f)) * fmt_block_bytes(f);
}
UAII_HD constexpr bool fmt_is_gguf(int f) { return f >= kQ4_0 && f <= kQ6_K; }

}  // namespace uaii_b200
