// ref_shim.cpp -- extern "C" entry points over the reference's OWN compiled code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// sixteen unmodified source files of the reference (arjun988/Universal-AI-Inference)
// into oracle/_ref/libuaii_ref.so.  Nothing here re-implements the reference:
// each function only builds the reference's TensorView arguments and calls
//   uaii::quant::dequant_gguf_row      (libs/uaii-quant/src/gguf_dequant.cpp:420-439)
//   uaii::kernels::moe_router_f32      (libs/uaii-kernels/src/transformer.cpp:446-481)
//   uaii::kernels::moe_experts_swiglu_f32 (libs/uaii-kernels/src/transformer.cpp:522-612)
//   uaii::kernels::matmul_f32          (libs/uaii-kernels/src/matmul.cpp:22-56)
//   uaii::kernels::quant_gemm_f32      (libs/uaii-kernels/src/quant_gemm.cpp:22-70)
//   uaii::kernels::rmsnorm_f32 / rope_f32 / attention_kv_f32 / embedding_f32 / softmax_f32
//                                      (libs/uaii-kernels/src/norm.cpp:89-130, transformer.cpp:61-345,
//                                       softmax.cpp:11-77)
//   uaii::loaders::gguf_read_header / gguf_load_tensor_f32 / gguf_load_tensor_raw /
//   gguf_write_f32                     (libs/uaii-loaders/src/gguf.cpp:374-650)
// It is used by tests/ to pin oracle/moe_oracle.c, by tests/golden/make_golden.py
// to produce fixtures, and by bench.py's reference arm as the timed CPU path.
#include "uaii/kernels/kernels.hpp"
#include "uaii/kernels/quant_gemm.hpp"
#include "uaii/loaders/gguf.hpp"
#include "uaii/quant/formats.hpp"
#include "uaii/quant/gguf_dequant.hpp"

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

using uaii::DType;
using uaii::kernels::TensorView;

namespace {

TensorView f32_view(const float* p, const std::int64_t* shape, std::size_t rank) {
  TensorView v;
  v.dtype = DType::F32;
  v.shape = shape;
  v.rank = rank;
  v.data = const_cast<float*>(p);
  std::size_t n = 1;
  for (std::size_t i = 0; i < rank; ++i) n *= static_cast<std::size_t>(shape[i]);
  v.nbytes = n * sizeof(float);
  return v;
}

thread_local std::string g_last;

int status(const uaii::Error& e) {
  g_last = e.message();
  return static_cast<int>(e.code());
}

}  // namespace

extern "C" {

const char* uref_last_error() { return g_last.c_str(); }

int uref_dequant_row(int fmt, const std::uint8_t* packed, std::int64_t cols, float* out) {
  return status(uaii::quant::dequant_gguf_row(static_cast<uaii::quant::QuantFormat>(fmt),
                                              packed, cols, out));
}

int uref_moe_router(const float* x, const float* gate, std::int64_t T, std::int64_t D,
                    std::int64_t E, float* probs, float* top) {
  const std::int64_t sx[2] = {T, D}, sg[2] = {E, D}, sp[2] = {T, E}, st[2] = {T, 1};
  TensorView vx = f32_view(x, sx, 2), vg = f32_view(gate, sg, 2);
  TensorView vp = f32_view(probs, sp, 2), vt = f32_view(top, st, 2);
  return status(uaii::kernels::moe_router_f32(vx, vg, &vp, &vt));
}

// Router logits through the reference GEMM (the path moe_router_f32 takes
// before its softmax): logits[T,E] = x[T,D] . gate[E,D]^T.
int uref_matmul_bt(const float* a, const float* b, std::int64_t M, std::int64_t K,
                   std::int64_t N, float* c) {
  const std::int64_t sa[2] = {M, K}, sb[2] = {N, K}, sc[2] = {M, N};
  TensorView va = f32_view(a, sa, 2), vb = f32_view(b, sb, 2), vc = f32_view(c, sc, 2);
  return status(uaii::kernels::matmul_f32(va, vb, &vc, false, true));
}

// MatMul with a packed B (the dispatch_cpu MatMul branch with transpose_b):
// c[M,N] = a[M,K] . dequant(b[N rows of K])^T.
int uref_quant_gemm(const float* a, std::int64_t M, std::int64_t K, const std::uint8_t* b, int fmt,
                    std::int64_t N, float* c) {
  const std::int64_t sa[2] = {M, K}, sb[2] = {N, K}, sc[2] = {M, N};
  TensorView va = f32_view(a, sa, 2), vc = f32_view(c, sc, 2);
  TensorView vb;
  vb.dtype = DType::Unknown;
  vb.shape = sb;
  vb.rank = 2;
  vb.data = const_cast<std::uint8_t*>(b);
  vb.quant_format = static_cast<uaii::quant::QuantFormat>(fmt);
  vb.nbytes = static_cast<std::size_t>(N) *
              uaii::quant::packed_nbytes(vb.quant_format, static_cast<std::size_t>(K));
  return status(uaii::kernels::quant_gemm_f32(va, vb, &vc, true));
}

// One tensor of a GGUF file through the reference loader: header, then the raw bytes.
// Returns the byte count (or -status); shape outermost first, type = ggml type.
std::int64_t uref_gguf_tensor_raw(const char* path, const char* name, std::uint8_t* out, std::int64_t cap,
                                  std::int64_t* shape, int* rank, int* type) {
  uaii::loaders::GgufFile file;
  uaii::Error e = uaii::loaders::gguf_read_header(path, &file);
  if (!e.ok()) return -status(e);
  std::vector<std::uint8_t> bytes;
  uaii::Shape shp;
  uaii::loaders::GgufType t{};
  e = uaii::loaders::gguf_load_tensor_raw(file, name, &bytes, &shp, &t);
  if (!e.ok()) return -status(e);
  if ((std::int64_t)bytes.size() > cap) return -1;
  std::copy(bytes.begin(), bytes.end(), out);
  *rank = (int)shp.dims.size();
  for (std::size_t i = 0; i < shp.dims.size() && i < 8; ++i) shape[i] = shp.dims[i];
  *type = static_cast<int>(t);
  return (std::int64_t)bytes.size();
}

// A tensor as the reference's Session loads it by default: gguf_load_tensor_f32,
// the load-time dequantization (libs/uaii-loaders/src/gguf.cpp:445-556).  Returns
// the element count, or minus the status.
std::int64_t uref_gguf_tensor_f32(const char* path, const char* name, float* out, std::int64_t cap) {
  uaii::loaders::GgufFile file;
  uaii::Error e = uaii::loaders::gguf_read_header(path, &file);
  if (!e.ok()) return -status(e);
  std::vector<float> vals;
  uaii::Shape shp;
  e = uaii::loaders::gguf_load_tensor_f32(file, name, &vals, &shp);
  if (!e.ok()) return -status(e);
  if ((std::int64_t)vals.size() > cap) return -1;
  std::copy(vals.begin(), vals.end(), out);
  return (std::int64_t)vals.size();
}

// ---- the decode step's other reference kernels, batch rows at a time (the reference runs
// them with batch 1 per sequence; each row is independent).
int uref_rmsnorm(const float* x, const float* w, std::int64_t rows, std::int64_t D, float eps, float* y) {
  const std::int64_t s[2] = {rows, D}, sw[1] = {D};
  TensorView vx = f32_view(x, s, 2), vy = f32_view(y, s, 2), vw = f32_view(w, sw, 1);
  return status(uaii::kernels::rmsnorm_f32(vx, &vw, &vy, eps));
}

// RoPE of rows [rows, dim] at positions[r] (f32), per head of head_dim (transformer.cpp:144-225).
int uref_rope(const float* x, const float* positions, std::int64_t rows, std::int64_t dim, float theta,
              std::int64_t head_dim, int mode, float* y) {
  const std::int64_t s[2] = {rows, dim}, sp[1] = {rows};
  TensorView vx = f32_view(x, s, 2), vy = f32_view(y, s, 2), vp = f32_view(positions, sp, 1);
  return status(uaii::kernels::rope_f32(vx, &vp, &vy, theta, head_dim, mode));
}

// One new position per sequence over past K/V [B, past, kv_dim] (transformer.cpp:227-345).
int uref_attention_kv(const float* q, const float* k, const float* v, std::int64_t B, std::int64_t q_dim,
                      std::int64_t kv_dim, int num_heads, const float* past_k, const float* past_v, std::int64_t past,
                      float* out) {
  const std::int64_t sq[2] = {B, q_dim}, sk[2] = {B, kv_dim}, sp[3] = {B, past, kv_dim};
  TensorView vq = f32_view(q, sq, 2), vk = f32_view(k, sk, 2), vv = f32_view(v, sk, 2), vo = f32_view(out, sq, 2);
  TensorView pk = f32_view(past_k, sp, 3), pv = f32_view(past_v, sp, 3);
  return status(uaii::kernels::attention_kv_f32(vq, vk, vv, &vo, num_heads, 0.0f, true, past > 0 ? &pk : nullptr,
                                                past > 0 ? &pv : nullptr, nullptr, nullptr));
}

// Token rows of a packed (GGUF) or f32 table [vocab, D] (transformer.cpp:61-138).
int uref_embedding(const float* tokens, std::int64_t B, const void* table, int fmt, std::int64_t vocab, std::int64_t D,
                   float* out) {
  const std::int64_t st[2] = {B, 1}, sw[2] = {vocab, D}, so[2] = {B, D};
  TensorView vt = f32_view(tokens, st, 2), vo = f32_view(out, so, 2);
  TensorView vw;
  vw.shape = sw;
  vw.rank = 2;
  vw.data = const_cast<void*>(table);
  if (fmt == 0) {
    vw.dtype = DType::F32;
    vw.nbytes = sizeof(float) * (std::size_t)(vocab * D);
  } else {
    vw.dtype = DType::Unknown;
    vw.quant_format = static_cast<uaii::quant::QuantFormat>(fmt);
    vw.quant_rows = vocab;
    vw.quant_cols = D;
    vw.nbytes = uaii::quant::packed_nbytes(vw.quant_format, (std::size_t)D) * (std::size_t)vocab;
  }
  return status(uaii::kernels::embedding_f32(vt, vw, &vo));
}

int uref_softmax(const float* x, std::int64_t rows, std::int64_t n, float* y) {
  const std::int64_t s[2] = {rows, n};
  TensorView vx = f32_view(x, s, 2), vy = f32_view(y, s, 2);
  return status(uaii::kernels::softmax_f32(vx, &vy, -1));
}

// A GGUF file written by the reference's own writer: f32 tensors (dims innermost
// first, as GGUF stores them) and two metadata keys.
int uref_gguf_write_f32(const char* path, int n, const char* const* names, const int* ranks,
                        const std::uint64_t* dims, const float* const* data) {
  std::unordered_map<std::string, uaii::loaders::GgufValue> kv;
  kv["general.architecture"] = std::string("llama");
  kv["llama.expert_count"] = std::uint32_t{4};
  std::vector<std::pair<uaii::loaders::GgufTensorInfo, std::vector<float>>> tensors;
  std::size_t d0 = 0;
  for (int i = 0; i < n; ++i) {
    uaii::loaders::GgufTensorInfo info;
    info.name = names[i];
    std::size_t numel = 1;
    for (int r = 0; r < ranks[i]; ++r) {
      info.dims.push_back(dims[d0 + r]);
      numel *= (std::size_t)dims[d0 + r];
    }
    d0 += (std::size_t)ranks[i];
    tensors.emplace_back(info, std::vector<float>(data[i], data[i] + numel));
  }
  return status(uaii::loaders::gguf_write_f32(path, kv, tensors));
}

int uref_moe_experts_swiglu(const float* x, const float* G, const float* U, const float* Dn,
                            const float* probs, std::int64_t T, std::int64_t D, std::int64_t E,
                            std::int64_t I, int top_k, float* y) {
  const std::int64_t sx[2] = {T, D}, sgu[3] = {E, I, D}, sd[3] = {E, D, I}, sp[2] = {T, E};
  TensorView vx = f32_view(x, sx, 2), vg = f32_view(G, sgu, 3), vu = f32_view(U, sgu, 3);
  TensorView vd = f32_view(Dn, sd, 3), vp = f32_view(probs, sp, 2), vy = f32_view(y, sx, 2);
  return status(uaii::kernels::moe_experts_swiglu_f32(vx, vg, vu, vd, vp, &vy,
                                                      static_cast<int>(E), top_k));
}

int uref_moe_experts(const float* x, const float* W, const float* top, std::int64_t B, std::int64_t D,
                     std::int64_t E, float* y) {
  const std::int64_t sx[2] = {B, D}, sw[3] = {E, D, D}, st[2] = {B, 1};
  TensorView vx = f32_view(x, sx, 2), vw = f32_view(W, sw, 3), vt = f32_view(top, st, 2);
  TensorView vy = f32_view(y, sx, 2);
  return status(uaii::kernels::moe_experts_f32(vx, vw, vt, &vy, static_cast<int>(E)));
}

// Same call, with the token rows split across `threads` host threads.  Each
// thread runs the unmodified reference function on its own contiguous token
// range (the function is independent per token row), so the arithmetic per
// token is exactly the reference's.  Used for the timed CPU baseline.
int uref_moe_experts_swiglu_mt(const float* x, const float* G, const float* U,
                               const float* Dn, const float* probs, std::int64_t T,
                               std::int64_t D, std::int64_t E, std::int64_t I, int top_k,
                               float* y, int threads) {
  if (threads <= 1 || T <= 1) {
    return uref_moe_experts_swiglu(x, G, U, Dn, probs, T, D, E, I, top_k, y);
  }
  if (threads > T) threads = static_cast<int>(T);
  std::vector<int> rc(static_cast<std::size_t>(threads), 0);
  std::vector<std::thread> pool;
  for (int i = 0; i < threads; ++i) {
    const std::int64_t t0 = T * i / threads, t1 = T * (i + 1) / threads;
    pool.emplace_back([=, &rc]() {
      rc[static_cast<std::size_t>(i)] = uref_moe_experts_swiglu(
          x + t0 * D, G, U, Dn, probs + t0 * E, t1 - t0, D, E, I, top_k, y + t0 * D);
    });
  }
  for (auto& th : pool) th.join();
  for (int v : rc) if (v != 0) return v;
  return 0;
}

}  // extern "C"
