// cudabackend_shim.cpp -- test infrastructure: C entry points that drive UAII's own CudaBackend
// (libs/uaii-backends/src/cuda_backend.cpp and host_executable.cpp, unmodified, built with
// UAII_WITH_CUDA) whose native layer is universal-ai-inference_b200/plugin/uaii_cuda_native.cpp.
// Device buffers come from the backend's allocate(); ops go through IBackend::dispatch with
// device-resident TensorViews (include/uaii/interfaces/backend.hpp:39-80), the path the
// reference takes for device tensors (cuda_backend.cpp:166-207).
#include "uaii/backends/factory.hpp"
#include "uaii/ir/attribute.hpp"
#include "uaii/kernels/tensor_view.hpp"
#include "uaii/memory/allocator.hpp"

#include <cstring>
#include <memory>
#include <string>
#include <vector>

namespace {
thread_local std::string g_last;
uaii::memory::Allocator& host_allocator() {
  static uaii::memory::Allocator a;
  return a;
}
int status(const uaii::Error& e) {
  g_last = e.ok() ? std::string() : e.message();
  return static_cast<int>(e.code());
}
uaii::IBackend* be(void* b) { return static_cast<uaii::IBackend*>(b); }
uaii::kernels::TensorView f32_view(void* p, const int64_t* shape, size_t rank) {
  uaii::kernels::TensorView v;
  v.dtype = uaii::DType::F32;
  v.shape = shape;
  v.rank = rank;
  v.data = p;
  size_t n = 1;
  for (size_t i = 0; i < rank; ++i) n *= static_cast<size_t>(shape[i]);
  v.nbytes = n * sizeof(float);
  return v;
}
}  // namespace

extern "C" {

const char* ucb_last_error() { return g_last.c_str(); }

// backend "cuda" with the native path preferred; native_available and the details string
// report whether the native layer initialised
int ucb_create(void** out, int* native_available, char* details, size_t cap) {
  std::unique_ptr<uaii::IBackend> b;
  uaii::backends::BackendCreateOptions o;
  o.allocator = &host_allocator();
  int st = status(uaii::backends::create_backend("cuda", o, &b));
  if (st != 0) return st;
  st = status(b->initialize());
  if (st != 0) return st;
  const uaii::BackendCapabilities c = b->capabilities();
  if (native_available) *native_available = c.native_available ? 1 : 0;
  if (details && cap) {
    std::strncpy(details, c.details.c_str(), cap - 1);
    details[cap - 1] = 0;
  }
  *out = b.release();
  return 0;
}

void ucb_destroy(void* b) {
  be(b)->shutdown();
  delete be(b);
}

int ucb_alloc(void* b, size_t bytes, void** p) { return status(be(b)->allocate(bytes, p)); }
int ucb_free(void* b, void* p) { return status(be(b)->free(p)); }
int ucb_h2d(void* b, const void* h, void* d, size_t n) { return status(be(b)->copy_h2d(h, d, n)); }
int ucb_d2h(void* b, const void* d, void* h, size_t n) { return status(be(b)->copy_d2h(d, h, n)); }
int ucb_sync(void* b) { return status(be(b)->synchronize()); }

// MoERouter: x [T, D], gate [E, D] -> probs [T, E], top [T, 1] (dispatch_cpu's arity and attrs)
int ucb_moe_router(void* b, void* x, void* gate, int64_t T, int64_t D, int64_t E, void* probs, void* top) {
  const int64_t sx[2] = {T, D}, sg[2] = {E, D}, sp[2] = {T, E}, st[2] = {T, 1};
  std::vector<uaii::kernels::TensorView> in{f32_view(x, sx, 2), f32_view(gate, sg, 2)};
  std::vector<uaii::kernels::TensorView> out{f32_view(probs, sp, 2), f32_view(top, st, 2)};
  std::vector<uaii::ir::Attribute> at{uaii::ir::make_int_attr("num_experts", E)};
  return status(be(b)->dispatch("MoERouter", "1", in, &out, at));
}

// MoEExpertsSwiGLU with packed GGUF experts (dtype Unknown, quant_format = fmt, nbytes packed,
// as the Session lays out keep_quantized weights, session.cpp:342-357)
int ucb_moe_swiglu(void* b, void* x, void* G, int gfmt, size_t gbytes, void* U, int ufmt, size_t ubytes, void* Dn,
                   int dfmt, size_t dbytes, void* probs, int64_t T, int64_t D, int64_t E, int64_t I, int64_t k,
                   void* y) {
  const int64_t sx[2] = {T, D}, sgu[3] = {E, I, D}, sd[3] = {E, D, I}, sp[2] = {T, E};
  auto packed = [](void* p, const int64_t* shape, int fmt, size_t bytes) {
    uaii::kernels::TensorView v;
    v.dtype = uaii::DType::Unknown;
    v.shape = shape;
    v.rank = 3;
    v.data = p;
    v.nbytes = bytes;
    v.quant_format = static_cast<uaii::quant::QuantFormat>(fmt);
    return v;
  };
  std::vector<uaii::kernels::TensorView> in{f32_view(x, sx, 2), packed(G, sgu, gfmt, gbytes),
                                            packed(U, sgu, ufmt, ubytes), packed(Dn, sd, dfmt, dbytes),
                                            f32_view(probs, sp, 2)};
  std::vector<uaii::kernels::TensorView> out{f32_view(y, sx, 2)};
  std::vector<uaii::ir::Attribute> at{uaii::ir::make_int_attr("num_experts", E), uaii::ir::make_int_attr("top_k", k)};
  return status(be(b)->dispatch("MoEExpertsSwiGLU", "1", in, &out, at));
}

// MatMul / MatMulRelu with a packed GGUF B [N, K] and transpose_b (dispatch_cpu's quant_gemm_f32
// branch, dispatch.cpp:85-89): a [M, K] f32 -> c [M, N]
int ucb_matmul_packed(void* b, void* a, int64_t M, int64_t K, void* B, int fmt, size_t bbytes, int64_t N, int relu,
                      void* c) {
  const int64_t sa[2] = {M, K}, sb[2] = {N, K}, sc[2] = {M, N};
  uaii::kernels::TensorView vb;
  vb.dtype = uaii::DType::Unknown;
  vb.shape = sb;
  vb.rank = 2;
  vb.data = B;
  vb.nbytes = bbytes;
  vb.quant_format = static_cast<uaii::quant::QuantFormat>(fmt);
  std::vector<uaii::kernels::TensorView> in{f32_view(a, sa, 2), vb};
  std::vector<uaii::kernels::TensorView> out{f32_view(c, sc, 2)};
  std::vector<uaii::ir::Attribute> at{uaii::ir::make_bool_attr("transpose_b", true)};
  return status(be(b)->dispatch(relu ? "MatMulRelu" : "MatMul", "1", in, &out, at));
}

// Softmax over the last axis of device-resident x [rows, cols]: an op the native layer
// declines, which CudaBackend stages through its host kernels (cuda_backend.cpp:199-204)
int ucb_softmax(void* b, void* x, int64_t rows, int64_t cols, void* y) {
  const int64_t s[2] = {rows, cols};
  std::vector<uaii::kernels::TensorView> in{f32_view(x, s, 2)};
  std::vector<uaii::kernels::TensorView> out{f32_view(y, s, 2)};
  std::vector<uaii::ir::Attribute> at{uaii::ir::make_int_attr("axis", -1)};
  return status(be(b)->dispatch("Softmax", "1", in, &out, at));
}

}  // extern "C"
