// uaii_cuda_native.cpp -- UAII's CUDA native layer (the functions CudaBackend calls,
// libs/uaii-backends/src/native_stubs.hpp:18-37) implemented over libuaii_moe.so.
//
// UAII's CudaBackend (libs/uaii-backends/src/cuda_backend.cpp) runs device-resident ops
// through native::cuda_dispatch and falls back to host staging when it returns an error
// (cuda_backend.cpp:199-204).  The reference's own implementation of this layer
// (cuda_runtime_api.cpp) has no MoE op; this one runs the MoE operators of libuaii_moe.so
// on the B200 -- MoERouter, MoEExperts, MoEExpertsSwiGLU, the fused MoEFFN and MatMul /
// MatMulRelu with a packed GGUF B (the quant_gemm_f32 branch of dispatch_cpu) -- and returns
// NotImplemented for every other op, which the backend then stages through the host kernels.
// A build of UAII with -DUAII_WITH_CUDA compiles this file in place of cuda_runtime_api.cpp
// (or merges its cuda_dispatch into that file's).
//
// Memory: cuda_allocate / cuda_free are cudaMalloc / cudaFree on the layer's device
// (UAII_MOE_DEVICE, default 0), tracked so that cuda_shutdown frees what is left, as the
// reference layer does.  Copies are synchronous except cuda_copy_h2d_async, which is
// ordered on the library backend's stream; cuda_synchronize waits for that stream.
#include "native_stubs.hpp"

#include "uaii_moe.h"

#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <set>
#include <string>
#include <vector>

namespace uaii {
namespace backends {
namespace native {
namespace {

std::mutex g_mu;
uaii_moe_backend* g_be = nullptr;
cudaStream_t g_stream = nullptr;
int g_device = 0;
std::set<void*> g_allocs;
std::atomic<unsigned long long> g_device_ops{0}, g_declined{0};

Error cuda_error(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Error::success();
  (void)cudaGetLastError();
  return Error::make(ErrorCode::Internal, std::string("CUDA ") + what + ": " + cudaGetErrorString(e));
}

Error moe_error(int st) {
  if (st == UAII_MOE_OK) return Error::success();
  return Error::make(static_cast<ErrorCode>(st), uaii_moe_last_error());
}

bool packed_matmul(const std::string& op, const std::vector<kernels::TensorView>& in,
                   const std::vector<ir::Attribute>& attrs) {
  if ((op != "MatMul" && op != "MatMulRelu") || in.size() != 2) return false;
  if (!quant::is_gguf_block_quant(in[1].quant_format)) return false;
  for (const auto& a : attrs)
    if (a.key == "transpose_b" && a.type == ir::AttributeType::Bool) return std::get<bool>(a.value);
  return false;
}

}  // namespace

bool cuda_compiled() noexcept { return true; }

const char* cuda_capability_details() noexcept {
  return "CUDA native (B200, libuaii_moe): MoERouter, MoEExperts, MoEExpertsSwiGLU, MoEFFN, packed-B MatMul on "
         "device; host_fallback: every other op";
}

Error cuda_init() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_be != nullptr) return Error::success();
  const char* dev = std::getenv("UAII_MOE_DEVICE");
  g_device = dev ? std::atoi(dev) : 0;
  const int st = uaii_moe_backend_create(g_device, nullptr, &g_be);
  if (st != UAII_MOE_OK) {
    g_be = nullptr;
    return moe_error(st);
  }
  void* stream = nullptr;
  (void)uaii_moe_backend_stream(g_be, &stream);
  g_stream = static_cast<cudaStream_t>(stream);
  return Error::success();
}

void cuda_shutdown() noexcept {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_be == nullptr) return;
  (void)uaii_moe_synchronize(g_be);
  for (void* p : g_allocs) (void)cudaFree(p);
  g_allocs.clear();
  uaii_moe_backend_destroy(g_be);
  g_be = nullptr;
  g_stream = nullptr;
}

Error cuda_allocate(std::size_t bytes, void** out_ptr) {
  if (out_ptr == nullptr) return Error::make(ErrorCode::InvalidArgument, "cuda_allocate out null");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_be == nullptr) return Error::make(ErrorCode::Internal, "CUDA native layer not initialised");
  Error err = cuda_error(cudaSetDevice(g_device), "SetDevice");
  if (!err.ok()) return err;
  err = cuda_error(cudaMalloc(out_ptr, bytes ? bytes : 1), "Malloc");
  if (err.ok()) g_allocs.insert(*out_ptr);
  return err;
}

Error cuda_free(void* ptr) noexcept {
  if (ptr == nullptr) return Error::success();
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_allocs.erase(ptr) == 0) return Error::make(ErrorCode::InvalidArgument, "cuda_free: unknown pointer");
  return cuda_error(cudaFree(ptr), "Free");
}

Error cuda_copy_h2d(const void* host, void* device, std::size_t bytes) {
  return cuda_error(cudaMemcpy(device, host, bytes, cudaMemcpyHostToDevice), "Memcpy(H2D)");
}

Error cuda_copy_h2d_async(const void* host, void* device, std::size_t bytes) {
  return cuda_error(cudaMemcpyAsync(device, host, bytes, cudaMemcpyHostToDevice, g_stream), "MemcpyAsync(H2D)");
}

bool cuda_probe_device() noexcept {
  int n = 0;
  const bool ok = cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
  (void)cudaGetLastError();
  return ok;
}

bool cuda_is_device_ptr(const void* p) noexcept {
  if (p == nullptr) return false;
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

Error cuda_copy_d2h(const void* device, void* host, std::size_t bytes) {
  if (g_stream) {
    const Error err = cuda_error(cudaStreamSynchronize(g_stream), "StreamSynchronize");
    if (!err.ok()) return err;
  }
  return cuda_error(cudaMemcpy(host, device, bytes, cudaMemcpyDeviceToHost), "Memcpy(D2H)");
}

Error cuda_copy_d2d(const void* src, void* dst, std::size_t bytes) {
  return cuda_error(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, g_stream), "MemcpyAsync(D2D)");
}

Error cuda_synchronize() {
  if (g_be == nullptr) return Error::success();
  return moe_error(uaii_moe_synchronize(g_be));
}

Error cuda_dispatch(const std::string& op_name, const std::string& op_version,
                    const std::vector<kernels::TensorView>& inputs, std::vector<kernels::TensorView>* outputs,
                    const std::vector<ir::Attribute>& attrs) {
  if (g_be == nullptr) return Error::make(ErrorCode::Internal, "CUDA native layer not initialised");
  if (!uaii_moe_supports_op(op_name.c_str()) && !packed_matmul(op_name, inputs, attrs)) {
    g_declined.fetch_add(1, std::memory_order_relaxed);
    return Error::make(ErrorCode::NotImplemented, "CUDA native op not implemented: " + op_name);
  }
  if (outputs == nullptr) return Error::make(ErrorCode::InvalidArgument, "dispatch outputs null");
  auto conv = [](const kernels::TensorView& t) {
    return uaii_moe_tensor{static_cast<int32_t>(t.dtype), static_cast<int32_t>(t.quant_format), t.shape, t.rank,
                           t.data, t.nbytes};
  };
  std::vector<uaii_moe_tensor> in, out;
  for (const auto& t : inputs) in.push_back(conv(t));
  for (const auto& t : *outputs) out.push_back(conv(t));
  std::vector<uaii_moe_attr> at;
  for (const auto& a : attrs) {
    if (a.type == ir::AttributeType::Int) at.push_back({a.key.c_str(), 1, std::get<std::int64_t>(a.value), 0.0});
    else if (a.type == ir::AttributeType::Float) at.push_back({a.key.c_str(), 2, 0, std::get<double>(a.value)});
    else if (a.type == ir::AttributeType::Bool) at.push_back({a.key.c_str(), 3, std::get<bool>(a.value) ? 1 : 0, 0.0});
  }
  std::lock_guard<std::mutex> lk(g_mu);
  const int st = uaii_moe_dispatch(g_be, op_name.c_str(), op_version.c_str(), in.data(), in.size(), out.data(),
                                   out.size(), at.data(), at.size());
  (st == UAII_MOE_OK ? g_device_ops : g_declined).fetch_add(1, std::memory_order_relaxed);
  return moe_error(st);
}

}  // namespace native
}  // namespace backends
}  // namespace uaii

// Ops this layer ran on the device, and ops it returned an error for (which CudaBackend then
// stages through the host kernels).
extern "C" __attribute__((visibility("default"))) void uaii_cuda_native_stats(unsigned long long* device_ops,
                                                                              unsigned long long* declined) {
  if (device_ops) *device_ops = uaii::backends::native::g_device_ops.load();
  if (declined) *declined = uaii::backends::native::g_declined.load();
}
