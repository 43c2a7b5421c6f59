// noalloc.cu -- the MoE FFN layer forward for callers that cannot allocate
// device memory.
//
// Some hosts of this operator cannot let it call cudaMalloc: a serving engine
// that has already reserved nearly all HBM for its own pools (KV cache,
// activations) would see an operator-level cudaMalloc fail or fragment its
// budget; an embedding runtime that owns every device allocation through its
// own allocator forbids allocation inside operators; and cudaMalloc/cudaFree
// synchronize the whole device, stalling the caller's other streams in the
// middle of a decode loop.  uaii_moe_ffn_forward_noalloc serves them: it runs
// the same kernels as uaii_moe_ffn_forward, but its scratch memory (routing
// tables, gathered activations, hidden activations, partial sums, the error
// flag) lives in one fixed array compiled into this library.
//
// The array is a file-scope static __device__ object, so every GPU that loads
// the library holds kScratchBytes of it until the process exits.  Host code
// may not use its name as a device address: the first call on each device
// looks the address up with cudaGetSymbolAddress (with that device current)
// and keeps it for later calls, so that first call should come before any
// stream capture.  Calls that need more scratch than the array holds are
// rejected with UAII_MOE_INVALID_ARGUMENT before any work is queued.  The
// device that was current when the call began is current again when it returns.
//
// Every call shares the array and finds the previous call's leftovers in it:
// the error flag, the split-work counters of the expert kernels and the expert
// routing mask are cleared on each call and every other buffer is fully
// rewritten before it is read.  Two calls whose GPU
// work overlapped would race on the shared array; this entry point prevents
// that inside one process by serializing calls with a lock and returning only
// after the call's GPU work has finished.
#include <mutex>

#include "../../include/uaii_moe.h"
#include "backend.hpp"

namespace uaii_b200 {
namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;  // 32 MiB per device
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_noalloc_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the array on the current device, looked up once per device.
Error scratch_address(int device, void** out) {
  if (device < 0 || device >= kMaxDevices)
    return Error::make(ErrorCode::InvalidArgument, "device index out of range");
  if (g_scratch_addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t st = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (st != cudaSuccess || p == nullptr) return cuda_status(st, "GetSymbolAddress(scratch)");
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return Error::success();
}

bool on_device_or_null(const void* p) { return p == nullptr || is_device_ptr(p); }

// Makes `device` current for the call and gives the caller back the device that
// was current before, on every return path.
struct DeviceGuard {
  int prev = -1;
  cudaError_t st = cudaSuccess;
  explicit DeviceGuard(int device) {
    st = cudaGetDevice(&prev);
    if (st == cudaSuccess) st = cudaSetDevice(device);
  }
  ~DeviceGuard() {
    if (prev >= 0) (void)cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace uaii_b200

using namespace uaii_b200;

extern "C" int uaii_moe_ffn_forward_noalloc(int device, void* stream, const uaii_moe_layer* layer,
                                            const float* x, int64_t T, float* y, float* probs) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (layer == nullptr || x == nullptr || y == nullptr)
    return report_status(Error::make(ErrorCode::InvalidArgument, "noalloc ffn: null argument"));
  DeviceGuard dg(device);
  if (dg.st != cudaSuccess) return report_status(cuda_status(dg.st, "SetDevice"));
  LayerArgs L;
  if (!layer_args_from_c(layer, &L))
    return report_status(Error::make(ErrorCode::InvalidArgument, "noalloc ffn: null expert weights"));
  // no staging without allocation: everything must already be on the device
  const void* must[] = {x, y, L.router_w, L.gate.data, L.up.data, L.down.data};
  for (const void* p : must)
    if (!is_device_ptr(p))
      return report_status(Error::make(ErrorCode::InvalidArgument,
                                       "noalloc ffn: inputs, outputs and weights must be device memory"));
  if (!on_device_or_null(probs) || (L.I_sh > 0 && (!is_device_ptr(L.gate_sh.data) || !is_device_ptr(L.up_sh.data) ||
                                                   !is_device_ptr(L.down_sh.data) ||
                                                   !on_device_or_null(L.gate_inp_sh))))
    return report_status(Error::make(ErrorCode::InvalidArgument,
                                     "noalloc ffn: inputs, outputs and weights must be device memory"));
  void* scratch = nullptr;
  Error e = scratch_address(device, &scratch);
  if (!e.ok()) return report_status(e);
  MoeCudaBackend exec;
  e = exec.attach_external(device, static_cast<cudaStream_t>(stream), scratch, kScratchBytes);
  if (e.ok()) e = exec.ffn(L, x, T, y, probs);
  if (e.ok()) e = exec.sync_and_check_public();
  else (void)cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  return report_status(e);
}
