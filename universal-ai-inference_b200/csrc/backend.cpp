// backend.cpp -- the MoE operators of UAII on a B200, behind the reference's
// operator seam (IBackend::dispatch, include/uaii/interfaces/backend.hpp:77-81),
// and the extern "C" shim declared in include/uaii_moe.h.
//
// Residency follows the reference CUDA backend: a pointer is device memory when
// cudaPointerGetAttributes says so (libs/uaii-backends/src/cuda_runtime_api.cpp:586-601).
// Host activations are staged through a backend-owned workspace and host
// outputs are copied back before the call returns (the reference's host
// staging, libs/uaii-backends/src/host_executable.cpp:169-233).  Host weights
// are staged per call unless registered; registered buffers are uploaded once
// into a backend-owned cache that shutdown() frees, like the reference's
// device_allocs_ (libs/uaii-backends/src/cuda_backend.cpp:68-78).
#include "backend.hpp"

#include <cmath>
#include <cstdlib>

#include <cstring>
#include <string>

#include "../../include/uaii_moe.h"
#include "gguf_format.hpp"
#include "operand_order.cuh"

namespace uaii_b200 {

bool is_device_ptr(const void* p) noexcept {
  if (p == nullptr) return false;
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

// CUDA errors map to Internal with the CUDA message
// (libs/uaii-backends/src/cuda_runtime_api.cpp:30-36).
Error cuda_status(cudaError_t st, const char* what) {
  if (st == cudaSuccess) return Error::success();
  return Error::make(ErrorCode::Internal, std::string("CUDA ") + what + ": " + cudaGetErrorString(st));
}


namespace {

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

bool fmt_supported(int f) { return f == kF32 || f == kF16 || fmt_is_gguf(f); }

uint64_t row_bytes(int fmt, int64_t cols) {
  if (fmt == kF32) return (uint64_t)cols * 4;
  if (fmt == kF16) return (uint64_t)cols * 2;
  return (uint64_t)fmt_row_bytes(fmt, cols);
}

Error check_cols(const char* what, int fmt, int64_t cols) {
  if (!fmt_supported(fmt))
    return Error::make(ErrorCode::NotImplemented, std::string(what) + ": unsupported weight format");
  const int qk = fmt_block_elems(fmt);  // 1 for dense rows: any length
  if (cols % qk != 0)
    return Error::make(ErrorCode::InvalidArgument,
                       std::string(what) + ": row length " + std::to_string(cols) +
                           " is not a multiple of " + std::to_string(qk));
  return Error::success();
}

}  // namespace

Error MoeCudaBackend::initialize(int device, cudaStream_t stream) {
  int count = 0;
  UAII_CUDA(cudaGetDeviceCount(&count), "GetDeviceCount");
  if (device < 0 || device >= count)
    return Error::make(ErrorCode::InvalidArgument, "no CUDA device " + std::to_string(device));
  UAII_CUDA(cudaSetDevice(device), "SetDevice");
  cudaDeviceProp prop{};
  UAII_CUDA(cudaGetDeviceProperties(&prop, device), "GetDeviceProperties");
  if (prop.major != 10)
    return Error::make(ErrorCode::NotImplemented,
                       std::string("device ") + prop.name + " is not sm_100 (this build targets B200 only)");
  device_ = device;
  // quad down in balanced ranges: "0" never, "1" always (where the buffers allow), unset: automatic
  const char* rg = std::getenv("UAII_MOE_DOWN_RANGES");
  ranges_mode_ = rg && rg[0] == '0' ? 0 : rg && rg[0] == '1' ? 1 : -1;
  UAII_CUDA(cudaMalloc(&dev_err_, sizeof(int)), "Malloc(error flag)");
  UAII_CUDA(cudaMemset(dev_err_, 0, sizeof(int)), "Memset(error flag)");
  // the quad schedule's tail-split partials and counters (the counters stay zero between launches)
  UAII_CUDA(cudaMalloc(&tail_.part, tail_bytes()), "Malloc(tail split)");
  tail_.cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(tail_.part) + tail_part_bytes());
  route_done_ = tail_.cnt + kTailMaxUnits;
  UAII_CUDA(cudaMemset(tail_.cnt, 0, sizeof(int) * (kTailMaxUnits + 16)), "Memset(tail split)");
  if (stream == nullptr) {
    UAII_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "StreamCreate");
    own_stream_ = true;
  } else {
    stream_ = stream;
    own_stream_ = false;
  }
  return Error::success();
}

Error MoeCudaBackend::attach_external(int device, cudaStream_t stream, void* scratch, size_t bytes) {
  const size_t fixed = kAlign + align_up(tail_bytes());
  if (scratch == nullptr || bytes < fixed + kAlign)
    return Error::make(ErrorCode::InvalidArgument, "external scratch too small");
  UAII_CUDA(cudaSetDevice(device), "SetDevice");
  device_ = device;
  stream_ = stream;
  own_stream_ = false;
  external_ = true;
  // first 256 bytes: the error flag; then the tail-split buffers and counters (the same plans as
  // the owning mode); the rest is the workspace.  The flag and the counters start at zero.
  dev_err_ = static_cast<int*>(scratch);
  tail_.part = reinterpret_cast<float*>(static_cast<char*>(scratch) + kAlign);
  tail_.cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(tail_.part) + tail_part_bytes());
  route_done_ = tail_.cnt + kTailMaxUnits;
  ws_ = static_cast<char*>(scratch) + fixed;
  ws_cap_ = bytes - fixed;
  ws_used_ = 0;
  UAII_CUDA(cudaMemsetAsync(tail_.cnt, 0, sizeof(int) * (kTailMaxUnits + 16), stream_), "MemsetAsync(counters)");
  return cuda_status(cudaMemsetAsync(dev_err_, 0, sizeof(int), stream_), "MemsetAsync(error flag)");
}

void MoeCudaBackend::shutdown() noexcept {
  if (device_ < 0) return;
  if (external_) {  // nothing here is ours to free
    if (stream_) (void)cudaStreamSynchronize(stream_);
    ws_ = nullptr;
    dev_err_ = nullptr;
    tail_ = TailSplit{};
    route_done_ = nullptr;
    ws_cap_ = ws_used_ = 0;
    stream_ = nullptr;
    device_ = -1;
    return;
  }
  (void)cudaSetDevice(device_);
  if (stream_) (void)cudaStreamSynchronize(stream_);
  drop_graphs();
  for (auto& kv : padded_) (void)cudaFree(kv.second.dev);
  padded_.clear();
  for (auto& kv : weights_) (void)cudaFree(kv.second);
  weights_.clear();
  const_dev_.clear();
  for (auto& m : marks_) { (void)cudaEventDestroy(m.start); (void)cudaEventDestroy(m.stop); }
  marks_.clear();
  for (auto e : event_pool_) (void)cudaEventDestroy(e);
  event_pool_.clear();
  if (ws_) (void)cudaFree(ws_);
  ws_ = nullptr;
  ws_cap_ = ws_used_ = 0;
  if (dev_err_) (void)cudaFree(dev_err_);
  dev_err_ = nullptr;
  if (tail_.part) (void)cudaFree(tail_.part);
  tail_ = TailSplit{};
  route_done_ = nullptr;
  for (auto e : chunk_events_) (void)cudaEventDestroy(e);
  chunk_events_.clear();
  if (in_stream_) (void)cudaStreamDestroy(in_stream_);
  if (out_stream_) (void)cudaStreamDestroy(out_stream_);
  in_stream_ = out_stream_ = nullptr;
  if (own_stream_ && stream_) (void)cudaStreamDestroy(stream_);
  stream_ = nullptr;
  device_ = -1;
}

Error MoeCudaBackend::synchronize() {
  std::lock_guard<std::mutex> lk(mu_);
  return sync_and_check();
}

// Wait for the stream and report a device-side failure recorded by a kernel
// (a bounded wait that ran out); the flag is cleared once reported.
Error MoeCudaBackend::sync_and_check() {
  UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
  int code = 0;
  UAII_CUDA(cudaMemcpy(&code, dev_err_, sizeof(int), cudaMemcpyDeviceToHost), "Memcpy(error flag)");
  if (code != 0) {
    (void)cudaMemset(dev_err_, 0, sizeof(int));
    if (tail_.cnt) (void)cudaMemset(tail_.cnt, 0, sizeof(int) * (kTailMaxUnits + 16));  // a kernel may have stopped mid-tile
    return Error::make(ErrorCode::Internal,
                       "tensor-core expert kernel gave up waiting (code " + std::to_string(code) + ")");
  }
  return Error::success();
}

Error MoeCudaBackend::reserve(size_t bytes) {
  ws_used_ = 0;
  if (bytes <= ws_cap_) return Error::success();
  if (external_)
    return Error::make(ErrorCode::InvalidArgument, "call needs " + std::to_string(bytes) +
                                                       " bytes of scratch; the fixed scratch holds " +
                                                       std::to_string(ws_cap_));
  UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
  drop_graphs();  // captured launches point into the old workspace
  if (ws_) UAII_CUDA(cudaFree(ws_), "Free");
  ws_ = nullptr;
  ws_cap_ = 0;
  const size_t cap = align_up(bytes + bytes / 4);
  UAII_CUDA(cudaMalloc(&ws_, cap), "Malloc(workspace)");
  ws_cap_ = cap;
  return Error::success();
}

void* MoeCudaBackend::carve(size_t bytes) {
  void* p = ws_ + ws_used_;
  ws_used_ += align_up(bytes);
  return p;
}

cudaEvent_t pool_event(std::vector<cudaEvent_t>& pool) {
  if (!pool.empty()) {
    cudaEvent_t e = pool.back();
    pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

void MoeCudaBackend::phase_begin(int phase) {
  if (!profiling_) return;
  open_phase_ = phase;
  open_start_ = pool_event(event_pool_);
  if (open_start_) (void)cudaEventRecord(open_start_, stream_);
}

void MoeCudaBackend::phase_end() {
  if (!profiling_ || open_phase_ < 0 || !open_start_) return;
  cudaEvent_t stop = pool_event(event_pool_);
  if (stop) {
    (void)cudaEventRecord(stop, stream_);
    marks_.push_back(PhaseMark{open_phase_, open_start_, stop});
  }
  open_phase_ = -1;
  open_start_ = nullptr;
}

Error MoeCudaBackend::profile_enable(bool on) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
  for (auto& m : marks_) { event_pool_.push_back(m.start); event_pool_.push_back(m.stop); }
  marks_.clear();
  for (int i = 0; i < kPhases; ++i) { phase_ms_[i] = 0.0; phase_calls_[i] = 0; }
  launches_ = 0;
  profiling_ = on;
  return Error::success();
}

Error MoeCudaBackend::profile_read(double* ms, uint64_t* calls, uint64_t* launches) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
  for (auto& m : marks_) {
    float t = 0.f;
    UAII_CUDA(cudaEventElapsedTime(&t, m.start, m.stop), "EventElapsedTime");
    phase_ms_[m.phase] += t;
    phase_calls_[m.phase] += 1;
    event_pool_.push_back(m.start);
    event_pool_.push_back(m.stop);
  }
  marks_.clear();
  for (int i = 0; i < kPhases; ++i) {
    if (ms) ms[i] = phase_ms_[i];
    if (calls) calls[i] = phase_calls_[i];
  }
  if (launches) *launches = launches_;
  return Error::success();
}

size_t MoeCudaBackend::weight_stage_bytes(const void* p, size_t bytes) const {
  if (p == nullptr || is_device_ptr(p)) return 0;
  if (weights_.count(std::make_pair(p, bytes))) return 0;
  return align_up(bytes);
}

Error MoeCudaBackend::stage_weight(const void* p, size_t bytes, const void** dev) {
  if (p == nullptr) return Error::make(ErrorCode::InvalidArgument, "null weight pointer");
  if (is_device_ptr(p)) {
    *dev = p;
    return Error::success();
  }
  auto it = weights_.find(std::make_pair(p, bytes));
  if (it != weights_.end()) {
    *dev = it->second;
    return Error::success();
  }
  void* scratch = carve(bytes);
  UAII_CUDA(cudaMemcpyAsync(scratch, p, bytes, cudaMemcpyHostToDevice, stream_), "MemcpyAsync(weights)");
  *dev = scratch;
  return Error::success();
}

bool MoeCudaBackend::weight_is_constant(const void* p, size_t bytes) const {
  if (weights_.count(std::make_pair(p, bytes))) return true;
  const char* c = static_cast<const char*>(p);
  auto it = const_dev_.upper_bound(p);  // first registered buffer starting after p
  if (it == const_dev_.begin()) return false;
  --it;
  const char* b = static_cast<const char*>(it->first);
  return c >= b && c + bytes <= b + it->second;
}

void MoeCudaBackend::drop_padded(const char* lo, const char* hi) {
  for (auto it = padded_.begin(); it != padded_.end();) {
    const char* src = static_cast<const char*>(std::get<0>(it->first));
    if (src >= lo && src < hi) {
      (void)cudaFree(it->second.dev);
      it = padded_.erase(it);
    } else {
      ++it;
    }
  }
}

Error MoeCudaBackend::register_weights(const void* p, size_t bytes) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  if (p == nullptr || bytes == 0) return Error::make(ErrorCode::InvalidArgument, "register_weights: empty buffer");
  drop_graphs();  // calls that used the unregistered weights launched differently
  if (is_device_ptr(p)) {  // nothing to upload; layouts derived from it may be kept
    size_t& have = const_dev_[p];
    if (bytes > have) have = bytes;
    return Error::success();
  }
  auto key = std::make_pair(p, bytes);
  if (weights_.count(key)) return Error::success();
  void* d = nullptr;
  UAII_CUDA(cudaMalloc(&d, align_up(bytes)), "Malloc(weights)");
  cudaError_t st = cudaMemcpy(d, p, bytes, cudaMemcpyHostToDevice);
  if (st != cudaSuccess) {
    (void)cudaFree(d);
    return cuda_status(st, "Memcpy(weights)");
  }
  weights_[key] = d;
  return Error::success();
}

Error MoeCudaBackend::release_weights(const void* host_ptr) {
  std::lock_guard<std::mutex> lk(mu_);
  drop_graphs();  // captured launches may read the copies freed here
  bool found = false;
  for (auto it = weights_.begin(); it != weights_.end();) {
    if (it->first.first == host_ptr) {
      UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
      const char* d = static_cast<const char*>(it->second);
      drop_padded(d, d + it->first.second);
      (void)cudaFree(it->second);
      it = weights_.erase(it);
      found = true;
    } else {
      ++it;
    }
  }
  auto dv = const_dev_.find(host_ptr);
  if (dv != const_dev_.end()) {
    UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
    const char* d = static_cast<const char*>(dv->first);
    drop_padded(d, d + dv->second);
    const_dev_.erase(dv);
    found = true;
  }
  return found ? Error::success()
               : Error::make(ErrorCode::NotFound, "pointer has no cached device copy");
}

Error MoeCudaBackend::stage_input(const void* p, size_t bytes, void* scratch, const void** dev,
                                  bool* was_host) {
  if (p == nullptr) return Error::make(ErrorCode::InvalidArgument, "null input pointer");
  if (is_device_ptr(p)) {
    *dev = p;
    *was_host = false;
    return Error::success();
  }
  UAII_CUDA(cudaMemcpyAsync(scratch, p, bytes, cudaMemcpyHostToDevice, stream_), "MemcpyAsync(H2D)");
  *dev = scratch;
  *was_host = true;
  return Error::success();
}

Error MoeCudaBackend::dequant_rows(int fmt, const void* packed, int64_t rows, int64_t cols,
                                   float* out) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  if (rows < 0 || cols <= 0) return Error::make(ErrorCode::InvalidArgument, "dequant: bad shape");
  UAII_TRY(check_cols("dequant", fmt, cols));
  if (!fmt_is_gguf(fmt) && cols % 32 != 0)
    return Error::make(ErrorCode::InvalidArgument, "dequant: dense rows must be a multiple of 32");
  const size_t in_bytes = (size_t)rows * row_bytes(fmt, cols);
  const size_t out_bytes = sizeof(float) * (size_t)rows * (size_t)cols;
  UAII_TRY(reserve(align_up(in_bytes) + align_up(out_bytes)));
  void* in_scratch = carve(in_bytes);
  float* out_scratch = static_cast<float*>(carve(out_bytes));
  const void* in_dev = nullptr;
  bool in_host = false;
  UAII_TRY(stage_input(packed, in_bytes, in_scratch, &in_dev, &in_host));
  const bool out_host = !is_device_ptr(out);
  float* o = out_host ? out_scratch : out;
  UAII_CUDA(launch_dequant_rows_f32(fmt, in_dev, rows, cols, (int64_t)row_bytes(fmt, cols), o, stream_),
            "dequant_rows");
  count_launches(rows > 0 ? 1 : 0);
  if (out_host) {
    UAII_CUDA(cudaMemcpyAsync(out, o, out_bytes, cudaMemcpyDeviceToHost, stream_), "MemcpyAsync(D2H)");
    UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
  }
  return Error::success();
}

// The token -> expert assignment of the fused layer: router logits and probabilities, then the
// top-k procedure ranking on the exact logits with weights from the probabilities (the
// selection inside moe_experts_swiglu_f32, transformer.cpp:564-580).  ids [T, k] in rank order.
Error MoeCudaBackend::route(const float* x, const float* gate_w, int64_t T, int64_t D, int64_t E, int k,
                            int norm_topk, int32_t* ids, float* w) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  if (T < 0 || D <= 0 || E <= 0 || k < 1 || k > 32 || k > E || E > 1024 || !x || !gate_w || !ids || !w)
    return Error::make(ErrorCode::InvalidArgument, "moe route arguments");
  if (T == 0) return Error::success();
  const size_t xb = sizeof(float) * (size_t)(T * D), pb = sizeof(float) * (size_t)(T * E);
  const size_t ib = sizeof(int32_t) * (size_t)(T * k), wb = sizeof(float) * (size_t)(T * k);
  const size_t rsb = router_scratch_bytes(T, D, E);
  UAII_TRY(reserve(align_up(xb) + 2 * align_up(pb) + 2 * align_up(ib) + 2 * align_up(wb) + align_up((size_t)(E * T)) +
                   2 * align_up(sizeof(int32_t) * (size_t)(T * k)) + align_up(rsb) + 10 * kAlign +
                   weight_stage_bytes(gate_w, sizeof(float) * (size_t)(E * D))));
  void* xs = carve(xb);
  float* logits = static_cast<float*>(carve(pb));
  float* probs = static_cast<float*>(carve(pb));
  RouteBuffers rb{};
  rb.topk_ids = static_cast<int32_t*>(carve(ib));
  rb.topk_w = static_cast<float*>(carve(wb));
  rb.mask = static_cast<uint8_t*>(carve((size_t)(E * T)));
  float* rscratch = rsb ? static_cast<float*>(carve(rsb)) : nullptr;
  const void *xd = nullptr, *wd = nullptr;
  bool xh = false;
  UAII_TRY(stage_input(x, xb, xs, &xd, &xh));
  UAII_TRY(stage_weight(gate_w, sizeof(float) * (size_t)(E * D), &wd));
  const bool ih = !is_device_ptr(ids), wh = !is_device_ptr(w);
  phase_begin(kRouter);
  UAII_CUDA(launch_router(static_cast<const float*>(xd), static_cast<const float*>(wd), T, D, E, logits, probs, nullptr,
                          stream_, rscratch, rsb),
            "router");
  phase_end();
  phase_begin(kRoute);
  UAII_CUDA(launch_route_topk(logits, probs, T, E, k, norm_topk, rb, stream_), "route_topk");
  phase_end();
  count_launches(3);
  if (ih) UAII_CUDA(cudaMemcpyAsync(ids, rb.topk_ids, ib, cudaMemcpyDeviceToHost, stream_), "D2H");
  else UAII_CUDA(cudaMemcpyAsync(ids, rb.topk_ids, ib, cudaMemcpyDeviceToDevice, stream_), "D2D");
  if (wh) UAII_CUDA(cudaMemcpyAsync(w, rb.topk_w, wb, cudaMemcpyDeviceToHost, stream_), "D2H");
  else UAII_CUDA(cudaMemcpyAsync(w, rb.topk_w, wb, cudaMemcpyDeviceToDevice, stream_), "D2D");
  if (ih || wh) UAII_TRY(sync_and_check());
  return Error::success();
}

Error MoeCudaBackend::router(const float* x, const float* gate_w, int64_t T, int64_t D,
                             int64_t E, float* probs, float* top, float* logits) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  if (T < 0 || D <= 0 || E <= 0) return Error::make(ErrorCode::InvalidArgument, "moe router ranks");
  if (!probs || !top) return Error::make(ErrorCode::InvalidArgument, "moe router outs");
  const size_t xb = sizeof(float) * (size_t)(T * D), pb = sizeof(float) * (size_t)(T * E),
               tb = sizeof(float) * (size_t)T;
  const size_t rsb = router_scratch_bytes(T, D, E);
  UAII_TRY(reserve(align_up(xb) + 3 * align_up(pb) + align_up(tb) + align_up(rsb) + 5 * kAlign +
                   weight_stage_bytes(gate_w, sizeof(float) * (size_t)(E * D))));
  void* xs = carve(xb);
  float* ls = static_cast<float*>(carve(pb));
  float* ps = static_cast<float*>(carve(pb));
  float* ts = static_cast<float*>(carve(tb));
  float* rscratch = rsb ? static_cast<float*>(carve(rsb)) : nullptr;
  const void* xd = nullptr;
  const void* wd = nullptr;
  bool xh = false;
  if (T == 0) return Error::success();
  UAII_TRY(stage_input(x, xb, xs, &xd, &xh));
  UAII_TRY(stage_weight(gate_w, sizeof(float) * (size_t)(E * D), &wd));
  const bool ph = !is_device_ptr(probs), th = !is_device_ptr(top);
  const bool lh = logits != nullptr && !is_device_ptr(logits);
  float* lo = (logits && !lh) ? logits : ls;
  float* po = ph ? ps : probs;
  float* to = th ? ts : top;
  phase_begin(kRouter);
  UAII_CUDA(launch_router(static_cast<const float*>(xd), static_cast<const float*>(wd), T, D, E,
                          lo, po, to, stream_, rscratch, rsb),
            "router");
  phase_end();
  count_launches(2);
  bool any_host = false;
  if (ph) { UAII_CUDA(cudaMemcpyAsync(probs, po, pb, cudaMemcpyDeviceToHost, stream_), "D2H"); any_host = true; }
  if (th) { UAII_CUDA(cudaMemcpyAsync(top, to, tb, cudaMemcpyDeviceToHost, stream_), "D2H"); any_host = true; }
  if (lh) { UAII_CUDA(cudaMemcpyAsync(logits, lo, pb, cudaMemcpyDeviceToHost, stream_), "D2H"); any_host = true; }
  if (any_host) UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
  return Error::success();
}

Error MoeCudaBackend::experts_linear(const float* x, const float* W, const float* top, int64_t B, int64_t D,
                                     int64_t E, float* y) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  if (B < 0 || D <= 0 || E <= 0) return Error::make(ErrorCode::InvalidArgument, "moe experts shape");
  if (!x || !W || !top || !y) return Error::make(ErrorCode::InvalidArgument, "moe experts out");
  const size_t xb = sizeof(float) * (size_t)(B * D), tb = sizeof(float) * (size_t)B;
  const size_t wb = sizeof(float) * (size_t)E * (size_t)(D * D);
  UAII_TRY(reserve(2 * align_up(xb) + align_up(tb) + 4 * kAlign + weight_stage_bytes(W, wb)));
  void* xs = carve(xb);
  void* ts = carve(tb);
  float* ys = static_cast<float*>(carve(xb));
  if (B == 0) return Error::success();
  const void *xd = nullptr, *td = nullptr, *wd = nullptr;
  bool xh = false, th = false;
  UAII_TRY(stage_input(x, xb, xs, &xd, &xh));
  UAII_TRY(stage_input(top, tb, ts, &td, &th));
  UAII_TRY(stage_weight(W, wb, &wd));
  const bool yh = !is_device_ptr(y);
  float* yo = yh ? ys : y;
  UAII_CUDA(launch_experts_linear(static_cast<const float*>(xd), static_cast<const float*>(wd),
                                  static_cast<const float*>(td), B, D, E, yo, stream_),
            "experts_linear");
  count_launches(1);
  if (yh) {
    UAII_CUDA(cudaMemcpyAsync(y, yo, xb, cudaMemcpyDeviceToHost, stream_), "D2H");
    UAII_CUDA(cudaStreamSynchronize(stream_), "StreamSynchronize");
  }
  return Error::success();
}

namespace {
constexpr int kSms = 148;
// K splits of a down-style projection: the split count whose last wave ends first.  A
// unit is one (tile, split); every unit costs its quads plus about two quads of
// pipeline fill and epilogue, and the units run in waves of one per SM.
int pick_down_splits(int64_t tiles, int kchunks) {
  if (tiles <= 0 || kchunks <= 1) return 1;
  int best = 1;
  double best_cost = 0;
  for (int sp = 1; sp <= 16 && sp <= kchunks; ++sp) {
    const double waves = (double)((tiles * sp + kSms - 1) / kSms);
    const double cost = waves * ((kchunks + sp - 1) / sp + 2);
    if (sp == 1 || cost < best_cost) {
      best = sp;
      best_cost = cost;
    }
  }
  return best;
}
}  // namespace

// Which expert-product schedule a layer call uses, and its tile shape.
// Automatic: tensor cores whenever the layer qualifies; the warp-MMA schedule
// when no expert gets more than 16 routed slots on average (decode), tcgen05
// above.  allow_warp_mma = false keeps the tcgen05 operand order (rows that
// arrive packed by another rank).
ExpertPlan MoeCudaBackend::plan_experts(const LayerArgs& L, int64_t T, int64_t slots, bool allow_warp_mma) const {
  ExpertPlan p;
  const int64_t S = slots >= 0 ? slots : T * L.top_k;
  const bool umma_ok = umma_shapes_supported(L.gate.fmt, L.down.fmt, L.D, L.I);
  const bool warp_ok = allow_warp_mma && warp_mma_shapes_supported(L.gate.fmt, L.down.fmt, L.D, L.I);
  p.umma = path_ != 1 && umma_ok;
  p.umma_refused = (path_ == 2 && !umma_ok) || ((path_ == 3 || path_ == 4) && allow_warp_mma && !warp_ok);
  // Slots an expert's tile must hold: the mean plus two standard deviations of a
  // Poisson count at small means (an expert just above a tile width costs a second
  // pass over its weights), the mean at large ones (half-empty tiles cost MMA time).
  auto need = [](double tpe) { return tpe < 32 ? tpe + 2.0 * std::sqrt(tpe) : tpe; };
  auto pick_bn = [&](double tpe) {
    const double n = need(tpe);
    return n <= 16 ? 16 : n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : 256;
  };
  // warp-MMA use: forced (path 3), never (paths 1, 2), or (path 0) when 8-slot tiles
  // hold every expert's slots -- measured faster than tcgen05 there, slower at 16 slots
  auto use_warp = [&](bool ok, double tpe) {
    return ok && (path_ == 3 || path_ == 4 || (path_ == 0 && need(tpe) <= 8));
  };
  auto warp_bn = [&](double tpe) { return need(tpe) <= 8 ? 8 : 16; };
  auto pick_splits = pick_down_splits;
  const int64_t active = S < L.E ? S : L.E;
  const double tpe = active > 0 ? (double)S / (double)active : 1.0;
  p.bn = pick_bn(tpe);
  if (p.umma) {
    p.warp_mma = use_warp(warp_ok, tpe);
    if (p.warp_mma) p.bn = warp_bn(tpe);
    // K-quant layers run the warp schedule over whole super-blocks (path 4 keeps the per-unit one)
    p.quad_mma = p.warp_mma && path_ != 4 && quad_mma_format(L.gate.fmt) && quad_mma_format(L.down.fmt);
    // Q4_K gate/up at 8-slot tiles: integer activations (path 5 keeps the f16 ones).  With 16-slot
    // tiles the integer variant measured slower than tcgen05 (Mixtral-shaped, 32 tokens: 0.218 vs
    // 0.183 ms; two slot octets of int32 sums spill under the 96-register cap).
    p.quad_i8 = p.quad_mma && !f16_quad_ && L.gate.fmt == kQ4_K && L.up.fmt == kQ4_K && p.bn == 8;
    // 16-slot tiles: the down projection is faster on the quad schedule, gate/up on tcgen05
    // (Mixtral-shaped layer, 32 tokens: down 0.160 -> 0.121 ms; gate/up 0.191 vs 0.247 ms)
    p.down_quad = !p.warp_mma && path_ == 0 && warp_ok && p.bn == 16 && quad_mma_format(L.gate.fmt) &&
                  quad_mma_format(L.down.fmt);

    const int64_t n_tiles = (int64_t)((tpe + p.bn - 1) / p.bn);
    p.splits = pick_splits(active * n_tiles * (L.D / 128), umma_kchunks(L.down.fmt, L.I));
    // A quad down with at least one tile per SM spreads its quads evenly over the SMs instead
    // (needs the tail-split buffers).  With fewer tiles most pieces would be partial and pay the
    // fix-up: Mixtral-shaped, 1 token (64 tiles): 41 us in ranges against 38 us in K splits;
    // 8 tokens (224 tiles): 97 against 110 us.
    const int64_t dn_tiles = active * n_tiles * (L.D / 128);
    const bool ranges_ok = (p.quad_mma || p.down_quad) && tail_.part != nullptr &&
                           2 * kSms * p.bn <= kTailMaxUnits * kTailMaxBn;
    if (ranges_ok && (ranges_mode_ == 1 || (ranges_mode_ < 0 && dn_tiles >= kSms))) {
      p.down_ranges = true;
      p.splits = 1;
    }
  }
  if (L.I_sh > 0) {
    p.sh_umma = p.umma && umma_shapes_supported(L.gate_sh.fmt, L.down_sh.fmt, L.D, L.I_sh);
    p.sh_bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
    if (p.sh_umma) {
      p.sh_warp_mma = warp_mma_shapes_supported(L.gate_sh.fmt, L.down_sh.fmt, L.D, L.I_sh) &&
                      (path_ == 3 || path_ == 4 || (path_ == 0 && T <= 8));
      if (p.sh_warp_mma) p.sh_bn = T <= 8 ? 8 : 16;  // the shared expert owns every token: no spread
      p.sh_splits = pick_splits(((T + p.sh_bn - 1) / p.sh_bn) * (L.D / 128), umma_kchunks(L.down_sh.fmt, L.I_sh));
    }
  }
  return p;
}

// Routing + expert products + combine for device-resident x.
// `scores` rank the experts; `probs_for_w` supplies the weights (may equal scores).
namespace {
size_t expert_bytes(const ExpertWeights& w, int64_t E) { return (size_t)(E * w.rows) * row_bytes(w.fmt, w.cols); }
}  // namespace

// Packed rows as the tensor-core path reads them: in place when the row pitch is a
// multiple of 16 bytes (TMA strides), else a copy with each row padded to 16 bytes.
Error MoeCudaBackend::umma_rows(const void* w, int fmt, int64_t rows, int64_t K, bool constant, const void** out,
                                int64_t* pitch) {
  const int64_t rb = (int64_t)row_bytes(fmt, K);
  if (rb % 16 == 0) {
    *out = w;
    *pitch = rb;
    return Error::success();
  }
  const int64_t pp = umma_pitch(fmt, K);
  if (constant) {  // registered weights: pad once, keep the copy until the buffer is released
    const auto key = std::make_tuple(w, fmt, K, rows);
    auto it = padded_.find(key);
    if (it == padded_.end()) {
      void* d = nullptr;
      UAII_CUDA(cudaMalloc(&d, (size_t)(rows * pp)), "Malloc(padded weights)");
      cudaError_t st = launch_pad_rows(w, rb, rows, rb, d, pp, stream_);
      if (st != cudaSuccess) {
        (void)cudaFree(d);
        return cuda_status(st, "pad_rows");
      }
      count_launches(1);
      it = padded_.emplace(key, Padded{d, pp}).first;
    }
    *out = it->second.dev;
    *pitch = it->second.pitch;
    return Error::success();
  }
  void* d = carve((size_t)(rows * pp));
  UAII_CUDA(launch_pad_rows(w, rb, rows, rb, d, pp, stream_), "pad_rows");
  count_launches(1);
  *out = d;
  *pitch = pp;
  return Error::success();
}

Error MoeCudaBackend::run_experts(const float* xd, const float* scores, const float* probs_for_w,
                                  const LayerArgs& L, const ExpertPlan& P, int64_t T, void* yd, const EpRows* ep,
                                  const DecodeRoute* dr) {
  last_plan_ = P;
  if (ep && !P.umma)
    return Error::make(ErrorCode::NotImplemented,
                       "expert-parallel rows need the tensor-core path (Q4_0/Q8_0/Q4_K/Q6_K, tile-multiple shapes)");
  const int64_t D = L.D, E = L.E, I = L.I;
  const int k = L.top_k;
  const int64_t S = T * k;
  if (P.umma_refused)
    return Error::make(ErrorCode::NotImplemented,
                       "tensor-core path needs Q4_0/Q8_0/Q4_K/Q6_K weights, d_ff % 64 == 0 and d_model % 128 == 0 "
                       "(Q4_K/Q6_K: both multiples of 256; warp-MMA schedule: both multiples of 128)");
  RouteBuffers rb{};
  rb.topk_ids = static_cast<int32_t*>(carve(sizeof(int32_t) * S));
  rb.topk_w = static_cast<float*>(carve(sizeof(float) * S));
  rb.mask = static_cast<uint8_t*>(carve((size_t)(E * T)));
  rb.slot_local = static_cast<int32_t*>(carve(sizeof(int32_t) * S));
  rb.slot_of = static_cast<int32_t*>(carve(sizeof(int32_t) * S));
  rb.token_of = static_cast<int32_t*>(carve(sizeof(int32_t) * S));
  rb.counts = static_cast<int32_t*>(carve(sizeof(int32_t) * E));
  rb.offsets = static_cast<int32_t*>(carve(sizeof(int32_t) * (E + 1)));
  int32_t* tile_base = static_cast<int32_t*>(carve(sizeof(int32_t) * (E + 1)));
  int32_t* tile_base_dn = static_cast<int32_t*>(carve(sizeof(int32_t) * (E + 1)));

  const void *gd = nullptr, *ud = nullptr, *dd = nullptr;
  UAII_TRY(stage_weight(L.gate.data, (size_t)(E * I) * row_bytes(L.gate.fmt, D), &gd));
  UAII_TRY(stage_weight(L.up.data, (size_t)(E * I) * row_bytes(L.up.fmt, D), &ud));
  UAII_TRY(stage_weight(L.down.data, (size_t)(E * D) * row_bytes(L.down.fmt, I), &dd));

  float* out = nullptr;
  int splits = 1;
  phase_begin(kRoute);
  if (dr) {  // router, softmax, top-k and slot numbering in one launch
    UAII_CUDA(launch_route_decode(xd, dr->router_w, T, D, E, k, L.norm_topk, dr->logits, dr->probs, rb, route_done_,
                                  stream_),
              "route_decode");
    count_launches(1);
  } else {
    if (ep) {
      UAII_CUDA(launch_ep_route(ep->ids, ep->w, T, E, k, rb, stream_, ep->e_pitch), "ep_route");
    } else {
      UAII_CUDA(launch_route_topk(scores, probs_for_w, T, E, k, L.norm_topk, rb, stream_), "route_topk");
    }
    UAII_CUDA(launch_route_scan(T, E, k, rb, stream_), "route_scan");
  }
  if (P.umma) {
    // operand orders: x in the gate/up kernel's, h in the down kernel's (operand_order.cuh)
    const int sched = P.quad_mma ? kSchedQuadMma : P.warp_mma ? kSchedWarpMma : kSchedTcgen05;
    const int dn_sched = P.down_quad ? kSchedQuadMma : sched;
    const int x_order = P.quad_i8    ? kOrderQ4KI8
                        : P.quad_mma ? (L.gate.fmt == kQ4_K ? kOrderQ4K : kOrderQ6K)
                        : P.warp_mma ? kOrderWm
                                     : kOrderTc;
    const int h_order = dn_sched == kSchedQuadMma ? (L.down.fmt == kQ4_K ? kOrderQ4K : kOrderQ6K)
                        : P.warp_mma                ? kOrderWm
                                                    : kOrderTc;
    void* xp16 = carve(2 * (size_t)(S * D));
    void* h16 = carve(2 * (size_t)(S * I));
    void* xsum = nullptr;    // Q4_K on the quad schedule: the activations' sub-block sums
    float* xscale = nullptr;  // ... and with integer activations their dequant scales
    splits = P.splits;
    out = static_cast<float*>(carve(sizeof(float) * (size_t)(splits * S * D)));
    if (ep) {  // rows arrive in the tcgen05 operand order
      if (P.warp_mma) return Error::make(ErrorCode::Internal, "expert-parallel rows planned on the warp-MMA schedule");
      UAII_CUDA(launch_route_gather16(ep->x16, T, D, E, k, rb, xp16, stream_, ep->x_pitch), "route_gather16");
    } else {
      TileTables tt;  // built by the gather from the same counts: no tile-table launches
      tt.gu = tile_base;
      tt.dn = tile_base_dn;
      tt.bn = P.bn;
      tt.gu_mtiles = (int)(I / 64);
      tt.dn_mtiles = (int)(D / 128);
      tt.dn_splits = std::min(splits, umma_kchunks(L.down.fmt, I));
      if (P.quad_mma && L.gate.fmt == kQ4_K) tt.xsum = carve(2 * (size_t)(S * (D / 256) * 16));
      if (P.quad_i8) tt.xscale = static_cast<float*>(carve(sizeof(float) * (size_t)(S * (D / 256))));
      xsum = tt.xsum;
      xscale = tt.xscale;
      UAII_CUDA(launch_route_gather(xd, T, D, E, k, rb, nullptr, xp16, stream_, x_order, &tt), "route_gather");
    }
    const bool tables = ep == nullptr;
    phase_end();
    count_launches(3);
    phase_begin(kGateUp);
    int64_t gpitch = 0, dpitch = 0;
    UAII_TRY(umma_rows(gd, L.gate.fmt, E * I, D, weight_is_constant(L.gate.data, expert_bytes(L.gate, E)), &gd, &gpitch));
    UAII_TRY(umma_rows(ud, L.up.fmt, E * I, D, weight_is_constant(L.up.data, expert_bytes(L.up, E)), &ud, &gpitch));
    UAII_TRY(umma_rows(dd, L.down.fmt, E * D, I, weight_is_constant(L.down.data, expert_bytes(L.down, E)), &dd,
                       &dpitch));
    UAII_CUDA(launch_gateup_umma(L.gate.fmt, gd, ud, gpitch, E, I, D, xp16, S, rb.counts, rb.offsets, tile_base, P.bn,
                                 h16, dev_err_, stream_, sched, h_order, tables, xsum, &tail_, xscale),
              "gateup(tensor cores)");
    phase_end();
    phase_begin(kDown);
    UAII_CUDA(launch_down_umma(L.down.fmt, dd, dpitch, E, D, I, h16, S, rb.counts, rb.offsets,
                               tables ? tile_base_dn : tile_base, P.bn, splits, out, dev_err_, stream_, dn_sched,
                               tables, P.down_ranges ? &tail_ : nullptr),
              "down(tensor cores)");
    phase_end();
    count_launches(tables ? 2 : 4);
  } else {
    float* xp = static_cast<float*>(carve(sizeof(float) * S * D));
    float* h = static_cast<float*>(carve(sizeof(float) * S * I));
    out = static_cast<float*>(carve(sizeof(float) * S * D));
    UAII_CUDA(launch_route_gather(xd, T, D, E, k, rb, xp, nullptr, stream_), "route_gather");
    phase_end();
    count_launches(3);
    phase_begin(kGateUp);
    UAII_CUDA(launch_gateup_simt(L.gate.fmt, gd, L.up.fmt, ud, E, I, D, (int64_t)row_bytes(L.gate.fmt, D),
                                 (int64_t)row_bytes(L.up.fmt, D), xp, rb.offsets, rb.counts, h, stream_),
              "gateup");
    phase_end();
    phase_begin(kDown);
    UAII_CUDA(launch_down_simt(L.down.fmt, dd, E, D, I, (int64_t)row_bytes(L.down.fmt, I), h, rb.offsets,
                               rb.counts, out, stream_),
              "down");
    phase_end();
    count_launches(2);
  }

  float* sh_out = nullptr;
  float* sh_gate = nullptr;
  int sh_splits = 1;
  if (L.I_sh > 0) {
    const int64_t Is = L.I_sh;
    int32_t* sh_route = static_cast<int32_t*>(carve(sizeof(int32_t) * 4));
    int32_t* sh_tiles = static_cast<int32_t*>(carve(sizeof(int32_t) * 2));
    const void *sg = nullptr, *su = nullptr, *sd = nullptr;
    UAII_TRY(stage_weight(L.gate_sh.data, (size_t)Is * row_bytes(L.gate_sh.fmt, D), &sg));
    UAII_TRY(stage_weight(L.up_sh.data, (size_t)Is * row_bytes(L.up_sh.fmt, D), &su));
    UAII_TRY(stage_weight(L.down_sh.data, (size_t)D * row_bytes(L.down_sh.fmt, Is), &sd));
    phase_begin(kShared);
    UAII_CUDA(launch_identity_route(sh_route, T, stream_), "identity_route");
    if (P.sh_umma) {
      void* x16 = carve(2 * (size_t)(T * D));
      void* sh_h16 = carve(2 * (size_t)(T * Is));
      sh_splits = P.sh_splits;
      sh_out = static_cast<float*>(carve(sizeof(float) * (size_t)(sh_splits * T * D)));
      UAII_CUDA(launch_to_f16(xd, T * D, x16, stream_, P.sh_warp_mma), "shared_to_f16");
      int64_t sgp = 0, sdp = 0;
      UAII_TRY(umma_rows(sg, L.gate_sh.fmt, Is, D, weight_is_constant(L.gate_sh.data, expert_bytes(L.gate_sh, 1)), &sg,
                         &sgp));
      UAII_TRY(umma_rows(su, L.up_sh.fmt, Is, D, weight_is_constant(L.up_sh.data, expert_bytes(L.up_sh, 1)), &su,
                         &sgp));
      UAII_TRY(umma_rows(sd, L.down_sh.fmt, D, Is, weight_is_constant(L.down_sh.data, expert_bytes(L.down_sh, 1)), &sd,
                         &sdp));
      UAII_CUDA(launch_gateup_umma(L.gate_sh.fmt, sg, su, sgp, 1, Is, D, x16, T, sh_route + 2, sh_route, sh_tiles,
                                   P.sh_bn, sh_h16, dev_err_, stream_, P.sh_warp_mma),
                "shared_gateup(tensor cores)");
      UAII_CUDA(launch_down_umma(L.down_sh.fmt, sd, sdp, 1, D, Is, sh_h16, T, sh_route + 2, sh_route, sh_tiles, P.sh_bn,
                                 sh_splits, sh_out, dev_err_, stream_, P.sh_warp_mma),
                "shared_down(tensor cores)");
      count_launches(6);
    } else {
      float* sh_h = static_cast<float*>(carve(sizeof(float) * T * Is));
      sh_out = static_cast<float*>(carve(sizeof(float) * T * D));
      UAII_CUDA(launch_gateup_simt(L.gate_sh.fmt, sg, L.up_sh.fmt, su, 1, Is, D, (int64_t)row_bytes(L.gate_sh.fmt, D),
                                   (int64_t)row_bytes(L.up_sh.fmt, D), xd, sh_route, sh_route + 2, sh_h, stream_),
                "shared_gateup");
      UAII_CUDA(launch_down_simt(L.down_sh.fmt, sd, 1, D, Is, (int64_t)row_bytes(L.down_sh.fmt, Is), sh_h, sh_route,
                                 sh_route + 2, sh_out, stream_),
                "shared_down");
      count_launches(3);
    }
    if (L.gate_inp_sh) {
      const void* gw = nullptr;
      UAII_TRY(stage_weight(L.gate_inp_sh, sizeof(float) * (size_t)D, &gw));
      sh_gate = static_cast<float*>(carve(sizeof(float) * T));
      UAII_CUDA(launch_shared_gate(xd, static_cast<const float*>(gw), T, D, sh_gate, stream_), "shared_gate");
      count_launches(1);
    }
    phase_end();
  }
  phase_begin(kCombine);
  UAII_CUDA(launch_combine(out, D, splits, S * D, T, D, k, rb, sh_out, sh_splits, T * D, sh_gate, yd, stream_,
                           ep != nullptr && ep->y_f16),
            "combine");
  phase_end();
  count_launches(1);
  return Error::success();
}

namespace {

// pad_*: how many padded row copies (gate and up: 0..2) live in the workspace
// (unregistered sources)
size_t experts_ws_bytes(const LayerArgs& L, int64_t T, const ExpertPlan& P, int pad_gateup, bool pad_down,
                        int pad_gateup_sh, bool pad_down_sh) {
  const int64_t S = T * L.top_k;
  size_t b = 0;
  b += 5 * align_up(sizeof(int32_t) * S) + align_up((size_t)(L.E * T));
  b += 4 * align_up(sizeof(int32_t) * (L.E + 1));  // counts, offsets, two tile tables
  if (P.umma) {
    b += align_up(2 * (size_t)(S * L.D)) + align_up(2 * (size_t)(S * L.I)) +
         align_up(sizeof(float) * (size_t)(P.splits * S * L.D));
    if (P.quad_mma && L.gate.fmt == kQ4_K) b += align_up(2 * (size_t)(S * (L.D / 256) * 16));  // sub-block sums
    if (row_bytes(L.gate.fmt, L.D) % 16)
      b += (size_t)pad_gateup * align_up((size_t)(L.E * L.I * umma_pitch(L.gate.fmt, L.D)));
    if (pad_down && row_bytes(L.down.fmt, L.I) % 16)
      b += align_up((size_t)(L.E * L.D * umma_pitch(L.down.fmt, L.I)));
  }
  else
    b += 2 * align_up(sizeof(float) * S * L.D) + align_up(sizeof(float) * S * L.I);
  if (L.I_sh > 0) {
    b += 2 * kAlign + align_up(sizeof(float) * T);
    if (P.sh_umma) {
      b += align_up(2 * (size_t)(T * L.D)) + align_up(2 * (size_t)(T * L.I_sh)) +
           align_up(sizeof(float) * (size_t)(P.sh_splits * T * L.D));
      if (row_bytes(L.gate_sh.fmt, L.D) % 16)
        b += (size_t)pad_gateup_sh * align_up((size_t)(L.I_sh * umma_pitch(L.gate_sh.fmt, L.D)));
      if (pad_down_sh && row_bytes(L.down_sh.fmt, L.I_sh) % 16)
        b += align_up((size_t)(L.D * umma_pitch(L.down_sh.fmt, L.I_sh)));
    }
    else
      b += align_up(sizeof(float) * T * L.I_sh) + align_up(sizeof(float) * T * L.D);
  }
  return b + 16 * kAlign;
}

Error check_layer(const LayerArgs& L) {
  if (L.D <= 0 || L.E <= 0 || L.I <= 0)
    return Error::make(ErrorCode::InvalidArgument, "moe swiglu shape mismatch");
  if (L.E > 1024) return Error::make(ErrorCode::NotImplemented, "more than 1024 experts");
  if (L.top_k > 32) return Error::make(ErrorCode::NotImplemented, "top_k above 32");
  if (L.gate.fmt != L.up.fmt)
    return Error::make(ErrorCode::NotImplemented, "gate and up experts must share one format");
  UAII_TRY(check_cols("gate_exps", L.gate.fmt, L.D));
  UAII_TRY(check_cols("up_exps", L.up.fmt, L.D));
  UAII_TRY(check_cols("down_exps", L.down.fmt, L.I));
  if (L.I_sh > 0) {
    if (L.gate_sh.fmt != L.up_sh.fmt)
      return Error::make(ErrorCode::NotImplemented, "shared gate and up must share one format");
    UAII_TRY(check_cols("gate_shexp", L.gate_sh.fmt, L.D));
    UAII_TRY(check_cols("up_shexp", L.up_sh.fmt, L.D));
    UAII_TRY(check_cols("down_shexp", L.down_sh.fmt, L.I_sh));
  }
  return Error::success();
}

}  // namespace

size_t MoeCudaBackend::experts_ws(const LayerArgs& L, int64_t T, const ExpertPlan& P) const {
  auto copies = [&](const ExpertWeights& w, int64_t E) { return weight_is_constant(w.data, expert_bytes(w, E)) ? 0 : 1; };
  const bool sh = L.I_sh > 0;
  return experts_ws_bytes(L, T, P, copies(L.gate, L.E) + copies(L.up, L.E), copies(L.down, L.E) != 0,
                          sh ? copies(L.gate_sh, 1) + copies(L.up_sh, 1) : 0, sh && copies(L.down_sh, 1) != 0);
}

// ---------------------------------------------------------------- expert parallelism

// Dense projection with a packed weight: the reference's quant_gemm_f32
// (libs/uaii-kernels/src/quant_gemm.cpp:22-70, reached from dispatch_cpu's MatMul case,
// libs/uaii-kernels/src/dispatch.cpp:82-100).  One "expert" owning every row: the
// tensor-core down projection (f16 operands, f32 accumulate, K splits added in order),
// or the CUDA-core f32 GEMV for formats and shapes the tensor path does not take.
Error MoeCudaBackend::quant_matmul(const float* x, int64_t M, int64_t K, const void* w, int fmt, int64_t N,
                                   float* y, bool relu) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  if (!x || !w || !y || M < 0 || K <= 0 || N <= 0)
    return Error::make(ErrorCode::InvalidArgument, "quant_gemm shape mismatch");
  if (!fmt_is_gguf(fmt)) return Error::make(ErrorCode::InvalidArgument, "quant_gemm B quant unsupported");
  UAII_TRY(check_cols("quant_gemm B", fmt, K));
  if (M == 0) return Error::success();
  const size_t wbytes = (size_t)N * row_bytes(fmt, K);
  const bool tc = path_ != 1 && umma_down_supported(fmt, N, K, false);
  const bool wm = tc && umma_down_supported(fmt, N, K, true) && (path_ == 3 || path_ == 4 || (path_ == 0 && M <= 8));
  if ((path_ == 2 && !tc) || ((path_ == 3 || path_ == 4) && !wm))
    return Error::make(ErrorCode::NotImplemented,
                       "tensor-core quant matmul needs Q4_0/Q8_0/Q4_K/Q6_K weights, N % 128 == 0 and K a multiple "
                       "of the format's tile (64; K-quants 256; warp-MMA schedule 128)");
  const int bn = wm ? (M <= 8 ? 8 : 16) : (M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256);
  const int splits = tc ? pick_down_splits(((M + bn - 1) / bn) * (N / 128), umma_kchunks(fmt, K)) : 1;
  const bool const_w = weight_is_constant(w, wbytes);
  const size_t xb = sizeof(float) * (size_t)(M * K), yb = sizeof(float) * (size_t)(M * N);
  const bool planes = tc && (splits > 1 || relu);
  size_t ws = align_up(xb) + align_up(yb) + 2 * kAlign + weight_stage_bytes(w, wbytes);
  if (tc) {
    ws += align_up(2 * (size_t)(M * K));
    if (planes) ws += align_up(sizeof(float) * (size_t)splits * (size_t)(M * N));
    if (!const_w && row_bytes(fmt, K) % 16) ws += align_up((size_t)N * (size_t)umma_pitch(fmt, K));
  }
  UAII_TRY(reserve(ws + 4 * kAlign));
  void* xs = carve(xb);
  float* ys = static_cast<float*>(carve(yb));
  int32_t* route = static_cast<int32_t*>(carve(sizeof(int32_t) * 4));
  int32_t* tiles = static_cast<int32_t*>(carve(sizeof(int32_t) * 2));
  const void *xd = nullptr, *wd = nullptr;
  bool xh = false;
  UAII_TRY(stage_input(x, xb, xs, &xd, &xh));
  UAII_TRY(stage_weight(w, wbytes, &wd));
  const bool yh = !is_device_ptr(y);
  float* yo = yh ? ys : y;
  ExpertPlan P;
  P.umma = tc;
  P.warp_mma = wm;
  P.bn = bn;
  P.splits = splits;
  last_plan_ = P;
  phase_begin(kDown);
  if (tc) {
    // one prep launch: f16 operand rows, the one-expert route (offsets {0, M}, counts {M}), the tile table
    void* x16 = carve(2 * (size_t)(M * K));
    UAII_CUDA(launch_to_f16_route(static_cast<const float*>(xd), M, K, x16, wm, route, tiles, bn, (int)(N / 128),
                                  std::min(splits, umma_kchunks(fmt, K)), stream_),
              "to_f16_route");
    int64_t pitch = 0;
    UAII_TRY(umma_rows(wd, fmt, N, K, const_w, &wd, &pitch));
    float* out = planes ? static_cast<float*>(carve(sizeof(float) * (size_t)splits * (size_t)(M * N))) : yo;
    UAII_CUDA(launch_down_umma(fmt, wd, pitch, 1, N, K, x16, M, route + 2, route, tiles, bn, splits, out, dev_err_,
                               stream_, wm, true),
              "quant_matmul(tensor cores)");
    count_launches(2);
    if (planes) {
      UAII_CUDA(launch_sum_planes(out, splits, M * N, M * N, yo, relu, stream_), "sum_planes");
      count_launches(1);
    }
  } else {
    UAII_CUDA(launch_identity_route(route, M, stream_), "identity_route");  // offsets {0, M}, counts {M}
    UAII_CUDA(launch_down_simt(fmt, wd, 1, N, K, (int64_t)row_bytes(fmt, K), static_cast<const float*>(xd), route,
                               route + 2, yo, stream_),
              "quant_matmul");
    count_launches(2);
    if (relu) {
      UAII_CUDA(launch_sum_planes(yo, 1, 0, M * N, yo, true, stream_), "relu");
      count_launches(1);
    }
  }
  phase_end();
  if (yh) {
    UAII_CUDA(cudaMemcpyAsync(y, yo, yb, cudaMemcpyDeviceToHost, stream_), "D2H");
    UAII_TRY(sync_and_check());
  }
  (void)xh;
  return Error::success();
}

Error MoeCudaBackend::ep_dispatch(const LayerArgs& L, const float* x, int64_t T, int rank, int world,
                                  void* send_x16, int32_t* send_ids, float* send_w, int32_t* send_token,
                                  int32_t* row_of, int32_t* send_counts, int32_t* send_entries, float* probs,
                                  int64_t x_pitch, int64_t e_pitch) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  const int64_t D = L.D, E = L.E;
  const int k = L.top_k;
  if (!L.router_w || D <= 0 || E <= 0 || k < 1 || k > 32 || k > E || T < 0)
    return Error::make(ErrorCode::InvalidArgument, "ep dispatch: router weight, d_model, n_experts, top_k");
  if (world < 1 || world > 255 || rank < 0 || rank >= world || E % world != 0)
    return Error::make(ErrorCode::InvalidArgument, "ep dispatch: world must divide n_experts (1..255 ranks)");
  for (const void* p : {static_cast<const void*>(x), static_cast<const void*>(L.router_w),
                        static_cast<const void*>(send_x16),
                        static_cast<const void*>(send_ids), static_cast<const void*>(send_w),
                        static_cast<const void*>(send_token), static_cast<const void*>(row_of),
                        static_cast<const void*>(send_counts), static_cast<const void*>(send_entries)})
    if (!is_device_ptr(p)) return Error::make(ErrorCode::InvalidArgument, "ep dispatch: arguments must be device memory");
  if (probs && !is_device_ptr(probs)) return Error::make(ErrorCode::InvalidArgument, "ep dispatch: probs must be device memory");
  const size_t lb = sizeof(float) * (size_t)(T * E);
  const size_t rsb = router_scratch_bytes(T, D, E);
  UAII_TRY(reserve(3 * align_up(lb) + 2 * align_up(sizeof(int32_t) * (size_t)(T * k)) + align_up((size_t)(E * T)) +
                   align_up((size_t)(world * T)) + align_up(sizeof(int32_t) * (size_t)(T * world)) +
                   align_up(sizeof(int32_t) * (size_t)world) + align_up(rsb) + 5 * kAlign));
  float* logits = static_cast<float*>(carve(lb));
  float* po = probs ? probs : static_cast<float*>(carve(lb));
  RouteBuffers rb{};
  rb.topk_ids = static_cast<int32_t*>(carve(sizeof(int32_t) * (size_t)(T * k)));
  rb.topk_w = static_cast<float*>(carve(sizeof(float) * (size_t)(T * k)));
  rb.mask = static_cast<uint8_t*>(carve((size_t)(E * T)));
  uint8_t* dmask = static_cast<uint8_t*>(carve((size_t)(world * T)));
  int32_t* rowpos = static_cast<int32_t*>(carve(sizeof(int32_t) * (size_t)(T * world)));
  int32_t* dcounts = static_cast<int32_t*>(carve(sizeof(int32_t) * (size_t)world));
  float* rscratch = rsb ? static_cast<float*>(carve(rsb)) : nullptr;
  const int epr = (int)(E / world);
  phase_begin(kRouter);
  UAII_CUDA(launch_router(x, L.router_w, T, D, E, logits, po, nullptr, stream_, rscratch, rsb), "router");
  phase_end();
  phase_begin(kRoute);
  UAII_CUDA(launch_route_topk(logits, po, T, E, k, L.norm_topk, rb, stream_), "route_topk");
  UAII_CUDA(launch_ep_plan(rb.topk_ids, T, k, world, epr, dmask, rowpos, dcounts, stream_), "ep_plan");
  UAII_CUDA(launch_ep_pack(x, T, D, k, world, epr, rb.topk_ids, rb.topk_w, dmask, rowpos, dcounts, send_x16, send_ids,
                           send_w, send_token, row_of, send_counts, send_entries, stream_, x_pitch, e_pitch),
            "ep_pack");
  phase_end();
  count_launches(7);
  (void)rank;
  return Error::success();
}

Error MoeCudaBackend::ep_experts(const LayerArgs& Lin, const void* recv_x16, const int32_t* recv_ids,
                                 const float* recv_w, int64_t N, int64_t entries, void* y_part, int64_t x_pitch,
                                 int64_t e_pitch, bool y_f16) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  LayerArgs L = Lin;
  UAII_TRY(check_layer(L));
  if (L.I_sh > 0)
    return Error::make(ErrorCode::NotImplemented, "ep experts: the shared expert runs on the token's own rank");
  if (N < 0 || entries < 0 || entries > N * L.top_k)
    return Error::make(ErrorCode::InvalidArgument, "ep experts: rows / entries");
  if (N == 0) return Error::success();
  for (const void* p : {static_cast<const void*>(recv_x16), static_cast<const void*>(recv_ids),
                        static_cast<const void*>(recv_w),
                        static_cast<const void*>(y_part)})
    if (!is_device_ptr(p)) return Error::make(ErrorCode::InvalidArgument, "ep experts: arguments must be device memory");
  const ExpertPlan P = plan_experts(L, N, entries, /*allow_warp_mma=*/false);
  UAII_TRY(reserve(experts_ws(L, N, P) + layer_stage_bytes(L)));
  if (y_f16 && L.D % 4 != 0) return Error::make(ErrorCode::InvalidArgument, "ep experts: f16 rows need d_model % 4 == 0");
  const EpRows rows{recv_x16, recv_ids, recv_w, x_pitch, e_pitch, y_f16};
  return run_experts(nullptr, nullptr, nullptr, L, P, N, y_part, &rows);
}

Error MoeCudaBackend::selftest_wait_timeout(int64_t budget_cycles) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  constexpr int kSelftestCode = 9;
  UAII_CUDA(launch_wait_timeout_selftest(dev_err_, (long long)budget_cycles, kSelftestCode, stream_),
            "wait_timeout_selftest");
  count_launches(1);
  return sync_and_check();
}

Error MoeCudaBackend::ep_combine(const void* y_back, const int32_t* row_of, int64_t T, int world, int64_t D,
                                 float* y, bool y_back_f16) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  if (T < 0 || D <= 0 || world < 1) return Error::make(ErrorCode::InvalidArgument, "ep combine: shapes");
  if (T == 0) return Error::success();
  for (const void* p : {static_cast<const void*>(y_back), static_cast<const void*>(row_of),
                        static_cast<const void*>(y)})
    if (!is_device_ptr(p)) return Error::make(ErrorCode::InvalidArgument, "ep combine: arguments must be device memory");
  phase_begin(kCombine);
  if (y_back_f16) UAII_CUDA(launch_ep_combine_f16(y_back, row_of, T, world, D, y, stream_), "ep_combine_f16");
  else UAII_CUDA(launch_ep_combine(static_cast<const float*>(y_back), row_of, T, world, D, y, stream_), "ep_combine");
  phase_end();
  count_launches(1);
  return Error::success();
}

size_t MoeCudaBackend::layer_stage_bytes(const LayerArgs& L) const {
  size_t b = weight_stage_bytes(L.gate.data, expert_bytes(L.gate, L.E)) +
             weight_stage_bytes(L.up.data, expert_bytes(L.up, L.E)) +
             weight_stage_bytes(L.down.data, expert_bytes(L.down, L.E));
  if (L.router_w) b += weight_stage_bytes(L.router_w, sizeof(float) * (size_t)(L.E * L.D));
  if (L.I_sh > 0) {
    b += weight_stage_bytes(L.gate_sh.data, expert_bytes(L.gate_sh, 1)) +
         weight_stage_bytes(L.up_sh.data, expert_bytes(L.up_sh, 1)) +
         weight_stage_bytes(L.down_sh.data, expert_bytes(L.down_sh, 1));
    if (L.gate_inp_sh) b += weight_stage_bytes(L.gate_inp_sh, sizeof(float) * (size_t)L.D);
  }
  return b;
}

Error MoeCudaBackend::experts(const float* x, const ExpertWeights& g, const ExpertWeights& u,
                              const ExpertWeights& d, const float* probs, int64_t T, int64_t D,
                              int64_t E, int64_t I, int top_k, int norm_topk, float* y) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  LayerArgs L;
  L.D = D; L.E = E; L.I = I;
  // transformer.cpp:562-563: k = top_k > 0 ? top_k : 1, clamped to E
  int k = top_k > 0 ? top_k : 1;
  if (k > E) k = (int)E;
  L.top_k = k;
  L.norm_topk = norm_topk;
  L.gate = g; L.up = u; L.down = d;
  UAII_TRY(check_layer(L));
  if (T < 0 || !x || !probs || !y) return Error::make(ErrorCode::InvalidArgument, "moe swiglu args");
  if (T == 0) return Error::success();
  const size_t xb = sizeof(float) * (size_t)(T * D), pb = sizeof(float) * (size_t)(T * E);
  const ExpertPlan P = plan_experts(L, T);
  UAII_TRY(reserve(experts_ws(L, T, P) + 2 * align_up(xb) + align_up(pb) + layer_stage_bytes(L)));
  void* xs = carve(xb);
  void* ps = carve(pb);
  float* ys = static_cast<float*>(carve(xb));
  const void *xd = nullptr, *pd = nullptr;
  bool xh = false, ph = false;
  UAII_TRY(stage_input(x, xb, xs, &xd, &xh));
  UAII_TRY(stage_input(probs, pb, ps, &pd, &ph));
  const bool yh = !is_device_ptr(y);
  float* yo = yh ? ys : y;
  UAII_TRY(run_experts(static_cast<const float*>(xd), static_cast<const float*>(pd),
                       static_cast<const float*>(pd), L, P, T, yo));
  if (yh) {
    UAII_CUDA(cudaMemcpyAsync(y, yo, xb, cudaMemcpyDeviceToHost, stream_), "MemcpyAsync(D2H)");
    UAII_TRY(sync_and_check());
  }
  return Error::success();
}

void MoeCudaBackend::drop_graphs() {
  for (auto& kv : graphs_)
    if (kv.second.exec) (void)cudaGraphExecDestroy(kv.second.exec);
  graphs_.clear();
}

// The launches of one layer forward (router, routing, expert GEMMs, combine).
Error MoeCudaBackend::ffn_launch(const LayerArgs& L, const ExpertPlan& P, int64_t T, const float* xd, const float* wd,
                                 float* logits, float* po, float* rscratch, size_t rsb, float* yo) {
  if (route_done_ != nullptr && route_decode_supported(T, L.D, L.E, L.top_k)) {  // one routing launch
    const DecodeRoute dr{wd, logits, po};
    return run_experts(xd, logits, po, L, P, T, yo, nullptr, &dr);
  }
  phase_begin(kRouter);
  UAII_CUDA(launch_router(xd, wd, T, L.D, L.E, logits, po, nullptr, stream_, rscratch, rsb), "router");
  phase_end();
  count_launches(2);
  // Rank on the exact logits (same order as the probabilities), weight with probs.
  return run_experts(xd, logits, po, L, P, T, yo);
}

Error MoeCudaBackend::ensure_copy_streams(int chunks) {
  if (!in_stream_) UAII_CUDA(cudaStreamCreateWithFlags(&in_stream_, cudaStreamNonBlocking), "StreamCreate(in)");
  if (!out_stream_) UAII_CUDA(cudaStreamCreateWithFlags(&out_stream_, cudaStreamNonBlocking), "StreamCreate(out)");
  while ((int)chunk_events_.size() < 2 * chunks + 1) {
    cudaEvent_t e = nullptr;
    UAII_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "EventCreate");
    chunk_events_.push_back(e);
  }
  return Error::success();
}

// Chunk c: its x rows go host -> device on in_stream_, the layer runs on stream_ once
// they have landed, and its y rows (and probabilities) go back on out_stream_ once the
// layer is done, so the copies of chunk c+1 (in) and c-1 (out) overlap the layer of c.
// Token rows are independent (the reference's GEMMs tile over rows only), so chunking
// changes only the order of work and, through each chunk's plan, the grouping of the
// down projection's f32 partial sums.  Returns after the last copy back.
Error MoeCudaBackend::ffn_host_chunked(const LayerArgs& L, const float* x, int64_t T, float* y, float* probs,
                                       int chunks) {
  const int64_t D = L.D, E = L.E;
  const int64_t tc_max = (T + chunks - 1) / chunks;
  const size_t xb = sizeof(float) * (size_t)(T * D), pb = sizeof(float) * (size_t)(T * E);
  const ExpertPlan Pmax = plan_experts(L, tc_max);
  const size_t rsb = router_scratch_bytes(tc_max, D, E);
  UAII_TRY(ensure_copy_streams(chunks));
  UAII_TRY(reserve(experts_ws(L, tc_max, Pmax) + 2 * align_up(xb) + 2 * align_up(pb) + align_up(rsb)));
  float* xs = static_cast<float*>(carve(xb));
  float* ys = static_cast<float*>(carve(xb));
  float* logits = static_cast<float*>(carve(pb));
  float* ps = static_cast<float*>(carve(pb));
  float* rscratch = rsb ? static_cast<float*>(carve(rsb)) : nullptr;
  const void* wd = nullptr;
  UAII_TRY(stage_weight(L.router_w, sizeof(float) * (size_t)(E * D), &wd));
  const size_t mark = ws_used_;
  cudaEvent_t* ev = chunk_events_.data();
  // the copies in must not overtake work of an earlier call that still reads the staging buffers
  UAII_CUDA(cudaEventRecord(ev[2 * chunks], stream_), "EventRecord");
  UAII_CUDA(cudaStreamWaitEvent(in_stream_, ev[2 * chunks], 0), "StreamWaitEvent");
  for (int c = 0; c < chunks; ++c) {
    const int64_t t0 = T * c / chunks, t1 = T * (c + 1) / chunks;
    UAII_CUDA(cudaMemcpyAsync(xs + t0 * D, x + t0 * D, sizeof(float) * (size_t)((t1 - t0) * D),
                              cudaMemcpyHostToDevice, in_stream_), "MemcpyAsync(H2D chunk)");
    UAII_CUDA(cudaEventRecord(ev[2 * c], in_stream_), "EventRecord");
  }
  ExpertPlan last{};
  for (int c = 0; c < chunks; ++c) {
    const int64_t t0 = T * c / chunks, t1 = T * (c + 1) / chunks, tc = t1 - t0;
    UAII_CUDA(cudaStreamWaitEvent(stream_, ev[2 * c], 0), "StreamWaitEvent");
    ws_used_ = mark;  // chunks run one after another on stream_: each reuses the same expert workspace
    const ExpertPlan P = plan_experts(L, tc);
    UAII_TRY(ffn_launch(L, P, tc, xs + t0 * D, static_cast<const float*>(wd), logits + t0 * E, ps + t0 * E, rscratch,
                        router_scratch_bytes(tc, D, E), ys + t0 * D));
    last = P;
    UAII_CUDA(cudaEventRecord(ev[2 * c + 1], stream_), "EventRecord");
    UAII_CUDA(cudaStreamWaitEvent(out_stream_, ev[2 * c + 1], 0), "StreamWaitEvent");
    UAII_CUDA(cudaMemcpyAsync(y + t0 * D, ys + t0 * D, sizeof(float) * (size_t)(tc * D), cudaMemcpyDeviceToHost,
                              out_stream_), "MemcpyAsync(D2H chunk)");
    if (probs)
      UAII_CUDA(cudaMemcpyAsync(probs + t0 * E, ps + t0 * E, sizeof(float) * (size_t)(tc * E), cudaMemcpyDeviceToHost,
                                out_stream_), "MemcpyAsync(D2H chunk)");
  }
  last_plan_ = last;
  UAII_CUDA(cudaStreamSynchronize(out_stream_), "StreamSynchronize(out)");
  return sync_and_check();
}

Error MoeCudaBackend::ffn(const LayerArgs& Lin, const float* x, int64_t T, float* y, float* probs) {
  std::lock_guard<std::mutex> lk(mu_);
  UAII_CUDA(cudaSetDevice(device_), "SetDevice");
  LayerArgs L = Lin;
  int k = L.top_k > 0 ? L.top_k : 1;
  if (k > L.E) k = (int)L.E;
  L.top_k = k;
  UAII_TRY(check_layer(L));
  if (!L.router_w || !x || !y) return Error::make(ErrorCode::InvalidArgument, "moe ffn args");
  if (T < 0) return Error::make(ErrorCode::InvalidArgument, "moe ffn: negative token count");
  if (T == 0) return Error::success();
  const int64_t D = L.D, E = L.E;
  // Large batches in and out of host memory: copies overlapped with the layer, in chunks
  // of at least 2048 tokens (at most 8 chunks), when no weight has to be staged per call.
  // Smaller chunks lose more in the expert products (each chunk decodes every weight tile
  // again, and its experts' last slot tiles are partly empty; Mixtral-shaped layer, 4096
  // tokens: one call 2.55 ms, 2 x 2048 tokens 3.06 ms, 4 x 1024 tokens 4.28 ms) than
  // their copies hide.
  if (!external_ && T >= 4096 && !is_device_ptr(x) && !is_device_ptr(y) && (!probs || !is_device_ptr(probs)) &&
      layer_stage_bytes(L) == 0)
    return ffn_host_chunked(L, x, T, y, probs, (int)std::min<int64_t>(8, T / 2048));
  const size_t xb = sizeof(float) * (size_t)(T * D), pb = sizeof(float) * (size_t)(T * E);
  const ExpertPlan P = plan_experts(L, T);
  const size_t rsb = router_scratch_bytes(T, D, E);
  UAII_TRY(reserve(experts_ws(L, T, P) + 2 * align_up(xb) + 2 * align_up(pb) + align_up(rsb) +
                   layer_stage_bytes(L)));
  void* xs = carve(xb);
  float* ys = static_cast<float*>(carve(xb));
  float* logits = static_cast<float*>(carve(pb));
  float* ps = static_cast<float*>(carve(pb));
  float* rscratch = rsb ? static_cast<float*>(carve(rsb)) : nullptr;
  const void *xd = nullptr, *wd = nullptr;
  bool xh = false;
  UAII_TRY(stage_input(x, xb, xs, &xd, &xh));
  UAII_TRY(stage_weight(L.router_w, sizeof(float) * (size_t)(E * D), &wd));
  const bool ph = probs != nullptr && !is_device_ptr(probs);
  float* po = (probs && !ph) ? probs : ps;
  const bool yh = !is_device_ptr(y);
  float* yo = yh ? ys : y;
  // Device-resident calls with device (or registered) weights are pure launch sequences:
  // replayed from a CUDA graph once the same call has been seen twice.
  const bool graphable = graphs_on_ && !profiling_ && !external_ && !xh && !yh && !ph && layer_stage_bytes(L) == 0;
  GraphEntry* ge = nullptr;
  if (graphable) {
    const std::vector<int64_t> key = {
        T, L.D, L.E, L.I, L.top_k, L.norm_topk, L.I_sh, path_,
        (int64_t)(uintptr_t)x, (int64_t)(uintptr_t)y, (int64_t)(uintptr_t)probs, (int64_t)(uintptr_t)L.router_w,
        (int64_t)(uintptr_t)L.gate.data, L.gate.fmt, (int64_t)(uintptr_t)L.up.data, L.up.fmt,
        (int64_t)(uintptr_t)L.down.data, L.down.fmt, (int64_t)(uintptr_t)L.gate_sh.data, L.gate_sh.fmt,
        (int64_t)(uintptr_t)L.up_sh.data, L.up_sh.fmt, (int64_t)(uintptr_t)L.down_sh.data, L.down_sh.fmt,
        (int64_t)(uintptr_t)L.gate_inp_sh, (int64_t)(uintptr_t)ws_};
    if (graphs_.size() >= 64 && !graphs_.count(key)) drop_graphs();  // bound the cache (varying batch sizes)
    ge = &graphs_[key];
    if (ge->exec) {
      UAII_CUDA(cudaGraphLaunch(ge->exec, stream_), "GraphLaunch");
      count_launches(ge->launches);
      last_plan_ = P;
      return Error::success();
    }
    if (ge->seen++ < 1) ge = nullptr;  // first sighting: plain launches (settles workspace and padded copies)
  }
  if (ge) {
    UAII_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "StreamBeginCapture");
    const uint64_t before = launches_;
    const Error e = ffn_launch(L, P, T, static_cast<const float*>(xd), static_cast<const float*>(wd), logits, po,
                               rscratch, rsb, yo);
    ge->launches = launches_ - before;
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(stream_, &graph);
    if (!e.ok()) {
      if (graph) (void)cudaGraphDestroy(graph);
      return e;
    }
    UAII_CUDA(ce, "StreamEndCapture");
    const cudaError_t ie = cudaGraphInstantiate(&ge->exec, graph, 0);
    (void)cudaGraphDestroy(graph);
    UAII_CUDA(ie, "GraphInstantiate");
    UAII_CUDA(cudaGraphLaunch(ge->exec, stream_), "GraphLaunch");
    return Error::success();
  }
  UAII_TRY(ffn_launch(L, P, T, static_cast<const float*>(xd), static_cast<const float*>(wd), logits, po, rscratch,
                      rsb, yo));
  bool any_host = false;
  if (yh) { UAII_CUDA(cudaMemcpyAsync(y, yo, xb, cudaMemcpyDeviceToHost, stream_), "D2H"); any_host = true; }
  if (ph) { UAII_CUDA(cudaMemcpyAsync(probs, po, pb, cudaMemcpyDeviceToHost, stream_), "D2H"); any_host = true; }
  if (any_host) UAII_TRY(sync_and_check());
  return Error::success();
}

// ---------------------------------------------------------------------------
// IBackend::dispatch seam.  Arity checks, attribute names and defaults follow
// kernels::dispatch_cpu (libs/uaii-kernels/src/dispatch.cpp:224-248); shape
// checks follow moe_router_f32 / moe_experts_swiglu_f32 (transformer.cpp:446-560).
namespace {

int64_t attr_int(const std::vector<Attribute>& attrs, const char* key, int64_t def) {
  for (const auto& a : attrs)
    if (a.key == key && (a.type == AttrType::Int || a.type == AttrType::Bool)) return a.i;
  return def;
}

Error weight_fmt(const TensorView& t, int* fmt) {
  if (fmt_is_gguf(t.quant_format)) { *fmt = t.quant_format; return Error::success(); }
  if (t.dtype == DType::F32) { *fmt = kF32; return Error::success(); }
  if (t.dtype == DType::F16) { *fmt = kF16; return Error::success(); }
  return Error::make(ErrorCode::NotImplemented, "unsupported expert weight type");
}

Error expert_view(const TensorView& t, const char* name, int64_t E, int64_t rows, int64_t cols,
                  ExpertWeights* w) {
  if (t.rank != 3 || t.dim(0) != E || t.dim(1) != rows || t.dim(2) != cols)
    return Error::make(ErrorCode::InvalidArgument, std::string("moe swiglu shape mismatch (") + name + ")");
  UAII_TRY(weight_fmt(t, &w->fmt));
  const uint64_t need = (uint64_t)(E * rows) * row_bytes(w->fmt, cols);
  if (t.nbytes != 0 && t.nbytes < need)
    return Error::make(ErrorCode::InvalidArgument, std::string(name) + ": buffer smaller than its shape");
  w->data = t.data;
  w->rows = rows;
  w->cols = cols;
  return Error::success();
}

Error f32_2d(const TensorView& t, const char* name) {
  if (t.dtype != DType::F32 || t.rank != 2 || t.data == nullptr)
    return Error::make(ErrorCode::InvalidArgument, std::string(name) + " must be rank-2 f32 with data");
  return Error::success();
}

}  // namespace

Error MoeCudaBackend::dispatch(const std::string& op_name, const std::string& /*op_version*/,
                               const std::vector<TensorView>& inputs,
                               std::vector<TensorView>* outputs,
                               const std::vector<Attribute>& attrs) {
  if (outputs == nullptr || outputs->empty())
    return Error::make(ErrorCode::InvalidArgument, "dispatch outputs empty");
  if (op_name == "MoERouter") {
    if (inputs.size() != 2 || outputs->size() < 2)
      return Error::make(ErrorCode::InvalidArgument, "MoERouter expects x,gate -> probs,top_expert");
    const TensorView &x = inputs[0], &g = inputs[1];
    TensorView &p = (*outputs)[0], &t = (*outputs)[1];
    if (x.rank != 2 || g.rank != 2) return Error::make(ErrorCode::InvalidArgument, "moe router ranks");
    UAII_TRY(f32_2d(x, "x"));
    UAII_TRY(f32_2d(g, "gate"));
    const int64_t T = x.dim(0), D = x.dim(1), E = g.dim(0);
    if (g.dim(1) != D) return Error::make(ErrorCode::InvalidArgument, "matmul shape mismatch");
    if (p.rank != 2 || p.dim(0) != T || p.dim(1) != E)
      return Error::make(ErrorCode::InvalidArgument, "matmul output shape mismatch");
    if (t.rank != 2 || t.dim(0) != T || t.dim(1) != 1)
      return Error::make(ErrorCode::InvalidArgument, "top_expert shape");
    return router(static_cast<const float*>(x.data), static_cast<const float*>(g.data), T, D, E,
                  static_cast<float*>(p.data), static_cast<float*>(t.data), nullptr);
  }
  if (op_name == "MoEExperts") {
    // checks in the order of dispatch_cpu and moe_experts_f32 (dispatch.cpp:231-238,
    // transformer.cpp:483-500); out and top_expert extents are checked as well here
    if (inputs.size() != 3 || outputs->size() != 1)
      return Error::make(ErrorCode::InvalidArgument, "MoEExperts expects x,experts_w,top_expert");
    const TensorView &x = inputs[0], &w = inputs[1], &top = inputs[2];
    TensorView& y = (*outputs)[0];
    if (x.rank != 2 || y.rank != 2 || w.rank != 3)
      return Error::make(ErrorCode::InvalidArgument, "moe experts expects x[B,D], W[E,D,D], out[B,D]");
    const int64_t B = x.dim(0), D = x.dim(1);
    const int64_t num_experts = attr_int(attrs, "num_experts", 1);
    if (w.dim(0) != num_experts || w.dim(1) != D || w.dim(2) != D)
      return Error::make(ErrorCode::InvalidArgument, "experts_w shape");
    if (y.dim(0) != B || y.dim(1) != D)
      return Error::make(ErrorCode::InvalidArgument, "moe experts expects x[B,D], W[E,D,D], out[B,D]");
    int64_t top_n = 1;
    for (size_t i = 0; i < top.rank; ++i) top_n *= top.shape[i];
    if (top.dtype != DType::F32 || top.data == nullptr || top_n < B)
      return Error::make(ErrorCode::InvalidArgument, "top_expert must be f32 with one id per row");
    if (w.dtype != DType::F32 || w.data == nullptr || fmt_is_gguf(w.quant_format))
      return Error::make(ErrorCode::NotImplemented, "MoEExperts takes dense f32 expert weights");
    UAII_TRY(f32_2d(x, "x"));
    UAII_TRY(f32_2d(y, "out"));
    return experts_linear(static_cast<const float*>(x.data), static_cast<const float*>(w.data),
                          static_cast<const float*>(top.data), B, D, num_experts, static_cast<float*>(y.data));
  }
  if (op_name == "MoEExpertsSwiGLU") {
    if (inputs.size() != 5 || outputs->size() != 1)
      return Error::make(ErrorCode::InvalidArgument, "MoEExpertsSwiGLU expects x,gate,up,down,probs");
    const TensorView& x = inputs[0];
    const TensorView& p = inputs[4];
    TensorView& y = (*outputs)[0];
    if (x.rank != 2 || y.rank != 2 || inputs[1].rank != 3 || inputs[2].rank != 3 ||
        inputs[3].rank != 3 || p.rank != 2)
      return Error::make(ErrorCode::InvalidArgument,
                         "moe swiglu expects x[B,D], gate/up[E,I,D], down[E,D,I], probs[B,E]");
    const int64_t T = x.dim(0), D = x.dim(1), E = inputs[1].dim(0), I = inputs[1].dim(1);
    const int64_t num_experts = attr_int(attrs, "num_experts", 1);
    if (E != num_experts || p.dim(0) != T || p.dim(1) != E || y.dim(0) != T || y.dim(1) != D)
      return Error::make(ErrorCode::InvalidArgument, "moe swiglu shape mismatch");
    ExpertWeights g, u, d;
    UAII_TRY(expert_view(inputs[1], "gate_exps", E, I, D, &g));
    UAII_TRY(expert_view(inputs[2], "up_exps", E, I, D, &u));
    UAII_TRY(expert_view(inputs[3], "down_exps", E, D, I, &d));
    UAII_TRY(f32_2d(x, "x"));
    UAII_TRY(f32_2d(p, "probs"));
    return experts(static_cast<const float*>(x.data), g, u, d, static_cast<const float*>(p.data), T, D,
                   E, I, (int)attr_int(attrs, "top_k", 2), (int)attr_int(attrs, "norm_topk", 1),
                   static_cast<float*>(y.data));
  }
  if (op_name == "MoEFFN") {
    if ((inputs.size() != 5 && inputs.size() != 8 && inputs.size() != 9) || outputs->empty() ||
        outputs->size() > 2)
      return Error::make(ErrorCode::InvalidArgument,
                         "MoEFFN expects x,gate,gate_exps,up_exps,down_exps[,shexp x3[,gate_inp_shexp]]");
    const TensorView& x = inputs[0];
    UAII_TRY(f32_2d(x, "x"));
    UAII_TRY(f32_2d(inputs[1], "gate"));
    const int64_t T = x.dim(0), D = x.dim(1), E = inputs[1].dim(0);
    if (inputs[2].rank != 3) return Error::make(ErrorCode::InvalidArgument, "gate_exps must be rank 3");
    const int64_t I = inputs[2].dim(1);
    LayerArgs L;
    L.D = D; L.E = E; L.I = I;
    L.top_k = (int)attr_int(attrs, "top_k", 2);
    L.norm_topk = (int)attr_int(attrs, "norm_topk", 1);
    L.router_w = static_cast<const float*>(inputs[1].data);
    if (inputs[1].dim(1) != D) return Error::make(ErrorCode::InvalidArgument, "router shape mismatch");
    UAII_TRY(expert_view(inputs[2], "gate_exps", E, I, D, &L.gate));
    UAII_TRY(expert_view(inputs[3], "up_exps", E, I, D, &L.up));
    UAII_TRY(expert_view(inputs[4], "down_exps", E, D, I, &L.down));
    if (inputs.size() >= 8) {
      if (inputs[5].rank != 2) return Error::make(ErrorCode::InvalidArgument, "gate_shexp must be rank 2");
      L.I_sh = inputs[5].dim(0);
      const int64_t one = 1;
      TensorView v;
      for (int j = 0; j < 3; ++j) {
        v = inputs[5 + j];
        const int64_t shp[3] = {one, v.dim(0), v.dim(1)};
        v.shape = shp;
        v.rank = 3;
        ExpertWeights* dst = j == 0 ? &L.gate_sh : j == 1 ? &L.up_sh : &L.down_sh;
        const int64_t rows = j == 2 ? D : L.I_sh, cols = j == 2 ? L.I_sh : D;
        UAII_TRY(expert_view(v, j == 0 ? "gate_shexp" : j == 1 ? "up_shexp" : "down_shexp", 1, rows, cols, dst));
      }
      if (inputs.size() == 9) L.gate_inp_sh = static_cast<const float*>(inputs[8].data);
    }
    TensorView& y = (*outputs)[0];
    if (y.rank != 2 || y.dim(0) != T || y.dim(1) != D)
      return Error::make(ErrorCode::InvalidArgument, "MoEFFN output shape mismatch");
    float* probs = outputs->size() == 2 ? static_cast<float*>((*outputs)[1].data) : nullptr;
    return ffn(L, static_cast<const float*>(x.data), T, static_cast<float*>(y.data), probs);
  }
  if (op_name == "MatMul" || op_name == "MatMulRelu") {
    // Only a packed B with transpose_b (the reference's quant_gemm_f32 branch) runs here; f32
    // operands stay with the backend's own MatMul (NotImplemented = its usual fallback signal).
    if (inputs.size() != 2 || outputs->size() != 1)
      return Error::make(ErrorCode::InvalidArgument, "MatMul expects 2 inputs / 1 output");
    const TensorView &a = inputs[0], &b = inputs[1];
    TensorView& c = (*outputs)[0];
    if (!fmt_is_gguf(b.quant_format) || attr_int(attrs, "transpose_b", 0) == 0)
      return Error::make(ErrorCode::NotImplemented, "CUDA native MatMul here takes packed GGUF B with transpose_b");
    if (a.dtype != DType::F32 || a.rank != 2 || a.data == nullptr)
      return Error::make(ErrorCode::InvalidArgument, "quant_gemm A must be f32 [M,K]");
    if (c.dtype != DType::F32 || c.rank != 2 || c.data == nullptr)
      return Error::make(ErrorCode::InvalidArgument, "quant_gemm C must be f32");
    const int64_t M = a.dim(0), K = a.dim(1), N = b.dim(0);
    if (b.dim(1) != K || c.dim(0) != M || c.dim(1) != N)
      return Error::make(ErrorCode::InvalidArgument, "quant_gemm shape mismatch");
    if (b.nbytes != 0 && b.nbytes < (size_t)N * row_bytes(b.quant_format, K))
      return Error::make(ErrorCode::InvalidArgument, "quant_gemm B: buffer smaller than its shape");
    return quant_matmul(static_cast<const float*>(a.data), M, K, b.data, b.quant_format, N,
                        static_cast<float*>(c.data), op_name == "MatMulRelu");
  }
  return Error::make(ErrorCode::NotImplemented, "CUDA native op not implemented: " + op_name);
}

}  // namespace uaii_b200

bool uaii_b200::layer_args_from_c(const uaii_moe_layer* l, LayerArgs* out) {
  LayerArgs& L = *out;
  L.D = l->d_model; L.E = l->n_experts; L.I = l->d_ff;
  L.top_k = l->top_k;
  L.norm_topk = l->norm_topk;
  L.router_w = l->router_w;
  L.gate = ExpertWeights{l->gate_exps, l->gate_fmt, L.I, L.D};
  L.up = ExpertWeights{l->up_exps, l->up_fmt, L.I, L.D};
  L.down = ExpertWeights{l->down_exps, l->down_fmt, L.D, L.I};
  if (!l->gate_exps || !l->up_exps || !l->down_exps) return false;
  if (l->shared_d_ff > 0) {
    if (!l->gate_shexp || !l->up_shexp || !l->down_shexp) return false;
    L.I_sh = l->shared_d_ff;
    L.gate_sh = ExpertWeights{l->gate_shexp, l->gate_shexp_fmt, L.I_sh, L.D};
    L.up_sh = ExpertWeights{l->up_shexp, l->up_shexp_fmt, L.I_sh, L.D};
    L.down_sh = ExpertWeights{l->down_shexp, l->down_shexp_fmt, L.D, L.I_sh};
    L.gate_inp_sh = l->gate_inp_shexp;
  }
  return true;
}

// ---------------------------------------------------------------------------
// extern "C" shim (include/uaii_moe.h)
using namespace uaii_b200;


namespace {
thread_local std::string g_last_error;
}  // namespace

int uaii_b200::report_status(const Error& e) {
  g_last_error = e.ok() ? std::string() : e.message();
  return static_cast<int>(e.code());
}

namespace {
int report(const Error& e) { return report_status(e); }

int no_backend() { return report(Error::make(ErrorCode::InvalidArgument, "null backend")); }

TensorView to_view(const uaii_moe_tensor& t) {
  TensorView v;
  v.dtype = static_cast<DType>(t.dtype);
  v.quant_format = t.quant_format;
  v.shape = t.shape;
  v.rank = (size_t)t.rank;
  v.data = t.data;
  v.nbytes = (size_t)t.nbytes;
  return v;
}
}  // namespace

extern "C" {

int uaii_moe_abi_version(void) { return UAII_MOE_ABI_VERSION; }

const char* uaii_moe_last_error(void) { return g_last_error.c_str(); }

int uaii_moe_backend_create(int device, void* stream, uaii_moe_backend** out) {
  if (out == nullptr) return report(Error::make(ErrorCode::InvalidArgument, "null out"));
  *out = nullptr;
  auto* b = new uaii_moe_backend();
  Error e = b->impl.initialize(device, static_cast<cudaStream_t>(stream));
  if (!e.ok()) {
    delete b;
    return report(e);
  }
  *out = b;
  return report(Error::success());
}

void uaii_moe_backend_destroy(uaii_moe_backend* b) { delete b; }

int uaii_moe_route(uaii_moe_backend* b, const float* x, const float* gate_w, int64_t T, int64_t D, int64_t E,
                   int top_k, int norm_topk, int32_t* topk_ids, float* topk_w) {
  if (!b) return no_backend();
  return report(b->impl.route(x, gate_w, T, D, E, top_k, norm_topk, topk_ids, topk_w));
}

int uaii_moe_set_graphs(uaii_moe_backend* b, int on) {
  if (!b) return no_backend();
  b->impl.set_graphs(on != 0);
  return report(Error::success());
}

int uaii_moe_backend_stream(uaii_moe_backend* b, void** stream) {
  if (!b) return no_backend();
  if (!stream) return report(Error::make(ErrorCode::InvalidArgument, "null stream pointer"));
  *stream = static_cast<void*>(b->impl.stream());
  return report(Error::success());
}

int uaii_moe_quant_matmul(uaii_moe_backend* b, const float* x, int64_t M, int64_t K, const void* w, int w_fmt,
                          int64_t N, int relu, float* y) {
  if (!b) return no_backend();
  return report(b->impl.quant_matmul(x, M, K, w, w_fmt, N, y, relu != 0));
}

int uaii_moe_synchronize(uaii_moe_backend* b) {
  if (!b) return no_backend();
  return report(b->impl.synchronize());
}

int uaii_moe_supports_op(const char* op) {
  if (!op) return 0;
  const std::string s(op);
  return (s == "MoERouter" || s == "MoEExperts" || s == "MoEExpertsSwiGLU" || s == "MoEFFN") ? 1 : 0;
}

int uaii_moe_dispatch(uaii_moe_backend* b, const char* op_name, const char* op_version,
                      const uaii_moe_tensor* inputs, size_t n_inputs, uaii_moe_tensor* outputs,
                      size_t n_outputs, const uaii_moe_attr* attrs, size_t n_attrs) {
  if (!b) return no_backend();
  if (!op_name || (n_inputs && !inputs) || (n_outputs && !outputs) || (n_attrs && !attrs))
    return report(Error::make(ErrorCode::InvalidArgument, "dispatch: null argument"));
  std::vector<TensorView> in, out;
  for (size_t i = 0; i < n_inputs; ++i) in.push_back(to_view(inputs[i]));
  for (size_t i = 0; i < n_outputs; ++i) out.push_back(to_view(outputs[i]));
  std::vector<Attribute> at;
  for (size_t i = 0; i < n_attrs; ++i) {
    Attribute a;
    a.key = attrs[i].key ? attrs[i].key : "";
    a.type = static_cast<AttrType>(attrs[i].type);
    a.i = attrs[i].i;
    a.f = attrs[i].f;
    at.push_back(a);
  }
  return report(b->impl.dispatch(op_name, op_version ? op_version : "1", in, &out, at));
}

int uaii_moe_dequant_rows(uaii_moe_backend* b, int fmt, const void* packed, int64_t rows,
                          int64_t cols, float* out) {
  if (!b) return no_backend();
  if (!packed || !out) return report(Error::make(ErrorCode::InvalidArgument, "dequant_gguf_row null"));
  return report(b->impl.dequant_rows(fmt, packed, rows, cols, out));
}

int uaii_moe_router_f32(uaii_moe_backend* b, const float* x, const float* gate_w, int64_t T,
                        int64_t D, int64_t E, float* probs, float* top_expert, float* logits) {
  if (!b) return no_backend();
  if (!x || !gate_w) return report(Error::make(ErrorCode::InvalidArgument, "moe router inputs"));
  return report(b->impl.router(x, gate_w, T, D, E, probs, top_expert, logits));
}

int uaii_moe_experts_swiglu(uaii_moe_backend* b, const float* x, const void* gate_exps,
                            int gate_fmt, const void* up_exps, int up_fmt,
                            const void* down_exps, int down_fmt, const float* probs, int64_t T,
                            int64_t D, int64_t E, int64_t I, int top_k, int norm_topk, float* y) {
  if (!b) return no_backend();
  ExpertWeights g{gate_exps, gate_fmt, I, D}, u{up_exps, up_fmt, I, D}, d{down_exps, down_fmt, D, I};
  if (!gate_exps || !up_exps || !down_exps)
    return report(Error::make(ErrorCode::InvalidArgument, "moe swiglu weights"));
  return report(b->impl.experts(x, g, u, d, probs, T, D, E, I, top_k, norm_topk, y));
}

int uaii_moe_ffn_forward(uaii_moe_backend* b, const uaii_moe_layer* l, const float* x, int64_t T,
                         float* y, float* probs) {
  if (!b) return no_backend();
  if (!l) return report(Error::make(ErrorCode::InvalidArgument, "null layer"));
  LayerArgs L;
  if (!layer_args_from_c(l, &L))
    return report(Error::make(ErrorCode::InvalidArgument, "moe ffn: null expert weights"));
  return report(b->impl.ffn(L, x, T, y, probs));
}

int uaii_moe_register_weights(uaii_moe_backend* b, const void* host_ptr, uint64_t bytes) {
  if (!b) return no_backend();
  return report(b->impl.register_weights(host_ptr, (size_t)bytes));
}

int uaii_moe_release_weights(uaii_moe_backend* b, const void* host_ptr) {
  if (!b) return no_backend();
  return report(b->impl.release_weights(host_ptr));
}

int uaii_moe_profile_enable(uaii_moe_backend* b, int enable) {
  if (!b) return no_backend();
  return report(b->impl.profile_enable(enable != 0));
}

int uaii_moe_profile_read(uaii_moe_backend* b, double* phase_ms, uint64_t* phase_calls,
                          uint64_t* kernel_launches) {
  if (!b) return no_backend();
  return report(b->impl.profile_read(phase_ms, phase_calls, kernel_launches));
}

int uaii_moe_ep_dispatch(uaii_moe_backend* b, const uaii_moe_layer* l, const float* x, int64_t T, int rank, int world,
                         void* send_x16, int32_t* send_ids, float* send_w, int32_t* send_token, int32_t* row_of,
                         int32_t* send_counts, int32_t* send_entries, float* probs) {
  if (!b) return no_backend();
  if (!l) return report(Error::make(ErrorCode::InvalidArgument, "null layer"));
  LayerArgs L{};
  L.D = l->d_model;
  L.E = l->n_experts;
  L.top_k = l->top_k;
  L.norm_topk = l->norm_topk;
  L.router_w = l->router_w;
  return report(b->impl.ep_dispatch(L, x, T, rank, world, send_x16, send_ids, send_w, send_token, row_of,
                                    send_counts, send_entries, probs));
}

namespace {
// Record of one exchanged row: f16 x (d_model), then top_k int32 ids, then top_k f32 weights.
Error record_layout(int64_t D, int k, int64_t rec_bytes) {
  if (D <= 0 || k < 1 || rec_bytes % 16 != 0 || rec_bytes < 2 * D + 8 * (int64_t)k || (2 * D) % 16 != 0)
    return Error::make(ErrorCode::InvalidArgument,
                       "ep records: rec_bytes must be a multiple of 16 and hold 2*d_model + 8*top_k bytes "
                       "(d_model a multiple of 8)");
  return Error::success();
}
}  // namespace

int uaii_moe_ep_dispatch_records(uaii_moe_backend* b, const uaii_moe_layer* l, const float* x, int64_t T, int rank,
                                 int world, void* send_rec, int64_t rec_bytes, int32_t* send_token, int32_t* row_of,
                                 int32_t* send_counts, int32_t* send_entries, float* probs) {
  if (!b) return no_backend();
  if (!l) return report(Error::make(ErrorCode::InvalidArgument, "null layer"));
  {
    const Error le = record_layout(l->d_model, (int)l->top_k, rec_bytes);
    if (!le.ok()) return report(le);
  }
  LayerArgs L{};
  L.D = l->d_model;
  L.E = l->n_experts;
  L.top_k = l->top_k;
  L.norm_topk = l->norm_topk;
  L.router_w = l->router_w;
  char* r = static_cast<char*>(send_rec);
  return report(b->impl.ep_dispatch(L, x, T, rank, world, r, reinterpret_cast<int32_t*>(r + 2 * L.D),
                                    reinterpret_cast<float*>(r + 2 * L.D + 4 * L.top_k), send_token, row_of,
                                    send_counts, send_entries, probs, rec_bytes / 2, rec_bytes / 4));
}

int uaii_moe_ep_experts_records(uaii_moe_backend* b, const uaii_moe_layer* l, const void* recv_rec, int64_t rec_bytes,
                                int64_t rows, int64_t entries, float* y_part) {
  if (!b) return no_backend();
  if (!l) return report(Error::make(ErrorCode::InvalidArgument, "null layer"));
  {
    const Error le = record_layout(l->d_model, (int)l->top_k, rec_bytes);
    if (!le.ok()) return report(le);
  }
  LayerArgs L;
  if (!layer_args_from_c(l, &L))
    return report(Error::make(ErrorCode::InvalidArgument, "ep experts: null expert weights"));
  const char* r = static_cast<const char*>(recv_rec);
  return report(b->impl.ep_experts(L, r, reinterpret_cast<const int32_t*>(r + 2 * L.D),
                                   reinterpret_cast<const float*>(r + 2 * L.D + 4 * L.top_k), rows, entries, y_part,
                                   rec_bytes / 2, rec_bytes / 4));
}

int uaii_moe_ep_experts_records_f16(uaii_moe_backend* b, const uaii_moe_layer* l, const void* recv_rec,
                                    int64_t rec_bytes, int64_t rows, int64_t entries, void* y_part_f16) {
  if (!b) return no_backend();
  if (!l) return report(Error::make(ErrorCode::InvalidArgument, "null layer"));
  {
    const Error le = record_layout(l->d_model, (int)l->top_k, rec_bytes);
    if (!le.ok()) return report(le);
  }
  LayerArgs L;
  if (!layer_args_from_c(l, &L))
    return report(Error::make(ErrorCode::InvalidArgument, "ep experts: null expert weights"));
  const char* r = static_cast<const char*>(recv_rec);
  return report(b->impl.ep_experts(L, r, reinterpret_cast<const int32_t*>(r + 2 * L.D),
                                   reinterpret_cast<const float*>(r + 2 * L.D + 4 * L.top_k), rows, entries,
                                   y_part_f16, rec_bytes / 2, rec_bytes / 4, /*y_f16=*/true));
}

int uaii_moe_ep_combine_f16(uaii_moe_backend* b, const void* y_back_f16, const int32_t* row_of, int64_t T, int world,
                            int64_t d_model, float* y) {
  if (!b) return no_backend();
  return report(b->impl.ep_combine(y_back_f16, row_of, T, world, d_model, y, /*y_back_f16=*/true));
}

int uaii_moe_ep_experts(uaii_moe_backend* b, const uaii_moe_layer* l, const void* recv_x16, const int32_t* recv_ids,
                        const float* recv_w, int64_t rows, int64_t entries, float* y_part) {
  if (!b) return no_backend();
  if (!l) return report(Error::make(ErrorCode::InvalidArgument, "null layer"));
  LayerArgs L;
  if (!layer_args_from_c(l, &L))
    return report(Error::make(ErrorCode::InvalidArgument, "ep experts: null expert weights"));
  return report(b->impl.ep_experts(L, recv_x16, recv_ids, recv_w, rows, entries, y_part));
}

int uaii_moe_ep_combine(uaii_moe_backend* b, const float* y_back, const int32_t* row_of, int64_t T, int world,
                        int64_t d_model, float* y) {
  if (!b) return no_backend();
  return report(b->impl.ep_combine(y_back, row_of, T, world, d_model, y));
}

int uaii_moe_selftest_wait_timeout(uaii_moe_backend* b, int64_t budget_cycles) {
  if (!b) return no_backend();
  return report(b->impl.selftest_wait_timeout(budget_cycles));
}

int uaii_moe_last_plan(uaii_moe_backend* b, int* tensor_cores, int* slot_tile, int* down_splits) {
  if (!b) return no_backend();
  const uaii_b200::ExpertPlan P = b->impl.last_plan();
  if (tensor_cores) *tensor_cores = P.umma ? (P.quad_i8 ? 4 : P.quad_mma ? 3 : P.warp_mma ? 2 : 1) : 0;
  if (slot_tile) *slot_tile = P.bn;
  if (down_splits) *down_splits = P.splits;
  return report(Error::success());
}

int uaii_moe_set_expert_path(uaii_moe_backend* b, int path) {
  if (!b) return no_backend();
  if (path < 0 || path > 5) return report(Error::make(ErrorCode::InvalidArgument, "path must be 0 .. 5"));
  b->impl.set_expert_path(path);
  return report(Error::success());
}

}  // extern "C"
