// backend.hpp -- C++17 host side of the B200 MoE backend.
//
// The types mirror the reference's operator interface so that the backend reads
// like a native op of UAII's CUDA backend:
//   ErrorCode / Error  <- uaii::ErrorCode, uaii::Error (include/uaii/core/error.hpp:12-51)
//   TensorView         <- kernels::TensorView (include/uaii/kernels/tensor_view.hpp:12-50)
//   Attribute          <- ir::Attribute (include/uaii/ir/attribute.hpp:10-30), scalar kinds
//   MoeCudaBackend::dispatch <- IBackend::dispatch (include/uaii/interfaces/backend.hpp:77-81)
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <tuple>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "kernels.hpp"

struct uaii_moe_layer;

namespace uaii_b200 {

enum class ErrorCode {
  Ok = 0, InvalidArgument = 1, NotFound = 2, IoError = 3, ConfigError = 4,
  PluginError = 5, AbiMismatch = 6, NotImplemented = 7, Internal = 8,
};

class Error {
 public:
  Error() = default;
  Error(ErrorCode c, std::string m) : code_(c), message_(std::move(m)) {}
  static Error success() { return Error{}; }
  static Error make(ErrorCode c, std::string m) { return Error{c, std::move(m)}; }
  bool ok() const noexcept { return code_ == ErrorCode::Ok; }
  ErrorCode code() const noexcept { return code_; }
  const std::string& message() const noexcept { return message_; }

 private:
  ErrorCode code_ = ErrorCode::Ok;
  std::string message_;
};

// uaii::DType values (include/uaii/interfaces/types.hpp:14-25)
enum class DType { Unknown = 0, F32 = 1, F16 = 2, BF16 = 3 };

struct TensorView {
  DType dtype = DType::Unknown;
  int quant_format = 0;  // uaii::quant::QuantFormat value
  const int64_t* shape = nullptr;
  size_t rank = 0;
  void* data = nullptr;
  size_t nbytes = 0;
  int64_t dim(size_t i) const { return i < rank ? shape[i] : 1; }
};

enum class AttrType { String = 0, Int = 1, Float = 2, Bool = 3 };
struct Attribute {
  std::string key;
  AttrType type = AttrType::Int;
  int64_t i = 0;
  double f = 0.0;
};

// Expert weights of one projection: [E, rows, cols] in `fmt`.
struct ExpertWeights {
  const void* data = nullptr;
  int fmt = 0;
  int64_t rows = 0, cols = 0;
};

struct LayerArgs {
  int64_t D = 0, E = 0, I = 0;
  int top_k = 2;
  int norm_topk = 1;
  const float* router_w = nullptr;  // [E, D] f32
  ExpertWeights gate, up, down;
  int64_t I_sh = 0;                 // shared expert width, 0 = none
  ExpertWeights gate_sh, up_sh, down_sh;
  const float* gate_inp_sh = nullptr;  // [D] f32 or null
};

struct ExpertPlan {
  bool umma = false;   // tensor-core grouped GEMM (else CUDA-core GEMV)
  bool warp_mma = false;      // ... on an mma.sync schedule (decode widths), else tcgen05
  bool quad_mma = false;      // ... the mma.sync schedule over whole K-quant super-blocks
  bool down_quad = false;     // the down projection alone on the quad schedule (16-slot tiles, gate/up on tcgen05)
  bool quad_i8 = false;       // quad gate/up (Q4_K, 8-slot tiles) on 16-bit integer activations, int8 mma.sync
  bool down_ranges = false;   // quad down in balanced ranges of the tile-major quad sequence (splits == 1)
  bool umma_refused = false;  // tensor cores forced but the layer does not qualify
  int bn = 16;         // slots per tile (MMA N)
  int splits = 1;      // K splits of the down projection
  bool sh_umma = false, sh_warp_mma = false;
  int sh_bn = 16, sh_splits = 1;
};

class MoeCudaBackend {
 public:
  ~MoeCudaBackend() { shutdown(); }
  Error initialize(int device, cudaStream_t stream);
  // Use caller-owned device memory as workspace and error flag, on the caller's
  // stream: nothing is allocated and shutdown() frees nothing.  Weights and
  // activations must then be device pointers.
  Error attach_external(int device, cudaStream_t stream, void* scratch, size_t bytes);
  void shutdown() noexcept;
  Error synchronize();

  Error dispatch(const std::string& op_name, const std::string& op_version,
                 const std::vector<TensorView>& inputs, std::vector<TensorView>* outputs,
                 const std::vector<Attribute>& attrs);

  Error dequant_rows(int fmt, const void* packed, int64_t rows, int64_t cols, float* out);
  Error router(const float* x, const float* gate_w, int64_t T, int64_t D, int64_t E,
               float* probs, float* top, float* logits);
  // MoEExperts (top-1 linear experts, moe_experts_f32): y[b] = x[b] . W[e_b]^T
  Error experts_linear(const float* x, const float* W, const float* top, int64_t B, int64_t D, int64_t E,
                       float* y);
  Error experts(const float* x, const ExpertWeights& g, const ExpertWeights& u,
                const ExpertWeights& d, const float* probs, int64_t T, int64_t D, int64_t E,
                int64_t I, int top_k, int norm_topk, float* y);
  Error ffn(const LayerArgs& L, const float* x, int64_t T, float* y, float* probs);
  // The fused layer's token -> expert assignment: ids [T, k] (rank order) and weights.
  Error route(const float* x, const float* gate_w, int64_t T, int64_t D, int64_t E, int k, int norm_topk,
              int32_t* ids, float* w);
  // y[M,N] = x[M,K] . dequant(W[N,K])^T (kernels::quant_gemm_f32), max(y, 0) with relu.
  Error quant_matmul(const float* x, int64_t M, int64_t K, const void* w, int fmt, int64_t N, float* y, bool relu);

  // Expert parallelism (device pointers only).  See include/uaii_moe.h.
  // x_pitch (f16 elements) / e_pitch (entries) between rows; 0 = dense.
  Error ep_dispatch(const LayerArgs& L, const float* x, int64_t T, int rank, int world, void* send_x16,
                    int32_t* send_ids, float* send_w, int32_t* send_token, int32_t* row_of, int32_t* send_counts,
                    int32_t* send_entries, float* probs, int64_t x_pitch = 0, int64_t e_pitch = 0);
  // y_part f32, or f16 when y_f16 (each row's sum rounded once: half the return bytes)
  Error ep_experts(const LayerArgs& L_local, const void* recv_x16, const int32_t* recv_ids, const float* recv_w,
                   int64_t rows, int64_t entries, void* y_part, int64_t x_pitch = 0, int64_t e_pitch = 0,
                   bool y_f16 = false);
  Error ep_combine(const void* y_back, const int32_t* row_of, int64_t T, int world, int64_t D, float* y,
                   bool y_back_f16 = false);
  // Runs the bounded-wait self-test kernel and returns the status the host observes.
  Error selftest_wait_timeout(int64_t budget_cycles);

  Error register_weights(const void* host_ptr, size_t bytes);
  Error release_weights(const void* host_ptr);
  Error profile_enable(bool on);
  Error profile_read(double* ms, uint64_t* calls, uint64_t* launches);
  // 0..4 as uaii_moe_set_expert_path; 5 = automatic with the Q4_K quad gate/up on f16 activations
  void set_expert_path(int p) {
    path_ = p == 5 ? 0 : p;
    f16_quad_ = p == 5;
    drop_graphs();
  }
  // Replay repeated device-resident layer calls from CUDA graphs (default on).
  void set_graphs(bool on) {
    graphs_on_ = on;
    if (!on) drop_graphs();
  }
  // Schedule chosen by the most recent expert-product call (routed experts).
  ExpertPlan last_plan() const { return last_plan_; }
  cudaStream_t stream() const { return stream_; }
  // Kernels launched on this backend's stream by code built on it (the decoder's own kernels),
  // added to the launch count uaii_moe_profile_read reports.
  void add_launches(uint64_t n) { count_launches(n); }
  int device() const { return device_; }

 private:
  struct Staged {  // an argument resolved to device memory
    const void* dev = nullptr;
    bool host = false;
  };
  // Device address of a weight: device pointers as they are, registered host
  // buffers from the cache, other host buffers copied into the workspace.
  Error stage_weight(const void* p, size_t bytes, const void** dev);
  size_t weight_stage_bytes(const void* p, size_t bytes) const;
  size_t layer_stage_bytes(const LayerArgs& L) const;
  Error stage_input(const void* p, size_t bytes, void* scratch, const void** dev, bool* was_host);
  Error reserve(size_t bytes);
  void* carve(size_t bytes);
  // `slots`: routed (token, expert) pairs when known (expert-parallel rows), else T * top_k.
  ExpertPlan plan_experts(const LayerArgs& L, int64_t T, int64_t slots = -1, bool allow_warp_mma = true) const;
  // Rows received by an expert-parallel rank: f16 activations in operand order and
  // top_k (local expert | -1, weight) entries per row; replaces the router output.
  struct EpRows {
    const void* x16;
    const int32_t* ids;
    const float* w;
    int64_t x_pitch, e_pitch;  // 0 = dense
    bool y_f16;                // the per-row sums written as f16
  };
  // Decode widths: the router runs inside the routing step (launch_route_decode), writing the
  // logits and probabilities here.
  struct DecodeRoute {
    const float* router_w;
    float* logits;
    float* probs;
  };
  Error run_experts(const float* x_dev, const float* scores, const float* probs_for_w,
                    const LayerArgs& L, const ExpertPlan& P, int64_t T, void* y_dev,
                    const EpRows* ep = nullptr, const DecodeRoute* dr = nullptr);
  Error sync_and_check();
  // Packed rows as the tensor-core path reads them (16-byte pitch).  `constant`: the
  // source is a registered buffer, so a padded copy is made once and kept.
  Error umma_rows(const void* w, int fmt, int64_t rows, int64_t K, bool constant, const void** out, int64_t* pitch);
  // Registered (host copy or device buffer): unchanged until released.
  bool weight_is_constant(const void* p, size_t bytes) const;
  size_t experts_ws(const LayerArgs& L, int64_t T, const ExpertPlan& P) const;

 public:
  Error sync_and_check_public() {
    std::lock_guard<std::mutex> lk(mu_);
    return sync_and_check();
  }

 private:

  // phase timing: events recorded around each phase while profiling is on
  static constexpr int kPhases = 6;
  enum Phase { kRouter = 0, kRoute = 1, kGateUp = 2, kDown = 3, kShared = 4, kCombine = 5 };
  struct PhaseMark {
    int phase;
    cudaEvent_t start, stop;
  };
  void phase_begin(int phase);
  void phase_end();
  void count_launches(uint64_t n) { launches_ += n; }
  bool profiling_ = false;
  std::vector<PhaseMark> marks_;
  std::vector<cudaEvent_t> event_pool_;
  int open_phase_ = -1;
  cudaEvent_t open_start_ = nullptr;
  double phase_ms_[kPhases] = {};
  uint64_t phase_calls_[kPhases] = {};
  uint64_t launches_ = 0;

  int device_ = -1;
  cudaStream_t stream_ = nullptr;
  bool own_stream_ = false;
  int path_ = 0;
  bool f16_quad_ = false;
  int ranges_mode_ = -1;  // UAII_MOE_DOWN_RANGES: 0 off, 1 forced, -1 automatic (quad down balanced ranges)
  ExpertPlan last_plan_{};
  int* dev_err_ = nullptr;
  TailSplit tail_{};  // quad schedule tail split and balanced down ranges (in external mode: carved from the scratch)
  static size_t tail_part_bytes() { return sizeof(float) * (size_t)kTailMaxUnits * 128 * kTailMaxBn; }
  static size_t tail_bytes() { return tail_part_bytes() + sizeof(int) * (size_t)(kTailMaxUnits + 16); }
  int* route_done_ = nullptr;  // launch_route_decode's counter (after the tail-split counters)
  bool external_ = false;  // workspace and error flag belong to the caller
  char* ws_ = nullptr;
  size_t ws_cap_ = 0;
  size_t ws_used_ = 0;
  std::map<std::pair<const void*, size_t>, void*> weights_;   // registered host buffer -> device copy
  std::map<const void*, size_t> const_dev_;                     // registered device buffers
  struct Padded {
    void* dev;
    int64_t pitch;
  };
  // (source device rows, format, K, rows) -> copy with 16-byte row pitch, for constant sources
  std::map<std::tuple<const void*, int, int64_t, int64_t>, Padded> padded_;
  void drop_padded(const char* lo, const char* hi);
  // CUDA graphs of device-resident layer calls, keyed by everything the launch sequence
  // depends on: captured on the second identical call, replayed from the third.
  struct GraphEntry {
    int seen = 0;
    cudaGraphExec_t exec = nullptr;
    uint64_t launches = 0;  // kernels in the captured sequence (counted again on every replay)
  };
  std::map<std::vector<int64_t>, GraphEntry> graphs_;
  bool graphs_on_ = true;
  void drop_graphs();
  Error ffn_launch(const LayerArgs& L, const ExpertPlan& P, int64_t T, const float* xd, const float* wd, float* logits,
                   float* po, float* rscratch, size_t rsb, float* yo);
  // Host x and y (and host or no probs) with device-resident weights: the batch in
  // chunks whose host copies overlap the neighbouring chunks' device work.
  Error ffn_host_chunked(const LayerArgs& L, const float* x, int64_t T, float* y, float* probs, int chunks);
  cudaStream_t in_stream_ = nullptr, out_stream_ = nullptr;  // host copies of the chunked path
  std::vector<cudaEvent_t> chunk_events_;
  Error ensure_copy_streams(int chunks);
  std::mutex mu_;
};

bool is_device_ptr(const void* p) noexcept;
// The C ABI layer description (include/uaii_moe.h) as LayerArgs; false if a
// required expert weight pointer is null.
bool layer_args_from_c(const struct uaii_moe_layer* l, LayerArgs* out);
// Record `e` as this thread's last error (uaii_moe_last_error) and return its status code.
int report_status(const Error& e);
Error cuda_status(cudaError_t st, const char* what);

}  // namespace uaii_b200

// The C ABI's opaque backend handle (include/uaii_moe.h).
struct uaii_moe_backend {
  uaii_b200::MoeCudaBackend impl;
};

#define UAII_TRY(expr)                   \
  do {                                   \
    ::uaii_b200::Error _e = (expr);      \
    if (!_e.ok()) return _e;             \
  } while (0)
#define UAII_CUDA(expr, what) UAII_TRY(::uaii_b200::cuda_status((expr), what))
