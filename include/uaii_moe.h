/*
 * uaii_moe.h -- C ABI of the B200-native GGUF mixture-of-experts FFN path.
 *
 * This library is a drop-in device implementation of the MoE operators of UAII
 * (arjun988/Universal-AI-Inference).  The reference runs these operators only
 * on the host: its CUDA backend has no MoE kernel and falls back to
 * kernels::dispatch_cpu (libs/uaii-backends/src/cuda_runtime_api.cpp:542-579,
 * libs/uaii-backends/src/cuda_backend.cpp:166-207).  Each entry point below
 * names the reference interface it replaces (paths are inside the reference
 * project).  Signatures use plain pointers and sizes only.
 *
 * Residency.  Every data pointer may be host memory or device memory of the
 * backend's device; the library tells them apart with cudaPointerGetAttributes,
 * exactly like the reference's CudaBackend (cuda_runtime_api.cpp:586-601).
 *   - Device pointers: work is queued on the backend's stream and the call
 *     returns without waiting.
 *   - Host pointers: inputs are copied in, outputs are copied back, and the
 *     call returns after the copy back has completed (the reference's
 *     host-staging behaviour, host_executable.cpp:169-233).
 *   - Host-resident weights are copied to the device on every call, unless
 *     the buffer was registered with uaii_moe_register_weights(): a
 *     registered buffer is uploaded once and its device copy is reused until
 *     uaii_moe_release_weights().  (Caching unregistered host buffers by
 *     address is unsafe: a freed buffer's address can come back holding
 *     different weights.)
 *
 * Errors.  Every int-returning function returns a uaii_moe_status; the message
 * of the last failure on the calling thread is uaii_moe_last_error().
 */
#ifndef UAII_MOE_H_
#define UAII_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UAII_MOE_ABI_VERSION 1

#if defined(__GNUC__)
#define UAII_MOE_API __attribute__((visibility("default")))
#else
#define UAII_MOE_API
#endif

/* Status codes: the values of uaii::ErrorCode (include/uaii/core/error.hpp:12-22)
 * and of uaii_status in the reference C ABI (include/uaii/c_api/uaii.h). */
typedef enum uaii_moe_status {
  UAII_MOE_OK = 0,
  UAII_MOE_INVALID_ARGUMENT = 1,
  UAII_MOE_NOT_FOUND = 2,
  UAII_MOE_IO_ERROR = 3,
  UAII_MOE_CONFIG_ERROR = 4,
  UAII_MOE_PLUGIN_ERROR = 5,
  UAII_MOE_ABI_MISMATCH = 6,
  UAII_MOE_NOT_IMPLEMENTED = 7,
  UAII_MOE_INTERNAL = 8
} uaii_moe_status;

/* Weight formats: the values of uaii::quant::QuantFormat
 * (include/uaii/quant/formats.hpp:10-29).  GGUF blocks are byte-identical to
 * the file format; rows are stored back to back (row pitch = packed bytes). */
typedef enum uaii_moe_format {
  UAII_MOE_F32 = 0,
  UAII_MOE_F16 = 1,
  UAII_MOE_Q4_0 = 7,
  UAII_MOE_Q4_1 = 8,
  UAII_MOE_Q5_0 = 9,
  UAII_MOE_Q5_1 = 10,
  UAII_MOE_Q8_0 = 11,
  UAII_MOE_Q2_K = 12,
  UAII_MOE_Q3_K = 13,
  UAII_MOE_Q4_K = 14,
  UAII_MOE_Q5_K = 15,
  UAII_MOE_Q6_K = 16
} uaii_moe_format;

/* Element types: the values of uaii::DType (include/uaii/interfaces/types.hpp:14-25). */
typedef enum uaii_moe_dtype {
  UAII_MOE_DTYPE_UNKNOWN = 0,
  UAII_MOE_DTYPE_F32 = 1,
  UAII_MOE_DTYPE_F16 = 2
} uaii_moe_dtype;

/* A non-owning tensor view: the C form of kernels::TensorView
 * (include/uaii/kernels/tensor_view.hpp:12-22).  Packed weights use
 * dtype = UNKNOWN, quant_format = Q*, nbytes = packed bytes (session.cpp:342-357). */
typedef struct uaii_moe_tensor {
  int32_t dtype;
  int32_t quant_format;
  const int64_t* shape;
  uint64_t rank;
  void* data;
  uint64_t nbytes;
} uaii_moe_tensor;

/* An operator attribute: the C form of ir::Attribute
 * (include/uaii/ir/attribute.hpp:10-30).  type: 1 = Int (value in i),
 * 2 = Float (value in f), 3 = Bool (value in i). */
typedef struct uaii_moe_attr {
  const char* key;
  int32_t type;
  int64_t i;
  double f;
} uaii_moe_attr;

typedef struct uaii_moe_backend uaii_moe_backend;

/* One MoE FFN layer (GGUF blk.N.ffn_* tensors, libs/uaii-loaders/src/gguf.cpp:1078-1128).
 * gate/up experts are [n_experts, d_ff, d_model], down experts [n_experts, d_model, d_ff];
 * the router weight ffn_gate_inp is f32 [n_experts, d_model].  The shared expert
 * is optional (shared_d_ff = 0 for none); gate_inp_shexp is an optional f32
 * [d_model] sigmoid gate of the shared expert (NULL = ungated, as in the reference). */
typedef struct uaii_moe_layer {
  int64_t d_model;
  int64_t n_experts;
  int64_t d_ff;
  int32_t top_k;
  int32_t norm_topk; /* 1 = renormalise the top-k weights (reference), 0 = raw probabilities */
  const float* router_w;
  const void* gate_exps;
  int32_t gate_fmt;
  const void* up_exps;
  int32_t up_fmt;
  const void* down_exps;
  int32_t down_fmt;
  int64_t shared_d_ff;
  const void* gate_shexp;
  int32_t gate_shexp_fmt;
  const void* up_shexp;
  int32_t up_shexp_fmt;
  const void* down_shexp;
  int32_t down_shexp_fmt;
  const float* gate_inp_shexp;
} uaii_moe_layer;

/* ABI version of this library (UAII_MOE_ABI_VERSION). */
UAII_MOE_API int uaii_moe_abi_version(void);

/* Message of the last failure on this thread ("" if none).
 * Replaces uaii_last_error (libs/uaii-capi/src/capi.cpp:17-44). */
UAII_MOE_API const char* uaii_moe_last_error(void);

/* Create a backend on CUDA device `device`; `stream` is a cudaStream_t or NULL
 * for a backend-owned stream.  Replaces CudaBackend::initialize
 * (libs/uaii-backends/src/cuda_backend.cpp:35-66) and native::cuda_init
 * (libs/uaii-backends/src/cuda_runtime_api.cpp:376-428). */
UAII_MOE_API int uaii_moe_backend_create(int device, void* stream, uaii_moe_backend** out);

/* Free every device allocation of the backend (workspace, cached weights).
 * Replaces CudaBackend::shutdown (cuda_backend.cpp:68-78). */
UAII_MOE_API void uaii_moe_backend_destroy(uaii_moe_backend* b);

/* CUDA-graph replay of layer calls (default on): a uaii_moe_ffn_forward whose
 * activations, outputs and weights are all device-resident (or registered)
 * is captured into a CUDA graph the second time the same call (same shapes,
 * pointers, schedule) is made and replayed from then on, so a decode loop pays
 * one graph launch per layer instead of ~10 kernel launches.  Replays read the
 * buffers' current contents.  Graphs are dropped when weights are registered
 * or released, the schedule changes or the workspace grows.  No reference
 * counterpart. */
UAII_MOE_API int uaii_moe_set_graphs(uaii_moe_backend* b, int on);

/* The CUDA stream (cudaStream_t) this backend queues its work on: the one given
 * to uaii_moe_backend_create, or the backend's own non-blocking stream when that
 * was NULL.  Callers that order other work against the backend's (collectives,
 * copies) use this stream.  No reference counterpart. */
UAII_MOE_API int uaii_moe_backend_stream(uaii_moe_backend* b, void** stream);

/* Wait for all work queued by this backend.  Replaces IBackend::synchronize
 * (include/uaii/interfaces/backend.hpp:74) / native::cuda_synchronize. */
UAII_MOE_API int uaii_moe_synchronize(uaii_moe_backend* b);

/* 1 if `op_name` runs natively on the device: "MoERouter", "MoEExpertsSwiGLU"
 * and the fused "MoEFFN".  Replaces the native op table of
 * native::cuda_dispatch (cuda_runtime_api.cpp:542-579). */
UAII_MOE_API int uaii_moe_supports_op(const char* op_name);

/* Execute one operator with TensorView-style arguments.  Replaces
 * IBackend::dispatch (include/uaii/interfaces/backend.hpp:77-81) as implemented
 * by CudaBackend::dispatch (cuda_backend.cpp:166-207); argument lists, arity
 * checks and attributes follow kernels::dispatch_cpu
 * (libs/uaii-kernels/src/dispatch.cpp:224-248):
 *   MoERouter         inputs {x[T,D], gate[E,D]}                 outputs {probs[T,E], top_expert[T,1]}
 *   MoEExpertsSwiGLU  inputs {x, gate_exps, up_exps, down_exps, probs}  outputs {y[T,D]}
 *                     attrs num_experts (default 1), top_k (default 2), norm_topk (default 1)
 *   MoEFFN            inputs {x, gate, gate_exps, up_exps, down_exps
 *                            [, gate_shexp, up_shexp, down_shexp [, gate_inp_shexp]]}
 *                     outputs {y[, probs]}; the two reference nodes fused.
 * Unknown ops return UAII_MOE_NOT_IMPLEMENTED (the reference's signal to fall
 * back to host staging). */
UAII_MOE_API int uaii_moe_dispatch(uaii_moe_backend* b, const char* op_name, const char* op_version,
                      const uaii_moe_tensor* inputs, size_t n_inputs, uaii_moe_tensor* outputs,
                      size_t n_outputs, const uaii_moe_attr* attrs, size_t n_attrs);

/* GGUF rows -> f32, bitwise equal to the reference for every finite value.
 * `rows` rows of `cols` elements, stored back to back.  Replaces
 * quant::dequant_gguf_row (include/uaii/quant/gguf_dequant.hpp:13-16) applied
 * row by row. */
UAII_MOE_API int uaii_moe_dequant_rows(uaii_moe_backend* b, int fmt, const void* packed, int64_t rows,
                          int64_t cols, float* out);

/* MoERouter: probs = softmax(x . gate^T), top_expert = first argmax as f32.
 * Replaces kernels::moe_router_f32 (libs/uaii-kernels/src/transformer.cpp:446-481).
 * `logits` may be NULL; when given it receives x . gate^T, bitwise equal to the
 * reference GEMM (libs/uaii-kernels/src/gemm_ref.cpp:45-75). */
UAII_MOE_API int uaii_moe_router_f32(uaii_moe_backend* b, const float* x, const float* gate_w, int64_t T,
                        int64_t D, int64_t E, float* probs, float* top_expert, float* logits);

/* MoEExpertsSwiGLU: y = sum over the top_k experts of w * down(silu(gate x) * up x).
 * Replaces kernels::moe_experts_swiglu_f32 (transformer.cpp:522-612);
 * norm_topk = 1 is the reference behaviour.  gate and up use the same format. */
UAII_MOE_API int uaii_moe_experts_swiglu(uaii_moe_backend* b, const float* x, const void* gate_exps,
                            int gate_fmt, const void* up_exps, int up_fmt,
                            const void* down_exps, int down_fmt, const float* probs, int64_t T,
                            int64_t D, int64_t E, int64_t I, int top_k, int norm_topk, float* y);

/* The token -> expert assignment the fused layer computes: router logits (the
 * reference GEMM order) and probabilities, then the top-k experts of every
 * token in rank order -- the selection of moe_experts_swiglu_f32
 * (libs/uaii-kernels/src/transformer.cpp:564-580) applied to the router's
 * output, ranked on the exact logits -- with their weights (renormalised when
 * norm_topk).  topk_ids [T, top_k] int32, topk_w [T, top_k] f32; host or device
 * memory.  Exposed so that callers and tests can check assignments bit for bit. */
UAII_MOE_API int uaii_moe_route(uaii_moe_backend* b, const float* x, const float* gate_w, int64_t T, int64_t D,
                                int64_t E, int top_k, int norm_topk, int32_t* topk_ids, float* topk_w);

/* The whole MoE FFN layer (router + experts [+ shared expert]) in one call:
 * the MoERouter -> MoEExpertsSwiGLU node pair (and the shared-expert nodes) the
 * reference GGUF loader emits per layer (libs/uaii-loaders/src/gguf.cpp:1078-1128).
 * `probs` (T x n_experts) may be NULL. */
UAII_MOE_API int uaii_moe_ffn_forward(uaii_moe_backend* b, const uaii_moe_layer* layer, const float* x,
                         int64_t T, float* y, float* probs);

/* ---- GGUF files, packed loading.  A file is mapped read-only;
 * header, metadata and tensor index are parsed once and tensor data is handed
 * out as pointers into the mapping (no copy; pass them to
 * uaii_moe_register_weights to upload once).  Replaces gguf_read_header /
 * gguf_load_tensor_raw (libs/uaii-loaders/src/gguf.cpp:374-443, :558-602),
 * which read the whole file into memory for the header and for every tensor.
 * Shapes are outermost first (the reference's dims_to_shape, gguf.cpp:272-280);
 * `fmt` is a uaii_moe_format, or -1 for tensor types without one (data NULL). */
typedef struct uaii_moe_gguf uaii_moe_gguf;
UAII_MOE_API int uaii_moe_gguf_open(const char* path, uaii_moe_gguf** out);
UAII_MOE_API void uaii_moe_gguf_close(uaii_moe_gguf* g);
UAII_MOE_API int64_t uaii_moe_gguf_tensor_count(const uaii_moe_gguf* g);
/* shape holds up to 8 entries; any output pointer may be NULL. */
UAII_MOE_API int uaii_moe_gguf_tensor_at(const uaii_moe_gguf* g, int64_t index, const char** name,
                                         const void** data, int* fmt, int64_t* shape, int* rank, uint64_t* nbytes);
UAII_MOE_API int uaii_moe_gguf_tensor(const uaii_moe_gguf* g, const char* name, const void** data, int* fmt,
                                      int64_t* shape, int* rank, uint64_t* nbytes);
/* Metadata: integer (any integer width, bool), number (integers and floats), string. */
UAII_MOE_API int uaii_moe_gguf_kv_int(const uaii_moe_gguf* g, const char* key, int64_t* out);
UAII_MOE_API int uaii_moe_gguf_kv_float(const uaii_moe_gguf* g, const char* key, double* out);
UAII_MOE_API int uaii_moe_gguf_kv_string(const uaii_moe_gguf* g, const char* key, const char** out);
/* The MoE FFN layer of block `block` as the reference's GGUF graph builds it
 * (gguf.cpp:1078-1128): blk.N.ffn_gate_inp (f32 router), ffn_{gate,up,down}_exps,
 * expert_count / expert_used_count from `{arch}.`, `llama.` or `general.` keys
 * (top_k default 2, clamped to the expert count), renormalised top-k, and the
 * ungated shared expert ffn_{gate,up,down}_shexp when present.  With flags &
 * UAII_MOE_GGUF_SHEXP_GATE the shared expert is also gated by sigmoid(x .
 * ffn_gate_inp_shexp) (Qwen2-MoE; the reference graph has no such gate).  The
 * layer's pointers point into the mapping: keep the file open while it is used. */
#define UAII_MOE_GGUF_SHEXP_GATE 1
UAII_MOE_API int uaii_moe_gguf_moe_layer(const uaii_moe_gguf* g, int block, int flags, uaii_moe_layer* layer);

/* Dense projection with a packed GGUF weight: y[M,N] = x[M,K] . dequant(w)^T,
 * w = N packed rows of K elements in w_fmt (any GGUF block format); relu != 0
 * applies max(y, 0) (the MatMulRelu op).  Replaces kernels::quant_gemm_f32
 * (libs/uaii-kernels/src/quant_gemm.cpp:22-70), which dispatch_cpu runs for
 * MatMul / MatMulRelu with a packed B and transpose_b
 * (libs/uaii-kernels/src/dispatch.cpp:82-100); uaii_moe_dispatch takes those ops
 * in the same form.  Q4_0/Q8_0/Q4_K/Q6_K with N % 128 == 0 run on the tensor
 * cores (f16 operands, f32 accumulate), everything else on the CUDA cores in f32.
 * Residency as above; x, y may be host or device memory. */
UAII_MOE_API int uaii_moe_quant_matmul(uaii_moe_backend* b, const float* x, int64_t M, int64_t K, const void* w,
                                       int w_fmt, int64_t N, int relu, float* y);

/* Declare a weight buffer constant until uaii_moe_release_weights().  A host
 * buffer is uploaded once and the device copy is reused whenever a call passes
 * the same (pointer, bytes).  For host and device buffers alike, layouts the
 * library derives from the weights (rows copied to a 16-byte pitch for the
 * tensor maps, when a format's row size is not a multiple of 16) are made on
 * first use and kept.  The caller keeps the buffer unchanged until it is
 * released.  No reference counterpart: the reference never uploads weights
 * (its Session keeps them in host memory, libs/uaii-runtime/src/session.cpp:259-367). */
UAII_MOE_API int uaii_moe_register_weights(uaii_moe_backend* b, const void* host_ptr, uint64_t bytes);

/* The whole MoE FFN layer, like uaii_moe_ffn_forward, for callers that cannot
 * allocate device memory (engines that pre-reserve HBM for their own pools,
 * runtimes that own every allocation, decode loops that must not be stalled by
 * the device-wide synchronization of cudaMalloc/cudaFree).  It allocates
 * nothing: its scratch is one fixed 32 MiB array compiled into the library,
 * held by every GPU that loads it until the process exits.  x, y, probs and all
 * weights must be device memory of `device`; work runs on `stream` (a
 * cudaStream_t, NULL for the default stream) and the call returns after it has
 * finished.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress), so make it before any stream capture.  A call that
 * needs more than 32 MiB of scratch returns UAII_MOE_INVALID_ARGUMENT: routing
 * tables, f16 activations, hidden activations and partial sums grow with T, so
 * this serves decode-sized batches (the Mixtral-shaped layer needs ~140 KB per
 * token: up to about 200 tokens), not large prefill batches.  Weights whose packed rows are not a
 * multiple of 16 bytes (e.g. Q8_0 rows of 1408 elements, the Qwen2-MoE down
 * projection) are copied with a 16-byte row pitch on every call, and that copy
 * is carved from the same 32 MiB, so such layers fit only when their padded
 * copy does (the Qwen2-MoE down stack needs ~180 MB and never fits).  All
 * calls share the array; calls are serialized inside one process because
 * overlapping GPU work on it would race.  The device current on entry is
 * current again on return.  No reference counterpart: the reference runs this
 * operator only on the host. */
UAII_MOE_API int uaii_moe_ffn_forward_noalloc(int device, void* stream, const uaii_moe_layer* layer,
                                              const float* x, int64_t T, float* y, float* probs);

/* Drop the device copy of a registered host weight buffer. */
UAII_MOE_API int uaii_moe_release_weights(uaii_moe_backend* b, const void* host_ptr);

/* Select the expert-product schedule: 0 = automatic (tensor cores when the layer
 * qualifies: the warp-MMA schedule at <= 16 routed slots per expert, tcgen05
 * above), 1 = CUDA-core f32 GEMV, 2 = tensor cores on the tcgen05 schedule only,
 * 3 = tensor cores on the warp-MMA (mma.sync) schedule for every slot count
 * (d_model and d_ff multiples of 128; expert-parallel rows stay on tcgen05),
 * 4 = as 3 with the per-32-element warp schedule for K-quants too,
 * 5 = automatic, with the Q4_K gate/up of 8-slot tiles on f16 activations instead
 * of 16-bit integer ones.  No reference counterpart. */
UAII_MOE_API int uaii_moe_set_expert_path(uaii_moe_backend* b, int path);

/* ---- Expert parallelism (one process per GPU, R ranks, rank r owns experts
 * [r*E/R, (r+1)*E/R)).  No reference counterpart: the reference runs the layer in
 * one host process (kernels::moe_experts_swiglu_f32,
 * libs/uaii-kernels/src/transformer.cpp:564-609).  The caller moves the buffers
 * between ranks (an all-to-all by rows, e.g. NCCL); every pointer is device
 * memory on this backend's device.
 *
 * Step 1, on each rank for its own T tokens: router + top-k exactly as
 * uaii_moe_ffn_forward, then each token is packed ONCE for every rank that owns
 * one of its experts.  Rows are grouped by destination rank (token order inside
 * a group).  Outputs (capacity T * min(top_k, world) rows):
 *   send_x16   [rows, d_model] f16, elements [0, 2, 1, 3] of every group of four;
 *   send_ids   [rows, top_k] destination-local expert id, -1 where that choice
 *              lives on another rank;  send_w [rows, top_k] routing weight;
 *   send_token [rows] source token;  row_of [T, world] row of (token, rank), -1;
 *   send_counts, send_entries [world] rows and valid entries per destination;
 *   probs [T, E] (optional).  `layer` supplies router_w, d_model, n_experts (all
 *   ranks), top_k, norm_topk; its expert pointers are not read. */
UAII_MOE_API int uaii_moe_ep_dispatch(uaii_moe_backend* b, const uaii_moe_layer* layer, const float* x, int64_t T,
                                      int rank, int world, void* send_x16, int32_t* send_ids, float* send_w,
                                      int32_t* send_token, int32_t* row_of, int32_t* send_counts,
                                      int32_t* send_entries, float* probs);

/* Step 2, on each rank for the rows it received (same layout as step 1's
 * output, `entries` = valid (row, expert) pairs): `layer` holds this rank's
 * experts (n_experts = E / world, their gate/up/down weights) and top_k; writes
 * y_part [rows, d_model] f32 = sum over the row's entries of weight * expert
 * output, in top-k order.  Tensor-core formats only; no shared expert. */
UAII_MOE_API int uaii_moe_ep_experts(uaii_moe_backend* b, const uaii_moe_layer* layer, const void* recv_x16,
                                     const int32_t* recv_ids, const float* recv_w, int64_t rows, int64_t entries,
                                     float* y_part);

/* Steps 1 and 2 with each exchanged row as ONE record, so that a single
 * all-to-all moves rows, ids and weights: record = f16 x [d_model] (operand
 * order as above), then top_k int32 ids, then top_k f32 weights, rec_bytes
 * apart (a multiple of 16, >= 2*d_model + 8*top_k; d_model a multiple of 8).
 * Same outputs and semantics as uaii_moe_ep_dispatch / uaii_moe_ep_experts. */
UAII_MOE_API int uaii_moe_ep_dispatch_records(uaii_moe_backend* b, const uaii_moe_layer* layer, const float* x,
                                              int64_t T, int rank, int world, void* send_rec, int64_t rec_bytes,
                                              int32_t* send_token, int32_t* row_of, int32_t* send_counts,
                                              int32_t* send_entries, float* probs);
UAII_MOE_API int uaii_moe_ep_experts_records(uaii_moe_backend* b, const uaii_moe_layer* layer, const void* recv_rec,
                                             int64_t rec_bytes, int64_t rows, int64_t entries, float* y_part);

/* Step 3, on each rank after the reverse exchange (y_back [rows, d_model] f32 in
 * its own send-row order): y[t] = sum over ranks d = 0..world-1 of
 * y_back[row_of[t, d]] (present rows, fixed rank order). */
UAII_MOE_API int uaii_moe_ep_combine(uaii_moe_backend* b, const float* y_back, const int32_t* row_of, int64_t T,
                                     int world, int64_t d_model, float* y);

/* Steps 2 and 3 with f16 return rows (half the bytes of the reverse exchange): each
 * received row's weighted expert sum is rounded once to f16 (d_model a multiple of 4),
 * and the source rank adds the returned f16 rows in f32, in rank order. */
UAII_MOE_API int uaii_moe_ep_experts_records_f16(uaii_moe_backend* b, const uaii_moe_layer* layer,
                                                 const void* recv_rec, int64_t rec_bytes, int64_t rows,
                                                 int64_t entries, void* y_part_f16);
UAII_MOE_API int uaii_moe_ep_combine_f16(uaii_moe_backend* b, const void* y_back_f16, const int32_t* row_of,
                                         int64_t T, int world, int64_t d_model, float* y);

/* Failure-path self-test: launches one block whose threads wait, through the
 * same bounded wait as the tensor-core kernels, on a barrier nothing arrives
 * on; they give up after budget_cycles (1e3..4e9 SM cycles) and record an
 * error code without faulting the device.  Returns UAII_MOE_INTERNAL with the
 * code in uaii_moe_last_error() when the path works; the backend stays usable.
 * Diagnostic; no reference counterpart. */
UAII_MOE_API int uaii_moe_selftest_wait_timeout(uaii_moe_backend* b, int64_t budget_cycles);

/* Schedule of the most recent expert-product call on this backend (routed
 * experts): *tensor_cores = 1 for the tcgen05 grouped GEMM, 2 for the warp-MMA
 * one, 3 for the warp-MMA over whole K-quant super-blocks (quad schedule), 4 for the
 * quad schedule with its Q4_K gate/up on 16-bit integer activations (int8 mma.sync),
 * 0 for the CUDA-core GEMV; *slot_tile = routed slots per tile (MMA N);
 * *down_splits = K splits of the down projection.  Any pointer may be NULL.
 * Diagnostic; no reference counterpart. */
UAII_MOE_API int uaii_moe_last_plan(uaii_moe_backend* b, int* tensor_cores, int* slot_tile, int* down_splits);

/* Device-side profile of the MoE phases, measured with CUDA events on the
 * backend's stream.  Phases: 0 router, 1 routing (top-k, permutation, gather),
 * 2 gate/up expert products + SwiGLU, 3 down expert products, 4 shared expert,
 * 5 weighted combine.  Replaces the host wall-clock scopes the reference wraps
 * around each dispatch (profiler::Profiler::Scope, libs/uaii-profiler/src/profiler.cpp:59,
 * used at libs/uaii-runtime/src/session.cpp:1128-1130) with device time.
 * uaii_moe_profile_enable resets the counters; uaii_moe_profile_read waits for
 * the stream and returns the accumulated milliseconds and call counts per
 * phase (arrays of UAII_MOE_N_PHASES) and the number of kernels this backend
 * launched since the reset (counted whether or not timing is enabled). */
#define UAII_MOE_N_PHASES 6
UAII_MOE_API int uaii_moe_profile_enable(uaii_moe_backend* b, int enable);
UAII_MOE_API int uaii_moe_profile_read(uaii_moe_backend* b, double* phase_ms, uint64_t* phase_calls,
                                       uint64_t* kernel_launches);

/* ---- Batched greedy decode of a GGUF MoE transformer on the device.  Replaces the
 * reference's decode loop, Session::generate (libs/uaii-runtime/src/session.cpp:910-1046),
 * over the seq-1 transformer graph its GGUF loader builds
 * (libs/uaii-loaders/src/gguf.cpp:905-1210) with a host f32 KV cache of batch 1
 * (include/uaii/runtime/kv_cache.hpp:16-190, session.cpp:852).  Here `batch`
 * sequences advance one position per step together, every activation and the KV
 * cache (f16, [batch, n_kv_heads, max_seq, head_dim] per layer) stay on the device:
 * embedding, per block RMSNorm -> Q/K/V projection (packed MatMul) -> RoPE -> KV
 * append -> grouped-query attention -> O projection -> residual Add -> RMSNorm -> MoE
 * FFN layer -> residual Add, then RMSNorm -> output projection -> arg-max (the
 * reference's greedy sampler, libs/uaii-runtime/src/sampling.cpp:38-50).  All weights
 * must be device memory and stay valid while the decoder lives. */
typedef struct uaii_moe_decoder_config {
  int64_t n_layers;
  int64_t d_model;
  int64_t n_heads;
  int64_t n_kv_heads;
  int64_t head_dim;  /* 128 */
  int64_t vocab;
  int64_t batch;
  int64_t max_seq;   /* cache positions per sequence */
  float rope_theta;
  float rms_eps;
  int32_t rope_mode; /* 0: pairs (2i, 2i+1) as for llama/Mixtral; 2: NeoX pairs (i, i + head_dim/2) */
} uaii_moe_decoder_config;

/* One block: attention (GGUF blk.N.attn_*) and the MoE FFN layer.  Norm weights f32 [d_model];
 * wq [n_heads*head_dim, d_model], wk / wv [n_kv_heads*head_dim, d_model], wo [d_model,
 * n_heads*head_dim] in GGUF block formats. */
typedef struct uaii_moe_decoder_block {
  const float* attn_norm;
  const void* wq;
  int32_t wq_fmt;
  const void* wk;
  int32_t wk_fmt;
  const void* wv;
  int32_t wv_fmt;
  const void* wo;
  int32_t wo_fmt;
  const float* ffn_norm;
  uaii_moe_layer moe;
} uaii_moe_decoder_block;

typedef struct uaii_moe_decoder uaii_moe_decoder;

/* blocks [n_layers]; output_norm f32 [d_model]; token_embd [vocab, d_model] (GGUF format, f16
 * or f32); output [vocab, d_model] (GGUF format) or NULL for tied embeddings (the reference
 * reuses the table, gguf.cpp:1195-1200).  The decode position starts at 0. */
UAII_MOE_API int uaii_moe_decoder_create(uaii_moe_backend* b, const uaii_moe_decoder_config* cfg,
                                         const uaii_moe_decoder_block* blocks, const float* output_norm,
                                         const void* token_embd, int embd_fmt, const void* output, int output_fmt,
                                         uaii_moe_decoder** out);
UAII_MOE_API void uaii_moe_decoder_destroy(uaii_moe_decoder* d);
/* Cache positions [0, n_pos) of layer `layer` from f32 k, v [batch, n_kv_heads, n_pos, head_dim]
 * (host or device; stored in f16); the decode position becomes n_pos. */
UAII_MOE_API int uaii_moe_decoder_set_kv(uaii_moe_decoder* d, int64_t layer, const float* k, const float* v,
                                         int64_t n_pos);
/* Synthetic prefill: K and V of every layer at positions [0, n_pos) drawn N(0, 1) from the
 * counter-based generator keyed by (seed, layer, sequence, head); the position becomes n_pos. */
UAII_MOE_API int uaii_moe_decoder_fill_kv(uaii_moe_decoder* d, int64_t n_pos, uint64_t seed);
/* One step at the current position: tokens [batch]; logits [batch, vocab] and next [batch]
 * (host, device or NULL).  Returns after the copies when an output is host memory. */
UAII_MOE_API int uaii_moe_decoder_step(uaii_moe_decoder* d, const int32_t* tokens, float* logits, int32_t* next);
/* `steps` greedy steps from tokens [batch]: out [steps, batch] token ids (host or device). */
UAII_MOE_API int uaii_moe_decoder_generate(uaii_moe_decoder* d, const int32_t* tokens, int64_t steps, int32_t* out);
UAII_MOE_API int64_t uaii_moe_decoder_position(const uaii_moe_decoder* d);

/* Device-side synthetic inputs (no reference counterpart): uaii_moe_fill_normal's draws
 * written on the backend's stream (equal to the host generator's up to the last bit of the
 * device's double-precision log/sin/cos), and uaii_moe_quantize_rows on the device (the same
 * bytes as the host quantizer for the same f32 input).  Device pointers only. */
UAII_MOE_API int uaii_moe_fill_normal_device(uaii_moe_backend* b, float* out, int64_t n, uint64_t seed, uint64_t stream,
                                             float mean, float std);
UAII_MOE_API int uaii_moe_quantize_rows_device(uaii_moe_backend* b, int fmt, const float* src, int64_t rows,
                                               int64_t cols, void* dst);

/* Bytes of one row of n elements in `fmt` (include/uaii/quant/formats.hpp:81-102). */
UAII_MOE_API uint64_t uaii_moe_packed_nbytes(int fmt, int64_t n);

/* Synthetic-input utilities (no reference counterpart: the reference has no
 * GGUF block quantizer, libs/uaii-quant/src/codec.cpp:81-179).
 * uaii_moe_quantize_rows: f32 rows -> GGUF blocks (Q4_0, Q8_0, Q4_K, Q6_K),
 * round to nearest with per-block scales, deterministic.
 * uaii_moe_fill_normal: out[i] = mean + std * N(0,1), a counter-based generator
 * keyed by (seed, stream, i); identical on every host and thread count. */
UAII_MOE_API int uaii_moe_quantize_rows(int fmt, const float* src, int64_t rows, int64_t cols, void* dst);
UAII_MOE_API int uaii_moe_fill_normal(float* out, int64_t n, uint64_t seed, uint64_t stream, float mean,
                         float std);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* UAII_MOE_H_ */
