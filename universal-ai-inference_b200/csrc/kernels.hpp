// kernels.hpp -- launch wrappers for the device kernels of the MoE FFN path.
// Plain pointers, sizes and a stream; every function returns a cudaError_t.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace uaii_b200 {

// ---- dequant.cu: exact GGUF rows -> f32 (parity kernel for dequant_gguf_row)
cudaError_t launch_dequant_rows_f32(int fmt, const void* packed, int64_t rows, int64_t cols,
                                    int64_t row_pitch, float* out, cudaStream_t st);

// ---- router.cu: logits in the reference GEMM order, softmax, argmax
// probs/top may be null when only logits are wanted; logits may be null.
cudaError_t launch_router(const float* x, const float* w, int64_t T, int64_t D, int64_t E,
                          float* logits, float* probs, float* top, cudaStream_t st, float* scratch = nullptr,
                          size_t scratch_bytes = 0);
// Scratch launch_router can use to split small batches across more blocks (0: none needed).
size_t router_scratch_bytes(int64_t T, int64_t D, int64_t E);

// ---- route.cu: top-k selection, stable permutation, gather, combine
struct RouteBuffers {
  int32_t* topk_ids;    // [T*k]
  float* topk_w;        // [T*k]
  uint8_t* mask;        // [E*T] rank+1 of token t in expert e's selection, 0 if absent
  int32_t* slot_local;  // [T*k] position of (t,r) inside its expert's list
  int32_t* slot_of;     // [T*k] global slot of (t,r)
  int32_t* token_of;    // [T*k] token of each slot
  int32_t* counts;      // [E]
  int32_t* offsets;     // [E+1]
};
// `scores` [T,E] rank the experts in the order of the reference's
// std::partial_sort (value descending, ties as the reference orders them); the
// routing weights are taken from `probs` [T,E] (which may be the same array).
// Decode widths: router + softmax + top-k + the per-expert slot numbering of tokens in ONE
// launch (T <= kDecodeRouteMaxT): logits, probs [T, E]; rb.topk_ids / topk_w / slot_local /
// counts as launch_route_topk + launch_route_scan leave them (rb.mask is not written).  `done`:
// one int, zero before the first launch (every launch leaves it zero).  cudaErrorNotSupported
// when the shapes do not fit (the caller then runs the separate kernels).
constexpr int64_t kDecodeRouteMaxT = 32;
bool route_decode_supported(int64_t T, int64_t D, int64_t E, int k);
cudaError_t launch_route_decode(const float* x, const float* w, int64_t T, int64_t D, int64_t E, int k, int norm_topk,
                                float* logits, float* probs, const RouteBuffers& rb, int* done, cudaStream_t st);
cudaError_t launch_route_topk(const float* scores, const float* probs, int64_t T, int64_t E,
                              int k, int norm_topk, const RouteBuffers& rb, cudaStream_t st);
// offsets = {0, T}, counts = {T} in buf[0..2]: one expert that owns every token.
cudaError_t launch_identity_route(int32_t* buf, int64_t T, cudaStream_t st);
cudaError_t launch_route_scan(int64_t T, int64_t E, int k, const RouteBuffers& rb,
                              cudaStream_t st);
// Self-test of the bounded-wait failure path (selftest.cu): one block waits on
// an mbarrier nothing arrives on, gives up after budget_cycles and records
// `code` in *err.  Faults nothing; the kernel returns normally.
cudaError_t launch_wait_timeout_selftest(int* err, long long budget_cycles, int code, cudaStream_t st);

// ---- expert parallelism (ep.cu).  Rank r of R owns experts [r*epr, (r+1)*epr).
// dmask [R*T] bytes, rowpos [T*R], dcounts [R]: which ranks each token goes to and
// its row inside each destination group (token order).
cudaError_t launch_ep_plan(const int32_t* topk_ids, int64_t T, int k, int R, int epr, uint8_t* dmask,
                           int32_t* rowpos, int32_t* dcounts, cudaStream_t st);
// Packs the send rows grouped by destination: f16 x (operand order), k (local
// expert | -1, weight) entries, source token; row_of [T*R] (-1 where none);
// send_counts / send_entries [R]: rows and valid entries per destination.
// x_pitch (f16 elements) and e_pitch (entries) between rows; 0 = dense (D, k).
cudaError_t launch_ep_pack(const float* x, int64_t T, int64_t D, int k, int R, int epr, const int32_t* topk_ids,
                           const float* topk_w, const uint8_t* dmask, const int32_t* rowpos,
                           const int32_t* dcounts, void* send_x16, int32_t* send_ids, float* send_w,
                           int32_t* send_token, int32_t* row_of, int32_t* send_counts, int32_t* send_entries,
                           cudaStream_t st, int64_t x_pitch = 0, int64_t e_pitch = 0);
// Receiving side: routing tables (topk_ids/w, expert mask) from received entries.
cudaError_t launch_ep_route(const int32_t* ids, const float* w, int64_t N, int64_t E, int k,
                            const RouteBuffers& rb, cudaStream_t st, int64_t e_pitch = 0);
// Gather of received f16 rows into expert-contiguous slots (absent entries skipped).
cudaError_t launch_route_gather16(const void* rows, int64_t N, int64_t D, int64_t E, int k, const RouteBuffers& rb,
                                  void* xp16, cudaStream_t st, int64_t x_pitch = 0);
// y[t] = sum over d = 0..R-1 of y_back[row_of[t*R+d]] (rows that exist), fixed order.
cudaError_t launch_ep_combine(const float* y_back, const int32_t* row_of, int64_t T, int R, int64_t D, float* y,
                              cudaStream_t st);
// launch_ep_combine on f16 returned rows (added in f32, the same rank order).
cudaError_t launch_ep_combine_f16(const void* y_back16, const int32_t* row_of, int64_t T, int R, int64_t D, float* y,
                                  cudaStream_t st);
// Gathers x rows into expert-contiguous slots: xp_f32 and/or xp_f16 (either may be null).
// xp_f16 rows are in an operand K order (operand_order.cuh, OperandOrder): tc_kpos for
// the tcgen05 schedule, wm_kpos (D % 128 == 0) for the warp-MMA one, q4k_kpos / q6k_kpos
// (D % 256 == 0) for the quad schedule.
// Optional: the gate/up and down expert GEMMs' tile tables ([E+1] each, as
// tile_table_kernel builds them) written by the gather from the same counts.
struct TileTables {
  int32_t* gu = nullptr;
  int32_t* dn = nullptr;
  int bn = 16, gu_mtiles = 0, dn_mtiles = 0, dn_splits = 1;
  // Quad schedule with Q4_K weights: the activations' 32-element sub-block sums (xsum_kpos order,
  // see launch_gateup_umma), or null.
  void* xsum = nullptr;
  // kOrderQ4KI8: the per (slot, quad) dequant scales of the integer activations [S][D / 256] f32.
  float* xscale = nullptr;
};
cudaError_t launch_route_gather(const float* x, int64_t T, int64_t D, int64_t E, int k,
                                const RouteBuffers& rb, float* xp_f32, void* xp_f16,
                                cudaStream_t st, int order = 0, const TileTables* tables = nullptr);
// The packed MatMul's operand prep in one launch: x [M, K] -> f16 operand order (tc_kpos, or
// wm_kpos), route = {0, M, M} (one expert owning every row) and its tile table {0, tiles}.
cudaError_t launch_to_f16_route(const float* x, int64_t M, int64_t K, void* out, bool wm_order, int32_t* route,
                                int32_t* tile_base, int bn, int m_tiles, int splits, cudaStream_t st);
// y[t] = sum_r w[t,r] * out[slot_of[t,r]] (rank order, from 0), then
// y[t] += gate[t] * shared_out[t] when shared_out is given (gate may be null = 1).
// `out` (and `shared_out`) may hold `splits` partial planes `split_stride`
// elements apart; the planes are added in order before weighting.  y is f32, or f16
// (y_f16: each sum rounded once; needs D and the strides to be multiples of 4).
cudaError_t launch_combine(const float* out, int64_t out_ld, int splits, int64_t split_stride,
                           int64_t T, int64_t D, int k, const RouteBuffers& rb,
                           const float* shared_out, int sh_splits, int64_t sh_split_stride,
                           const float* shared_gate, void* y, cudaStream_t st, bool y_f16 = false);
// y[i] = sum over s of planes[s*plane_stride + i] (in plane order), max(., 0) when relu; y may alias planes.
cudaError_t launch_sum_planes(const float* planes, int splits, int64_t plane_stride, int64_t n, float* y, bool relu,
                              cudaStream_t st);
// x rows -> f16 copy (shared-expert operand in token order; operand K order tc_kpos,
// or wm_kpos with wm_order and n % 128 == 0)
cudaError_t launch_to_f16(const float* x, int64_t n, void* out, cudaStream_t st, bool wm_order = false);
// gate[t] = sigmoid(x[t] . w) with the reference GEMM summation order
cudaError_t launch_shared_gate(const float* x, const float* w, int64_t T, int64_t D,
                               float* gate, cudaStream_t st);

// ---- experts_simt.cu: CUDA-core grouped GEMV (f32 end to end)
// Gate/up for every (expert, slot): h[slot, i] = silu(x.G[e,i]) * (x.U[e,i]).
cudaError_t launch_gateup_simt(int gfmt, const void* G, int ufmt, const void* U, int64_t E,
                               int64_t I, int64_t D, int64_t g_pitch, int64_t u_pitch,
                               const float* xp, const int32_t* offsets, const int32_t* counts,
                               float* h, cudaStream_t st);
// Down for every (expert, slot): out[slot, o] = h[slot] . Dn[e, o].
cudaError_t launch_down_simt(int dfmt, const void* Dn, int64_t E, int64_t D, int64_t I,
                             int64_t d_pitch, const float* h, const int32_t* offsets,
                             const int32_t* counts, float* out, cudaStream_t st);

// MoEExperts (top-1 linear experts): y[b] = x[b] . W[e_b]^T, W [E, D, D] f32, e_b = (int)top[b]
// (expert 0 outside [0, E)), sequential f32 sums in the reference order.
cudaError_t launch_experts_linear(const float* x, const float* W, const float* top, int64_t B, int64_t D,
                                  int64_t E, float* y, cudaStream_t st);

// ---- experts_umma.cu: tensor-core grouped GEMM (tcgen05 + TMEM + TMA)
bool umma_format_supported(int fmt);
// whole-layer check: formats, K chunking and tile multiples (any row pitch: rows that
// are not 16-byte aligned are staged with a padded pitch, see launch_pad_rows)
bool umma_shapes_supported(int gate_fmt, int down_fmt, int64_t D, int64_t I);
int umma_kchunks(int fmt, int64_t K);
// Row pitch the tensor-core path reads a packed matrix with: row_bytes rounded up to 16.
int64_t umma_pitch(int fmt, int64_t K);
// The warp-MMA schedule (mma.sync, slot tiles of 8 or 16) also needs D and I to be
// multiples of 128; its operand rows are in wm_kpos order (operand_order.cuh).
bool warp_mma_shapes_supported(int gate_fmt, int down_fmt, int64_t D, int64_t I);
// A single projection out[N] = W[N, K] . x on tensor cores (launch_down_umma with E = 1):
// format and K chunking, N a multiple of 128 (and K of 128 for the warp-MMA schedule).
bool umma_down_supported(int fmt, int64_t N, int64_t K, bool warp_mma);
// Expert-product schedules on the tensor cores.
enum ExpertSchedule : int {
  kSchedTcgen05 = 0,  // tcgen05/TMEM/TMA, slot tiles 16..256, operands in tc_kpos order
  kSchedWarpMma = 1,  // mma.sync, slot tiles 8 or 16, a 32-element unit per lane and row, wm_kpos order
  kSchedQuadMma = 2,  // mma.sync over whole K-quant super-blocks (Q4_K, Q6_K), q4k_kpos / q6k_kpos order
};
// The schedules the quad kernel takes: K-quant formats with whole super-blocks.
inline bool quad_mma_format(int fmt) { return fmt == 14 || fmt == 16; }
// h16[slot, i] = silu(x.G[e,i]) * (x.U[e,i]) in f16; x is xp16 [S_rows, D] f16.
// G, U rows `pitch` bytes apart (a multiple of 16).  sched selects the schedule; x is
// in that schedule's order for the gate format; h is written in the tc_kpos
// (tcgen05), wm_kpos (warp-MMA) or h_order (quad: the order of the down format) order.
// tile_base: scratch of E+1 ints.  *err receives a nonzero code if a wait timed out.
// table_ready: tile_base already holds the tile table (route_gather or the prep kernel built
// it), so no tile-table kernel is launched.  xsum (quad schedule, Q4_K): per slot and 256-element
// quad, the f32 sums of the eight 32-element sub-blocks of the f16 activations as 8 f16 values
// then their 8 f16 remainders ([S_rows][kquads][16] f16, route_gather writes them), so the Q4_K
// minima take two MMAs per quad instead of one per k-step.
// xscale (quad schedule, Q4_K gate/up, 8-slot tiles): x holds 16-bit integer activations as
// int8 hi / lo planes per 256-element quad (route_gather's kOrderQ4KI8: [S_rows][kquads][512]
// bytes in the xp16 buffer), xscale their per (slot, quad) dequant scales [S_rows][kquads] f32,
// and xsum the planes' integer sub-block sums / 1024; the products run on integer mma.sync.
// Tail split of the quad schedule's gate/up launch (see the kernel): part holds
// kTailMaxUnits x 128 x kTailMaxBn f32, cnt kTailMaxUnits ints, zero before the first launch
// (every launch leaves them zero).  A null or absent TailSplit turns the split off.
constexpr int kTailMaxUnits = 320, kTailMaxBn = 16;
struct TailSplit {
  float* part = nullptr;
  int* cnt = nullptr;
};
cudaError_t launch_gateup_umma(int fmt, const void* G, const void* U, int64_t pitch, int64_t E, int64_t I, int64_t D,
                               const void* xp16, int64_t S_rows, const int32_t* counts,
                               const int32_t* offsets, int32_t* tile_base, int bn, void* h16, int* err,
                               cudaStream_t st, int sched = kSchedTcgen05, int h_order = 0,
                               bool table_ready = false, const void* xsum = nullptr,
                               const TailSplit* tail = nullptr, const float* xscale = nullptr);
// out[split][slot, o] = partial of h16[slot] . Dn[e, o] over the split's K range (f32).
// ranges (quad schedule, splits == 1, the same TailSplit buffers as the gate/up tail split, BN x 2
// x SMs <= kTailMaxUnits x kTailMaxBn): every CTA takes an equal share of the tile-major sequence
// of all tiles' quads; a tile cut between CTAs is finished by the CTA that completes its last
// piece, which adds the pieces in order.  Null: whole tiles (or `splits` K ranges) per unit.
cudaError_t launch_down_umma(int fmt, const void* Dn, int64_t pitch, int64_t E, int64_t D, int64_t I, const void* h16,
                             int64_t S_rows, const int32_t* counts, const int32_t* offsets,
                             int32_t* tile_base, int bn, int splits, float* out, int* err, cudaStream_t st,
                             int sched = kSchedTcgen05, bool table_ready = false, const TailSplit* ranges = nullptr);
// Copies `rows` packed rows of row_bytes (even) from src (src_pitch apart) to dst
// (dst_pitch apart, a multiple of 16), zero-filling each row's padding.
cudaError_t launch_pad_rows(const void* src, int64_t src_pitch, int64_t rows, int64_t row_bytes, void* dst,
                            int64_t dst_pitch, cudaStream_t st);

}  // namespace uaii_b200
