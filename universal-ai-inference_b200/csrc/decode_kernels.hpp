// decode_kernels.hpp -- launch wrappers of the batched decode step's device kernels
// (decode_model.cu).  Plain pointers, sizes and a stream; each returns a cudaError_t.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace uaii_b200 {

// x[b] = row tokens[b] of the embedding table (any GGUF block format, f16 or f32 rows),
// bitwise the reference's embedding_f32; an out-of-range token writes zeros and sets *err.
cudaError_t launch_embed(int fmt, const void* table, int64_t vocab, int64_t D, const int32_t* tokens, int64_t B,
                         float* x, int* err, cudaStream_t st);
// x += delta (if delta); y = RMSNorm(x) * w (if w), rows of D.
cudaError_t launch_add_rmsnorm(float* x, const float* delta, const float* w, int64_t B, int64_t D, float eps, float* y,
                               cudaStream_t st);
// RoPE of the q and k parts of qkv [B, H*hd + 2*Hkv*hd] at position pos (freq [hd/2]);
// q_out [B, H*hd] f32; k and v appended to the f16 caches [B, Hkv, max_seq, hd] at pos.
cudaError_t launch_rope_append(const float* qkv, int64_t B, int64_t H, int64_t Hkv, int64_t hd, const float* freq,
                               int64_t pos, int mode, float* q_out, void* kc, void* vc, int64_t max_seq,
                               cudaStream_t st);
// Splits (of 128 positions) of the attention over len positions; partial buffers hold
// B*H*splits*hd (po) and B*H*splits (pm, pl) floats.
int attn_splits(int64_t len);
// TMA map (128 bytes, CUtensorMap) of an f16 KV cache of `rows` rows of 128 elements.
constexpr int kKvMapBytes = 128;
bool make_kv_map(void* map, const void* cache, int64_t rows);
// out [B, H*hd] = attention of q over the first len cached positions (hd = 128) on the tensor
// cores; kmap / vmap from make_kv_map.  A copy that never lands sets *err after about a
// second instead of hanging.
cudaError_t launch_attn_decode(const void* kmap, const void* vmap, const float* q, int64_t B, int64_t H, int64_t Hkv,
                               int64_t hd, int64_t len, int64_t max_seq, float* po, float* pm, float* pl, float* out,
                               int* err, cudaStream_t st);
// dst[r * dst_pitch + c] = f16(src[r * cols + c]) (KV-cache rows from f32).
cudaError_t launch_to_half_rows(const float* src, int64_t rows, int64_t cols, void* dst, int64_t dst_pitch,
                                cudaStream_t st);
// out[b] = first index of the largest logit of row b (the reference's greedy sampler).
cudaError_t launch_argmax(const float* logits, int64_t B, int64_t V, int32_t* out, cudaStream_t st);
// Device-side synthetic inputs: the counter-based normals of uaii_moe_fill_normal (f32, or
// rounded to f16 row by row) and the GGUF block quantizers of uaii_moe_quantize_rows.
uint64_t normal_key(uint64_t seed, uint64_t stream);
cudaError_t launch_fill_normal(float* out, int64_t n, uint64_t seed, uint64_t stream, float mean, float std,
                               cudaStream_t st);
// rows of cols f16 draws, pitch elements apart; row r uses generator stream stream0 + r.
cudaError_t launch_fill_normal_f16_rows(void* out, int64_t rows, int64_t cols, int64_t pitch, uint64_t seed,
                                        uint64_t stream0, float mean, float std, cudaStream_t st);
cudaError_t launch_quantize_rows(int fmt, const float* src, int64_t rows, int64_t cols, void* dst, cudaStream_t st);

}  // namespace uaii_b200
