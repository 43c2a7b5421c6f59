// decoder.cpp -- batched greedy decode of a GGUF MoE transformer on the device.
//
// The reference decodes through its seq-1 transformer graph one token per
// Session::run with a batch-1 host KV cache (libs/uaii-runtime/src/session.cpp:
// 910-1046, libs/uaii-loaders/src/gguf.cpp:905-1210, include/uaii/runtime/
// kv_cache.hpp:16-190).  Here a batch of B sequences advances one position per
// step with every activation and the KV cache resident on the device:
//
//   x = embed(tokens)
//   per layer:  n = RMSNorm(x += ff_prev);  qkv = n . [Wq; Wk; Wv]^T;  RoPE(q, k) at pos,
//               k, v -> cache;  a = attention(q, cache[0 .. pos]);  o = a . Wo^T;
//               n2 = RMSNorm(x += o);  ff = MoE(n2)
//   logits = RMSNorm(x += ff) . W_out^T;  next = argmax(logits)
//
// Projections with packed weights run on the packed-MatMul kernels
// (MoeCudaBackend::quant_matmul), the MoE layer on the fused layer path
// (MoeCudaBackend::ffn: router, top-k, grouped expert GEMMs, combine), the rest on
// the kernels of decode_model.cu.  All positions of the batch advance together;
// the cache holds max_seq positions per sequence in f16.
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/uaii_moe.h"
#include "backend.hpp"
#include "decode_kernels.hpp"
#include "gguf_format.hpp"

namespace uaii_b200 {

struct DecoderBlock {
  const float* attn_norm = nullptr;
  const void* wq = nullptr;
  const void* wk = nullptr;
  const void* wv = nullptr;
  const void* wo = nullptr;
  int wq_fmt = 0, wk_fmt = 0, wv_fmt = 0, wo_fmt = 0;
  const float* ffn_norm = nullptr;
  LayerArgs moe;
  void* wqkv = nullptr;  // owned: [q_dim + 2 kv_dim] packed rows when the three share a format
};

class Decoder {
 public:
  ~Decoder() { release(); }

  Error create(MoeCudaBackend* be, const uaii_moe_decoder_config& c, const uaii_moe_decoder_block* blocks,
               const float* out_norm, const void* embd, int embd_fmt, const void* output, int output_fmt) {
    be_ = be;
    cfg_ = c;
    const int64_t L = c.n_layers, D = c.d_model, H = c.n_heads, Hkv = c.n_kv_heads, hd = c.head_dim;
    if (L <= 0 || D <= 0 || H <= 0 || Hkv <= 0 || H % Hkv || hd != 128 || c.vocab <= 0 || c.batch <= 0 ||
        c.max_seq <= 0 || (c.rope_mode != 0 && c.rope_mode != 2))
      return Error::make(ErrorCode::InvalidArgument,
                         "decoder config: layers, d_model, vocab, batch, max_seq > 0; n_heads a multiple of "
                         "n_kv_heads; head_dim 128; rope_mode 0 or 2");
    if (!blocks || !out_norm || !embd) return Error::make(ErrorCode::InvalidArgument, "decoder: null weights");
    if (D % 32 != 0) return Error::make(ErrorCode::InvalidArgument, "decoder: d_model must be a multiple of 32");
    q_dim_ = H * hd;
    kv_dim_ = Hkv * hd;
    out_norm_ = out_norm;
    embd_ = embd;
    embd_fmt_ = embd_fmt;
    output_ = output ? output : embd;  // tied embeddings: the lm_head reuses the table (gguf.cpp:1195-1200)
    output_fmt_ = output ? output_fmt : embd_fmt;
    if (!fmt_is_gguf(output_fmt_))
      return Error::make(ErrorCode::NotImplemented, "decoder: the output projection must be a GGUF block format");
    UAII_CUDA(cudaSetDevice(be_->device()), "SetDevice");
    cudaStream_t st = be_->stream();
    blocks_.resize((size_t)L);
    for (int64_t l = 0; l < L; ++l) {
      const uaii_moe_decoder_block& s = blocks[l];
      DecoderBlock& b = blocks_[(size_t)l];
      if (!s.attn_norm || !s.wq || !s.wk || !s.wv || !s.wo || !s.ffn_norm)
        return Error::make(ErrorCode::InvalidArgument, "decoder: null weight in block " + std::to_string(l));
      if (!layer_args_from_c(&s.moe, &b.moe))
        return Error::make(ErrorCode::InvalidArgument, "decoder: null expert weights in block " + std::to_string(l));
      if (b.moe.D != D) return Error::make(ErrorCode::InvalidArgument, "decoder: MoE d_model differs from the model's");
      b.attn_norm = s.attn_norm;
      b.ffn_norm = s.ffn_norm;
      b.wq = s.wq; b.wq_fmt = s.wq_fmt;
      b.wk = s.wk; b.wk_fmt = s.wk_fmt;
      b.wv = s.wv; b.wv_fmt = s.wv_fmt;
      b.wo = s.wo; b.wo_fmt = s.wo_fmt;
      for (const void* p : {(const void*)s.attn_norm, s.wq, s.wk, s.wv, s.wo, (const void*)s.ffn_norm})
        if (!is_device_ptr(p)) return Error::make(ErrorCode::InvalidArgument, "decoder: weights must be device memory");
      for (int f : {b.wq_fmt, b.wk_fmt, b.wv_fmt, b.wo_fmt})
        if (!fmt_is_gguf(f)) return Error::make(ErrorCode::NotImplemented, "decoder: attention weights must be GGUF blocks");
      // one projection for q, k and v when they share a format: their packed rows back to back
      if (b.wq_fmt == b.wk_fmt && b.wk_fmt == b.wv_fmt) {
        const size_t rb = (size_t)fmt_row_bytes(b.wq_fmt, D);
        UAII_CUDA(cudaMalloc(&b.wqkv, rb * (size_t)(q_dim_ + 2 * kv_dim_)), "Malloc(wqkv)");
        char* dst = static_cast<char*>(b.wqkv);
        UAII_CUDA(cudaMemcpyAsync(dst, b.wq, rb * q_dim_, cudaMemcpyDeviceToDevice, st), "Memcpy(wq)");
        UAII_CUDA(cudaMemcpyAsync(dst + rb * q_dim_, b.wk, rb * kv_dim_, cudaMemcpyDeviceToDevice, st), "Memcpy(wk)");
        UAII_CUDA(cudaMemcpyAsync(dst + rb * (q_dim_ + kv_dim_), b.wv, rb * kv_dim_, cudaMemcpyDeviceToDevice, st),
                  "Memcpy(wv)");
      }
    }
    // RoPE frequencies exactly as rope_f32 computes them (libs/uaii-kernels/src/transformer.cpp:201-222)
    std::vector<float> freq((size_t)(hd / 2));
    for (int64_t i = 0; i < hd / 2; ++i)
      freq[(size_t)i] = c.rope_mode == 2
                            ? 1.0f / std::pow(c.rope_theta, (2.0f * (float)i) / (float)hd)
                            : 1.0f / std::pow(c.rope_theta, (float)(2 * i) / (float)hd);
    const int64_t B = c.batch;
    const int ns = attn_splits(c.max_seq);
    auto dmalloc = [&](void** p, size_t bytes, const char* what) { return cuda_status(cudaMalloc(p, bytes), what); };
    UAII_TRY(dmalloc((void**)&freq_, sizeof(float) * freq.size(), "Malloc(freq)"));
    UAII_CUDA(cudaMemcpy(freq_, freq.data(), sizeof(float) * freq.size(), cudaMemcpyHostToDevice), "Memcpy(freq)");
    const size_t kv_bytes = sizeof(uint16_t) * (size_t)(B * Hkv) * (size_t)c.max_seq * (size_t)hd;
    kc_.assign((size_t)L, nullptr);
    vc_.assign((size_t)L, nullptr);
    maps_.assign((size_t)(2 * L), KvMap{});
    for (int64_t l = 0; l < L; ++l) {
      UAII_TRY(dmalloc(&kc_[(size_t)l], kv_bytes, "Malloc(K cache)"));
      UAII_TRY(dmalloc(&vc_[(size_t)l], kv_bytes, "Malloc(V cache)"));
      UAII_CUDA(cudaMemsetAsync(kc_[(size_t)l], 0, kv_bytes, st), "Memset(K cache)");
      UAII_CUDA(cudaMemsetAsync(vc_[(size_t)l], 0, kv_bytes, st), "Memset(V cache)");
      if (!make_kv_map(maps_[(size_t)(2 * l)].bytes, kc_[(size_t)l], B * Hkv * c.max_seq) ||
          !make_kv_map(maps_[(size_t)(2 * l + 1)].bytes, vc_[(size_t)l], B * Hkv * c.max_seq))
        return Error::make(ErrorCode::Internal, "decoder: KV-cache tensor map");
    }
    UAII_TRY(dmalloc((void**)&x_, sizeof(float) * (size_t)(B * D), "Malloc(x)"));
    UAII_TRY(dmalloc((void**)&n_, sizeof(float) * (size_t)(B * D), "Malloc(n)"));
    UAII_TRY(dmalloc((void**)&o_, sizeof(float) * (size_t)(B * D), "Malloc(o)"));
    UAII_TRY(dmalloc((void**)&ff_, sizeof(float) * (size_t)(B * D), "Malloc(ff)"));
    UAII_TRY(dmalloc((void**)&qkv_, sizeof(float) * (size_t)(B * (q_dim_ + 2 * kv_dim_)), "Malloc(qkv)"));
    UAII_TRY(dmalloc((void**)&q_, sizeof(float) * (size_t)(B * q_dim_), "Malloc(q)"));
    UAII_TRY(dmalloc((void**)&attn_, sizeof(float) * (size_t)(B * q_dim_), "Malloc(attn)"));
    UAII_TRY(dmalloc((void**)&po_, sizeof(float) * (size_t)(B * H * ns * hd), "Malloc(attn partials)"));
    UAII_TRY(dmalloc((void**)&pm_, sizeof(float) * (size_t)(B * H * ns), "Malloc(attn maxima)"));
    UAII_TRY(dmalloc((void**)&pl_, sizeof(float) * (size_t)(B * H * ns), "Malloc(attn sums)"));
    UAII_TRY(dmalloc((void**)&logits_, sizeof(float) * (size_t)(B * c.vocab), "Malloc(logits)"));
    UAII_TRY(dmalloc((void**)&tokens_, sizeof(int32_t) * (size_t)B, "Malloc(tokens)"));
    UAII_TRY(dmalloc((void**)&next_, sizeof(int32_t) * (size_t)B, "Malloc(next)"));
    UAII_TRY(dmalloc((void**)&err_, sizeof(int), "Malloc(error flag)"));
    UAII_CUDA(cudaMemsetAsync(err_, 0, sizeof(int), st), "Memset(error flag)");
    UAII_CUDA(cudaStreamSynchronize(st), "StreamSynchronize");
    pos_ = 0;
    return Error::success();
  }

  void release() noexcept {
    if (!be_) return;
    (void)cudaSetDevice(be_->device());
    (void)cudaStreamSynchronize(be_->stream());
    for (auto& b : blocks_) (void)cudaFree(b.wqkv);
    blocks_.clear();
    for (void* p : kc_) (void)cudaFree(p);
    for (void* p : vc_) (void)cudaFree(p);
    kc_.clear();
    vc_.clear();
    for (void* p : {(void*)freq_, (void*)x_, (void*)n_, (void*)o_, (void*)ff_, (void*)qkv_, (void*)q_, (void*)attn_,
                    (void*)po_, (void*)pm_, (void*)pl_, (void*)logits_, (void*)tokens_, (void*)next_, (void*)err_})
      (void)cudaFree(p);
    be_ = nullptr;
  }

  int64_t position() const { return pos_; }

  // Cache positions [0, n) of one layer from f32 K and V [batch, kv_heads, n, head_dim]
  // (host or device), rounded to f16; the decode position becomes n.
  Error set_kv(int64_t layer, const float* k, const float* v, int64_t n) {
    if (layer < 0 || layer >= cfg_.n_layers || n < 0 || n > cfg_.max_seq || !k || !v)
      return Error::make(ErrorCode::InvalidArgument, "decoder set_kv: layer or position count out of range");
    UAII_CUDA(cudaSetDevice(be_->device()), "SetDevice");
    const int64_t rows = cfg_.batch * cfg_.n_kv_heads, hd = cfg_.head_dim;
    const size_t bytes = sizeof(float) * (size_t)(rows * n * hd);
    float* tmp = nullptr;
    UAII_CUDA(cudaMalloc(&tmp, bytes ? bytes : 4), "Malloc(kv staging)");
    Error e = Error::success();
    cudaStream_t st = be_->stream();
    for (int kv = 0; kv < 2 && e.ok(); ++kv) {
      e = cuda_status(cudaMemcpyAsync(tmp, kv ? v : k, bytes, cudaMemcpyDefault, st), "Memcpy(kv)");
      if (e.ok()) e = cuda_status(launch_to_half_rows(tmp, rows, n * hd, kv ? vc_[(size_t)layer] : kc_[(size_t)layer],
                                                      cfg_.max_seq * hd, st),
                                  "kv to f16");
    }
    if (e.ok()) e = cuda_status(cudaStreamSynchronize(st), "StreamSynchronize");
    (void)cudaFree(tmp);
    if (e.ok()) pos_ = n;
    return e;
  }

  // Synthetic prefill: every layer's K and V at positions [0, n) drawn N(0, 1) (seeded,
  // counter-based); the decode position becomes n.
  Error fill_kv(int64_t n, uint64_t seed) {
    if (n < 0 || n > cfg_.max_seq) return Error::make(ErrorCode::InvalidArgument, "decoder fill_kv: n out of range");
    UAII_CUDA(cudaSetDevice(be_->device()), "SetDevice");
    const int64_t rows = cfg_.batch * cfg_.n_kv_heads, hd = cfg_.head_dim;
    for (int64_t l = 0; l < cfg_.n_layers; ++l)
      for (int kv = 0; kv < 2; ++kv)  // (sequence, kv head) rows of n * head_dim values, max_seq * head_dim apart
        UAII_CUDA(launch_fill_normal_f16_rows(kv ? vc_[(size_t)l] : kc_[(size_t)l], rows, n * hd, cfg_.max_seq * hd,
                                              seed, (uint64_t)((l * 2 + kv) * rows), 0.0f, 1.0f, be_->stream()),
                  "fill_kv");
    UAII_CUDA(cudaStreamSynchronize(be_->stream()), "StreamSynchronize");
    pos_ = n;
    return Error::success();
  }

  // One decode step at the current position for every sequence: tokens [batch] (host or
  // device); logits [batch, vocab] and next [batch] (host, device or null).
  Error step(const int32_t* tokens, float* logits, int32_t* next) {
    if (!tokens) return Error::make(ErrorCode::InvalidArgument, "decoder step: null tokens");
    if (pos_ >= cfg_.max_seq) return Error::make(ErrorCode::InvalidArgument, "decoder step: the cache is full");
    UAII_CUDA(cudaSetDevice(be_->device()), "SetDevice");
    cudaStream_t st = be_->stream();
    const int64_t B = cfg_.batch, D = cfg_.d_model, H = cfg_.n_heads, Hkv = cfg_.n_kv_heads, hd = cfg_.head_dim;
    UAII_CUDA(cudaMemcpyAsync(tokens_, tokens, sizeof(int32_t) * (size_t)B, cudaMemcpyDefault, st), "Memcpy(tokens)");
    UAII_CUDA(launch_embed(embd_fmt_, embd_, cfg_.vocab, D, tokens_, B, x_, err_, st), "embed");
    for (int64_t l = 0; l < cfg_.n_layers; ++l) {
      const DecoderBlock& b = blocks_[(size_t)l];
      UAII_CUDA(launch_add_rmsnorm(x_, l ? ff_ : nullptr, b.attn_norm, B, D, cfg_.rms_eps, n_, st), "rmsnorm(attn)");
      if (b.wqkv) {
        UAII_TRY(be_->quant_matmul(n_, B, D, b.wqkv, b.wq_fmt, q_dim_ + 2 * kv_dim_, qkv_, false));
      } else {  // separate projections into the same row layout: q | k | v
        UAII_TRY(project_into(b.wq, b.wq_fmt, q_dim_, 0));
        UAII_TRY(project_into(b.wk, b.wk_fmt, kv_dim_, q_dim_));
        UAII_TRY(project_into(b.wv, b.wv_fmt, kv_dim_, q_dim_ + kv_dim_));
      }
      UAII_CUDA(launch_rope_append(qkv_, B, H, Hkv, hd, freq_, pos_, cfg_.rope_mode, q_, kc_[(size_t)l],
                                   vc_[(size_t)l], cfg_.max_seq, st),
                "rope_append");
      UAII_CUDA(launch_attn_decode(maps_[(size_t)(2 * l)].bytes, maps_[(size_t)(2 * l + 1)].bytes, q_, B, H, Hkv, hd,
                                   pos_ + 1, cfg_.max_seq, po_, pm_, pl_, attn_, err_, st),
                "attention");
      UAII_TRY(be_->quant_matmul(attn_, B, q_dim_, b.wo, b.wo_fmt, D, o_, false));
      UAII_CUDA(launch_add_rmsnorm(x_, o_, b.ffn_norm, B, D, cfg_.rms_eps, n_, st), "rmsnorm(ffn)");
      UAII_TRY(be_->ffn(b.moe, n_, B, ff_, nullptr));
    }
    UAII_CUDA(launch_add_rmsnorm(x_, ff_, out_norm_, B, D, cfg_.rms_eps, n_, st), "rmsnorm(out)");
    UAII_TRY(be_->quant_matmul(n_, B, D, output_, output_fmt_, cfg_.vocab, logits_, false));
    UAII_CUDA(launch_argmax(logits_, B, cfg_.vocab, next_, st), "argmax");
    be_->add_launches(3 + 5 * (uint64_t)cfg_.n_layers);  // embed, per block 2 norms + rope + 2 attention, norm, argmax
    if (logits)
      UAII_CUDA(cudaMemcpyAsync(logits, logits_, sizeof(float) * (size_t)(B * cfg_.vocab), cudaMemcpyDefault, st),
                "Memcpy(logits)");
    if (next) UAII_CUDA(cudaMemcpyAsync(next, next_, sizeof(int32_t) * (size_t)B, cudaMemcpyDefault, st), "Memcpy(next)");
    ++pos_;
    const bool host_out = (logits && !is_device_ptr(logits)) || (next && !is_device_ptr(next));
    if (host_out) UAII_TRY(check_flag());
    return Error::success();
  }

  // `steps` greedy steps from tokens [batch]: out [steps, batch] (host or device); each
  // step's arg-max is the next step's input, without leaving the device.
  Error generate(const int32_t* tokens, int64_t steps, int32_t* out) {
    if (!tokens || !out || steps < 0) return Error::make(ErrorCode::InvalidArgument, "decoder generate: bad arguments");
    if (pos_ + steps > cfg_.max_seq) return Error::make(ErrorCode::InvalidArgument, "decoder generate: cache too short");
    UAII_CUDA(cudaSetDevice(be_->device()), "SetDevice");
    const int64_t B = cfg_.batch;
    const int32_t* in = tokens;
    for (int64_t s = 0; s < steps; ++s) {
      UAII_TRY(step(in, nullptr, nullptr));
      UAII_CUDA(cudaMemcpyAsync(out + s * B, next_, sizeof(int32_t) * (size_t)B, cudaMemcpyDefault, be_->stream()),
                "Memcpy(tokens out)");
      in = next_;  // the next step copies it to its input on the stream before the arg-max overwrites it
    }
    return check_flag();
  }

 private:
  Error project_into(const void* w, int fmt, int64_t rows, int64_t col0) {
    // the packed-MatMul writes [B, rows] densely: project into o_ scratch, then place the columns
    const int64_t B = cfg_.batch;
    float* tmp = rows <= cfg_.d_model ? ff_ : nullptr;
    if (!tmp) return Error::make(ErrorCode::NotImplemented, "decoder: separate q projection wider than d_model");
    UAII_TRY(be_->quant_matmul(n_, B, cfg_.d_model, w, fmt, rows, tmp, false));
    UAII_CUDA(cudaMemcpy2DAsync(qkv_ + col0, sizeof(float) * (size_t)(q_dim_ + 2 * kv_dim_), tmp,
                                sizeof(float) * (size_t)rows, sizeof(float) * (size_t)rows, (size_t)B,
                                cudaMemcpyDeviceToDevice, be_->stream()),
              "Memcpy2D(qkv)");
    return Error::success();
  }

  Error check_flag() {
    UAII_TRY(be_->sync_and_check_public());
    int flag = 0;
    UAII_CUDA(cudaMemcpy(&flag, err_, sizeof(int), cudaMemcpyDeviceToHost), "Memcpy(error flag)");
    if (flag) {
      (void)cudaMemset(err_, 0, sizeof(int));
      if (flag == 17) return Error::make(ErrorCode::Internal, "attention: a KV-cache copy did not complete");
      return Error::make(ErrorCode::InvalidArgument, "embedding token id out of range");
    }
    return Error::success();
  }

  MoeCudaBackend* be_ = nullptr;
  uaii_moe_decoder_config cfg_{};
  int64_t q_dim_ = 0, kv_dim_ = 0, pos_ = 0;
  std::vector<DecoderBlock> blocks_;
  const float* out_norm_ = nullptr;
  const void* embd_ = nullptr;
  const void* output_ = nullptr;
  int embd_fmt_ = 0, output_fmt_ = 0;
  float* freq_ = nullptr;
  std::vector<void*> kc_, vc_;
  struct KvMap {
    alignas(64) unsigned char bytes[kKvMapBytes];
  };
  std::vector<KvMap> maps_;  // TMA maps of each layer's K and V caches
  float *x_ = nullptr, *n_ = nullptr, *o_ = nullptr, *ff_ = nullptr, *qkv_ = nullptr, *q_ = nullptr, *attn_ = nullptr;
  float *po_ = nullptr, *pm_ = nullptr, *pl_ = nullptr, *logits_ = nullptr;
  int32_t *tokens_ = nullptr, *next_ = nullptr;
  int* err_ = nullptr;
};

}  // namespace uaii_b200

using namespace uaii_b200;

struct uaii_moe_decoder {
  Decoder impl;
};

extern "C" {

int uaii_moe_decoder_create(uaii_moe_backend* b, const uaii_moe_decoder_config* cfg,
                            const uaii_moe_decoder_block* blocks, const float* output_norm, const void* token_embd,
                            int embd_fmt, const void* output, int output_fmt, uaii_moe_decoder** out) {
  if (!b || !cfg || !out) return report_status(Error::make(ErrorCode::InvalidArgument, "decoder create: null argument"));
  *out = nullptr;
  auto* d = new uaii_moe_decoder();
  const Error e = d->impl.create(&b->impl, *cfg, blocks, output_norm, token_embd, embd_fmt, output, output_fmt);
  if (!e.ok()) {
    delete d;
    return report_status(e);
  }
  *out = d;
  return report_status(Error::success());
}

void uaii_moe_decoder_destroy(uaii_moe_decoder* d) { delete d; }

int uaii_moe_decoder_set_kv(uaii_moe_decoder* d, int64_t layer, const float* k, const float* v, int64_t n_pos) {
  if (!d) return report_status(Error::make(ErrorCode::InvalidArgument, "null decoder"));
  return report_status(d->impl.set_kv(layer, k, v, n_pos));
}

int uaii_moe_decoder_fill_kv(uaii_moe_decoder* d, int64_t n_pos, uint64_t seed) {
  if (!d) return report_status(Error::make(ErrorCode::InvalidArgument, "null decoder"));
  return report_status(d->impl.fill_kv(n_pos, seed));
}

int uaii_moe_decoder_step(uaii_moe_decoder* d, const int32_t* tokens, float* logits, int32_t* next) {
  if (!d) return report_status(Error::make(ErrorCode::InvalidArgument, "null decoder"));
  return report_status(d->impl.step(tokens, logits, next));
}

int uaii_moe_decoder_generate(uaii_moe_decoder* d, const int32_t* tokens, int64_t steps, int32_t* out) {
  if (!d) return report_status(Error::make(ErrorCode::InvalidArgument, "null decoder"));
  return report_status(d->impl.generate(tokens, steps, out));
}

int64_t uaii_moe_decoder_position(const uaii_moe_decoder* d) { return d ? d->impl.position() : -1; }

int uaii_moe_fill_normal_device(uaii_moe_backend* b, float* out, int64_t n, uint64_t seed, uint64_t stream, float mean,
                                float std) {
  if (!b || !out || n < 0) return report_status(Error::make(ErrorCode::InvalidArgument, "fill_normal_device args"));
  if (!is_device_ptr(out)) return report_status(Error::make(ErrorCode::InvalidArgument, "out must be device memory"));
  return report_status(cuda_status(launch_fill_normal(out, n, seed, stream, mean, std, b->impl.stream()), "fill_normal"));
}

int uaii_moe_quantize_rows_device(uaii_moe_backend* b, int fmt, const float* src, int64_t rows, int64_t cols,
                                  void* dst) {
  if (!b || !src || !dst || rows < 0 || cols <= 0)
    return report_status(Error::make(ErrorCode::InvalidArgument, "quantize_rows_device args"));
  if (!(fmt == kQ4_0 || fmt == kQ8_0 || fmt == kQ4_K || fmt == kQ6_K))
    return report_status(Error::make(ErrorCode::NotImplemented, "quantize_rows_device: Q4_0, Q8_0, Q4_K, Q6_K only"));
  if (cols % fmt_block_elems(fmt) != 0)
    return report_status(Error::make(ErrorCode::InvalidArgument, "quantize_rows_device: cols not a block multiple"));
  if (!is_device_ptr(src) || !is_device_ptr(dst))
    return report_status(Error::make(ErrorCode::InvalidArgument, "src and dst must be device memory"));
  return report_status(cuda_status(launch_quantize_rows(fmt, src, rows, cols, dst, b->impl.stream()), "quantize"));
}

}  // extern "C"
