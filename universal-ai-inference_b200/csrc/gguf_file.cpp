// gguf_file.cpp -- GGUF files mapped read-only.
//
// The header, metadata and tensor index are parsed once; tensor data is handed out
// as pointers into the mapping, so a layer's packed expert stacks are never copied
// on the host (they go to the device once, through uaii_moe_register_weights).
// The reference reads the whole file into memory for the header and again for every
// tensor it loads (gguf_read_header, gguf_load_tensor_raw:
// libs/uaii-loaders/src/gguf.cpp:374-443, :558-602, through ByteReader::from_file,
// libs/uaii-loaders/src/binary_io.hpp:20-35), which cannot load a 30 GB Mixtral file.
//
// Format (GGUF v2/v3, as the reference parses it): "GGUF", u32 version, u64 tensor
// count, u64 metadata count; metadata = (string key, u32 value type, value); tensor
// infos = (string name, u32 n_dims, u64 dims[n_dims] innermost first, u32 ggml type,
// u64 offset); data starts at the next multiple of the alignment.  Strings are a u64
// length and bytes.  Every read is bounds-checked against the file size.
//
// Differences from the reference, on purpose: the data alignment honours
// `general.alignment` (the GGUF rule) where the reference always uses 32 (the same
// for files that do not set it); tensor types the reference does not map (I8 and
// wider) are listed with format -1 instead of rejected at parse time.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/uaii_moe.h"
#include "backend.hpp"
#include "gguf_format.hpp"

using namespace uaii_b200;

struct uaii_moe_gguf {
  int fd = -1;
  const uint8_t* base = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32;
  uint64_t data_offset = 0;
  struct Value {
    uint32_t type = 0;  // GGUF value type
    int64_t i = 0;      // integer and bool types
    double f = 0.0;     // float types
    std::string s;      // strings
    uint64_t count = 0; // arrays: element count (elements not kept)
  };
  std::map<std::string, Value> kv;
  struct Tensor {
    std::string name;
    std::vector<int64_t> shape;  // outermost first (the reference's dims_to_shape)
    uint32_t ggml_type = 0;
    int fmt = -1;
    uint64_t offset = 0, nbytes = 0;
  };
  std::vector<Tensor> tensors;
  std::map<std::string, size_t> by_name;
  ~uaii_moe_gguf() {
    if (base) munmap(const_cast<uint8_t*>(base), size);
    if (fd >= 0) close(fd);
  }
};

namespace {

enum : uint32_t { kU8 = 0, kI8, kU16, kI16, kU32, kI32, kF32v, kBool, kString, kArray, kU64, kI64, kF64v };

// ggml tensor type -> uaii::quant::QuantFormat (include/uaii/quant/formats.hpp:10-29), -1 if none
int fmt_of_ggml(uint32_t t) {
  switch (t) {
    case 0: return kF32;
    case 1: return kF16;
    case 2: return kQ4_0;
    case 3: return kQ4_1;
    case 6: return kQ5_0;
    case 7: return kQ5_1;
    case 8: return kQ8_0;
    case 10: return kQ2_K;
    case 11: return kQ3_K;
    case 12: return kQ4_K;
    case 13: return kQ5_K;
    case 14: return kQ6_K;
    default: return -1;
  }
}

struct Cursor {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  template <class T>
  T get() {
    T v{};
    if (!ok || n - pos < sizeof(T)) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  bool skip(uint64_t bytes) {
    if (!ok || bytes > n - pos) return ok = false;
    pos += (size_t)bytes;
    return true;
  }
  std::string str() {
    const uint64_t len = get<uint64_t>();
    if (!ok || len > n - pos) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p + pos), (size_t)len);
    pos += (size_t)len;
    return s;
  }
};

size_t scalar_bytes(uint32_t t) {
  switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32v: return 4;
    case kU64: case kI64: case kF64v: return 8;
    default: return 0;
  }
}

bool read_value(Cursor& c, uint32_t type, uaii_moe_gguf::Value* v, int depth) {
  v->type = type;
  switch (type) {
    case kU8: v->i = c.get<uint8_t>(); break;
    case kI8: v->i = c.get<int8_t>(); break;
    case kU16: v->i = c.get<uint16_t>(); break;
    case kI16: v->i = c.get<int16_t>(); break;
    case kU32: v->i = c.get<uint32_t>(); break;
    case kI32: v->i = c.get<int32_t>(); break;
    case kU64: v->i = (int64_t)c.get<uint64_t>(); break;
    case kI64: v->i = c.get<int64_t>(); break;
    case kBool: v->i = c.get<int8_t>() != 0; break;
    case kF32v: v->f = c.get<float>(); break;
    case kF64v: v->f = c.get<double>(); break;
    case kString: v->s = c.str(); break;
    case kArray: {
      if (depth > 0) return c.ok = false;  // arrays of arrays: not in GGUF model files
      const uint32_t et = c.get<uint32_t>();
      const uint64_t count = c.get<uint64_t>();
      v->count = count;
      if (!c.ok) return false;
      if (et == kString) {
        for (uint64_t i = 0; i < count && c.ok; ++i) (void)c.str();
      } else {
        const size_t b = scalar_bytes(et);
        if (b == 0 || count > (c.n - c.pos) / b) return c.ok = false;
        c.skip(count * b);
      }
      break;
    }
    default: return c.ok = false;
  }
  return c.ok;
}

Error parse(uaii_moe_gguf* g) {
  Cursor c{g->base, g->size};
  char magic[4];
  for (char& m : magic) m = (char)c.get<uint8_t>();
  if (!c.ok || std::memcmp(magic, "GGUF", 4) != 0) return Error::make(ErrorCode::InvalidArgument, "not a GGUF file");
  g->version = c.get<uint32_t>();
  const uint64_t n_tensors = c.get<uint64_t>();
  const uint64_t n_kv = c.get<uint64_t>();
  if (!c.ok || g->version < 2) return Error::make(ErrorCode::InvalidArgument, "unsupported GGUF version (v2/v3)");
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = c.str();
    const uint32_t vt = c.get<uint32_t>();
    uaii_moe_gguf::Value v;
    if (!c.ok || !read_value(c, vt, &v, 0))
      return Error::make(ErrorCode::InvalidArgument, "GGUF metadata truncated or of unknown type");
    g->kv[std::move(key)] = std::move(v);
  }
  auto al = g->kv.find("general.alignment");
  if (al != g->kv.end() && al->second.type != kString && al->second.type != kArray && al->second.i > 0)
    g->alignment = (uint64_t)al->second.i;
  if ((g->alignment & (g->alignment - 1)) != 0) return Error::make(ErrorCode::InvalidArgument, "GGUF alignment");
  if (n_tensors > (g->size - c.pos) / 24) return Error::make(ErrorCode::InvalidArgument, "GGUF tensor count");
  g->tensors.reserve((size_t)n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    uaii_moe_gguf::Tensor t;
    t.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (!c.ok || nd == 0 || nd > 8) return Error::make(ErrorCode::InvalidArgument, "GGUF tensor info");
    std::vector<uint64_t> dims(nd);
    for (auto& d : dims) d = c.get<uint64_t>();
    t.ggml_type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (!c.ok) return Error::make(ErrorCode::InvalidArgument, "GGUF tensor info truncated");
    uint64_t numel = 1;
    for (auto it = dims.rbegin(); it != dims.rend(); ++it) {
      if (*it == 0 || *it > (1ull << 40) || numel > (1ull << 62) / *it)
        return Error::make(ErrorCode::InvalidArgument, "GGUF tensor dims");
      numel *= *it;
      t.shape.push_back((int64_t)*it);
    }
    t.fmt = fmt_of_ggml(t.ggml_type);
    if (t.fmt >= 0) {
      const uint64_t row = dims[0];
      if (row % (uint64_t)fmt_block_elems(t.fmt) != 0)
        return Error::make(ErrorCode::InvalidArgument, "GGUF tensor " + t.name + ": row not whole blocks");
      t.nbytes = (uint64_t)fmt_row_bytes(t.fmt, (long long)row) * (numel / row);
    }
    g->by_name[t.name] = g->tensors.size();
    g->tensors.push_back(std::move(t));
  }
  g->data_offset = (c.pos + g->alignment - 1) / g->alignment * g->alignment;
  for (const auto& t : g->tensors)
    if (t.fmt >= 0 && (t.offset > g->size || g->data_offset > g->size - t.offset ||
                       t.nbytes > g->size - g->data_offset - t.offset))
      return Error::make(ErrorCode::InvalidArgument, "GGUF tensor " + t.name + " extends past the end of the file");
  return Error::success();
}

const uaii_moe_gguf::Tensor* find(const uaii_moe_gguf* g, const std::string& name) {
  auto it = g->by_name.find(name);
  return it == g->by_name.end() ? nullptr : &g->tensors[it->second];
}

bool kv_int(const uaii_moe_gguf* g, const std::string& key, int64_t* out) {
  auto it = g->kv.find(key);
  if (it == g->kv.end() || it->second.type == kString || it->second.type == kArray || it->second.type == kF32v ||
      it->second.type == kF64v)
    return false;
  *out = it->second.i;
  return true;
}

// `{architecture}.suffix`, then `llama.suffix`, then `general.suffix` (the reference's
// kv_i64_arch, libs/uaii-loaders/src/gguf.cpp:734-748); negative values count as absent
int64_t kv_arch(const uaii_moe_gguf* g, const std::string& arch, const char* suffix, int64_t def) {
  int64_t v = -1;
  if (!arch.empty() && kv_int(g, arch + "." + suffix, &v) && v >= 0) return v;
  if (kv_int(g, std::string("llama.") + suffix, &v) && v >= 0) return v;
  if (kv_int(g, std::string("general.") + suffix, &v) && v >= 0) return v;
  return def;
}

int report(const Error& e) { return report_status(e); }

}  // namespace

extern "C" {

int uaii_moe_gguf_open(const char* path, uaii_moe_gguf** out) {
  if (!path || !out) return report(Error::make(ErrorCode::InvalidArgument, "gguf open: null argument"));
  *out = nullptr;
  auto* g = new uaii_moe_gguf();
  g->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (g->fd < 0) {
    delete g;
    return report(Error::make(ErrorCode::NotFound, std::string("cannot open ") + path));
  }
  struct stat st {};
  if (fstat(g->fd, &st) != 0 || st.st_size < 24) {
    delete g;
    return report(Error::make(ErrorCode::InvalidArgument, "not a GGUF file (too short)"));
  }
  g->size = (size_t)st.st_size;
  void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
  if (m == MAP_FAILED) {
    delete g;
    return report(Error::make(ErrorCode::Internal, "mmap failed"));
  }
  g->base = static_cast<const uint8_t*>(m);
  const Error e = parse(g);
  if (!e.ok()) {
    delete g;
    return report(e);
  }
  *out = g;
  return report(Error::success());
}

void uaii_moe_gguf_close(uaii_moe_gguf* g) { delete g; }

int64_t uaii_moe_gguf_tensor_count(const uaii_moe_gguf* g) { return g ? (int64_t)g->tensors.size() : -1; }

int uaii_moe_gguf_tensor_at(const uaii_moe_gguf* g, int64_t index, const char** name, const void** data, int* fmt,
                            int64_t* shape, int* rank, uint64_t* nbytes) {
  if (!g || index < 0 || index >= (int64_t)g->tensors.size())
    return report(Error::make(ErrorCode::InvalidArgument, "gguf tensor index"));
  const auto& t = g->tensors[(size_t)index];
  if (name) *name = t.name.c_str();
  if (data) *data = t.fmt >= 0 ? g->base + g->data_offset + t.offset : nullptr;
  if (fmt) *fmt = t.fmt;
  if (rank) *rank = (int)t.shape.size();
  if (shape)
    for (size_t i = 0; i < t.shape.size() && i < 8; ++i) shape[i] = t.shape[i];
  if (nbytes) *nbytes = t.nbytes;
  return report(Error::success());
}

int uaii_moe_gguf_tensor(const uaii_moe_gguf* g, const char* name, const void** data, int* fmt, int64_t* shape,
                         int* rank, uint64_t* nbytes) {
  if (!g || !name) return report(Error::make(ErrorCode::InvalidArgument, "gguf tensor: null argument"));
  auto it = g->by_name.find(name);
  if (it == g->by_name.end())
    return report(Error::make(ErrorCode::NotFound, std::string("tensor not in gguf: ") + name));
  return uaii_moe_gguf_tensor_at(g, (int64_t)it->second, nullptr, data, fmt, shape, rank, nbytes);
}

int uaii_moe_gguf_kv_int(const uaii_moe_gguf* g, const char* key, int64_t* out) {
  if (!g || !key || !out) return report(Error::make(ErrorCode::InvalidArgument, "gguf kv: null argument"));
  if (!kv_int(g, key, out)) return report(Error::make(ErrorCode::NotFound, std::string("no integer key ") + key));
  return report(Error::success());
}

int uaii_moe_gguf_kv_float(const uaii_moe_gguf* g, const char* key, double* out) {
  if (!g || !key || !out) return report(Error::make(ErrorCode::InvalidArgument, "gguf kv: null argument"));
  auto it = g->kv.find(key);
  if (it == g->kv.end() || it->second.type == kString || it->second.type == kArray)
    return report(Error::make(ErrorCode::NotFound, std::string("no number key ") + key));
  *out = (it->second.type == kF32v || it->second.type == kF64v) ? it->second.f : (double)it->second.i;
  return report(Error::success());
}

int uaii_moe_gguf_kv_string(const uaii_moe_gguf* g, const char* key, const char** out) {
  if (!g || !key || !out) return report(Error::make(ErrorCode::InvalidArgument, "gguf kv: null argument"));
  auto it = g->kv.find(key);
  if (it == g->kv.end() || it->second.type != kString)
    return report(Error::make(ErrorCode::NotFound, std::string("no string key ") + key));
  *out = it->second.s.c_str();
  return report(Error::success());
}

int uaii_moe_gguf_moe_layer(const uaii_moe_gguf* g, int block, int flags, uaii_moe_layer* L) {
  if (!g || !L || block < 0) return report(Error::make(ErrorCode::InvalidArgument, "gguf moe layer: argument"));
  std::memset(L, 0, sizeof(*L));
  std::string arch = "llama";
  auto a = g->kv.find("general.architecture");
  if (a != g->kv.end() && a->second.type == kString) arch = a->second.s;
  const std::string pfx = "blk." + std::to_string(block) + ".";
  const auto* router = find(g, pfx + "ffn_gate_inp.weight");
  const auto* gate = find(g, pfx + "ffn_gate_exps.weight");
  const auto* up = find(g, pfx + "ffn_up_exps.weight");
  const auto* down = find(g, pfx + "ffn_down_exps.weight");
  if (!router || !gate || !up || !down)
    return report(Error::make(ErrorCode::NotFound, "block " + std::to_string(block) + " has no MoE FFN tensors"));
  if (router->fmt != kF32 || router->shape.size() != 2)
    return report(Error::make(ErrorCode::NotImplemented, pfx + "ffn_gate_inp.weight must be f32 [E, D]"));
  if (gate->shape.size() != 3 || up->shape != gate->shape || down->shape.size() != 3)
    return report(Error::make(ErrorCode::InvalidArgument, pfx + "expert stacks must be rank 3"));
  const int64_t E = gate->shape[0], I = gate->shape[1], D = gate->shape[2];
  if (router->shape[0] != E || router->shape[1] != D || down->shape[0] != E || down->shape[1] != D ||
      down->shape[2] != I)
    return report(Error::make(ErrorCode::InvalidArgument, pfx + "MoE tensor shapes disagree"));
  if (gate->fmt < 0 || up->fmt < 0 || down->fmt < 0)
    return report(Error::make(ErrorCode::NotImplemented, pfx + "expert tensor type not supported"));
  int64_t n_experts = kv_arch(g, arch, "expert_count", 0);
  if (n_experts <= 0) n_experts = E;
  if (n_experts != E) return report(Error::make(ErrorCode::InvalidArgument, "expert_count disagrees with the tensors"));
  int64_t top_k = kv_arch(g, arch, "expert_used_count", 2);  // the reference's default and clamp (gguf.cpp:1088-1090)
  if (top_k <= 0) top_k = 2;
  if (top_k > E) top_k = E;
  const auto ptr = [g](const uaii_moe_gguf::Tensor* t) { return static_cast<const void*>(g->base + g->data_offset + t->offset); };
  L->d_model = D;
  L->n_experts = E;
  L->d_ff = I;
  L->top_k = (int32_t)top_k;
  L->norm_topk = 1;  // the reference always renormalises (transformer.cpp:574-580)
  L->router_w = static_cast<const float*>(ptr(router));
  L->gate_exps = ptr(gate);
  L->gate_fmt = gate->fmt;
  L->up_exps = ptr(up);
  L->up_fmt = up->fmt;
  L->down_exps = ptr(down);
  L->down_fmt = down->fmt;
  const auto* gs = find(g, pfx + "ffn_gate_shexp.weight");
  const auto* us = find(g, pfx + "ffn_up_shexp.weight");
  const auto* ds = find(g, pfx + "ffn_down_shexp.weight");
  if (gs && us && ds) {  // the reference adds SwiGLU(x) of the shared expert without a gate (gguf.cpp:1107-1128)
    if (gs->shape.size() != 2 || us->shape != gs->shape || ds->shape.size() != 2 || gs->shape[1] != D ||
        ds->shape[0] != D || ds->shape[1] != gs->shape[0] || gs->fmt < 0 || us->fmt < 0 || ds->fmt < 0)
      return report(Error::make(ErrorCode::InvalidArgument, pfx + "shared expert shapes"));
    L->shared_d_ff = gs->shape[0];
    L->gate_shexp = ptr(gs);
    L->gate_shexp_fmt = gs->fmt;
    L->up_shexp = ptr(us);
    L->up_shexp_fmt = us->fmt;
    L->down_shexp = ptr(ds);
    L->down_shexp_fmt = ds->fmt;
    const auto* gi = find(g, pfx + "ffn_gate_inp_shexp.weight");
    if ((flags & UAII_MOE_GGUF_SHEXP_GATE) && gi) {  // Qwen2-MoE's sigmoid gate (no reference counterpart)
      if (gi->fmt != kF32 || gi->nbytes != sizeof(float) * (uint64_t)D)
        return report(Error::make(ErrorCode::NotImplemented, pfx + "ffn_gate_inp_shexp.weight must be f32 [D]"));
      L->gate_inp_shexp = static_cast<const float*>(ptr(gi));
    }
  }
  return report(Error::success());
}

}  // extern "C"
