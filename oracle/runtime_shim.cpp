// runtime_shim.cpp -- test infrastructure: C entry points into the reference runtime build
// (oracle/_ref/libuaii_ref_runtime.so) for what its own C API (include/uaii/c_api/uaii.h)
// does not expose: loading a plugin (uaii::PluginRegistry::load_path,
// include/uaii/core/plugin.hpp:56-80) and the reference's MoE smoke demo
// (uaii::runtime::run_moe_smoke_demo, libs/uaii-runtime/src/demos_phase4.cpp:186-282),
// and Sessions created the way the reference C API creates them
// (uaii_session_create / set_f32 / run / get_f32, libs/uaii-capi/src/capi.cpp:121-227:
// load_graph or load_model, SessionOptions from uaii_session_options_init's defaults,
// Session::create).  The C API's own file is not in this build: it includes a header
// that CMake generates at configure time.
#include "uaii/core/plugin.hpp"
#include "uaii/ir/serialize.hpp"
#include "uaii/loaders/registry.hpp"
#include "uaii/plugins/operator_host.hpp"
#include "uaii/runtime/session.hpp"

#include <cstring>
#include <memory>
#include <string>
#include <vector>

namespace {
thread_local std::string g_last;
uaii::PluginRegistry& registry() {
  static uaii::PluginRegistry reg;  // plugins stay loaded until exit
  return reg;
}
int status(const uaii::Error& e) {
  g_last = e.ok() ? std::string() : e.message();
  return static_cast<int>(e.code());
}
}  // namespace

extern "C" {

const char* urt_last_error() { return g_last.c_str(); }

int urt_plugin_load(const char* path) { return status(registry().load_path(path)); }

int urt_operator_registered(const char* op) {
  return uaii::plugins::OperatorHostRegistry::instance().has(op) ? 1 : 0;
}

int urt_moe_smoke_demo(int* ok) {
  bool good = false;
  const int st = status(uaii::runtime::run_moe_smoke_demo(&good));
  if (ok) *ok = good ? 1 : 0;
  return st;
}

// path: .uaii.json IR (or a model file); backend: "cpu", "cuda", ...; options otherwise
// as uaii_session_options_init leaves them, with keep_quantized_weights and
// enable_memory_reuse given.
int urt_session_create(const char* path, const char* backend, const char* weights_dir, int keep_quantized,
                       int memory_reuse, void** out) {
  if (!path || !out) return status(uaii::Error::make(uaii::ErrorCode::InvalidArgument, "path/out null"));
  *out = nullptr;
  uaii::ir::Graph graph;
  const std::string p(path);
  const bool ir = p.size() > 10 && (p.rfind(".uaii.json") == p.size() - 10);
  uaii::Error err = ir ? uaii::ir::load_graph(p, &graph) : uaii::loaders::load_model(p, &graph);
  if (!err.ok()) return status(err);
  uaii::runtime::SessionOptions o;
  o.backend_name = backend ? backend : "cpu";
  if (weights_dir) o.weights_dir = weights_dir;
  o.weight_init = uaii::runtime::WeightInit::None;
  o.enable_fusion = true;
  o.enable_memory_reuse = memory_reuse != 0;
  o.keep_quantized_weights = keep_quantized != 0;
  auto s = std::make_unique<uaii::runtime::Session>();
  err = s->create(std::move(graph), o);
  if (!err.ok()) return status(err);
  *out = s.release();
  return 0;
}

void urt_session_destroy(void* s) { delete static_cast<uaii::runtime::Session*>(s); }

int urt_session_set_f32(void* s, const char* name, const float* data, size_t n) {
  return status(static_cast<uaii::runtime::Session*>(s)->set_tensor_f32(name, std::vector<float>(data, data + n)));
}

int urt_session_run(void* s) { return status(static_cast<uaii::runtime::Session*>(s)->run()); }

int urt_session_get_f32(void* s, const char* name, float* out, size_t cap, size_t* n) {
  std::vector<float> v;
  const int st = status(static_cast<uaii::runtime::Session*>(s)->get_tensor_f32(name, &v));
  if (st != 0) return st;
  *n = v.size();
  if (out && cap >= v.size()) std::memcpy(out, v.data(), v.size() * sizeof(float));
  return 0;
}

// Session::generate (libs/uaii-runtime/src/session.cpp:910-1046), greedy, as uaii_session_generate
// calls it: the prompt is prefilled one token per run, then max_new tokens are sampled.
int urt_session_generate(void* s, const int64_t* prompt, size_t n, int64_t max_new, int64_t* out, size_t cap,
                         size_t* out_n) {
  std::vector<std::int64_t> toks;
  const int st = status(static_cast<uaii::runtime::Session*>(s)->generate(
      std::vector<std::int64_t>(prompt, prompt + n), max_new, &toks));
  if (st != 0) return st;
  *out_n = toks.size() < cap ? toks.size() : cap;
  for (size_t i = 0; i < *out_n; ++i) out[i] = toks[i];
  return 0;
}

const char* urt_session_backend_details(void* s) {
  static thread_local std::string d;
  const auto* b = static_cast<uaii::runtime::Session*>(s)->backend();
  d = b ? b->capabilities().details : std::string();
  return d.c_str();
}

}  // extern "C"
