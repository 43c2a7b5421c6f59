// uaii_moe_plugin.cpp -- a UAII OPERATOR plugin that runs the reference's MoE operators
// on the B200 through libuaii_moe.so.
//
// The reference loads operator plugins with Plugin::load / PluginRegistry::load_path
// (libs/uaii-core/src/plugin.cpp:139-187): it resolves uaii_plugin_get_info / init /
// shutdown (include/uaii/c_api/plugin_abi.h:40-48), checks the ABI version and calls
// init.  Init registers MoERouter, MoEExperts and MoEExpertsSwiGLU in
// plugins::OperatorHostRegistry (include/uaii/plugins/operator_host.hpp), the table that
// kernels::dispatch_cpu consults before its builtins (libs/uaii-kernels/src/dispatch.cpp:
// 76-80).  So every Session whose ops run through host dispatch -- backend "cpu", and
// backend "cuda" for host-resident session tensors (libs/uaii-backends/src/
// cuda_backend.cpp:189-192), which is every Session tensor today (session.cpp:259-367)
// -- runs these three operators on the device without a change to the reference.
//
// Each call converts the reference's TensorView / Attribute vectors to the C ABI of
// include/uaii_moe.h and calls uaii_moe_dispatch; the library stages host tensors
// through its device workspace and returns the reference's status codes and messages.
// Shapes the device path does not take (NotImplemented) run the reference's own f32
// kernel instead (moe_router_f32 / moe_experts_f32 / moe_experts_swiglu_f32,
// include/uaii/kernels/kernels.hpp), as the reference's CUDA backend falls back for
// its unimplemented native ops; uaii_moe_plugin_stats() counts both outcomes.
//
// Init fails (the plugin does not load, Plugin::load returns PluginError) when no
// CUDA device can be opened: the plugin never registers a host implementation.
//
// Environment:
//   UAII_MOE_DEVICE          CUDA device ordinal (default 0)
//   UAII_MOE_CONST_WEIGHTS   "1": expert and router weights are constant for the
//                            process lifetime (a loaded Session's weights are); each
//                            weight buffer is registered on first use and uploaded once
//                            (uaii_moe_register_weights).  Default: staged per call.
//
// Built against the reference's public headers; the symbols it uses from the host
// process (OperatorHostRegistry::instance, the three f32 kernels) resolve when the host
// loads it, as for the reference's own example operator plugin (plugins/example_op).
#include "uaii/c_api/plugin_abi.h"
#include "uaii/core/error.hpp"
#include "uaii/ir/attribute.hpp"
#include "uaii/kernels/kernels.hpp"
#include "uaii/kernels/tensor_view.hpp"
#include "uaii/plugins/operator_host.hpp"

#include "uaii_moe.h"

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

namespace {

using uaii::Error;
using uaii::ErrorCode;
using uaii::ir::Attribute;
using uaii::ir::AttributeType;
using uaii::kernels::TensorView;

uaii_plugin_info g_info{};
uaii_moe_backend* g_backend = nullptr;
std::mutex g_mu;                                    // one call at a time on the backend
std::set<std::pair<const void*, uint64_t>> g_registered;
bool g_const_weights = false;
std::atomic<uint64_t> g_device_calls{0}, g_host_calls{0};

void fill_info() {
  std::memset(&g_info, 0, sizeof(g_info));
  g_info.abi_version = UAII_PLUGIN_ABI_VERSION;
  g_info.kind = UAII_PLUGIN_KIND_OPERATOR;
  std::strncpy(g_info.name, "uaii_moe_b200", UAII_PLUGIN_NAME_MAX - 1);
  std::strncpy(g_info.version, "1.0.0", UAII_PLUGIN_VERSION_MAX - 1);
  std::strncpy(g_info.description,
               "MoERouter, MoEExperts, MoEExpertsSwiGLU on the B200 (GGUF blocks dequantized on the device)",
               UAII_PLUGIN_DESC_MAX - 1);
}

uaii_moe_tensor to_c(const TensorView& t) {
  uaii_moe_tensor c;
  c.dtype = static_cast<int32_t>(t.dtype);
  c.quant_format = static_cast<int32_t>(t.quant_format);
  c.shape = t.shape;
  c.rank = t.rank;
  c.data = t.data;
  c.nbytes = t.nbytes;
  return c;
}

// Weight inputs of each op (registered once when UAII_MOE_CONST_WEIGHTS=1).
std::vector<size_t> weight_inputs(const std::string& op) {
  if (op == "MoERouter" || op == "MoEExperts") return {1};
  if (op == "MoEExpertsSwiGLU") return {1, 2, 3};
  return {};
}

Error host_kernel(const std::string& op, const std::vector<TensorView>& in, std::vector<TensorView>* out,
                  const std::vector<Attribute>& attrs) {
  auto attr_int = [&](const char* key, int64_t def) {
    for (const auto& a : attrs)
      if (a.key == key && a.type == AttributeType::Int) return std::get<int64_t>(a.value);
    return def;
  };
  ++g_host_calls;
  if (op == "MoERouter") return uaii::kernels::moe_router_f32(in[0], in[1], &(*out)[0], &(*out)[1]);
  if (op == "MoEExperts")
    return uaii::kernels::moe_experts_f32(in[0], in[1], in[2], &(*out)[0], (int)attr_int("num_experts", 1));
  return uaii::kernels::moe_experts_swiglu_f32(in[0], in[1], in[2], in[3], in[4], &(*out)[0],
                                               (int)attr_int("num_experts", 1), (int)attr_int("top_k", 2));
}

Error run_op(const std::string& op, const std::vector<TensorView>& in, std::vector<TensorView>* out,
             const std::vector<Attribute>& attrs) {
  if (out == nullptr || out->empty()) return Error::make(ErrorCode::InvalidArgument, "dispatch outputs empty");
  std::vector<uaii_moe_tensor> ci, co;
  for (const auto& t : in) ci.push_back(to_c(t));
  for (const auto& t : *out) co.push_back(to_c(t));
  std::vector<uaii_moe_attr> ca;
  for (const auto& a : attrs) {
    if (a.type == AttributeType::Int) ca.push_back({a.key.c_str(), 1, std::get<int64_t>(a.value), 0.0});
    else if (a.type == AttributeType::Float) ca.push_back({a.key.c_str(), 2, 0, std::get<double>(a.value)});
    else if (a.type == AttributeType::Bool) ca.push_back({a.key.c_str(), 3, std::get<bool>(a.value) ? 1 : 0, 0.0});
  }
  int st;
  std::string msg;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_const_weights) {
      for (size_t i : weight_inputs(op)) {
        if (i >= in.size() || in[i].data == nullptr || in[i].nbytes == 0) continue;
        const auto key = std::make_pair(static_cast<const void*>(in[i].data), (uint64_t)in[i].nbytes);
        if (g_registered.count(key)) continue;
        if (uaii_moe_register_weights(g_backend, key.first, key.second) == UAII_MOE_OK) g_registered.insert(key);
      }
    }
    st = uaii_moe_dispatch(g_backend, op.c_str(), "1", ci.data(), ci.size(), co.data(), co.size(), ca.data(),
                           ca.size());
    if (st != UAII_MOE_OK) msg = uaii_moe_last_error();
  }
  if (st == UAII_MOE_OK) {
    ++g_device_calls;
    return Error::success();
  }
  if (st == UAII_MOE_NOT_IMPLEMENTED) return host_kernel(op, in, out, attrs);
  return Error::make(static_cast<ErrorCode>(st), msg);
}

template <const char* kName>
Error op_fn(const std::vector<TensorView>& in, std::vector<TensorView>* out, const std::vector<Attribute>& attrs) {
  return run_op(kName, in, out, attrs);
}
constexpr char kRouter[] = "MoERouter";
constexpr char kExperts[] = "MoEExperts";
constexpr char kSwiGLU[] = "MoEExpertsSwiGLU";

}  // namespace

extern "C" {

__attribute__((visibility("default"))) const uaii_plugin_info* uaii_plugin_get_info(void) {
  if (g_info.abi_version == 0) fill_info();
  return &g_info;
}

__attribute__((visibility("default"))) int uaii_plugin_init(void) {
  if (g_info.abi_version == 0) fill_info();
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_backend == nullptr) {
    const char* dev = std::getenv("UAII_MOE_DEVICE");
    const char* cw = std::getenv("UAII_MOE_CONST_WEIGHTS");
    g_const_weights = cw != nullptr && std::strcmp(cw, "1") == 0;
    const int st = uaii_moe_backend_create(dev ? std::atoi(dev) : 0, nullptr, &g_backend);
    if (st != UAII_MOE_OK) return st;  // no device: the plugin does not load
  }
  auto& reg = uaii::plugins::OperatorHostRegistry::instance();
  reg.register_op(kRouter, &op_fn<kRouter>);
  reg.register_op(kExperts, &op_fn<kExperts>);
  reg.register_op(kSwiGLU, &op_fn<kSwiGLU>);
  return 0;
}

// The registry has no removal: the registered entries keep pointing at this library,
// so a host must not unload it while sessions may still dispatch (as for every
// operator plugin of the reference).  The device backend stays alive until exit.
__attribute__((visibility("default"))) void uaii_plugin_shutdown(void) {}

// Calls served on the device / by the reference's host kernel (NotImplemented shapes).
__attribute__((visibility("default"))) void uaii_moe_plugin_stats(uint64_t* device_calls, uint64_t* host_calls) {
  if (device_calls) *device_calls = g_device_calls.load();
  if (host_calls) *host_calls = g_host_calls.load();
}

}  // extern "C"
