// exl3_model.cu -- the model seam over the EXL3 linears (C ABI): bill, load, the forward over the linears, unload.
//
// The reference's model plugin exports a ModelTable {claims, parse, bill, load, unload, forward, ...}
// (plugins/turboexl3_qwen38/plugin.zig:38-53) that serves a whole Qwen3.8 EXL3 pack.  On this path only the entries
// that touch the EXL3 linears are in scope, and they are here, over this library's quant seam:
//   bill     -- the resident bytes: every EXL3 tensor of the pack's layers as the pack stores it (EXL3 weights stay
//               resident as stored, plugins/turboexl3_ds41/config.zig:57-61);
//   load     -- the config parse (exl3_model_parse), then every EXL3 linear of every layer uploaded once under the
//               trunk block's rules and every routed bank (<bank>.experts.<e>.<proj>) under the expert block's; the
//               linears of a layer that read one input (q|k|v, gate|up) are also stacked into one launch
//               (SX/linear.zig:39-72 linearShared); the dense MLP's intermediate buffers are reserved for `max_rows`;
//   forward  -- one linear, linears that read one input (one stacked launch where the load stacked them), the dense
//               SwiGLU MLP, and the routed experts with the layer's shared expert (exl3_swiglu_shared);
//   unload   -- releases every weight and the buffers.
// Names follow the pack: <prefix>.layers.<i>.<module>.{trellis,suh,svh} (src/direct/config.zig weight_prefix).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "../../include/exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_json.h"

struct exl3_model {
  exl3_model_config cfg{};
  std::string prefix;
  int device = 0;
  int max_rows = 0;
  std::map<std::pair<int, std::string>, exl3_weight> lin;      // (layer, module) -> one linear
  std::map<std::pair<int, std::string>, exl3_weight> stacked;  // (layer, "a|b|c") -> the stacked launch
  std::map<std::pair<int, std::string>, std::map<std::string, exl3_weight>> banks;  // (layer, bank) -> proj -> bank
  uint8_t* scratch = nullptr;  // the dense MLP's gate|up output and its SwiGLU, max_rows rows
  size_t scratch_bytes = 0;
};

namespace {

exl3_verdict refuse_model(int32_t code, const char* why) { return {code, why}; }
constexpr exl3_verdict kModelOk = {EXL3_OK, nullptr};

size_t dtype_bytes(int32_t dt) {
  switch (dt) {
    case EXL3_F32: case EXL3_I32: case EXL3_U32: return 4;
    default: return 2;
  }
}

std::string str_of(exl3_str s) { return s.ptr ? std::string(s.ptr, s.len) : std::string(); }

bool host_tensor(const exl3_source* src, const std::string& name, exl3_host_tensor& out) {
  if (!src || !src->tensor) return false;
  memset(&out, 0, sizeof out);
  exl3_str s{name.data(), name.size()};
  return src->tensor(src->ctx, s, &out) == 0;
}

// The pack's EXL3 modules of every layer: (layer, module) of plain linears, (layer, bank) -> projections of routed
// banks, from the names <prefix>.layers.<i>.<module>.trellis (a bank member is <bank>.experts.<e>.<proj>).
struct PackPlan {
  std::map<int, std::vector<std::string>> linears;
  std::map<int, std::map<std::string, std::vector<std::string>>> banks;
};

bool plan_pack(const std::string& prefix, const exl3_str* names, int32_t count, uint32_t layers, PackPlan& plan) {
  const std::string head = prefix + ".layers.", tail = ".trellis", experts = ".experts.";
  std::set<std::pair<int, std::string>> seen;
  for (int32_t i = 0; i < count; ++i) {
    const std::string n = str_of(names[i]);
    if (n.size() <= head.size() + tail.size() || n.compare(0, head.size(), head) != 0 ||
        n.compare(n.size() - tail.size(), tail.size(), tail) != 0)
      continue;
    const std::string rest = n.substr(head.size(), n.size() - head.size() - tail.size());  // <i>.<module>
    const size_t dot = rest.find('.');
    if (dot == std::string::npos || dot == 0) continue;
    int layer = 0;
    for (size_t k = 0; k < dot; ++k) {
      if (rest[k] < '0' || rest[k] > '9' || layer > 1000000) return false;
      layer = layer * 10 + (rest[k] - '0');
    }
    if (static_cast<uint32_t>(layer) >= layers) return false;
    const std::string module = rest.substr(dot + 1);
    const size_t ex = module.find(experts);
    if (ex != std::string::npos) {
      const std::string bank = module.substr(0, ex), after = module.substr(ex + experts.size());  // <e>.<proj>
      const size_t d2 = after.find('.');
      if (bank.empty() || d2 == std::string::npos || d2 == 0) continue;
      const std::string proj = after.substr(d2 + 1);
      if (seen.insert({layer, bank + "|" + proj}).second) plan.banks[layer][bank].push_back(proj);
    } else if (seen.insert({layer, module}).second) {
      plan.linears[layer].push_back(module);
    }
  }
  return true;
}

const exl3_weight* find(const std::map<std::pair<int, std::string>, exl3_weight>& m, int layer, const std::string& k) {
  auto it = m.find({layer, k});
  return it == m.end() ? nullptr : &it->second;
}

// y[r][c] = RN(silu(g[r][c]) * u[r][c]) with g | u the stacked gate|up output's two segments (each [rows][inter],
// back to back), in the activations' dtype; silu in f32.
__global__ void silu_mul_kernel(const void* gu, void* h, int64_t n, int32_t dt) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float g = exl3::load_act(gu, static_cast<size_t>(i), dt), u = exl3::load_act(gu, static_cast<size_t>(n + i), dt);
  exl3::store_act(h, static_cast<size_t>(i), g / (1.0f + expf(-g)) * u, dt);
}

exl3_tensor view(void* data, int32_t dt, int64_t rows, int64_t cols) {
  exl3_tensor t{};
  t.data = data;
  t.dtype = dt;
  t.ndim = 2;
  t.shape[0] = rows;
  t.shape[1] = cols;
  return t;
}

int64_t rows_of(const exl3_tensor* x) {
  int64_t r = 1;
  for (int i = 0; i + 1 < x->ndim; ++i) r *= x->shape[i];
  return r;
}

void release_all(exl3_model* m) {
  for (auto& kv : m->stacked) exl3_release(&kv.second);
  for (auto& kv : m->lin) exl3_release(&kv.second);
  for (auto& kv : m->banks)
    for (auto& p : kv.second) exl3_release(&p.second);
  m->stacked.clear();
  m->lin.clear();
  m->banks.clear();
  if (m->scratch) {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(m->device);
    cudaFree(m->scratch);
    if (prev >= 0) cudaSetDevice(prev);
    m->scratch = nullptr;
  }
}

// The dense MLP's stacks: (gate_proj, up_proj) per module prefix; q|k|v per attention prefix.
const char* const kStacks[][3] = {{"q_proj", "k_proj", "v_proj"}, {"gate_proj", "up_proj", nullptr}};

}  // namespace

extern "C" {

uint64_t exl3_model_bill(exl3_str config_json, const exl3_source* source, const exl3_str* names, int32_t count) {
  exl3_model_config cfg{};
  cfg.size = sizeof cfg;
  if (exl3_model_parse(config_json, &cfg).code != EXL3_OK || (count > 0 && !names)) return 0;
  const std::string head = std::string(cfg.weight_prefix) + ".layers.";
  uint64_t total = 0;
  for (int32_t i = 0; i < count; ++i) {
    const std::string n = str_of(names[i]);
    const bool ours = n.compare(0, head.size(), head) == 0 &&
                      (n.size() > 8 && (n.compare(n.size() - 8, 8, ".trellis") == 0 ||
                                        n.compare(n.size() - 4, 4, ".suh") == 0 ||
                                        n.compare(n.size() - 4, 4, ".svh") == 0));
    exl3_host_tensor t;
    if (!ours || !host_tensor(source, n, t)) continue;
    uint64_t e = 1;
    for (int d = 0; d < t.ndim && d < 4; ++d) e *= static_cast<uint64_t>(t.shape[d]);
    total += e * dtype_bytes(t.dtype);
  }
  return total;
}

exl3_verdict exl3_model_load(exl3_str config_json, const exl3_source* source, const exl3_str* names, int32_t count,
                             int32_t device, int32_t max_rows, void* stream, exl3_model** out) {
  if (!out || !source || !source->tensor || (count > 0 && !names) || count < 0 || max_rows < 1 || max_rows > 65536)
    return refuse_model(EXL3_FAILED, "exl3_b200: bad model load arguments");
  *out = nullptr;
  exl3_model_config cfg{};
  cfg.size = sizeof cfg;
  exl3_verdict v = exl3_model_parse(config_json, &cfg);
  if (v.code != EXL3_OK) return v;
  exl3::JVal root;
  if (!exl3::parse_json(config_json, root) || root.kind != exl3::JVal::Obj)
    return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: InvalidConfig");
  std::string trunk, expert;
  exl3::dump_json(*root.get("trunk_quant"), trunk);  // (exl3_model_parse refuses a pack without it)
  if (const exl3::JVal* e = root.get("expert_quant"); e && e->kind == exl3::JVal::Obj) exl3::dump_json(*e, expert);
  else expert = trunk;
  PackPlan plan;
  if (!plan_pack(cfg.weight_prefix, names, count, cfg.num_hidden_layers, plan))
    return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: InvalidConfigField");

  exl3_model* m = new exl3_model;
  m->cfg = cfg;
  m->prefix = cfg.weight_prefix;
  m->device = device;
  m->max_rows = max_rows;
  exl3_load_ctx ctx{};
  ctx.size = sizeof ctx;
  ctx.config_json = config_json;
  ctx.source = *source;
  ctx.device = device;
  ctx.stream = stream;
  auto fail = [&](exl3_verdict why) {
    release_all(m);
    delete m;
    return why;
  };
  // the trunk's linears, then the stacks of the linears that read one input
  ctx.block_json = {trunk.data(), trunk.size()};
  if (!plan.linears.empty()) {
    if ((v = exl3_open(&ctx)).code != EXL3_OK) return fail(v);
    for (const auto& [layer, modules] : plan.linears)
      for (const std::string& mod : modules) {
        const std::string name = m->prefix + ".layers." + std::to_string(layer) + "." + mod;
        exl3_host_tensor tr;
        if (!host_tensor(source, name + ".trellis", tr) || tr.ndim != 3) {
          exl3_close(&ctx);
          return fail(refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: MissingTensor"));
        }
        exl3_weight w{};
        v = exl3_load_tensor(&ctx, {name.data(), name.size()}, static_cast<uint32_t>(tr.shape[0] * 16), &w);
        if (v.code != EXL3_OK) {
          exl3_close(&ctx);
          return fail(v);
        }
        m->lin[{layer, mod}] = w;
      }
    exl3_close(&ctx);
    for (const auto& [layer, modules] : plan.linears)
      for (const std::string& mod : modules) {
        const size_t dot = mod.rfind('.');
        const std::string base = dot == std::string::npos ? std::string() : mod.substr(0, dot + 1);
        for (const auto& group : kStacks) {
          if (mod != base + group[0]) continue;
          std::vector<exl3_weight> parts;
          std::string key;
          for (int j = 0; j < 3 && group[j]; ++j) {
            const exl3_weight* w = find(m->lin, layer, base + group[j]);
            if (!w) break;
            parts.push_back(*w);
            key += (j ? "|" : "") + base + group[j];
          }
          const int want = group[2] ? 3 : 2;
          if (static_cast<int>(parts.size()) != want) continue;
          exl3_weight st{};
          if ((v = exl3_weight_stack(parts.data(), want, stream, &st)).code != EXL3_OK) return fail(v);
          m->stacked[{layer, key}] = st;
        }
      }
  }
  // the routed banks under the expert block
  if (!plan.banks.empty()) {
    ctx.block_json = {expert.data(), expert.size()};
    if ((v = exl3_open(&ctx)).code != EXL3_OK) return fail(v);
    for (const auto& [layer, banks] : plan.banks)
      for (const auto& [bank, projs] : banks)
        for (const std::string& proj : projs) {
          const std::string stem = m->prefix + ".layers." + std::to_string(layer) + "." + bank + ".experts.";
          exl3_host_tensor tr;
          if (!host_tensor(source, stem + "0." + proj + ".trellis", tr) || tr.ndim != 3) {
            exl3_close(&ctx);
            return fail(refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: MissingTensor"));
          }
          const std::string name = stem + proj;
          exl3_weight w{};
          v = exl3_load_bank(&ctx, {name.data(), name.size()}, static_cast<uint32_t>(tr.shape[0] * 16), &w);
          if (v.code != EXL3_OK) {
            exl3_close(&ctx);
            return fail(v);
          }
          m->banks[{layer, bank}][proj] = w;
        }
    exl3_close(&ctx);
  }
  // the dense MLP's buffers: the widest gate|up stack's output and its SwiGLU, f32-sized, max_rows rows
  size_t widest = 0;
  for (const auto& kv : m->stacked)
    if (kv.first.second.find("gate_proj|") != std::string::npos)
      widest = widest > static_cast<size_t>(kv.second.out_features) ? widest : static_cast<size_t>(kv.second.out_features);
  if (widest) {
    m->scratch_bytes = static_cast<size_t>(max_rows) * widest * 4 * 3 / 2;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    const bool ok = cudaMalloc(&m->scratch, m->scratch_bytes) == cudaSuccess;
    if (prev >= 0) cudaSetDevice(prev);
    if (!ok) {
      m->scratch = nullptr;
      return fail(refuse_model(EXL3_TOO_LARGE, "exl3_b200: the dense MLP's buffers do not fit"));
    }
  }
  *out = m;
  return kModelOk;
}

void exl3_model_unload(exl3_model* m) {
  if (!m) return;
  release_all(m);
  delete m;
}

int32_t exl3_model_weight(const exl3_model* m, int32_t layer, exl3_str module, exl3_weight* out) {
  if (!m || !out) return 0;
  const std::string k = str_of(module);
  if (const exl3_weight* w = find(m->lin, layer, k)) *out = *w;
  else if (const exl3_weight* s = find(m->stacked, layer, k)) *out = *s;
  else return 0;
  return 1;
}

exl3_verdict exl3_model_linear(const exl3_model* m, int32_t layer, exl3_str module, const exl3_tensor* x, void* stream,
                               exl3_tensor* out) {
  if (!m) return refuse_model(EXL3_FAILED, "exl3_b200: no model");
  const exl3_weight* w = find(m->lin, layer, str_of(module));
  if (!w) return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: MissingLinear");
  return exl3_matmul(w, x, stream, out);
}

exl3_verdict exl3_model_linears(const exl3_model* m, int32_t layer, const exl3_str* modules, int32_t count,
                                const exl3_tensor* x, void* stream, exl3_tensor* out) {
  if (!m || !modules || count < 1 || count > EXL3_MAX_SEGMENTS || !x || !out || x->ndim < 1)
    return refuse_model(EXL3_FAILED, "exl3_b200: bad arguments");
  std::string key;
  std::vector<const exl3_weight*> ws;
  int64_t total = 0;
  for (int32_t i = 0; i < count; ++i) {
    const std::string mod = str_of(modules[i]);
    const exl3_weight* w = find(m->lin, layer, mod);
    if (!w) return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: MissingLinear");
    ws.push_back(w);
    total += w->out_features;
    key += (i ? "|" : "") + mod;
  }
  const int64_t rows = rows_of(x);
  int64_t numel = 1;
  for (int i = 0; i < out->ndim; ++i) numel *= out->shape[i];
  if (numel != rows * total || out->dtype != x->dtype)
    return refuse_model(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (out holds every linear's [rows, out] back to back)");
  if (const exl3_weight* st = find(m->stacked, layer, key)) {
    exl3_tensor o = view(out->data, out->dtype, rows, total);
    exl3_tensor xv = view(x->data, x->dtype, rows, x->shape[x->ndim - 1]);
    return exl3_matmul(st, &xv, stream, &o);
  }
  const size_t es = dtype_bytes(x->dtype);
  int64_t c0 = 0;
  for (const exl3_weight* w : ws) {
    exl3_tensor o = view(static_cast<uint8_t*>(out->data) + static_cast<size_t>(rows * c0) * es, out->dtype, rows,
                         w->out_features);
    exl3_tensor xv = view(x->data, x->dtype, rows, x->shape[x->ndim - 1]);
    exl3_verdict v = exl3_matmul(w, &xv, stream, &o);
    if (v.code != EXL3_OK) return v;
    c0 += w->out_features;
  }
  return kModelOk;
}

exl3_verdict exl3_model_mlp(const exl3_model* m, int32_t layer, exl3_str module, const exl3_tensor* x, void* stream,
                            exl3_tensor* out) {
  if (!m || !x || !out || x->ndim < 1) return refuse_model(EXL3_FAILED, "exl3_b200: bad arguments");
  const std::string mod = str_of(module);
  const std::string gk = mod + ".gate_proj", uk = mod + ".up_proj", dk = mod + ".down_proj";
  const exl3_weight* st = find(m->stacked, layer, gk + "|" + uk);
  const exl3_weight* down = find(m->lin, layer, dk);
  if (!st || !down) return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: MissingLinear");
  const int64_t rows = rows_of(x);
  const int64_t inter = st->out_features / 2;
  if (rows > m->max_rows) return refuse_model(EXL3_TOO_LARGE, "exl3_b200: more rows than the model's max_rows");
  if (down->in_features != inter) return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: BadExl3Shape");
  const size_t es = dtype_bytes(x->dtype);
  uint8_t* gu = m->scratch;
  uint8_t* h = m->scratch + static_cast<size_t>(rows) * 2 * inter * es;
  exl3_tensor xv = view(x->data, x->dtype, rows, x->shape[x->ndim - 1]);
  exl3_tensor guv = view(gu, x->dtype, rows, 2 * inter);
  exl3_verdict v = exl3_matmul(st, &xv, stream, &guv);
  if (v.code != EXL3_OK) return v;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != m->device) cudaSetDevice(m->device);
  const int64_t n = rows * inter;
  silu_mul_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(gu, h, n,
                                                                                                         x->dtype);
  const cudaError_t e = cudaGetLastError();
  if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
  if (e != cudaSuccess) return refuse_model(EXL3_FAILED, "exl3_b200: SwiGLU launch failed");
  exl3_tensor hv = view(h, x->dtype, rows, inter);
  exl3_tensor ov = view(out->data, out->dtype, rows, down->out_features);
  return exl3_matmul(down, &hv, stream, &ov);
}

exl3_verdict exl3_model_experts(const exl3_model* m, int32_t layer, exl3_str bank, exl3_str shared,
                                const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores,
                                const void* shared_logit, void* stream, exl3_tensor* out) {
  if (!m) return refuse_model(EXL3_FAILED, "exl3_b200: no model");
  auto it = m->banks.find({layer, str_of(bank)});
  if (it == m->banks.end()) return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: MissingBank");
  const auto& b = it->second;
  auto g = b.find("gate_proj"), u = b.find("up_proj"), d = b.find("down_proj");
  if (g == b.end() || u == b.end() || d == b.end()) return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: MissingBank");
  const std::string sh = str_of(shared);
  const exl3_weight* sg = sh.empty() ? nullptr : find(m->lin, layer, sh + ".gate_proj");
  const exl3_weight* su = sh.empty() ? nullptr : find(m->lin, layer, sh + ".up_proj");
  const exl3_weight* sd = sh.empty() ? nullptr : find(m->lin, layer, sh + ".down_proj");
  if (!sg || !su || !sd) {
    if (shared_logit) return refuse_model(EXL3_UNSUPPORTED, "turboexl3_qwen38: a shared gate without a shared expert");
    return exl3_swiglu(&g->second, &u->second, &d->second, x, inds, scores, nullptr, stream, out);
  }
  exl3_shared_swiglu o{};
  o.size = sizeof o;
  o.gate = sg;
  o.up = su;
  o.down = sd;
  o.logit = shared_logit;
  return exl3_swiglu_shared(&g->second, &u->second, &d->second, x, inds, scores, &o, stream, out);
}

}  // extern "C"
