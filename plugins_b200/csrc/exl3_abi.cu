// exl3_abi.cu -- the C ABI of libexl3b200.so (include/exl3_b200.h): the reference plugin's quant seam over device
// buffers.  Host code only; the kernels live in exl3_gemv.cu, exl3_decode.cu and exl3_moe.cu.
#include <cuda_runtime.h>

#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/exl3_b200.h"
#include "exl3_internal.h"
#include "exl3_json.h"
#include "exl3_moe.h"

namespace {

using exl3::JParser;
using exl3::JVal;
using exl3::parse_json;
using exl3::str_is;

// ------------------------------------------------------------------ verdicts

constexpr exl3_verdict kOk = {EXL3_OK, nullptr};
exl3_verdict refuse(int32_t code, const char* why) { return {code, why}; }


// ------------------------------------------------------------------ per-device state

struct DeviceState {
  bool ready = false;
  uint8_t* base = nullptr;
  size_t bytes = 0;
  float* partials = nullptr;
  size_t partial_floats = 0;
  uint32_t* counters = nullptr;
  uint32_t* err = nullptr;
  uint8_t* image = nullptr;  // prefill GEMM operand images (A rows, then B columns)
  size_t image_bytes = 0;
  int sms = 0;
  int gemm_min_rows = exl3::kGemmMinRows;
};

constexpr int kMaxDevices = 64;
constexpr size_t kCounterCount = 8192;           // out / 128 <= 8192
constexpr size_t kPartialBytes = 128u << 20;     // decode-GEMV split partials
constexpr size_t kImageBytes = 256u << 20;       // prefill GEMM operand images

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

namespace exl3 {
__device__ uint32_t g_device_error;  // kErr* bits, one word per device

uint32_t* device_error_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
  return static_cast<uint32_t*>(p);
}

uint64_t* trace_alloc() {
  const char* e = getenv("EXL3_TRACE");
  if (!e || strcmp(e, "1") != 0) return nullptr;
  const size_t bytes = sizeof(uint64_t) * kTraceSteps * kTraceStamps;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return nullptr;
  }
  return static_cast<uint64_t*>(p);
}

bool trace_copy(const uint64_t* ring, const uint32_t* step_word, uint64_t* out) {
  if (!ring || !step_word || !out) return false;
  uint64_t host[kTraceSteps * kTraceStamps];
  uint32_t step = 0;
  if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&step, step_word, 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemcpy(host, ring, sizeof host, cudaMemcpyDeviceToHost) != cudaSuccess)
    return false;
  for (int i = 0; i < kTraceSteps; ++i) {  // oldest first: steps step - 15 .. step
    const uint32_t s = step - static_cast<uint32_t>(kTraceSteps - 1 - i);
    const bool ran = static_cast<int32_t>(step) - (kTraceSteps - 1 - i) >= 1;
    for (int j = 0; j < kTraceStamps; ++j)
      out[i * kTraceStamps + j] = ran ? host[(s % kTraceSteps) * kTraceStamps + j] : 0;
  }
  return true;
}
}

namespace {

// Creates the device workspace once (load time, never inside matmul).
exl3_verdict ensure_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return refuse(EXL3_UNSUPPORTED, "exl3_b200: device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (d.ready) return kOk;
  DeviceGuard guard(dev);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return refuse(EXL3_FAILED, "exl3_b200: no CUDA device");
  if (prop.major != 10) return refuse(EXL3_UNSUPPORTED, "exl3_b200: the kernels are built for sm_100a (B200) only");
  d.sms = prop.multiProcessorCount;
  const size_t counter_bytes = kCounterCount * 4;
  d.bytes = kImageBytes + kPartialBytes + counter_bytes + 256;
  if (cudaMalloc(&d.base, d.bytes) != cudaSuccess) return refuse(EXL3_TOO_LARGE, "exl3_b200: workspace allocation failed");
  d.image = d.base;
  d.image_bytes = kImageBytes;
  d.partials = reinterpret_cast<float*>(d.base + kImageBytes);
  d.partial_floats = kPartialBytes / 4;
  d.counters = reinterpret_cast<uint32_t*>(d.base + kImageBytes + kPartialBytes);
  // tuning override for measurement runs
  if (const char* e = getenv("EXL3_GEMM_MIN_ROWS")) {
    const int v = atoi(e);
    if (v >= 1) d.gemm_min_rows = v;
  }
  if (cudaMemset(d.counters, 0, counter_bytes) != cudaSuccess) return refuse(EXL3_FAILED, "exl3_b200: workspace init failed");
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&d.err), exl3::g_device_error) != cudaSuccess)
    return refuse(EXL3_FAILED, "exl3_b200: error word lookup failed");
  if (cudaMemset(d.err, 0, 4) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
    return refuse(EXL3_FAILED, "exl3_b200: workspace init failed");
  d.ready = true;
  return kOk;
}

DeviceState* device_state(int dev) {
  if (dev < 0 || dev >= kMaxDevices || !g_dev[dev].ready) return nullptr;
  return &g_dev[dev];
}

bool rate_served(int n) { return exl3::rate_served_n(n); }

exl3_verdict check_linear_shape(int groups, int in_f, int out_f, int n) {
  if (groups < 1 || in_f <= 0 || out_f <= 0) return refuse(EXL3_UNSUPPORTED, "exl3_b200: empty weight");
  if (in_f % 128 != 0 || out_f % 128 != 0)
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: in and out features must be multiples of 128 (the Hadamard blocks)");
  if (!(n % 2 == 0 && n >= 16 && n <= 128)) return refuse(EXL3_UNSUPPORTED, "exl3_b200: not an admitted rate (n even, 16..128)");
  if (!rate_served(n))
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: rates off the half-bit grid or above 6 bits are not served by the sm_100a kernels");
  if (out_f / 128 > static_cast<int>(kCounterCount)) return refuse(EXL3_TOO_LARGE, "exl3_b200: out_features too large");
  return kOk;
}

int64_t numel(const exl3_tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

bool act_dtype(int32_t dt) { return dt == EXL3_F16 || dt == EXL3_BF16 || dt == EXL3_F32; }

// ------------------------------------------------------------------ host loads

std::string name_of(exl3_str s) { return s.ptr ? std::string(s.ptr, s.len) : std::string(); }

bool source_get(const exl3_load_ctx* ctx, const std::string& name, exl3_host_tensor& out) {
  if (!ctx || !ctx->source.tensor) return false;
  exl3_str s{name.data(), name.size()};
  memset(&out, 0, sizeof out);
  return ctx->source.tensor(ctx->source.ctx, s, &out) == 0 && out.data != nullptr;
}

struct LinearParts {
  exl3_host_tensor tr, su, sv;
};

// <base>.trellis / .suh / .svh as exllamav3 stores a linear (plugin.zig:96-103); 0 = missing, -1 = misshaped.
int parts_of(const exl3_load_ctx* ctx, const std::string& base, uint32_t in_dim, LinearParts& p) {
  if (!source_get(ctx, base + ".trellis", p.tr)) return 0;
  if (!source_get(ctx, base + ".suh", p.su) || !source_get(ctx, base + ".svh", p.sv)) return 0;
  if (p.tr.ndim != 3 || p.su.ndim != 1 || p.sv.ndim != 1) return -1;
  if (p.su.shape[0] != p.tr.shape[0] * 16 || p.sv.shape[0] != p.tr.shape[1] * 16) return -1;
  if (in_dim != 0 && p.su.shape[0] != static_cast<int64_t>(in_dim)) return -1;
  if (p.su.dtype != EXL3_F16 || p.sv.dtype != EXL3_F16) return -1;
  if (p.tr.dtype != EXL3_I16 && p.tr.dtype != EXL3_U16) return -1;
  return 1;
}

const exl3_verdict kNotShaped = {EXL3_UNSUPPORTED,
                                 "exl3_b200: not an EXL3 linear of the expected input width (trellis [in/16, out/16, n], "
                                 "suh f16 [in], svh f16 [out])"};

// The block's codebook and codeword window as weight flags (EXL3_WEIGHT_MCG, EXL3_WEIGHT_WINDOW); 0 for mul1 at the
// full window.
uint32_t block_window_flags(exl3_str block_json) {
  JVal b;
  if (!parse_json(block_json, b) || b.kind != JVal::Obj) return 0;
  const JVal* w = b.get("window");
  uint32_t f = str_is(b.get("codebook"), "mcg") ? EXL3_WEIGHT_MCG : 0u;
  if (!w || w->kind != JVal::Num || !w->is_int || w->num < 8 || w->num > 16) return f;
  return f | EXL3_WEIGHT_WINDOW(static_cast<int>(w->num));
}

exl3_verdict upload_stack(const exl3_load_ctx* ctx, const std::vector<LinearParts>& parts, uint32_t flags,
                          exl3_weight* out) {
  const LinearParts& p0 = parts[0];
  const int in_f = static_cast<int>(p0.su.shape[0]);
  const int out_f = static_cast<int>(p0.sv.shape[0]);
  const int n = static_cast<int>(p0.tr.shape[2]);
  for (const auto& p : parts)
    if (p.su.shape[0] != in_f || p.sv.shape[0] != out_f || p.tr.shape[2] != n) return kNotShaped;
  const int groups = static_cast<int>(parts.size());
  exl3_verdict v = check_linear_shape(groups, in_f, out_f, n);
  if (v.code != EXL3_OK) return v;
  v = ensure_device(ctx->device);
  if (v.code != EXL3_OK) return v;
  DeviceGuard guard(ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(ctx->stream);
  const size_t tw = static_cast<size_t>(in_f / 16) * (out_f / 16) * n;
  uint16_t *tr = nullptr, *su = nullptr, *sv = nullptr;
  if (cudaMalloc(&tr, tw * groups * 2) != cudaSuccess || cudaMalloc(&su, static_cast<size_t>(in_f) * groups * 2) != cudaSuccess ||
      cudaMalloc(&sv, static_cast<size_t>(out_f) * groups * 2) != cudaSuccess) {
    cudaFree(tr);
    cudaFree(su);
    cudaFree(sv);
    return refuse(EXL3_TOO_LARGE, "exl3_b200: out of device memory");
  }
  bool ok = true;
  for (int g = 0; g < groups && ok; ++g) {
    ok = cudaMemcpyAsync(tr + g * tw, parts[g].tr.data, tw * 2, cudaMemcpyHostToDevice, st) == cudaSuccess &&
         cudaMemcpyAsync(su + static_cast<size_t>(g) * in_f, parts[g].su.data, static_cast<size_t>(in_f) * 2,
                         cudaMemcpyHostToDevice, st) == cudaSuccess &&
         cudaMemcpyAsync(sv + static_cast<size_t>(g) * out_f, parts[g].sv.data, static_cast<size_t>(out_f) * 2,
                         cudaMemcpyHostToDevice, st) == cudaSuccess;
  }
  ok = ok && cudaStreamSynchronize(st) == cudaSuccess;  // host data is only valid during the call
  if (!ok) {
    cudaFree(tr);
    cudaFree(su);
    cudaFree(sv);
    return refuse(EXL3_FAILED, "exl3_b200: upload failed");
  }
  memset(out, 0, sizeof *out);
  out->size = sizeof(exl3_weight);
  out->flags = EXL3_WEIGHT_OWNED | flags | block_window_flags(ctx->block_json);
  out->trellis = tr;
  out->suh = su;
  out->svh = sv;
  out->groups = groups;
  out->in_features = in_f;
  out->out_features = out_f;
  out->n = n;
  out->device = ctx->device;
  out->nseg = 1;
  out->seg_cols[0] = 0;
  out->seg_cols[1] = out_f;
  return kOk;
}

// ------------------------------------------------------------------ resident decoded matrices

// A kept weight's GEMM B image (W_hat^T blocks of 128 columns x 64 k, f16; the layout images_kernel writes), per
// group, with two column blocks of padding so a ragged last tile's reads stay inside it.  Keyed on the weight's
// device pointers and shape.
struct Resident {
  int device;
  const uint16_t *trellis, *suh, *svh;
  int groups, in_f, out_f, n, nseg;
  size_t group_bytes;
  uint8_t* image;
  bool filled;
};
std::mutex g_res_mu;
std::vector<std::unique_ptr<Resident>> g_res;

size_t resident_group_bytes(const exl3_weight* w) {
  return static_cast<size_t>(w->out_features / 128 + 2) * w->in_features * 256;  // in/64 blocks of 16 KiB per column block
}

bool resident_is(const Resident& r, const exl3_weight* w) {
  return r.device == w->device && r.trellis == w->trellis && r.suh == w->suh && r.svh == w->svh &&
         r.groups == w->groups && r.in_f == w->in_features && r.out_f == w->out_features && r.n == w->n &&
         r.nseg == w->nseg;
}

void resident_free(Resident& r) {
  DeviceGuard guard(r.device);
  cudaFree(r.image);
}

exl3_verdict check_weight(const exl3_weight* w) {
  if (!w || w->size != sizeof(exl3_weight) || !w->trellis || !w->suh || !w->svh)
    return refuse(EXL3_FAILED, "exl3_b200: not a loaded weight");
  if (w->nseg < 1 || w->nseg > EXL3_MAX_SEGMENTS) return refuse(EXL3_FAILED, "exl3_b200: bad segment count");
  if (exl3::flags_window_bits(w->flags) < 8) return refuse(EXL3_UNSUPPORTED, "exl3_b200: Exl3WindowUnsupported");
  return check_linear_shape(w->groups, w->in_features, w->out_features, w->n);
}

// The prefill path: per group, segment and chunk of rows, the A image of the rotated rows; per chunk of columns, the
// B image of the decoded weights and one tensor-core GEMM into y.  The chunks keep both images inside the workspace's
// image region, so the call allocates nothing.
// The GEMM's tile shape for an m x n launch: the fewest tile-waves over the SMs, weighted by the tile's area (its MMA
// time) and divided by the shape's measured throughput on B200 relative to 256 x 256 (4096 x 12288 at 4 bpw:
// 128 x 128 0.72, 128 x 256 0.93, 256 x 128 0.83 -- narrower tiles re-read more operand bytes per flop).
// EXL3_GEMM_SHAPE (0..3) overrides it, for measurement runs.
int gemm_shape_for(int64_t m, int64_t n, int sms) {
  if (const char* e = getenv("EXL3_GEMM_SHAPE")) {
    const int v = atoi(e);
    if (v >= 0 && v <= 3) return v;
  }
  static const int64_t kEff[4] = {72, 93, 83, 100};
  int best = 0;
  int64_t best_cost = -1;
  for (int shape : {1, 3, 2, 0}) {
    const int64_t bm = exl3::gemm_block_m(shape), bn = exl3::gemm_block_n(shape);
    const int64_t tiles = ((m + bm - 1) / bm) * ((n + bn - 1) / bn);
    const int64_t cost = (tiles + sms - 1) / sms * bm * bn * 100 / kEff[shape];
    if (best_cost < 0 || cost < best_cost) {
      best = shape;
      best_cost = cost;
    }
  }
  return best;
}

exl3_verdict run_gemm(DeviceState* d, const exl3_weight* w, const void* x, int32_t x_dtype, int64_t rows, void* y,
                      int32_t y_dtype, uint32_t flags, cudaStream_t st, void* const* ev) {
  bool first = true;
  auto mark = [&](int i) {
    if (ev && first && ev[i]) cudaEventRecord(static_cast<cudaEvent_t>(ev[i]), st);
  };
  mark(0);
  const int in_f = w->in_features, out_f = w->out_features, groups = w->groups;
  const bool grouped = (w->flags & EXL3_WEIGHT_GROUPED) != 0;
  constexpr int bm = 256, bn = 256;  // chunk granularity: a multiple of every tile shape
  const size_t tile_halfs = static_cast<size_t>(in_f / 16) * (out_f / 16) * w->n;
  const size_t xsz = x_dtype == EXL3_F32 ? 4 : 2;
  const size_t ysz = y_dtype == EXL3_F32 ? 4 : 2;
  const size_t row_bytes = static_cast<size_t>(in_f) * 2;  // one image row (A) or column (B)
  // rows per chunk: at most half the region; columns: what the rows leave
  int64_t mc = static_cast<int64_t>(d->image_bytes / 2 / row_bytes) / bm * bm;
  const int64_t rows_padded = (rows + bm - 1) / bm * bm;
  if (mc > rows_padded) mc = rows_padded;
  if (mc < bm) return refuse(EXL3_TOO_LARGE, "exl3_b200: in_features too large for the prefill image region");
  uint8_t* a_img = d->image;
  uint8_t* b_img = d->image + static_cast<size_t>(mc) * row_bytes;
  // a multiple of the tile width, so a ragged last tile's reads stay inside the B region
  int64_t nc_cap = static_cast<int64_t>((d->image_bytes - static_cast<size_t>(mc) * row_bytes) / row_bytes) / bn * bn;
  if (nc_cap < bn) return refuse(EXL3_TOO_LARGE, "exl3_b200: in_features too large for the prefill image region");
  const int gcount = grouped ? groups : 1;
  const uint32_t cw_mask = exl3::window_mask(exl3::flags_window_bits(w->flags));
  const int mcg = (w->flags & EXL3_WEIGHT_MCG) ? 1 : 0;
  // a kept weight: its B image is decoded once (the first call fills it, on this stream) and read from there
  uint8_t* kept = nullptr;
  size_t kept_group = 0;
  bool fill = false;
  {
    std::lock_guard<std::mutex> lk(g_res_mu);
    for (auto& r : g_res)
      if (resident_is(*r, w)) {
        kept = r->image;
        kept_group = r->group_bytes;
        fill = !r->filled;
        r->filled = true;
        break;
      }
  }
  // W_hat^T decoded inside the GEMM (no B image; the same bytes): taken on request (EXL3_GEMM_FUSED=1) for the full
  // mul1 window without a kept image.  Measured on config 3's layer at 64 / 128 / 256 rows it is not the default: its
  // 128-column tiles keep 96 of the 148 SMs decoding (68.8 / 71.2 / 85.7 us against the image path's 63.6 / 66.5 /
  // 74.8); the routed experts' prefill, whose tiles fill every SM, takes it by default (exl3_moe_prefill.cu)
  const char* fz = getenv("EXL3_GEMM_FUSED");
  const bool fused = !kept && !cw_mask && !mcg && fz && atoi(fz) == 1;
  if (kept || fused) {
    nc_cap = (static_cast<int64_t>(out_f) + bn - 1) / bn * bn;  // no column chunks: no B image (or the kept one)
    for (int g = 0; fill && g < gcount; ++g)
      if (exl3::launch_images(nullptr, x_dtype, 0, 0, 0, nullptr, 0, nullptr, w->trellis + static_cast<size_t>(g) * tile_halfs,
                              in_f, out_f, 0, out_f, w->n, kept + static_cast<size_t>(g) * kept_group, st,
                              cw_mask, mcg) != cudaSuccess)
        return refuse(EXL3_FAILED, "exl3_b200: resident image launch failed");
  }
  for (int g = 0; g < gcount; ++g) {
    const int64_t x_stride = grouped ? static_cast<int64_t>(groups) * in_f : in_f;
    const uint8_t* xg = static_cast<const uint8_t*>(x) + static_cast<size_t>(g) * in_f * xsz;
    const uint16_t* trg = w->trellis + static_cast<size_t>(g) * tile_halfs;
    for (int s = 0; s < w->nseg; ++s) {
      const int c0 = w->seg_cols[s], c1 = w->seg_cols[s + 1], seg_w = c1 - c0;
      const uint16_t* suh = w->suh + (static_cast<size_t>(g) * w->nseg + s) * in_f;
      const uint16_t* svh = w->svh + static_cast<size_t>(g) * out_f + c0;
      // y element (row, column j of this segment)
      uint8_t* yseg;
      int64_t ystride;
      if (w->nseg == 1) {
        ystride = grouped ? static_cast<int64_t>(groups) * out_f : out_f;
        yseg = static_cast<uint8_t*>(y) + static_cast<size_t>(g) * out_f * ysz;
      } else {
        ystride = seg_w;
        yseg = static_cast<uint8_t*>(y) + static_cast<size_t>(rows) * c0 * ysz;
      }
      for (int64_t r0 = 0; r0 < rows; r0 += mc) {
        const int m = static_cast<int>(rows - r0 < mc ? rows - r0 : mc);
        const int mp = (m + bm - 1) / bm * bm;  // padded rows: whole tiles of every shape
        for (int j0 = 0; j0 < seg_w; j0 += static_cast<int>(nc_cap)) {
          const int nc = static_cast<int>(seg_w - j0 < nc_cap ? seg_w - j0 : nc_cap);
          // the A image with the first column chunk's B image, in one launch
          if (exl3::launch_images(xg + static_cast<size_t>(r0) * x_stride * xsz, x_dtype, x_stride, m, mp, suh,
                                  (flags & EXL3_MATMUL_PREPARED) ? 1 : 0, j0 == 0 ? a_img : nullptr, trg, in_f, out_f,
                                  c0 + j0, nc, w->n, (kept || fused) ? nullptr : b_img, st, cw_mask, mcg) != cudaSuccess)
            return refuse(EXL3_FAILED, "exl3_b200: prefill operand images launch failed");
          mark(1);
          // fused: 128 or 256-row tiles (above 256 rows each row tile decodes its B blocks again), 128-column tiles to
          // spread the decode over more SMs unless the columns fill them twice over
          const int shape = fused ? (m > 128 ? 2 : 0) + (nc % 256 == 0 && nc / 128 >= 2 * d->sms ? 1 : 0)
                                  : gemm_shape_for(m, nc, d->sms);
          const int tbm = exl3::gemm_block_m(shape), tbn = exl3::gemm_block_n(shape);
          exl3::GemmParams gp{};
          gp.a_img = a_img;
          gp.b_img = kept ? kept + static_cast<size_t>(g) * kept_group + static_cast<size_t>((c0 + j0) / 128) * in_f * 256
                          : b_img;
          gp.svh = svh + j0;
          uint8_t* yp = yseg + (static_cast<size_t>(r0) * ystride + j0) * ysz;
          gp.y = yp;
          gp.y_dtype = y_dtype;
          gp.y_row_stride = ystride;
          gp.m = m;
          gp.ncols = nc;
          gp.tiles_m = (m + tbm - 1) / tbm;
          gp.tiles_n = (nc + tbn - 1) / tbn;
          gp.kb = in_f / 64;
          gp.inner_only = (flags & EXL3_MATMUL_INNER) ? 1 : 0;
          gp.vec_store = exl3::store_width(yp, ystride * ysz);
          gp.err = d->err;
          if (fused) {
            gp.b_img = nullptr;
            gp.trellis = trg;
            gp.out_tiles = out_f / 16;
            gp.tn0 = (c0 + j0) / 16;
            gp.n = w->n;
          }
          if ((fused ? exl3::launch_gemm_fused(gp, shape, d->sms, st) : exl3::launch_gemm_image(gp, shape, d->sms, st)) !=
              cudaSuccess)
            return refuse(EXL3_FAILED, "exl3_b200: prefill GEMM launch failed");
          mark(2);
          first = false;
        }
      }
    }
  }
  if (ev && ev[3]) cudaEventRecord(static_cast<cudaEvent_t>(ev[3]), st);
  return kOk;
}

// The most rows a cluster-split GEMV launch rotates in each CTA; more take the prepare launch.
constexpr int kCtaRotateRows = 1;

// Rows from the GEMM threshold on take the tensor-core GEMM; fewer rows take one decode-GEMV launch per group and
// per 16 rows.
exl3_verdict run_linear(const exl3_weight* w, const void* x, int32_t x_dtype, int64_t rows, void* y, int32_t y_dtype,
                        uint32_t flags, cudaStream_t st, void* const* ev = nullptr) {
  DeviceState* d = device_state(w->device);
  if (!d) return refuse(EXL3_FAILED, "exl3_b200: no workspace on this device (exl3_open or a weight load creates it)");
  DeviceGuard guard(w->device);
  // the GEMM's prepare reads four elements per vector load
  const size_t vec = x_dtype == EXL3_F32 ? 16 : 8;
  const bool x_vec = reinterpret_cast<uintptr_t>(x) % vec == 0;
  const bool gemm = x_vec && ((flags & EXL3_MATMUL_GEMM) != 0 ||
                              ((flags & EXL3_MATMUL_GEMV) == 0 && rows >= d->gemm_min_rows));
  if (gemm) return run_gemm(d, w, x, x_dtype, rows, y, y_dtype, flags, st, ev);
  if (ev && ev[0]) cudaEventRecord(static_cast<cudaEvent_t>(ev[0]), st);
  // measurement overrides: EXL3_GEMV=4 takes the grid-stride GEMV, =5 the cluster-split one, =6 the persistent one;
  // EXL3_GEMV_SPLIT the cluster size
  const char* gv = getenv("EXL3_GEMV");
  const int gv_pick = gv ? atoi(gv) : 0;
  const bool gemv_v5 = gv_pick != 4;
  const char* sp = getenv("EXL3_GEMV_SPLIT");
  const int split = sp ? atoi(sp) : 0;
  const int in_f = w->in_features, out_f = w->out_features, groups = w->groups;
  const bool grouped = (w->flags & EXL3_WEIGHT_GROUPED) != 0;
  const bool imma = (flags & EXL3_MATMUL_DP4A) == 0;
  const size_t tile_halfs = static_cast<size_t>(in_f / 16) * (out_f / 16) * w->n;
  const size_t xsz = x_dtype == EXL3_F32 ? 4 : 2;
  const size_t ysz = y_dtype == EXL3_F32 ? 4 : 2;
  const int gcount = grouped ? groups : 1;
  for (int g = 0; g < gcount; ++g) {
    for (int64_t r0 = 0; r0 < rows; r0 += exl3::kMaxRows) {
      const int rc = static_cast<int>(rows - r0 < exl3::kMaxRows ? rows - r0 : exl3::kMaxRows);
      const int rg = rc <= 8 ? 1 : 2;
      exl3::GemvParams gp{};
      const int64_t x_stride = grouped ? static_cast<int64_t>(groups) * in_f : in_f;
      gp.trellis = w->trellis + static_cast<size_t>(g) * tile_halfs;
      gp.suh = w->suh + static_cast<size_t>(g) * w->nseg * in_f;
      gp.svh = w->svh + static_cast<size_t>(g) * out_f;
      gp.x = static_cast<const uint8_t*>(x) + static_cast<size_t>(g) * in_f * xsz;
      gp.x_dtype = x_dtype;
      gp.x_row_stride = x_stride;
      const int64_t y_stride = grouped ? static_cast<int64_t>(groups) * out_f : out_f;
      gp.y = static_cast<uint8_t*>(y) + static_cast<size_t>(g) * out_f * ysz;
      gp.y_dtype = y_dtype;
      gp.y_row_stride = y_stride;
      gp.row0 = static_cast<int32_t>(r0);
      gp.rows_total = static_cast<int32_t>(rows);
      gp.partials = d->partials;
      gp.counters = d->counters;
      gp.err = d->err;
      gp.in_features = in_f;
      gp.out_features = out_f;
      gp.rows = rc;
      gp.nseg = w->nseg;
      for (int s = 0; s <= w->nseg; ++s) gp.seg_cb[s] = w->seg_cols[s] / 128;
      for (int s = w->nseg + 1; s <= exl3::kMaxSegments; ++s) gp.seg_cb[s] = gp.seg_cb[w->nseg];
      gp.prepared = (flags & EXL3_MATMUL_PREPARED) ? 1 : 0;
      gp.inner_only = (flags & EXL3_MATMUL_INNER) ? 1 : 0;
      gp.cw_mask = exl3::window_mask(exl3::flags_window_bits(w->flags));
      gp.mcg = (w->flags & EXL3_WEIGHT_MCG) ? 1 : 0;
      if ((gp.cw_mask || gp.mcg) && !imma)
        return refuse(EXL3_UNSUPPORTED, "exl3_b200: a narrowed codeword window or mcg takes the tensor-pipe order (no dp4a)");
      const char* why = nullptr;
      // the persistent GEMV for large launches (every row count of a shape takes the same kernel, so a row's bits do
      // not depend on the rows batched with it), the cluster-split one below (and for a narrowed codeword window)
      const bool v6 = imma && !gp.cw_mask && !gp.mcg && (gv_pick == 6 || (gv_pick == 0 && exl3::gemv6_prefers(gp)));
      if (v6 && exl3::gemv6_scratch_bytes(gp, d->sms) <= d->partial_floats * 4) {
        if (exl3::launch_gemv6(gp, w->n, d->sms, d->partials, d->counters, st) != cudaSuccess)
          return refuse(EXL3_FAILED, "exl3_b200: GEMV launch failed");
        continue;
      }
      // the cluster-split GEMV where a split fits (every served width), else the grid-stride one with global partials
      if (gemv_v5 && exl3::gemv5_geometry(gp, w->n, d->sms, rg, split, &why)) {
        // more than four rows: x is rotated once by a prepare launch instead of by every CTA for its slabs
        if (imma && rc > kCtaRotateRows && exl3::gemv_prep_bytes(gp, rg) <= d->partial_floats * 4) {
          if (exl3::launch_gemv_prep(gp, rg, d->partials, st) != cudaSuccess)
            return refuse(EXL3_FAILED, "exl3_b200: GEMV launch failed");
          gp.xf = d->partials;
        }
        if (exl3::launch_gemv5(gp, w->n, rg, imma, st, true) != cudaSuccess)
          return refuse(EXL3_FAILED, "exl3_b200: GEMV launch failed");
        continue;
      }
      if (gp.cw_mask || gp.mcg)
        return refuse(EXL3_UNSUPPORTED, "exl3_b200: a narrowed codeword window or mcg needs a cluster split of this input width");
      if (!exl3::gemv_geometry(gp, d->sms, rg, d->partial_floats, &why)) return refuse(EXL3_TOO_LARGE, why);
      if (exl3::launch_gemv(gp, w->n, rg, imma, st, true) != cudaSuccess)
        return refuse(EXL3_FAILED, "exl3_b200: GEMV launch failed");
    }
  }
  if (ev && ev[3]) cudaEventRecord(static_cast<cudaEvent_t>(ev[3]), st);
  return kOk;
}

}  // namespace

// ====================================================================== the C ABI

extern "C" {

const char* exl3_version(void) { return "exl3_b200 1 (sm_100a)"; }

exl3_claim exl3_claims(exl3_str block_json, exl3_str config_json) {
  (void)config_json;
  JVal b;
  if (!parse_json(block_json, b) || b.kind != JVal::Obj) return EXL3_CLAIM_NO;
  if (str_is(b.get("quant_method"), "exl3") || str_is(b.get("format"), "exl3")) return EXL3_CLAIM_BY_MARKER;
  return EXL3_CLAIM_NO;
}

exl3_verdict exl3_validate(exl3_str block_json, exl3_str config_json) {
  (void)config_json;
  JVal b;
  if (!parse_json(block_json, b) || b.kind != JVal::Obj) return refuse(EXL3_UNSUPPORTED, "exl3_b200: the block is not a JSON object");
  if (!str_is(b.get("quant_method"), "exl3") && !str_is(b.get("format"), "exl3"))
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: not an exllamav3 block");
  const JVal* cb = b.get("codebook");
  if (!str_is(cb, "mul1")) return refuse(EXL3_UNSUPPORTED, "exl3_b200: the codebook is not mul1");
  if (const JVal* w = b.get("window")) {
    if (w->kind != JVal::Num || !w->is_int || w->num < 8 || w->num > 16)
      return refuse(EXL3_UNSUPPORTED, "exl3_b200: Exl3WindowUnsupported");
  }
  if (const JVal* k = b.get("k")) {
    if (k->kind != JVal::Num) return refuse(EXL3_UNSUPPORTED, "exl3_b200: Exl3RateUnsupported");
    const double scaled = k->num * 16.0, n = std::round(scaled);
    if (std::fabs(scaled - n) > 1e-6 || n < 16 || n > 128 || std::fmod(n, 2.0) != 0)
      return refuse(EXL3_UNSUPPORTED, "exl3_b200: Exl3RateUnsupported");
    if (!rate_served(static_cast<int>(n)))
      return refuse(EXL3_UNSUPPORTED, "exl3_b200: rates off the half-bit grid or above 6 bits are not served by the sm_100a kernels");
  }
  return kOk;
}

uint64_t exl3_bill(exl3_str block_json, exl3_str model_dir, uint64_t stored) {
  (void)block_json;
  (void)model_dir;
  return stored;
}

// ---------------------------------------------------------------- the model seam's parse (linears only)
//
// plugins/turboexl3_qwen38/config.zig:19-119 (claims, parse, checkPack / checkBlock) and src/direct/config.zig:301-420
// (parseJson): MLX-free and bounds-checked, the EXL3 blocks refused with the reference's names, narrowed to what this
// library decodes (the mul1 or mcg codebook named; windows 8..16; whole and half bits per weight 1..6).

namespace {

constexpr uint32_t kModelMaxTopK = 32;  // the widest top-k the routed reduction holds (config.zig:16)

bool is_qwen38(const std::string& mt) { return mt == "qwen4_exp" || mt == "qwen4_exp_text"; }

const char* check_model_block(const JVal& o, bool bank, uint32_t* rate_n) {
  if (!str_is(o.get("format"), "exl3")) return "turboexl3_qwen38: NotExl3";
  // mul1 or mcg (the reference also lets a trunk block leave its codebook unnamed; here it is named)
  if (!str_is(o.get("codebook"), "mul1") && !str_is(o.get("codebook"), "mcg"))
    return "turboexl3_qwen38: Exl3CodebookUnsupported";
  if (const JVal* w = o.get("window"))
    if (w->kind != JVal::Num || !w->is_int || w->num < 8 || w->num > 16) return "turboexl3_qwen38: Exl3WindowUnsupported";
  if (bank) {
    const JVal* k = o.get("k");
    if (!k || k->kind != JVal::Num) return "turboexl3_qwen38: Exl3RateUnsupported";
    const double scaled = k->num * 16.0, n = std::round(scaled);
    if (!std::isfinite(scaled) || std::fabs(scaled - n) > 1e-6 || !exl3::rate_served_n(static_cast<int>(n)))
      return "turboexl3_qwen38: Exl3RateUnsupported";
    *rate_n = static_cast<uint32_t>(n);
  }
  return nullptr;
}

// A u32 field: absent keeps the default; anything but a non-negative integer below 2^32 is refused.
bool model_u32(const JVal& o, const char* key, uint32_t* v) {
  const JVal* f = o.get(key);
  if (!f) return true;
  if (f->kind != JVal::Num || !f->is_int || f->num < 0 || f->num > 4294967295.0) return false;
  *v = static_cast<uint32_t>(f->num);
  return true;
}

}  // namespace

exl3_claim exl3_model_claims(exl3_str model_type, exl3_str config_json) {
  if (!is_qwen38(name_of(model_type))) return EXL3_CLAIM_NO;
  JVal doc;
  if (!parse_json(config_json, doc) || doc.kind != JVal::Obj) return EXL3_CLAIM_NO;
  const JVal* t = doc.get("trunk_quant");
  return (t && t->kind != JVal::Null) ? EXL3_CLAIM_BY_MARKER : EXL3_CLAIM_NO;
}

exl3_verdict exl3_model_parse(exl3_str config_json, exl3_model_config* out) {
  if (!out || out->size != sizeof(exl3_model_config)) return refuse(EXL3_FAILED, "exl3_b200: bad model config");
  JVal root;
  if (!parse_json(config_json, root) || root.kind != JVal::Obj) return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: InvalidConfig");
  exl3_model_config c{};
  c.size = sizeof(exl3_model_config);
  // the pack's EXL3 blocks first (config.zig:35-41: checkPack runs before the model's parse)
  const JVal* t = root.get("trunk_quant");
  if (t && t->kind == JVal::Null) t = nullptr;
  if (t) {
    if (t->kind != JVal::Obj) return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: TrunkQuantNotAnObject");
    if (const char* why = check_model_block(*t, false, nullptr)) return refuse(EXL3_UNSUPPORTED, why);
  }
  const JVal* tc = root.get("text_config");
  if (tc && tc->kind != JVal::Obj) return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: InvalidConfigField");
  const JVal& text = tc ? *tc : root;
  const JVal* e = root.get("expert_quant");
  if (e && e->kind == JVal::Null) e = nullptr;
  if (e) {
    if (e->kind != JVal::Obj) return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: NotExl3");
    if (const char* why = check_model_block(*e, true, &c.expert_rate_n)) return refuse(EXL3_UNSUPPORTED, why);
    if (const JVal* k = text.get("num_experts_per_tok"))
      if (k->kind == JVal::Num && k->is_int && k->num > kModelMaxTopK)
        return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: Exl3TopKExceedsReduceBank");
  }
  if (!t) return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: Unsupported");  // a K pack is fully EXL3
  // src/direct/config.zig:24-78 defaults
  c.hidden_size = 3840, c.intermediate_size = 15360, c.num_hidden_layers = 48, c.num_attention_heads = 16;
  c.num_key_value_heads = 8, c.head_dim = 256;
  const struct { const char* key; uint32_t* v; } fields[] = {
      {"hidden_size", &c.hidden_size}, {"intermediate_size", &c.intermediate_size},
      {"num_hidden_layers", &c.num_hidden_layers}, {"num_attention_heads", &c.num_attention_heads},
      {"num_key_value_heads", &c.num_key_value_heads}, {"head_dim", &c.head_dim}, {"num_experts", &c.num_experts},
      {"num_experts_per_tok", &c.num_experts_per_tok}, {"moe_intermediate_size", &c.moe_intermediate_size},
      {"shared_expert_intermediate_size", &c.shared_expert_intermediate_size}};
  for (const auto& f : fields)
    if (!model_u32(text, f.key, f.v)) return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: InvalidConfigField");
  // the bounds the linears need: whole 128-column blocks, heads that divide, a routed bank when experts are named
  if (c.hidden_size == 0 || c.hidden_size % 128 || c.num_hidden_layers == 0 || c.num_key_value_heads == 0 ||
      c.num_attention_heads % c.num_key_value_heads || c.intermediate_size % 128 || c.moe_intermediate_size % 128 ||
      c.shared_expert_intermediate_size % 128)
    return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: InvalidConfigField");
  if (c.num_experts && (!e || c.num_experts_per_tok == 0 || c.num_experts_per_tok > c.num_experts ||
                        c.num_experts > 1024 || c.moe_intermediate_size == 0))
    return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: InvalidConfigField");
  const char* prefix = "language_model.model";
  if (const JVal* wp = root.get("weight_prefix"))
    if (wp->kind == JVal::Str) prefix = wp->str.c_str();
  if (strlen(prefix) >= sizeof(c.weight_prefix)) return refuse(EXL3_UNSUPPORTED, "turboexl3_qwen38: InvalidConfigField");
  strcpy(c.weight_prefix, prefix);
  *out = c;
  return kOk;
}

exl3_verdict exl3_open(exl3_load_ctx* ctx) {
  if (!ctx || ctx->size != sizeof(exl3_load_ctx)) return refuse(EXL3_FAILED, "exl3_b200: bad load context");
  if (exl3_claims(ctx->block_json, ctx->config_json) == EXL3_CLAIM_NO)
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: not an exllamav3 mul1 block");
  // a pack the model seam claims (qwen38) loads by that seam's block rules (mul1 or mcg, windows 8..16,
  // config.zig:86-104); the quant seam's own validate is the ds41 plugin's (mul1 only, config.zig:49-53)
  JVal cfg, blk;
  if (parse_json(ctx->config_json, cfg) && cfg.kind == JVal::Obj && cfg.get("model_type") &&
      cfg.get("model_type")->kind == JVal::Str && is_qwen38(cfg.get("model_type")->str) &&
      parse_json(ctx->block_json, blk) && blk.kind == JVal::Obj) {
    uint32_t rate_n = 0;
    if (const char* why = check_model_block(blk, blk.get("k") != nullptr, &rate_n)) return refuse(EXL3_UNSUPPORTED, why);
    return ensure_device(ctx->device);
  }
  exl3_verdict v = exl3_validate(ctx->block_json, ctx->config_json);
  if (v.code != EXL3_OK) return v;
  return ensure_device(ctx->device);
}

void exl3_close(exl3_load_ctx* ctx) { (void)ctx; }

exl3_verdict exl3_load_tensor(const exl3_load_ctx* ctx, exl3_str name, uint32_t in_dim, exl3_weight* out) {
  if (!ctx || !out) return refuse(EXL3_FAILED, "exl3_b200: bad arguments");
  const std::string base = name_of(name);
  if (base.size() > 160) return refuse(EXL3_FAILED, "exl3_b200: a name too long");
  LinearParts p;
  const int got = parts_of(ctx, base, in_dim, p);
  if (got < 0) return kNotShaped;
  if (got == 1) return upload_stack(ctx, {p}, 0, out);
  // grouped linear: <base>.slice.<g>
  std::vector<LinearParts> parts;
  for (int g = 0;; ++g) {
    LinearParts q;
    const int r = parts_of(ctx, base + ".slice." + std::to_string(g), in_dim, q);
    if (r < 0) return kNotShaped;
    if (r == 0) break;
    parts.push_back(q);
  }
  if (parts.empty()) return refuse(EXL3_FAILED, "MissingWeight");
  return upload_stack(ctx, parts, EXL3_WEIGHT_GROUPED, out);
}

exl3_verdict exl3_load_bank(const exl3_load_ctx* ctx, exl3_str name, uint32_t in_dim, exl3_weight* out) {
  if (!ctx || !out) return refuse(EXL3_FAILED, "exl3_b200: bad arguments");
  const std::string full = name_of(name);
  const size_t dot = full.rfind('.');
  if (dot == std::string::npos) return refuse(EXL3_FAILED, "MissingWeight");
  const std::string prefix = full.substr(0, dot), suffix = full.substr(dot);
  std::vector<LinearParts> parts;
  for (int e = 0;; ++e) {
    LinearParts q;
    const int r = parts_of(ctx, prefix + "." + std::to_string(e) + suffix, in_dim, q);
    if (r < 0) return kNotShaped;
    if (r == 0) break;
    parts.push_back(q);
  }
  if (parts.empty()) return refuse(EXL3_FAILED, "MissingWeight");
  // every expert the router scores (plugin.zig:142-151)
  const std::string tail = ".experts";
  bool routed_ok = false;
  if (prefix.size() > tail.size() && prefix.compare(prefix.size() - tail.size(), tail.size(), tail) == 0) {
    exl3_host_tensor gate;
    if (source_get(ctx, prefix.substr(0, prefix.size() - tail.size()) + ".gate.weight", gate) && gate.ndim == 2)
      routed_ok = gate.shape[0] == static_cast<int64_t>(parts.size());
  }
  if (!routed_ok)
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: the bank holds another count of experts than its router scores");
  exl3_verdict v = upload_stack(ctx, parts, EXL3_WEIGHT_BANK, out);
  if (v.code == EXL3_OK) {
    v = exl3::moe_reserve(out->device, out->in_features, out->out_features);
    if (v.code != EXL3_OK) exl3_release(out);
  }
  return v;
}

void exl3_release(exl3_weight* w) {
  if (!w) return;
  if (w->size == sizeof(exl3_weight)) {  // its kept matrices go with it
    std::lock_guard<std::mutex> lk(g_res_mu);
    for (size_t i = 0; i < g_res.size();)
      if (resident_is(*g_res[i], w)) {
        resident_free(*g_res[i]);
        g_res.erase(g_res.begin() + static_cast<std::ptrdiff_t>(i));
      } else {
        ++i;
      }
  }
  if ((w->flags & EXL3_WEIGHT_OWNED) && w->size == sizeof(exl3_weight)) {
    DeviceGuard guard(w->device);
    cudaFree(w->trellis);
    cudaFree(w->suh);
    cudaFree(w->svh);
  }
  memset(w, 0, sizeof *w);
}

exl3_verdict exl3_matmul_ex(const exl3_weight* w, const exl3_tensor* x, uint32_t flags, void* stream, exl3_tensor* out) {
  return exl3_matmul_timed(w, x, flags, stream, out, nullptr);
}

exl3_verdict exl3_matmul_timed(const exl3_weight* w, const exl3_tensor* x, uint32_t flags, void* stream,
                               exl3_tensor* out, void* const* events) {
  exl3_verdict v = check_weight(w);
  if (v.code != EXL3_OK) return v;
  if (!x || !out || x->ndim < 1 || x->ndim > 4 || out->ndim != x->ndim) return refuse(EXL3_FAILED, "exl3_b200: bad tensors");
  if ((numel(x) > 0 && !x->data) || (numel(out) > 0 && !out->data)) return refuse(EXL3_FAILED, "exl3_b200: bad tensors");
  if (!act_dtype(x->dtype)) return refuse(EXL3_UNSUPPORTED, "exl3_b200: activations must be f16, bf16 or f32");
  if ((flags & EXL3_MATMUL_GEMV) && (flags & EXL3_MATMUL_GEMM))
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: GEMV and GEMM forced together");
  if ((flags & EXL3_MATMUL_PREPARED) && x->dtype != EXL3_F16)
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: prepared rows are f16");
  const bool grouped = (w->flags & EXL3_WEIGHT_GROUPED) != 0;
  if (w->groups > 1 && !grouped) return refuse(EXL3_UNSUPPORTED, "exl3_b200: a bank runs through swiglu, not matmul");
  const int64_t last = x->shape[x->ndim - 1];
  if (last != w->in_features) return refuse(EXL3_UNSUPPORTED, "exl3_b200: x's last dim is not the weight's input width");
  int64_t rows = numel(x) / last;
  if (grouped) {
    if (x->ndim < 2 || x->shape[x->ndim - 2] != w->groups)
      return refuse(EXL3_UNSUPPORTED, "exl3_b200: a grouped linear takes x [rows, groups, in]");
    rows /= w->groups;
  }
  const int32_t y_dtype = (flags & EXL3_MATMUL_INNER) ? EXL3_F32 : (flags & EXL3_MATMUL_PREPARED) ? out->dtype : x->dtype;
  if (out->dtype != y_dtype || (flags & EXL3_MATMUL_PREPARED && !act_dtype(out->dtype)))
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: the output has the wrong dtype");
  for (int i = 0; i < x->ndim - 1; ++i)
    if (out->shape[i] != x->shape[i]) return refuse(EXL3_UNSUPPORTED, "exl3_b200: the output has the wrong shape");
  if (out->shape[out->ndim - 1] != w->out_features) return refuse(EXL3_UNSUPPORTED, "exl3_b200: the output has the wrong shape");
  if (rows == 0) return kOk;
  if (rows > (1 << 24)) return refuse(EXL3_TOO_LARGE, "exl3_b200: too many rows");
  return run_linear(w, x->data, x->dtype, rows, out->data, y_dtype, flags, static_cast<cudaStream_t>(stream), events);
}

exl3_verdict exl3_matmul_tp(const exl3_weight* w, const exl3_tensor* x, exl3_tp* tp, int32_t slot,
                            const int64_t* seg_col0, const int64_t* seg_total, void* stream) {
  exl3_verdict v = check_weight(w);
  if (v.code != EXL3_OK) return v;
  const exl3::TpDev* td = exl3::tp_device(tp);
  if (!td) return refuse(EXL3_FAILED, "exl3_matmul_tp: not a connected exchange");
  if (exl3::tp_device_index(tp) != w->device) return refuse(EXL3_UNSUPPORTED, "exl3_matmul_tp: weight and exchange on different devices");
  if (slot < 0 || slot >= exl3::tp_slots(tp)) return refuse(EXL3_UNSUPPORTED, "exl3_matmul_tp: slot out of range");
  if (w->groups != 1 || (w->flags & EXL3_WEIGHT_GROUPED)) return refuse(EXL3_UNSUPPORTED, "exl3_matmul_tp: one ungrouped weight");
  if (!x || x->ndim < 1 || x->ndim > 4 || !act_dtype(x->dtype)) return refuse(EXL3_FAILED, "exl3_matmul_tp: bad x");
  if (x->shape[x->ndim - 1] != w->in_features) return refuse(EXL3_UNSUPPORTED, "exl3_matmul_tp: x's last dim is not the input width");
  const int64_t rows = numel(x) / w->in_features;
  if (rows < 1 || rows > exl3::kMaxRows) return refuse(EXL3_UNSUPPORTED, "exl3_matmul_tp: 1..16 rows (one launch)");
  if (!x->data || !seg_col0 || !seg_total) return refuse(EXL3_FAILED, "exl3_matmul_tp: bad arguments");
  const size_t esize = x->dtype == EXL3_F32 ? 4 : 2;
  int64_t total = 0;
  for (int s = 0; s < w->nseg; ++s) {
    const int64_t width = w->seg_cols[s + 1] - w->seg_cols[s];
    if (seg_total[s] % 128 != 0 || seg_col0[s] % 128 != 0 || seg_col0[s] < 0 || seg_col0[s] + width > seg_total[s])
      return refuse(EXL3_UNSUPPORTED, "exl3_matmul_tp: a segment's columns do not fit its gathered width");
    total += seg_total[s];
  }
  if (total / 128 > exl3::tp_max_cb(tp)) return refuse(EXL3_TOO_LARGE, "exl3_matmul_tp: gathered width beyond the exchange's flags");
  if (static_cast<int64_t>(rows * total * esize) > exl3::tp_slot_bytes(tp))
    return refuse(EXL3_TOO_LARGE, "exl3_matmul_tp: gathered rows beyond the exchange's slot");
  DeviceState* d = device_state(w->device);
  if (!d) return refuse(EXL3_FAILED, "exl3_b200: no workspace on this device (exl3_open or a weight load creates it)");
  DeviceGuard guard(w->device);
  exl3::GemvParams gp{};
  gp.trellis = w->trellis;
  gp.suh = w->suh;
  gp.svh = w->svh;
  gp.x = x->data;
  gp.x_dtype = x->dtype;
  gp.x_row_stride = w->in_features;
  gp.y = nullptr;
  gp.y_dtype = x->dtype;
  gp.row0 = 0;
  gp.rows_total = static_cast<int32_t>(rows);
  gp.err = d->err;
  gp.in_features = w->in_features;
  gp.out_features = w->out_features;
  gp.rows = static_cast<int32_t>(rows);
  gp.nseg = w->nseg;
  for (int s = 0; s <= w->nseg; ++s) gp.seg_cb[s] = w->seg_cols[s] / 128;
  for (int s = w->nseg + 1; s <= exl3::kMaxSegments; ++s) gp.seg_cb[s] = gp.seg_cb[w->nseg];
  int64_t base = 0;
  int32_t cbb = 0;
  for (int s = 0; s < w->nseg; ++s) {
    gp.tp_total[s] = seg_total[s];
    gp.tp_col0[s] = seg_col0[s];
    gp.tp_seg_base[s] = base;
    gp.tp_cb_base[s] = cbb;
    base += rows * seg_total[s];
    cbb += static_cast<int32_t>(seg_total[s] / 128);
  }
  gp.tp = td;
  gp.cw_mask = exl3::window_mask(exl3::flags_window_bits(w->flags));
  gp.mcg = (w->flags & EXL3_WEIGHT_MCG) ? 1 : 0;
  gp.tp_slot = slot;
  gp.tp_meta_cb = static_cast<uint32_t>(cbb);
  gp.tp_meta_bytes = static_cast<uint32_t>(rows * total * esize);
  const int rg = rows <= 8 ? 1 : 2;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the shard takes the kernel exl3_matmul gives its shape: the persistent GEMV where preferred, else the cluster
  // split (with the prepare launch from two rows)
  if (!gp.cw_mask && !gp.mcg && exl3::gemv6_prefers(gp) && exl3::gemv6_scratch_bytes(gp, d->sms) <= d->partial_floats * 4) {
    if (exl3::launch_gemv6(gp, w->n, d->sms, d->partials, d->counters, st) != cudaSuccess)
      return refuse(EXL3_FAILED, "exl3_matmul_tp: GEMV launch failed");
    return kOk;
  }
  const char* why = nullptr;
  if (!exl3::gemv5_geometry(gp, w->n, d->sms, rg, 0, &why)) return refuse(EXL3_UNSUPPORTED, why);
  if (rows > kCtaRotateRows && exl3::gemv_prep_bytes(gp, rg) <= d->partial_floats * 4) {
    if (exl3::launch_gemv_prep(gp, rg, d->partials, st) != cudaSuccess)
      return refuse(EXL3_FAILED, "exl3_matmul_tp: GEMV launch failed");
    gp.xf = d->partials;
  }
  if (exl3::launch_gemv5(gp, w->n, rg, true, st, true) != cudaSuccess)
    return refuse(EXL3_FAILED, "exl3_matmul_tp: GEMV launch failed");
  return kOk;
}

exl3_verdict exl3_matmul(const exl3_weight* w, const exl3_tensor* x, void* stream, exl3_tensor* out) {
  return exl3_matmul_ex(w, x, 0, stream, out);
}

exl3_verdict exl3_moe(const exl3_weight*, const exl3_tensor*, const exl3_tensor*, const exl3_tensor*, int32_t, void*,
                      exl3_tensor*) {
  return refuse(EXL3_UNSUPPORTED, "exl3_b200: routed experts run through swiglu");
}

exl3_verdict exl3_swiglu(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down, const exl3_tensor* x,
                         const exl3_tensor* inds, const exl3_tensor* scores, const exl3_swiglu_opts* opts, void* stream,
                         exl3_tensor* out) {
  return exl3::moe_swiglu(gate, up, down, x, inds, scores, opts, stream, out);
}

exl3_verdict exl3_moe_prefill_reserve(int32_t device, int32_t experts, int32_t hidden, int32_t inter, int32_t max_slots,
                                      uint64_t* bytes) {
  return exl3::moe_prefill_reserve(device, experts, hidden, inter, max_slots, bytes);
}

exl3_verdict exl3_swiglu_shared(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                                const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores,
                                const exl3_shared_swiglu* opts, void* stream, exl3_tensor* out) {
  return exl3::moe_swiglu_shared(gate, up, down, x, inds, scores, opts, stream, out);
}

exl3_verdict exl3_weight_view(uint16_t* trellis, uint16_t* suh, uint16_t* svh, int32_t groups, int32_t in_features,
                              int32_t out_features, int32_t n, int32_t device, exl3_weight* out) {
  if (!out || !trellis || !suh || !svh) return refuse(EXL3_FAILED, "exl3_b200: bad arguments");
  exl3_verdict v = check_linear_shape(groups, in_features, out_features, n);
  if (v.code != EXL3_OK) return v;
  if ((reinterpret_cast<uintptr_t>(trellis) & 15u) != 0)
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: the trellis must be 16-byte aligned");
  v = ensure_device(device);
  if (v.code != EXL3_OK) return v;
  memset(out, 0, sizeof *out);
  out->size = sizeof(exl3_weight);
  out->flags = groups > 1 ? EXL3_WEIGHT_BANK : 0;
  out->trellis = trellis;
  out->suh = suh;
  out->svh = svh;
  out->groups = groups;
  out->in_features = in_features;
  out->out_features = out_features;
  out->n = n;
  out->device = device;
  out->nseg = 1;
  out->seg_cols[1] = out_features;
  if (groups > 1) {  // a bank: make sure the routed-expert path has its workspace
    v = exl3::moe_reserve(device, in_features, out_features);
    if (v.code != EXL3_OK) return v;
  }
  return kOk;
}

exl3_verdict exl3_weight_stack(const exl3_weight* parts, int32_t count, void* stream, exl3_weight* out) {
  if (!parts || !out || count < 2 || count > EXL3_MAX_SEGMENTS)
    return refuse(EXL3_UNSUPPORTED, "exl3_b200: stack 2..4 linears");
  const exl3_weight& p0 = parts[0];
  int total = 0;
  for (int i = 0; i < count; ++i) {
    exl3_verdict v = check_weight(&parts[i]);
    if (v.code != EXL3_OK) return v;
    if (parts[i].groups != 1 || parts[i].nseg != 1 || parts[i].in_features != p0.in_features || parts[i].n != p0.n ||
        parts[i].device != p0.device || ((parts[i].flags ^ p0.flags) & (EXL3_WEIGHT_WINDOW_MASK | EXL3_WEIGHT_MCG)))
      return refuse(EXL3_UNSUPPORTED, "exl3_b200: stacked linears share one input width, rate, codebook, codeword window and device");
    total += parts[i].out_features;
  }
  exl3_verdict v = check_linear_shape(1, p0.in_features, total, p0.n);
  if (v.code != EXL3_OK) return v;
  DeviceGuard guard(p0.device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int KT = p0.in_features / 16, n = p0.n;
  uint16_t *tr = nullptr, *su = nullptr, *sv = nullptr;
  if (cudaMalloc(&tr, static_cast<size_t>(KT) * (total / 16) * n * 2) != cudaSuccess ||
      cudaMalloc(&su, static_cast<size_t>(count) * p0.in_features * 2) != cudaSuccess ||
      cudaMalloc(&sv, static_cast<size_t>(total) * 2) != cudaSuccess) {
    cudaFree(tr);
    cudaFree(su);
    cudaFree(sv);
    return refuse(EXL3_TOO_LARGE, "exl3_b200: out of device memory");
  }
  memset(out, 0, sizeof *out);
  int col = 0;
  bool ok = true;
  for (int i = 0; i < count && ok; ++i) {
    const size_t row_bytes = static_cast<size_t>(parts[i].out_features / 16) * n * 2;
    const size_t dst_pitch = static_cast<size_t>(total / 16) * n * 2;
    ok = cudaMemcpy2DAsync(reinterpret_cast<uint8_t*>(tr) + static_cast<size_t>(col / 16) * n * 2, dst_pitch,
                           parts[i].trellis, row_bytes, row_bytes, KT, cudaMemcpyDeviceToDevice, st) == cudaSuccess &&
         cudaMemcpyAsync(su + static_cast<size_t>(i) * p0.in_features, parts[i].suh, static_cast<size_t>(p0.in_features) * 2,
                         cudaMemcpyDeviceToDevice, st) == cudaSuccess &&
         cudaMemcpyAsync(sv + col, parts[i].svh, static_cast<size_t>(parts[i].out_features) * 2, cudaMemcpyDeviceToDevice,
                         st) == cudaSuccess;
    out->seg_cols[i] = col;
    col += parts[i].out_features;
  }
  if (!ok || cudaStreamSynchronize(st) != cudaSuccess) {
    cudaFree(tr);
    cudaFree(su);
    cudaFree(sv);
    memset(out, 0, sizeof *out);
    return refuse(EXL3_FAILED, "exl3_b200: stacking copy failed");
  }
  out->seg_cols[count] = total;
  out->size = sizeof(exl3_weight);
  out->flags = EXL3_WEIGHT_OWNED | (p0.flags & (EXL3_WEIGHT_WINDOW_MASK | EXL3_WEIGHT_MCG));
  out->trellis = tr;
  out->suh = su;
  out->svh = sv;
  out->groups = 1;
  out->in_features = p0.in_features;
  out->out_features = total;
  out->n = n;
  out->device = p0.device;
  out->nseg = count;
  return kOk;
}

exl3_verdict exl3_decode_dense(const exl3_weight* w, int32_t group, uint16_t* out, uint32_t flags, void* stream) {
  exl3_verdict v = check_weight(w);
  if (v.code != EXL3_OK) return v;
  if (group < 0 || group >= w->groups || !out) return refuse(EXL3_FAILED, "exl3_b200: bad arguments");
  DeviceGuard guard(w->device);
  const size_t tw = static_cast<size_t>(w->in_features / 16) * (w->out_features / 16) * w->n;
  if (exl3::launch_decode_dense(w->trellis + group * tw, w->in_features, w->out_features, w->n, out,
                                (flags & EXL3_MATMUL_DP4A) ? 0 : 1, static_cast<cudaStream_t>(stream),
                                exl3::window_mask(exl3::flags_window_bits(w->flags)),
                                (w->flags & EXL3_WEIGHT_MCG) ? 1 : 0) != cudaSuccess)
    return refuse(EXL3_FAILED, "exl3_b200: decode launch failed");
  return kOk;
}

exl3_verdict exl3_reconstruct_public(const exl3_weight* w, int32_t group, uint16_t* out, void* stream) {
  exl3_verdict v = check_weight(w);
  if (v.code != EXL3_OK) return v;
  if (group < 0 || group >= w->groups || !out) return refuse(EXL3_FAILED, "exl3_b200: bad arguments");
  if (w->nseg != 1) return refuse(EXL3_UNSUPPORTED, "exl3_b200: the dense effective W of one linear (not a stack)");
  DeviceGuard guard(w->device);
  const size_t tw = static_cast<size_t>(w->in_features / 16) * (w->out_features / 16) * w->n;
  if (exl3::launch_reconstruct_public(w->trellis + group * tw, w->suh + static_cast<size_t>(group) * w->in_features,
                                      w->svh + static_cast<size_t>(group) * w->out_features, w->in_features,
                                      w->out_features, w->n, out, static_cast<cudaStream_t>(stream),
                                      exl3::window_mask(exl3::flags_window_bits(w->flags)),
                                      (w->flags & EXL3_WEIGHT_MCG) ? 1 : 0) != cudaSuccess)
    return refuse(EXL3_FAILED, "exl3_b200: reconstruct launch failed");
  return kOk;
}

exl3_verdict exl3_encode_trellis(const float* target, int32_t in_features, int32_t out_features, int32_t n,
                                 uint16_t* trellis, void* stream) {
  if (!target || !trellis) return refuse(EXL3_FAILED, "exl3_b200: bad arguments");
  exl3_verdict v = check_linear_shape(1, in_features, out_features, n);
  if (v.code != EXL3_OK) return v;
  if (n % 16 != 0) return refuse(EXL3_UNSUPPORTED, "exl3_b200: the encoder searches whole-bit trellises only");
  if (exl3::launch_encode(target, in_features, out_features, n, trellis, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return refuse(EXL3_FAILED, "exl3_b200: encoder launch failed");
  return kOk;
}

exl3_verdict exl3_resident(const exl3_weight* ws, int32_t count, uint64_t room, void* stream, uint64_t* bytes) {
  (void)stream;  // the memory is reserved here and filled by the first prefill call, on that call's stream
  std::lock_guard<std::mutex> lk(g_res_mu);
  uint64_t held = 0;
  if (count == 0) {
    for (auto& r : g_res) resident_free(*r);
    g_res.clear();
  } else {
    if (!ws || count < 0) return refuse(EXL3_FAILED, "exl3_b200: bad arguments");
    for (const auto& r : g_res) held += static_cast<uint64_t>(r->group_bytes) * r->groups;
    std::vector<const exl3_weight*> add;
    uint64_t more = 0;
    for (int i = 0; i < count; ++i) {
      const exl3_weight* w = &ws[i];
      exl3_verdict v = check_weight(w);
      if (v.code != EXL3_OK) return v;
      if ((w->flags & EXL3_WEIGHT_BANK) && !(w->flags & EXL3_WEIGHT_GROUPED))
        return refuse(EXL3_UNSUPPORTED, "exl3_b200: routed banks are not kept (their calls are decode GEMVs)");
      bool kept = false;
      for (const auto& r : g_res) kept = kept || resident_is(*r, w);
      for (const exl3_weight* a : add) kept = kept || (a->device == w->device && a->trellis == w->trellis);
      if (kept) continue;
      add.push_back(w);
      more += static_cast<uint64_t>(resident_group_bytes(w)) * w->groups;
    }
    if (room > 0 && held + more > room) return refuse(EXL3_TOO_LARGE, "exl3_b200: the kept matrices pass the room");
    std::vector<std::unique_ptr<Resident>> made;
    for (const exl3_weight* w : add) {
      auto r = std::make_unique<Resident>();
      *r = Resident{w->device, w->trellis, w->suh, w->svh, w->groups, w->in_features, w->out_features, w->n, w->nseg,
                    resident_group_bytes(w), nullptr, false};
      DeviceGuard guard(w->device);
      if (cudaMalloc(&r->image, r->group_bytes * w->groups) != cudaSuccess) {
        for (auto& m : made) resident_free(*m);
        return refuse(EXL3_TOO_LARGE, "exl3_b200: out of device memory for the kept matrices");
      }
      made.push_back(std::move(r));
    }
    for (auto& r : made) g_res.push_back(std::move(r));
    held += more;
  }
  if (bytes) *bytes = held;
  return kOk;
}

uint64_t exl3_resident_pending(void) {
  std::lock_guard<std::mutex> lk(g_res_mu);
  uint64_t pending = 0;
  for (const auto& r : g_res)
    if (!r->filled) pending += static_cast<uint64_t>(r->group_bytes) * r->groups;
  return pending;
}

exl3_verdict exl3_device_error(int32_t device, uint32_t* bits, int32_t clear) {
  if (!bits || device < 0 || device >= kMaxDevices) return refuse(EXL3_FAILED, "exl3_b200: bad arguments");
  DeviceGuard guard(device);
  uint32_t* err = exl3::device_error_ptr();  // the word exists on every device, workspace or not
  if (!err) return refuse(EXL3_FAILED, "exl3_b200: no device error word on this device");
  if (cudaMemcpy(bits, err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return refuse(EXL3_FAILED, "exl3_b200: read failed");
  if (clear) {
    // a launch that gave up may have left block counters raised: reset them with the error word
    DeviceState* d = device_state(device);
    if (cudaMemset(err, 0, 4) != cudaSuccess ||
        (d && cudaMemset(d->counters, 0, kCounterCount * 4) != cudaSuccess) || cudaDeviceSynchronize() != cudaSuccess)
      return refuse(EXL3_FAILED, "exl3_b200: reset failed");
  }
  return kOk;
}

}  // extern "C"
