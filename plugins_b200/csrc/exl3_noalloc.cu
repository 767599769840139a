// exl3_noalloc.cu -- exl3_matmul_noalloc: the decode GEMV for callers that cannot allocate device memory.
//
// Some hosts cannot let a library call cudaMalloc: a serving process that reserves its device memory up front and
// admits nothing beyond what it billed (the plugin seam bills a pack as its stored bytes), or an embedding runtime
// whose allocator owns every device byte.  exl3_matmul needs a per-device workspace, which the library allocates the
// first time a weight is registered.  This entry point runs the same kernel with its scratch (the split partials,
// the per-column-block counters and an error word) in one static device array instead, so the caller passes the
// weight, the input and the output and nothing is allocated -- no cudaMalloc, no cudaFree, no allocating library.
// The kernel is the grid-stride decode GEMV (exl3_gemv.cu): the same decode and the same f32 accumulation as
// exl3_matmul, within its 2e-3 rel-L2 bar of the f32 truth, but not bit-identical to it (exl3_matmul picks other
// kernels by shape, and their sums run in another order).  Kernel errors land in the device error word that
// exl3_device_error reads and clears.
//
// Limits and rules:
//   * the static array holds 8 MiB of split partials and 8192 counters; a call whose layer needs more partials
//     (large in_features x out_features at many rows) is refused with EXL3_TOO_LARGE before any launch;
//   * every device that loads the library holds the array (about 8 MiB) until the process exits;
//   * the first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device
//     current) and clears the counters with a memset on the caller's stream; make that first call before any
//     stream capture;
//   * all calls share the array and it keeps the last call's contents: the kernel returns every counter it raised
//     to zero, and calls that overlap on the GPU (concurrent streams, or two devices' calls racing through one
//     device) race on it -- order them on one stream.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "../../include/exl3_b200.h"
#include "exl3_internal.h"

namespace {

constexpr size_t kPartialFloats = size_t(2) << 20;  // 8 MiB of split partials
constexpr size_t kCounters = 8192;                   // column blocks (out_features <= 1,048,576)
constexpr size_t kScratchWords = kPartialFloats + kCounters;

// The scratch.  In host code this name is only a stand-in for the device array: its device address comes from
// cudaGetSymbolAddress, per device.
static __device__ __align__(256) uint32_t g_noalloc_scratch[kScratchWords];

struct Scratch {
  bool ready = false;
  float* partials = nullptr;
  uint32_t* counters = nullptr;
  uint32_t* err = nullptr;  // the library's device error word (exl3_device_error), not part of the array
  int sms = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_mu;
Scratch g_scratch[kMaxDevices];

exl3_verdict refuse(int32_t code, const char* why) { return {code, why}; }

// Once per device, with that device current: the array's device address, the SM count, the counters zeroed on the
// caller's stream.
exl3_verdict scratch_for(int dev, cudaStream_t st, Scratch** out) {
  if (dev < 0 || dev >= kMaxDevices) return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  Scratch& s = g_scratch[dev];
  if (!s.ready) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10)
      return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: the kernels are built for sm_100a (B200) only");
    if (cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return refuse(EXL3_FAILED, "exl3_matmul_noalloc: no SM count");
    void* base = nullptr;
    if (cudaGetSymbolAddress(&base, g_noalloc_scratch) != cudaSuccess || base == nullptr)
      return refuse(EXL3_FAILED, "exl3_matmul_noalloc: cudaGetSymbolAddress of the static scratch failed");
    uint32_t* words = static_cast<uint32_t*>(base);
    s.partials = reinterpret_cast<float*>(words);
    s.counters = words + kPartialFloats;
    s.err = exl3::device_error_ptr();
    if (s.err == nullptr) return refuse(EXL3_FAILED, "exl3_matmul_noalloc: no device error word");
    if (cudaMemsetAsync(s.counters, 0, kCounters * sizeof(uint32_t), st) != cudaSuccess)
      return refuse(EXL3_FAILED, "exl3_matmul_noalloc: clearing the static scratch failed");
    s.ready = true;
  }
  *out = &s;
  return {EXL3_OK, nullptr};
}

int64_t numel(const exl3_tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

}  // namespace

extern "C" exl3_verdict exl3_matmul_noalloc(const exl3_weight* w, const exl3_tensor* x, void* stream,
                                            exl3_tensor* out) {
  if (!w || w->size != sizeof(exl3_weight) || !w->trellis || !w->suh || !w->svh)
    return refuse(EXL3_FAILED, "exl3_matmul_noalloc: not a weight");
  if (w->groups != 1 || w->nseg < 1 || w->nseg > EXL3_MAX_SEGMENTS || (w->flags & EXL3_WEIGHT_GROUPED))
    return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: one ungrouped weight (stacked segments allowed)");
  const int in_f = w->in_features, out_f = w->out_features, n = w->n;
  if (in_f <= 0 || out_f <= 0 || in_f % 128 != 0 || out_f % 128 != 0)
    return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: in and out features must be multiples of 128");
  if (w->flags & (EXL3_WEIGHT_WINDOW_MASK | EXL3_WEIGHT_MCG))
    return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: narrowed codeword windows and mcg take exl3_matmul");
  if (!exl3::rate_served_n(n))
    return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: rates off the half-bit grid or above 6 bits are not served");
  // stacked segments: bounds from 0 to out_features, each a multiple of 128 and above the one before (a weight
  // struct filled by hand is checked here; the launch geometry divides by each segment's width)
  if (w->seg_cols[0] != 0 || w->seg_cols[w->nseg] != out_f)
    return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: seg_cols must run from 0 to out_features");
  for (int s = 0; s < w->nseg; ++s)
    if (w->seg_cols[s + 1] <= w->seg_cols[s] || w->seg_cols[s + 1] % 128 != 0)
      return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: seg_cols must rise in steps of whole 128-column blocks");
  if (out_f / 128 > static_cast<int>(kCounters))
    return refuse(EXL3_TOO_LARGE, "exl3_matmul_noalloc: out_features beyond the static scratch's 8192 column blocks");
  if ((reinterpret_cast<uintptr_t>(w->trellis) & 15u) != 0)
    return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: the trellis must be 16-byte aligned");
  if (!x || !out || x->ndim < 1 || x->ndim > 4 || out->ndim != x->ndim)
    return refuse(EXL3_FAILED, "exl3_matmul_noalloc: bad tensors");
  if (x->dtype != EXL3_F16 && x->dtype != EXL3_BF16 && x->dtype != EXL3_F32)
    return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: activations must be f16, bf16 or f32");
  if (x->shape[x->ndim - 1] != in_f || out->shape[out->ndim - 1] != out_f || out->dtype != x->dtype)
    return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: x [..., in] -> out [..., out] in x's dtype");
  for (int i = 0; i < x->ndim - 1; ++i)
    if (out->shape[i] != x->shape[i]) return refuse(EXL3_UNSUPPORTED, "exl3_matmul_noalloc: the output has the wrong shape");
  const int64_t rows = numel(x) / in_f;
  if (rows > (int64_t{1} << 24)) return refuse(EXL3_TOO_LARGE, "exl3_matmul_noalloc: more than 2^24 rows");
  if (rows == 0) return {EXL3_OK, nullptr};
  if (!x->data || !out->data) return refuse(EXL3_FAILED, "exl3_matmul_noalloc: bad tensors");

  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != w->device && cudaSetDevice(w->device) != cudaSuccess)
    return refuse(EXL3_FAILED, "exl3_matmul_noalloc: cannot select the weight's device");
  Scratch* sc = nullptr;
  exl3_verdict v = scratch_for(w->device, static_cast<cudaStream_t>(stream), &sc);
  for (int64_t r0 = 0; v.code == EXL3_OK && r0 < rows; r0 += exl3::kMaxRows) {
    const int rc = static_cast<int>(rows - r0 < exl3::kMaxRows ? rows - r0 : exl3::kMaxRows);
    const int rg = rc <= 8 ? 1 : 2;
    exl3::GemvParams gp{};
    gp.trellis = w->trellis;
    gp.suh = w->suh;
    gp.svh = w->svh;
    gp.x = x->data;
    gp.x_dtype = x->dtype;
    gp.x_row_stride = in_f;
    gp.y = out->data;
    gp.y_dtype = out->dtype;
    gp.y_row_stride = out_f;
    gp.row0 = static_cast<int32_t>(r0);
    gp.rows_total = static_cast<int32_t>(rows);
    gp.partials = sc->partials;
    gp.counters = sc->counters;
    gp.err = sc->err;
    gp.in_features = in_f;
    gp.out_features = out_f;
    gp.rows = rc;
    gp.nseg = w->nseg;
    for (int s = 0; s <= w->nseg; ++s) gp.seg_cb[s] = w->seg_cols[s] / 128;
    for (int s = w->nseg + 1; s <= exl3::kMaxSegments; ++s) gp.seg_cb[s] = gp.seg_cb[w->nseg];
    const char* why = nullptr;
    if (!exl3::gemv_geometry(gp, sc->sms, rg, ~size_t(0), &why)) {
      v = refuse(EXL3_TOO_LARGE, why);
      break;
    }
    const size_t need = static_cast<size_t>(out_f / 128) * gp.kc * gp.contrib_max * static_cast<size_t>(rc) * 128;
    if (need > kPartialFloats) {
      v = refuse(EXL3_TOO_LARGE, "exl3_matmul_noalloc: the layer needs more split partials than the 8 MiB static scratch");
      break;
    }
    if (exl3::launch_gemv(gp, n, rg, true, static_cast<cudaStream_t>(stream), true) != cudaSuccess)
      v = refuse(EXL3_FAILED, "exl3_matmul_noalloc: GEMV launch failed");
  }
  if (prev >= 0 && prev != w->device) cudaSetDevice(prev);
  return v;
}
