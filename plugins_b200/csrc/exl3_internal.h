// exl3_internal.h -- launch parameter blocks shared by the kernels and the C-ABI layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <type_traits>

namespace exl3 {

// One kernel's launch setup, per device: dynamic shared memory above 48 KiB is opted into in each device's context,
// and the resident CTAs per SM it leaves are that device's.  Launchers keep one (a function-local static per kernel
// instantiation); the first launch on a device, or one needing more shared memory than any before it, takes the
// mutex, so concurrent first launches from several host threads set the attribute once and in order.
struct KernelSetup {
  static constexpr int kDevices = 64;
  std::atomic<int> smem[kDevices] = {};    // bytes opted into on the device (0: none yet)
  std::atomic<int> per_sm[kDevices] = {};  // resident CTAs per SM found at that opt-in (when asked for)
  std::mutex mu;
};

// Opts `kern` into `smem` bytes (and, with `cluster`, non-portable cluster sizes) on the current device, once per
// device and size; with `per_sm` non-null, also returns the kernel's resident CTAs per SM there at `threads` threads,
// clamped to 1 .. cap (kernels whose shared memory does not vary from launch to launch).
template <typename Kern>
cudaError_t kernel_setup(KernelSetup& s, Kern kern, int threads, size_t smem, bool cluster = false,
                         int* per_sm = nullptr, int cap = 1) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= KernelSetup::kDevices) return cudaErrorInvalidDevice;
  const int bytes = static_cast<int>(smem);
  if (s.smem[dev].load(std::memory_order_acquire) < bytes || (per_sm && s.per_sm[dev].load(std::memory_order_acquire) == 0)) {
    std::lock_guard<std::mutex> lk(s.mu);
    if (s.smem[dev].load(std::memory_order_relaxed) < bytes || (per_sm && s.per_sm[dev].load(std::memory_order_relaxed) == 0)) {
      const int set = bytes > s.smem[dev].load(std::memory_order_relaxed) ? bytes : s.smem[dev].load(std::memory_order_relaxed);
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, set);
      if (e != cudaSuccess) return e;
      if (cluster) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
      }
      if (per_sm) {
        int occ = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
        if (e != cudaSuccess) return e;
        s.per_sm[dev].store(occ < 1 ? 1 : (occ > cap ? cap : occ), std::memory_order_release);
      }
      s.smem[dev].store(set, std::memory_order_release);
    }
  }
  if (per_sm) *per_sm = s.per_sm[dev].load(std::memory_order_acquire);
  return cudaSuccess;
}

// The rates the kernels serve: n halfwords per 256-weight tile, 16 x bits per weight, whole and half bits 1..6.
inline bool rate_served_n(int n) { return n % 8 == 0 && n >= 16 && n <= 96; }

// Calls f(std::integral_constant<int, N>{}) for the served rate n; false (nothing called) for any other n.
template <typename F>
inline bool with_rate(int n, F&& f) {
  switch (n) {
    case 16: f(std::integral_constant<int, 16>{}); return true;
    case 24: f(std::integral_constant<int, 24>{}); return true;
    case 32: f(std::integral_constant<int, 32>{}); return true;
    case 40: f(std::integral_constant<int, 40>{}); return true;
    case 48: f(std::integral_constant<int, 48>{}); return true;
    case 56: f(std::integral_constant<int, 56>{}); return true;
    case 64: f(std::integral_constant<int, 64>{}); return true;
    case 72: f(std::integral_constant<int, 72>{}); return true;
    case 80: f(std::integral_constant<int, 80>{}); return true;
    case 88: f(std::integral_constant<int, 88>{}); return true;
    case 96: f(std::integral_constant<int, 96>{}); return true;
    default: return false;
  }
}

// The codeword mask of a window of `bits` (8..16): 0 for the full 16-bit window (no masking instantiation).
inline uint32_t window_mask(int bits) { return bits >= 16 ? 0u : (1u << bits) - 1u; }
// A weight's window bits from its flags (bits 8..11 hold 16 - w: EXL3_WEIGHT_WINDOW in exl3_b200.h).
inline int flags_window_bits(uint32_t flags) { return 16 - static_cast<int>((flags >> 8) & 0xFu); }

// The decode spec of a weight: 0 mul1 at the full window, 1 mul1 at a narrowed window, 2 mcg.
inline int decode_spec(uint32_t cw_mask, bool mcg) { return mcg ? 2 : (cw_mask ? 1 : 0); }

// with_rate and the decode spec: f(N, DS) for the served rate n, DS = decode_spec(cw_mask, mcg).
template <typename F>
inline bool with_rate_decode(int n, uint32_t cw_mask, bool mcg, F&& f) {
  return with_rate(n, [&](auto N) {
    switch (decode_spec(cw_mask, mcg)) {
      case 0: f(N, std::integral_constant<int, 0>{}); break;
      case 1: f(N, std::integral_constant<int, 1>{}); break;
      default: f(N, std::integral_constant<int, 2>{}); break;
    }
  });
}
// The codeword mask a decode spec reads: the window's, or all 16 bits for mcg at the full window.
constexpr uint32_t spec_mask(uint32_t cw_mask) { return cw_mask ? cw_mask : 0xFFFFu; }

constexpr int kMaxSegments = 4;  // linears stacked into one launch (the reference's SHARED_MAX, linear.zig:39-40)
constexpr int kMaxRows = 16;     // decode-GEMV rows per launch (two m16n8k16 row groups)

constexpr int kGemvCtasPerSm = 3;  // the decode GEMV's persistent grid: CTAs per SM (fixed: rows and byte-sum path
                                   // do not change a row's sum order)

// Column-parallel exchange (exl3_tp.cu): this rank's view of every rank's exchange buffer.
constexpr int kMaxTpRanks = 8;
struct TpDev {
  uint8_t* y[kMaxTpRanks];      // rank q's gathered outputs: [2 parities][slots][slot_bytes]
  uint32_t* flag[kMaxTpRanks];  // rank q's done words: [world], the last step each rank published there
  uint32_t* step;               // this rank's step counter
  uint32_t* meta;               // this rank's slot metadata: [slots][4] (gathered column blocks, bytes)
  int32_t world, rank, slots, max_cb;
  int64_t slot_bytes;
  uint64_t* trace;              // the phase timeline ring, or null: 0 begin, 1 publish (the step's GEMVs done), 2 every
                                // rank's columns seen, 3 gather copied
};

struct GemvParams {
  const uint16_t* trellis;  // [in/16][out/16][n]
  const uint16_t* suh;      // [nseg][in] f16 bits (unused when prepared)
  const uint16_t* svh;      // [out] f16 bits
  const void* x;            // [rows_total][x_row_stride] activations of the whole call
  int32_t x_dtype;          // exl3::DType
  int64_t x_row_stride;     // elements
  void* y;                  // one segment: y[row][col] at row * y_row_stride; several: [rows_total][width_s] each,
  int32_t y_dtype;          //   segments back to back
  int64_t y_row_stride;     // elements (single segment)
  int32_t row0, rows_total; // this launch's first row, and all rows of the call
  float* partials;          // split partials, [pair][contributor][rows][128]
  uint32_t* counters;       // [out/128], zero between launches
  uint32_t* err;            // device error word
  int32_t in_features, out_features, rows, nseg;
  int32_t seg_cb[kMaxSegments + 1];  // segment bounds in 128-column blocks
  int32_t prepared;         // x already holds f16(H(x*suh)/sqrt(128)): no rotation
  int32_t inner_only;       // skip the output Hadamard and svh: y = the f32 inner product
  const void* xf;           // cluster-split GEMV: x already rotated into fragment order by launch_gemv_prep
                            //   ([nseg][in/16][row groups][128 halfs]), or null: each CTA rotates its slabs itself
  uint32_t cw_mask;         // a narrowed codeword window's mask (window_mask), 0 for the full 16-bit window
  int32_t mcg;              // the mcg codebook (else mul1)
  // geometry (gemv_geometry)
  int32_t kt, kr, kc;       // 16-row slabs, slabs per chunk, chunks
  int32_t contrib_max;      // most CTAs contributing to one (segment, chunk, column block)
  int64_t xp_bytes;         // shared memory for the rotated activations a share touches
  int32_t grid;
  int32_t stages;           // cluster-split GEMV: units in flight per warp
  // column-parallel exchange (cluster-split GEMV only): y goes to every rank's slot instead of p.y
  const TpDev* tp;          // device pointer, null without exchange
  int32_t tp_slot;
  int64_t tp_total[kMaxSegments];    // per segment: the gathered width
  int64_t tp_col0[kMaxSegments];     // per segment: this rank's first column in it
  int64_t tp_seg_base[kMaxSegments]; // per segment: first element of its [rows][width] block in the slot
  int32_t tp_cb_base[kMaxSegments];  // per segment: first gathered column block
  uint32_t tp_meta_cb, tp_meta_bytes; // the slot's gathered column blocks and bytes (for the gather)
};

// The exchange handle's fields the launch needs (exl3_tp.cu).
}  // namespace exl3
struct exl3_tp;
namespace exl3 {
const TpDev* tp_device(const exl3_tp* tp);
int tp_device_index(const exl3_tp* tp);
int tp_max_cb(const exl3_tp* tp);
int tp_slots(const exl3_tp* tp);
int64_t tp_slot_bytes(const exl3_tp* tp);

// Fills the geometry fields of `p` for `sms` SMs; false (with a reason) when the shape does not fit one launch.
bool gemv_geometry(GemvParams& p, int sms, int row_groups, size_t partial_capacity_floats, const char** why);
cudaError_t launch_gemv(const GemvParams& p, int n, int row_groups, bool imma, cudaStream_t st, bool pdl);

// The persistent work-balanced decode GEMV (exl3_gemv6.cu), 1..16 rows, no column-parallel exchange: a prepare
// launch (x rotated into fragment order in `scratch`) and the GEMV (runs' partials in `scratch` after the prepared x;
// `counters` [out/128] zero between launches, each reset by the run that uses it).  Preferred (measured faster than
// the cluster split at 1, 2, 8 and 16 rows) from kGemv6MinSlabs 16-row slabs of 128 columns per launch, for inputs of
// 8192 and more from kGemv6MinSlabsDeep (where the cluster split needs 12-16 CTAs per cluster), and for narrow
// outputs -- at most kGemv6NarrowCb column blocks -- from kGemv6NarrowSlabs (config 2's o and q|k|v: 11.6 / 11.8 us
// against 11.9 / 12.8 at one row, 15.1 / 15.3 against 17.8 / 17.9 at eight); in between (config 2's 4096 x 12288:
// 17.5 against 19.2 us) the cluster split wins.
constexpr int64_t kGemv6MinSlabs = 49152;
constexpr int64_t kGemv6MinSlabsDeep = 16384;
constexpr int kGemv6NarrowCb = 64;
constexpr int64_t kGemv6NarrowSlabs = 8192;
bool gemv6_prefers(const GemvParams& p);
// x of the launch's rows rotated once into the GEMVs' fragment order (IMMA k order) at xf: [nseg][in/16][row_groups]
// [128 halfs], rows past the launch's zero; chained to the next launch with programmatic dependent launch.
size_t gemv_prep_bytes(const GemvParams& p, int row_groups);
cudaError_t launch_gemv_prep(const GemvParams& p, int row_groups, void* xf, cudaStream_t st);
size_t gemv6_scratch_bytes(const GemvParams& p, int sms);
cudaError_t launch_gemv6(const GemvParams& p, int n, int sms, void* scratch, uint32_t* counters, cudaStream_t st);

// The cluster-split decode GEMV (exl3_gemv5.cu): one thread-block cluster per 128-column block, its CTAs splitting
// the input (kc = CTAs per cluster, kr = slabs per CTA), partials summed over distributed shared memory.
// split_override > 0 forces the CTAs per cluster (measurement); false when no split fits.
bool gemv5_geometry(GemvParams& p, int n, int sms, int row_groups, int split_override, const char** why);
cudaError_t launch_gemv5(const GemvParams& p, int n, int row_groups, bool imma, cudaStream_t st, bool pdl);

// decode a whole trellis to W_hat (f16 bits, row-major [in][out]); one warp per tile
cudaError_t launch_decode_dense(const uint16_t* trellis, int in_features, int out_features, int n, uint16_t* out,
                                int imma, cudaStream_t st, uint32_t cw_mask = 0, int mcg = 0);

// the dense effective W (f16 bits, row-major [in][out]) of one group: svh * H (suh * H W_hat), per 128 x 128 block
cudaError_t launch_reconstruct_public(const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh,
                                      int in_features, int out_features, int n, uint16_t* out, cudaStream_t st,
                                      uint32_t cw_mask = 0, int mcg = 0);

// trellis encoder (exl3_encode.cu): target [in][out] f32 (rotated, unit variance) -> trellis [in/16][out/16][n]
cudaError_t launch_encode(const float* target, int in_features, int out_features, int n, uint16_t* trellis,
                          cudaStream_t st);

// ---------------------------------------------------------------- prefill GEMM (exl3_gemm.cu)

constexpr int kGemmMinRows = 64;  // rows from which matmul takes the tensor-core GEMM instead of the decode GEMV

struct GemmParams {
  const uint8_t* a_img;  // [tiles_m * BM / 128][kb] image blocks of xp
  const uint8_t* b_img;  // [tiles_n * BN / 128][kb] image blocks of W_hat^T
  const uint16_t* svh;   // [tiles_n * BN] f16 bits, this launch's columns
  void* y;               // y[row * y_row_stride + col], col relative to this launch's first column
  int32_t y_dtype;
  int64_t y_row_stride;
  int32_t m;             // valid rows
  int32_t ncols;         // valid columns (tiles past them are computed but not stored)
  int32_t tiles_m, tiles_n, kb;  // kb = in_features / 64
  int32_t inner_only;    // y = the f32 inner product (no output Hadamard, no svh)
  int32_t vec_store;     // y and y_row_stride allow 16-byte (1) or 32-byte (2) stores
  uint32_t* err;
  // grouped (the routed experts' prefill, 128-row blocks only): the blocks [mt_range[0], mt_range[1]) of the padded
  // rows (device words; null: blocks 0 .. tiles_m), block b's expert m_group[b]; expert e's B image at
  // b_img + (e - group0) * b_group_bytes, its svh at svh + e * svh_group (svh2 + e * svh_group - svh_split for the
  // columns from svh_split on: a stacked gate|up)
  const int32_t* mt_range;
  const int32_t* m_group;
  int32_t group0;
  int64_t b_group_bytes;
  int64_t svh_group;
  const uint16_t* svh2;
  int32_t svh_split;
  // the decode-in-the-GEMM form (launch_gemm_fused; b_img unused): W_hat^T blocks decoded from the trellis into shared
  // memory at every k-step; the launch's columns start at tile column tn0 of a weight of out_tiles tile columns and n
  // halfwords per tile; grouped, block b's expert e = m_group[b] has its trellis at trellis + (e - group0) * tr_group
  const uint16_t* trellis;
  int64_t tr_group;
  int32_t out_tiles, tn0, n;
};

// One launch writes the A image of xp rows [0, mp) (rows >= m are zeros; prepared = x already holds xp; skipped when
// a_img is null) and the B image of the trellis columns [col0, col0 + ncols) (skipped when b_img is null).
cudaError_t launch_images(const void* x, int32_t x_dtype, int64_t x_row_stride, int m, int mp, const uint16_t* suh,
                          int prepared, uint8_t* a_img, const uint16_t* trellis, int in_features, int out_features,
                          int col0, int ncols, int n, uint8_t* b_img, cudaStream_t st, uint32_t cw_mask = 0,
                          int mcg = 0);
// The routed experts' prefill (exl3_moe_prefill.cu): operand images of rows sorted by expert, each expert's rows
// padded to whole 128-row blocks (row_slot[row] = token * topk + k, -1 for padding; m_group[row / 128] = expert).
struct MoeImages {
  const int32_t* row_slot;
  const int32_t* m_group;
  const int32_t* rows_total;  // device: the call's padded rows (A images)
  const int32_t* row_range;   // device: {first row, end row} (the down input's A image)
  int32_t topk;
  const void* x;
  int32_t x_dtype;
  int32_t x_vec;  // x's rows take vector loads: 4 elements and 16 bytes aligned (row strides are multiples of 128)
  int64_t x_row_stride;
  int32_t hidden, inter;
  const uint16_t *suh_g, *suh_u, *suh_d;  // [E][hidden], [E][hidden], [E][inter]
  uint8_t *a_g, *a_u, *a_d;               // A images: [rows / 128][hidden / 64] (gate, up), [rows / 128][inter / 64]
  const float* gu;                         // the gate|up GEMMs' outputs, [rows][gu_stride] f32
  int64_t gu_stride;
  float limit;
};
cudaError_t launch_moe_a_images(const MoeImages& j, int sms, cudaStream_t st);
cudaError_t launch_moe_mid_images(const MoeImages& j, int sms, cudaStream_t st);
// B images (W_hat^T) of the bank's experts e0 .. e0 + count - 1 (experts with counts[e] == 0 skipped), expert e at
// b_img + (e - e0) * b_group_bytes.
cudaError_t launch_moe_b_images(const uint16_t* trellis, int in_features, int out_features, int n, int e0, int count,
                                const int32_t* counts, uint8_t* b_img, int64_t b_group_bytes, cudaStream_t st,
                                uint32_t cw_mask = 0, int mcg = 0);

// shape: 0 = 128x128 tiles, 1 = 128x256, 2 = 256x128, 3 = 256x256 (rows x columns)
// GemmParams::vec_store for output rows at y, row_bytes apart: 2 = 32-byte stores, 1 = 16-byte, 0 = element stores
inline int32_t store_width(const void* y, int64_t row_bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(y);
  if (a % 32 == 0 && row_bytes % 32 == 0) return 2;
  return (a % 16 == 0 && row_bytes % 16 == 0) ? 1 : 0;
}
int gemm_block_m(int shape);
int gemm_block_n(int shape);
cudaError_t launch_gemm_image(const GemmParams& p, int shape, int sms, cudaStream_t st);
// The same GEMM with W_hat^T decoded inside it (exl3_gemm_fused.cu): eight decode warps fill each k-step's B block in
// shared memory from the trellis, so no B image is written or read.  Shapes 0..3 as above (256-row blocks for the
// dense launch only), the full 16-bit mul1 window only.
cudaError_t launch_gemm_fused(const GemmParams& p, int shape, int sms, cudaStream_t st);

// the device error word of the current device (exl3_device_error reads it), or null
uint32_t* device_error_ptr();

// A launch that may begin while the previous kernel in the stream finishes (programmatic dependent launch): the
// kernel calls pdl_wait() before it touches anything an earlier launch in the stream wrote or reads.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_k(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// An exchange's phase timeline: with EXL3_TRACE=1 in the environment when the exchange is created, its kernels write
// %globaltimer stamps (ns) into a device ring of kTraceStamps per step for the last kTraceSteps steps (a null ring
// records nothing).  trace_alloc: that ring (zeroed) on the current device, or null without EXL3_TRACE=1; trace_copy
// waits for the device and writes the ring to out oldest step first, given the exchange's step word (the step of the
// newest stamps).
constexpr int kTraceSteps = 16, kTraceStamps = 8;
uint64_t* trace_alloc();
bool trace_copy(const uint64_t* ring, const uint32_t* step_word, uint64_t* out);

#if defined(__CUDACC__)
__device__ __forceinline__ uint64_t trace_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// one thread's stamp
__device__ __forceinline__ void trace_at(uint64_t* ring, uint32_t step, int i) {
  if (ring) ring[(step % kTraceSteps) * kTraceStamps + i] = trace_now();
}
// every CTA of a launch as it leaves: the latest is kept
__device__ __forceinline__ void trace_last(uint64_t* ring, uint32_t step, int i) {
  if (ring)
    atomicMax(reinterpret_cast<unsigned long long*>(ring) + (step % kTraceSteps) * kTraceStamps + i,
              static_cast<unsigned long long>(trace_now()));
}
#endif


}  // namespace exl3
