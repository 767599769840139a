// exl3_gemv.cu -- the EXL3 decode GEMV for 1..16 rows (sm_100a).
//
// Computes, per the reference (plugins/sushi_ds41/src/sushi/exl3/project_rows.zig:170-308, the multi-row kernel,
// and expert_exl3.zig:490-566, the scalar definition):
//   xp = f16(H128(x * suh) / sqrt(128))            per 128-block of the input     (prep kernel)
//   inner[c] = sum_k xp[k] W_hat[k, c]             f32 accumulation                (stream-K kernel)
//   y = H128(inner) / sqrt(128) * svh              per 128-block of the output     (stream-K epilogue)
//
// Design (B200):
//  * persistent stream-K grid: (output 128-column block, k-row of 16) units are split evenly over SMs x occupancy
//    CTAs, so every shape fills all 148 SMs with equal work and no wave tail;
//  * each of a CTA's four warps prefetches its own units -- a unit's 8 tiles (16n bytes, contiguous in the pack
//    layout) and its activation fragments -- with 16-byte cp.async copies into a private 8-stage shared-memory ring;
//  * the warps decode each 16x16 tile in registers: lane t's eight windows ARE the m16n8k16 A fragment of
//    W^T, so a tile is one tensor-core MMA against the rows (B = x^T, 8 rows per MMA) with f32 accumulation;
//    the mul1 byte sums run either on dp4a or on the tensor pipe (u8 IMMA);
//  * block partials that a CTA does not own completely are summed by the last contributing CTA in CTA order
//    (deterministic), which also applies the output Hadamard and svh.
#include <cuda_runtime.h>

#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace exl3 {

#ifndef EXL3_GEMV_STAGES
#define EXL3_GEMV_STAGES 4
#endif
#ifndef EXL3_GEMV_WARPS
#define EXL3_GEMV_WARPS 4
#endif
#ifndef EXL3_GEMV_CTAS_PER_SM
#define EXL3_GEMV_CTAS_PER_SM 6  // the stream-K partition's CTAs per SM, the same for every instantiation
#endif
constexpr int kStages = EXL3_GEMV_STAGES;
constexpr int kConsumerWarps = EXL3_GEMV_WARPS;
constexpr int kThreads = kConsumerWarps * 32;
constexpr int kRedStride = 132;  // floats per row of the reduction buffer (conflict-free fragment stores)

// ------------------------------------------------------------------ prep: activations -> fragment-major f16

// xpf layout: [seg][KT][RG][32 lanes][4 halves]; lane (g, q) of row-group rg holds row 8 rg + g at
//   IMMA order : k = 4q + e
//   dp4a order : k = 2q + (e & 1) + 8 (e >> 1)
__global__ void __launch_bounds__(128) prep_kernel(PrepParams p) {
  pdl_wait();  // xpf may still be read by the previous GEMV on this stream
  pdl_launch_dependents();
  const uint32_t lane = threadIdx.x & 31u;
  const int blk = blockIdx.x * 4 + (threadIdx.x >> 5);  // 128-block of the input
  const int row = blockIdx.y;                          // 0 .. RG*8-1
  const int seg = blockIdx.z;
  if (blk * 128 >= p.in_features) return;
  float v[4];
  if (row < p.rows) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const size_t k = static_cast<size_t>(blk) * 128 + lane + 32 * i;
      const float xv = load_act(p.x, static_cast<size_t>(row) * p.x_row_stride + k, p.x_dtype);
      v[i] = p.prepared ? xv : xv * f16_bits_to_float(p.suh[static_cast<size_t>(seg) * p.in_features + k]);
    }
    if (!p.prepared) {
      fwht128_warp(v, lane);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] *= kHadScale;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = 0.0f;
  }
  const int kt_total = p.in_features / 16;
  const int rg = row >> 3, g = row & 7;
  __half* out = reinterpret_cast<__half*>(p.xpf);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = blk * 128 + lane + 32 * i;
    const int tk = k >> 4, kk = k & 15;
    int q, e;
    if (p.imma_order) {
      q = kk >> 2;
      e = kk & 3;
    } else {
      q = (kk & 7) >> 1;
      e = (kk & 1) | ((kk >> 3) << 1);
    }
    const size_t at = ((static_cast<size_t>(seg) * kt_total + tk) * p.row_groups + rg) * 128 + (g * 4 + q) * 4 + e;
    out[at] = __float2half_rn(v[i]);
  }
}

// ------------------------------------------------------------------ the stream-K decode GEMV

struct Partition {
  uint64_t U, G;
  __device__ __forceinline__ uint32_t start(uint32_t c) const { return static_cast<uint32_t>(U * c / G); }
  // the CTA whose range holds unit u
  __device__ __forceinline__ uint32_t owner(uint32_t u) const {
    return static_cast<uint32_t>(((static_cast<uint64_t>(u) + 1) * G + U - 1) / U) - 1u;
  }
};

// Segment lookups with static indexing only (dynamic indexing of the parameter block would spill it to the stack).
__device__ __forceinline__ int seg_of(const GemvParams& p, int cb) {
  int seg = 0;
#pragma unroll
  for (int t = 1; t < kMaxSegments; ++t)
    if (t < p.nseg && cb >= p.seg_cb[t]) seg = t;
  return seg;
}
__device__ __forceinline__ int seg_bound(const GemvParams& p, int s) {
  int v = p.seg_cb[0];
#pragma unroll
  for (int t = 1; t <= kMaxSegments; ++t)
    if (t == s) v = p.seg_cb[t];
  return v;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int K, int RG, bool IMMA>
__global__ void __launch_bounds__(kThreads, RG == 1 ? EXL3_GEMV_CTAS_PER_SM : EXL3_GEMV_CTAS_PER_SM / 2) gemv_kernel(GemvParams p) {
  constexpr uint32_t kTileBytes = 32u * K;            // 2n bytes, n = 16K
  constexpr uint32_t kUnitTrellis = 8u * kTileBytes;  // 8 tiles: one 128-column block, one 16-row k slab
  constexpr uint32_t kUnitX = RG * 256u;
  constexpr uint32_t kUnitBytes = kUnitTrellis + kUnitX;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  const int kRB = p.rows;  // rows of the reduction buffer (the launch's rows; MMA rows beyond them are padding)
  uint8_t* ring = smem + warp * (kStages * kUnitBytes);  // this warp's private ring
  float* red = reinterpret_cast<float*>(smem + kConsumerWarps * kStages * kUnitBytes);  // [W][rows][kRedStride]
  volatile int* s_flags = reinterpret_cast<volatile int*>(red + kConsumerWarps * kRB * kRedStride);

  const int KT = p.in_features / 16;
  const int CB = p.out_features / 128;
  const Partition part{static_cast<uint64_t>(CB) * KT, gridDim.x};
  const uint32_t c = blockIdx.x;
  const uint32_t u0 = part.start(c), u1 = part.start(c + 1);
  const uint32_t nunits = u1 - u0;
  // this warp's units: u0 + warp + W i
  constexpr uint32_t W = kConsumerWarps;
  const uint32_t mine = nunits > warp ? (nunits - warp + W - 1u) / W : 0u;
  const uint8_t* trellis = reinterpret_cast<const uint8_t*>(p.trellis);

  auto unit_of = [&](uint32_t i) { return u0 + warp + W * i; };
  auto issue_trellis = [&](uint32_t i) {
    if (i >= mine) return;
    const uint32_t u = unit_of(i), cb = u / KT, tk = u % KT;
    const uint8_t* src = trellis + (static_cast<size_t>(tk) * (CB * 8) + cb * 8u) * kTileBytes;
    uint8_t* dst = ring + (i % kStages) * kUnitBytes;
#pragma unroll
    for (uint32_t ch = lane; ch < kUnitTrellis / 16u; ch += 32u) cp_async16(dst + ch * 16u, src + ch * 16u);
  };
  auto issue_x = [&](uint32_t i) {
    if (i >= mine) return;
    const uint32_t u = unit_of(i), cb = u / KT, tk = u % KT;
    const int seg = seg_of(p, static_cast<int>(cb));
    const uint8_t* src = p.xpf + (static_cast<size_t>(seg) * KT + tk) * kUnitX;
    uint8_t* dst = ring + (i % kStages) * kUnitBytes + kUnitTrellis;
#pragma unroll
    for (uint32_t ch = lane; ch < kUnitX / 16u; ch += 32u) cp_async16(dst + ch * 16u, src + ch * 16u);
  };

  pdl_launch_dependents();  // the next launch on this stream may be scheduled now; it waits for this grid to finish
  // prologue: weights first (they do not depend on the prep kernel), one group; then the activations, one group
  // per unit.  Group i+1 then always holds unit i, so every wait is cp.async.wait_group(kStages - 2).
  for (uint32_t i = 0; i + 1 < static_cast<uint32_t>(kStages); ++i) issue_trellis(i);
  cp_async_commit();
  pdl_wait();
  for (uint32_t i = 0; i + 1 < static_cast<uint32_t>(kStages); ++i) {
    issue_x(i);
    cp_async_commit();
  }

  LaneWindows<K> lw;
  lw.init(lane);
  ImmaIndicator ind;
  ind.init(lane);
  const uint32_t g = lane >> 2, q = lane & 3u;
  if (tid == 0) s_flags[1] = 0;

  uint32_t i = 0;  // this warp's next unit
  const uint32_t cb_first = u0 / KT;
  const uint32_t cb_last = nunits ? (u1 - 1u) / KT : cb_first - 1u;
  for (uint32_t cb = cb_first; nunits && cb <= cb_last; ++cb) {
    const uint32_t blk0 = cb * KT, blk1 = blk0 + KT;
    const uint32_t ua = u0 > blk0 ? u0 : blk0;
    const uint32_t ub = u1 < blk1 ? u1 : blk1;
    float acc[8][RG][4];
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int r = 0; r < RG; ++r)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][r][e] = 0.0f;

    for (; i < mine && unit_of(i) < ub; ++i) {
      cp_async_wait<kStages - 2>();
      __syncwarp();
      const uint8_t* st = ring + (i % kStages) * kUnitBytes;
      const uint32_t* tw = reinterpret_cast<const uint32_t*>(st);
      const uint2* xf = reinterpret_cast<const uint2*>(st + kUnitTrellis);
      uint32_t b0[RG], b1[RG];
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const uint2 xv = xf[r * 32 + lane];
        b0[r] = xv.x;
        b1[r] = xv.y;
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        uint32_t w[8], a[4];
        lane_codewords<K>(tw + t * (8u * K), lw, w);
        if constexpr (IMMA) decode_afrag_imma(w, ind, a);
        else decode_afrag_dp4a(w, a);
#pragma unroll
        for (int r = 0; r < RG; ++r) mma_16816(acc[t][r], a, b0[r], b1[r]);
      }
      __syncwarp();
      // refill the stage read in the previous iteration with unit i + kStages - 1
      issue_trellis(i + kStages - 1);
      issue_x(i + kStages - 1);
      cp_async_commit();
    }

    // warp partial -> shared: D[col 16t + g (+8)][row 2q + {0,1} + 8r]
    float* rw = red + warp * kRB * kRedStride;
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const int col = 16 * t + g, row = 8 * r + 2 * q;
        if (row < kRB) {
          rw[row * kRedStride + col] = acc[t][r][0];
          rw[row * kRedStride + col + 8] = acc[t][r][2];
        }
        if (row + 1 < kRB) {
          rw[(row + 1) * kRedStride + col] = acc[t][r][1];
          rw[(row + 1) * kRedStride + col + 8] = acc[t][r][3];
        }
      }
    named_barrier_sync(1, kConsumerWarps * 32);

    // sum the warps (fixed order) into warp 0's slab
    const int rows = p.rows;
    for (int idx = tid; idx < rows * 128; idx += kConsumerWarps * 32) {
      const int row = idx >> 7, col = idx & 127;
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) v += red[(w * kRB + row) * kRedStride + col];
      red[row * kRedStride + col] = v;
    }
    named_barrier_sync(1, kConsumerWarps * 32);

    const bool full_block = (ua == blk0 && ub == blk1);
    bool finish = full_block;
    if (!full_block) {
      const uint32_t slot = (cb == cb_first) ? 0u : 1u;
      float* out = p.partials + (static_cast<size_t>(c) * 2 + slot) * 16 * 128;
      for (int idx = tid; idx < rows * 128; idx += kConsumerWarps * 32) {
        const int row = idx >> 7, col = idx & 127;
        out[row * 128 + col] = red[row * kRedStride + col];
      }
      __threadfence();
      named_barrier_sync(1, kConsumerWarps * 32);
      const uint32_t cfirst = part.owner(blk0), clast = part.owner(blk1 - 1u);
      if (tid == 0) {
        const uint32_t old = atomicAdd(&p.counters[cb], 1u);
        s_flags[1] = (old == clast - cfirst) ? 1 : 0;
      }
      named_barrier_sync(1, kConsumerWarps * 32);
      finish = s_flags[1] != 0;
      if (finish) {
        __threadfence();
        for (int idx = tid; idx < rows * 128; idx += kConsumerWarps * 32) {
          const int row = idx >> 7, col = idx & 127;
          float v = 0.0f;
          for (uint32_t cc = cfirst; cc <= clast; ++cc) {
            const uint32_t sl = (part.start(cc) / KT == cb) ? 0u : 1u;
            v += __ldcg(p.partials + (static_cast<size_t>(cc) * 2 + sl) * 16 * 128 + row * 128 + col);
          }
          red[row * kRedStride + col] = v;
        }
        if (tid == 0) p.counters[cb] = 0u;  // ready for the next launch
        named_barrier_sync(1, kConsumerWarps * 32);
      }
    }
    if (finish) {
      // output Hadamard + svh (or the raw inner product), one warp per row
      const int seg = seg_of(p, static_cast<int>(cb));
      const int seg_c0 = seg_bound(p, seg) * 128;
      const int seg_w = seg_bound(p, seg + 1) * 128 - seg_c0;
      for (int row = warp; row < rows; row += kConsumerWarps) {
        const size_t grow = static_cast<size_t>(p.row0 + row);
        const size_t ybase = p.nseg == 1 ? grow * p.y_row_stride
                                         : static_cast<size_t>(p.rows_total) * seg_c0 + grow * seg_w - seg_c0;
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = red[row * kRedStride + lane + 32 * k];
        if (!p.inner_only) {
          fwht128_warp(v, lane);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            v[k] = v[k] * kHadScale * f16_bits_to_float(p.svh[cb * 128 + lane + 32 * k]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) store_act(p.y, ybase + cb * 128 + lane + 32 * k, v[k], p.y_dtype);
      }
    }
    named_barrier_sync(1, kConsumerWarps * 32);
  }
  cp_async_wait<0>();  // no copy outlives the CTA
}

// ------------------------------------------------------------------ host launch

template <int K, int RG, bool IMMA>
static size_t gemv_smem_bytes(int rows) {
  constexpr size_t unit = 8u * 32u * K + RG * 256u;
  return kConsumerWarps * kStages * unit + static_cast<size_t>(kConsumerWarps) * rows * kRedStride * 4 + 16;
}

template <int K, int RG, bool IMMA>
static bool gemv_prepare() {
  static int ready = 0;  // per instantiation
  if (!ready) {
    auto kern = gemv_kernel<K, RG, IMMA>;
    const size_t smem = gemv_smem_bytes<K, RG, IMMA>(RG * 8);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
      return false;
    ready = 1;
  }
  return true;
}

// The stream-K partition uses EXL3_GEMV_CTAS_PER_SM CTAs per SM for every instantiation, so a row's f32 sum order
// (and so its bytes) does not depend on how many rows share the launch or which byte-sum path runs; an
// instantiation that fits fewer CTAs per SM runs the equal shares in waves.
template <int K, int RG, bool IMMA>
static cudaError_t launch_gemv_t(const GemvParams& p0, int sms, cudaStream_t st, bool pdl) {
  auto kern = gemv_kernel<K, RG, IMMA>;
  if (!gemv_prepare<K, RG, IMMA>()) return cudaErrorInvalidConfiguration;
  GemvParams p = p0;
  const uint64_t U = static_cast<uint64_t>(p.out_features / 128) * (p.in_features / 16);
  uint64_t G = static_cast<uint64_t>(sms) * EXL3_GEMV_CTAS_PER_SM;
  if (G > static_cast<uint64_t>(p.max_ctas)) G = p.max_ctas;
  if (G > U) G = U;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(G));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = gemv_smem_bytes<K, RG, IMMA>(p.rows);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int RG, bool IMMA>
static cudaError_t launch_gemv_k(const GemvParams& p, int K, int sms, cudaStream_t st, bool pdl) {
  switch (K) {
    case 1: return launch_gemv_t<1, RG, IMMA>(p, sms, st, pdl);
    case 2: return launch_gemv_t<2, RG, IMMA>(p, sms, st, pdl);
    case 3: return launch_gemv_t<3, RG, IMMA>(p, sms, st, pdl);
    case 4: return launch_gemv_t<4, RG, IMMA>(p, sms, st, pdl);
    case 5: return launch_gemv_t<5, RG, IMMA>(p, sms, st, pdl);
    case 6: return launch_gemv_t<6, RG, IMMA>(p, sms, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_prep(const PrepParams& p, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.in_features / 128 + 3) / 4, p.row_groups * 8, p.nseg);
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prep_kernel, p);
}

cudaError_t launch_gemv(const GemvParams& p, int K, int row_groups, bool imma, int sms, cudaStream_t st, bool pdl) {
  if (row_groups == 1) return imma ? launch_gemv_k<1, true>(p, K, sms, st, pdl) : launch_gemv_k<1, false>(p, K, sms, st, pdl);
  if (row_groups == 2) return imma ? launch_gemv_k<2, true>(p, K, sms, st, pdl) : launch_gemv_k<2, false>(p, K, sms, st, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace exl3
