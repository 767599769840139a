// exl3_gemv5.cu -- the EXL3 decode GEMV with split-K inside a thread-block cluster (sm_100a).
//
// The same three steps as exl3_gemv.cu (the reference's multi-row kernel, plugins/sushi_ds41/src/sushi/exl3/
// project_rows.zig:170-308, and the scalar definition, expert_exl3.zig:490-566):
//   xp = f16(H128(x * suh) / sqrt(128))            per 128-block of the input     (fused prologue)
//   inner[c] = sum_k xp[k] W_hat[k, c]             f32 accumulation                (main loop)
//   y = H128(inner) / sqrt(128) * svh              per 128-block of the output     (epilogue)
//
// Work split.  One thread-block cluster per 128-column block of the output (all segments of a stacked weight in
// order); the cluster's S CTAs split the input: CTA rank r takes the 16-row slabs [r KT/S, (r+1) KT/S).  A CTA's
// four warps take its slabs round-robin; a slab of one column block is one unit (8 tiles, contiguous in the pack
// layout), prefetched with 16-byte cp.async into the warp's deep ring (8-16 units) before griddepcontrol.wait, so the weight stream
// overlaps the previous kernel.  After the input rotation of its k-range (shared memory, MMA B-fragment order) each
// warp decodes its tiles in registers (lane t's windows ARE the A fragment of W^T) into mma.sync m16n8k16.
// Reduction: the warps' partials are summed in warp order into the CTA's partial; then the cluster's rank 0 reads the
// other ranks' partials over distributed shared memory and adds them in rank order -- deterministic, no global
// partials, no atomics, no fences -- applies the output Hadamard and svh and stores y.  Cluster barriers are
// hardware barriers of the co-scheduled cluster (no spinning).
#include <cuda_runtime.h>

#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace exl3 {

namespace {

constexpr int kW5 = 4;              // warps per CTA
constexpr int kT5 = kW5 * 32;
// Units in flight per warp: a deep ring (prefetch measured faster at every shape) or a shallow one, whichever is the
// deepest that keeps three CTAs per SM beside the CTA's rotated input (a unit is 16 n bytes; n = 16 x bits).
constexpr int deep_stages_n(int n) { return n <= 32 ? 16 : (n <= 64 ? 12 : (n <= 80 ? 10 : 8)); }
constexpr int shallow_stages_n(int n) { return n <= 64 ? 8 : 6; }
template <int N>
constexpr int deep_stages() { return deep_stages_n(N); }
template <int N>
constexpr int shallow_stages() { return shallow_stages_n(N); }
constexpr int kRed5 = 132;          // row stride of the reduction buffer (floats)

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// f32 at this CTA's shared address `local` in cluster CTA `rank`
__device__ __forceinline__ float ld_dsmem(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

}  // namespace

template <int N, int RG, bool IMMA, int ST, int DS>
__global__ void __launch_bounds__(kT5, 3) gemv5_kernel(GemvParams p) {
  constexpr uint32_t kTileBytes = 2u * N;
  constexpr uint32_t kUnitBytes = 8u * kTileBytes;
  constexpr uint32_t kSlabX = RG * 256u;
  constexpr int kStages5 = ST;

  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  const int rows = p.rows;
  const int S = p.kc;                       // CTAs per cluster (input splits)
  const int KR = p.kr;                      // slabs per CTA
  const uint32_t rank = S > 1 ? cluster_rank() : 0u;
  const int cbg = static_cast<int>(blockIdx.x) / S;  // global column block of this cluster
  const int t0 = static_cast<int>(rank) * KR;        // first slab
  uint8_t* xps = smem;                                                  // [KR][RG][32][8 B]
  uint8_t* ring = smem + p.xp_bytes + warp * (kStages5 * kUnitBytes);
  // after the main loop, the reduction buffer [kW5][rows][kRed5] overlays the rotated input and the rings (both dead
  // by then), and the exchange's staging rows follow it: the launch takes the larger of the two footprints
  float* red = reinterpret_cast<float*>(smem);

  // segment of this column block
  int s = 0;
#pragma unroll
  for (int i = 1; i < kMaxSegments; ++i)
    if (i < p.nseg && cbg >= p.seg_cb[i]) s = i;
  int seg_lo = p.seg_cb[0], seg_hi = p.seg_cb[1];
#pragma unroll
  for (int i = 1; i < kMaxSegments; ++i)
    if (i == s) {
      seg_lo = p.seg_cb[i];
      seg_hi = p.seg_cb[i + 1];
    }

  const size_t OT = static_cast<size_t>(p.out_features / 16);
  const uint8_t* src0 = reinterpret_cast<const uint8_t*>(p.trellis) +
                        (static_cast<size_t>(t0) * OT + static_cast<size_t>(cbg) * 8u) * kTileBytes;
  const size_t slab_stride = OT * kTileBytes;  // bytes from one slab's unit to the next
  const int mine = KR > static_cast<int>(warp) ? (KR - static_cast<int>(warp) + kW5 - 1) / kW5 : 0;

  pdl_launch_dependents();

  // ---- weights: this warp's units (slabs warp, warp + 4, ...), independent of the previous kernel
  auto issue = [&](int i) {
    const uint8_t* src = src0 + static_cast<size_t>(static_cast<int>(warp) + kW5 * i) * slab_stride;
    uint8_t* dst = ring + (i % kStages5) * kUnitBytes;
#pragma unroll
    for (uint32_t ch = lane; ch < kUnitBytes / 16u; ch += 32u) cp_async16(dst + ch * 16u, src + ch * 16u);
  };
#pragma unroll 1
  for (int i = 0; i + 1 < kStages5; ++i) {
    if (i < mine) issue(i);
    cp_async_commit();
  }

  // ---- activations: after the previous kernel, rotate the CTA's k-range into fragment order
  pdl_wait();
  {
    const int per_row = KR / 8;  // 128-wide input blocks
    const int jobs = p.xf ? 0 : per_row * rows;
    __half* xh = reinterpret_cast<__half*>(xps);
    if (p.xf) {
      // rotated once by the prepare launch (the same arithmetic, so the same bits): this CTA's slabs, rows past the
      // launch's already zero
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.xf) +
                                                        (static_cast<size_t>(s) * p.kt + t0) * kSlabX);
      uint4* dst = reinterpret_cast<uint4*>(xps);
      const uint32_t n16 = static_cast<uint32_t>(KR) * kSlabX / 16u;
      for (uint32_t i = tid; i < n16; i += 4 * kT5) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i + u * kT5 < n16) v[u] = __ldcg(src + i + u * kT5);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i + u * kT5 < n16) dst[i + u * kT5] = v[u];
      }
    }
    if (!p.xf && (rows % 8 != 0 || RG * 8 != rows)) {  // rows that no job writes must read as zero
      uint4* z = reinterpret_cast<uint4*>(xps);
      const uint32_t nz = static_cast<uint32_t>(KR) * kSlabX / 16u;
      for (uint32_t i = tid; i < nz; i += kT5) z[i] = make_uint4(0, 0, 0, 0);
      __syncthreads();
    }
    // four of the warp's jobs at a time: every job's loads (x, suh) are issued before the first rotation, so their
    // latency is paid once per four jobs (the same arithmetic per job, so the same bits)
    constexpr int kJobBatch = 4;
    for (int base = static_cast<int>(warp); base < jobs; base += kJobBatch * kW5) {
      float v[kJobBatch][4];
#pragma unroll
      for (int u = 0; u < kJobBatch; ++u) {
        const int job = base + u * kW5;
        if (job >= jobs) continue;  // (warp-uniform)
        const int h = job / rows, row = job % rows;
        const int k0 = (t0 + h * 8) * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const size_t k = static_cast<size_t>(k0) + lane + 32 * i;
          v[u][i] = load_act(p.x, static_cast<size_t>(p.row0 + row) * p.x_row_stride + k, p.x_dtype);
          if (!p.prepared) v[u][i] *= f16_bits_to_float(p.suh[static_cast<size_t>(s) * p.in_features + k]);
        }
      }
#pragma unroll
      for (int u = 0; u < kJobBatch; ++u) {
        const int job = base + u * kW5;
        if (job >= jobs) continue;
        const int h = job / rows, row = job % rows;
        if (!p.prepared) {
          fwht128_warp(v[u], lane);
#pragma unroll
          for (int i = 0; i < 4; ++i) v[u][i] *= kHadScale;
        }
        const int rg = row >> 3, g = row & 7;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk_all = static_cast<int>(lane) + 32 * i;
          const int t = h * 8 + (kk_all >> 4), kk = kk_all & 15;
          int q, e;
          if (IMMA) {
            q = kk >> 2;
            e = kk & 3;
          } else {
            q = (kk & 7) >> 1;
            e = (kk & 1) | ((kk >> 3) << 1);
          }
          xh[(static_cast<size_t>(t) * RG + rg) * 128 + (g * 4 + q) * 4 + e] = __float2half_rn(v[u][i]);
        }
      }
    }
    __syncthreads();
  }

  // ---- main loop
  LaneWin<N> lwin;
  lwin.init(lane);
  lwin.mask = spec_mask(p.cw_mask);
  ImmaIndicator ind;
  ind.init(lane);
  ImmaWin<N> iwin;
  if constexpr (IMMA && DS == 2) iwin.init(lane, lwin.mask);
  const uint32_t g = lane >> 2, q = lane & 3u;
  float acc[8][RG][4];
#pragma unroll
  for (int t = 0; t < 8; ++t)
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[t][r][e] = 0.0f;
#pragma unroll 1
  for (int i = 0; i < mine; ++i) {
    cp_async_wait<kStages5 - 2>();
    __syncwarp();
    const uint32_t* tw = reinterpret_cast<const uint32_t*>(ring + (i % kStages5) * kUnitBytes);
    const uint8_t* xs = xps + static_cast<size_t>(static_cast<int>(warp) + kW5 * i) * kSlabX;
    uint32_t b0[RG], b1[RG];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const uint2 xv = reinterpret_cast<const uint2*>(xs + r * 256)[lane];
      b0[r] = xv.x;
      b1[r] = xv.y;
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      uint32_t a[4];
      if constexpr (IMMA) decode_tile_imma<N, DS, ST == deep_stages<N>()>(tw + t * (kTileBytes / 4u), lwin, iwin, ind, a);
      else decode_tile_natural<N, DS>(tw + t * (kTileBytes / 4u), lwin, a);
#pragma unroll
      for (int r = 0; r < RG; ++r) mma_16816(acc[t][r], a, b0[r], b1[r]);
    }
    __syncwarp();
    if (i + kStages5 - 1 < mine) issue(i + kStages5 - 1);
    cp_async_commit();
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is past the main loop: the rotated input and the rings are free

  // ---- the CTA's partial: the warps' sums in warp order, into red[0]
  float* rw = red + warp * rows * kRed5;
#pragma unroll
  for (int t = 0; t < 8; ++t)
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const int col = 16 * t + static_cast<int>(g), row = 8 * r + 2 * static_cast<int>(q);
      if (row < rows) {
        rw[row * kRed5 + col] = acc[t][r][0];
        rw[row * kRed5 + col + 8] = acc[t][r][2];
      }
      if (row + 1 < rows) {
        rw[(row + 1) * kRed5 + col] = acc[t][r][1];
        rw[(row + 1) * kRed5 + col + 8] = acc[t][r][3];
      }
    }
  __syncthreads();
  for (int idx = static_cast<int>(tid); idx < rows * 128; idx += kT5) {
    const int row = idx >> 7, col = idx & 127;
    float v = red[row * kRed5 + col];
#pragma unroll
    for (int w2 = 1; w2 < kW5; ++w2) v += red[(w2 * rows + row) * kRed5 + col];
    red[row * kRed5 + col] = v;
  }

  // ---- the cluster's sum, in rank order, by rank 0; then the output rotation and store
  if (S > 1) {
    cluster_sync();  // every rank's partial is complete and visible
    if (rank == 0) {
      for (int idx = static_cast<int>(tid); idx < rows * 128; idx += kT5) {
        const int at = (idx >> 7) * kRed5 + (idx & 127);
        float v = red[at];
        for (int r = 1; r < S; ++r) v += ld_dsmem(red + at, static_cast<uint32_t>(r));
        red[at] = v;
      }
    }
    cluster_sync();  // no rank leaves while rank 0 still reads its shared memory
    if (rank != 0) return;
  } else {
    __syncthreads();
  }
  __syncthreads();
  const int seg_c0 = seg_lo * 128, seg_w = (seg_hi - seg_lo) * 128;
  if (p.tp) {
    // column-parallel exchange: this block's columns into every rank's slot (published by the step's gather)
    const TpDev& tp = *p.tp;
    const uint32_t step = *reinterpret_cast<volatile uint32_t*>(tp.step);
    const size_t esize = p.y_dtype == kF32 ? 4 : 2;
    const size_t slot_off = (static_cast<size_t>(step & 1u) * tp.slots + p.tp_slot) * tp.slot_bytes;
    int64_t tot = p.tp_total[0], c0 = p.tp_col0[0], sb = p.tp_seg_base[0];
    int cbb = p.tp_cb_base[0];
#pragma unroll
    for (int i = 1; i < kMaxSegments; ++i)
      if (i == s) {
        tot = p.tp_total[i];
        c0 = p.tp_col0[i];
        sb = p.tp_seg_base[i];
        cbb = p.tp_cb_base[i];
      }
    const int64_t col = c0 + (cbg * 128 - seg_c0);  // first gathered column of this block
    // each warp: its row's 128 outputs through a shared-memory staging row, then 16-byte stores into every rank
    uint8_t* stage = smem + static_cast<size_t>(kW5) * rows * kRed5 * 4 + warp * 512u;  // this warp's row, after red
    const uint32_t row_bytes = 128u * static_cast<uint32_t>(esize);
    for (int row = static_cast<int>(warp); row < rows; row += kW5) {
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = red[row * kRed5 + lane + 32 * k];
      if (!p.inner_only) {
        fwht128_warp(v, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = v[k] * kHadScale * f16_bits_to_float(p.svh[cbg * 128 + lane + 32 * k]);
      }
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 4; ++k) store_act(stage, lane + 32 * k, v[k], p.y_dtype);
      __syncwarp();
      const size_t at = (static_cast<size_t>(sb + static_cast<int64_t>(p.row0 + row) * tot + col)) * esize;
      if (lane * 16u < row_bytes) {
        const uint4 chunk = reinterpret_cast<const uint4*>(stage)[lane];
        for (int q = 0; q < tp.world; ++q)
          reinterpret_cast<uint4*>(tp.y[q] + slot_off + at)[lane] = chunk;
      }
    }
    if (blockIdx.x == 0 && tid == 0) {  // the slot's size, for this rank's gather (same on every rank)
      tp.meta[p.tp_slot * 4 + 0] = p.tp_meta_cb;
      tp.meta[p.tp_slot * 4 + 1] = p.tp_meta_bytes;
    }
    (void)cbb;  // the step's gather releases every rank's columns at once (one system-scope fence per step)
    return;
  }
  for (int row = static_cast<int>(warp); row < rows; row += kW5) {
    const size_t grow = static_cast<size_t>(p.row0 + row);
    const size_t ybase = p.nseg == 1 ? grow * p.y_row_stride
                                     : static_cast<size_t>(p.rows_total) * seg_c0 + grow * seg_w - seg_c0;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = red[row * kRed5 + lane + 32 * k];
    if (!p.inner_only) {
      fwht128_warp(v, lane);
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = v[k] * kHadScale * f16_bits_to_float(p.svh[cbg * 128 + lane + 32 * k]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) store_act(p.y, ybase + static_cast<size_t>(cbg) * 128 + lane + 32 * k, v[k], p.y_dtype);
  }
}

// ------------------------------------------------------------------ host

template <int N, int RG, bool IMMA, int ST, int DS>
static cudaError_t launch5_t(const GemvParams& p, cudaStream_t st, bool pdl) {
  auto kern = gemv5_kernel<N, RG, IMMA, ST, DS>;
  const size_t loop = static_cast<size_t>(p.xp_bytes) + static_cast<size_t>(kW5) * ST * 8u * 2u * N;
  const size_t tail = static_cast<size_t>(kW5) * p.rows * kRed5 * 4 + kW5 * 512u;
  const size_t smem = loop > tail ? loop : tail;
  static KernelSetup setup;
  if (cudaError_t e = kernel_setup(setup, kern, kT5, smem, true); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid));
  cfg.blockDim = dim3(kT5);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(p.kc);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int N, int RG, bool IMMA, int DS>
static cudaError_t launch5_s(const GemvParams& p, cudaStream_t st, bool pdl) {
  return p.stages == deep_stages<N>() ? launch5_t<N, RG, IMMA, deep_stages<N>(), DS>(p, st, pdl)
                                      : launch5_t<N, RG, IMMA, shallow_stages<N>(), DS>(p, st, pdl);
}

// A narrowed codeword window or the mcg codebook takes the tensor-pipe operand order only.
template <int RG, bool IMMA>
static cudaError_t launch5_k(const GemvParams& p, int n, cudaStream_t st, bool pdl) {
  cudaError_t e = cudaErrorInvalidValue;
  if constexpr (IMMA)
    with_rate_decode(n, p.cw_mask, p.mcg != 0, [&](auto N, auto DS) {
      e = launch5_s<decltype(N)::value, RG, IMMA, decltype(DS)::value>(p, st, pdl);
    });
  else if (!p.cw_mask && !p.mcg)
    with_rate(n, [&](auto N) { e = launch5_s<decltype(N)::value, RG, IMMA, 0>(p, st, pdl); });
  return e;
}

// The launch's shared memory: the main loop's (rotated input + rings) or, overlaying it, the tail's (reduction buffer
// + exchange staging), whichever is larger.
static size_t gemv5_smem_for(int n, int stages, int KR, int row_groups, int rows) {
  const size_t loop = static_cast<size_t>(KR) * row_groups * 256 + static_cast<size_t>(kW5) * stages * 8u * 2u * n;
  const size_t tail = static_cast<size_t>(kW5) * rows * kRed5 * 4 + kW5 * 512u;
  return loop > tail ? loop : tail;
}

bool gemv5_geometry(GemvParams& p, int n, int sms, int row_groups, int split_override, const char** why) {
  const int KT = p.in_features / 16;
  const int CB = p.out_features / 128;
  constexpr size_t kThreePerSm = 74 * 1024;  // shared memory that still fits three CTAs on an SM
  const int deep = deep_stages_n(n), shallow = shallow_stages_n(n);
  // CTAs per column block: a divisor of KT leaving whole 128-input blocks (8 slabs) per CTA, at most 16 (the
  // cluster limit) and at most 128 slabs per CTA.  The split fixes a row's summation order (slabs per warp, CTA
  // partials in rank order), so it is chosen for every width at once -- a row's bytes must not depend on the rows
  // batched with it: splits whose shared memory (with the shallow ring) fits at the widest launch, preferred by their
  // footprint at 8 rows: those that keep three CTAs per SM, among them the largest whose grid still fits one wave of
  // three CTAs per SM, else the smallest.  Only the ring depth follows the launch's rows (it sets prefetch, not the
  // order of the sums): the deep ring where it still keeps three CTAs per SM.
  int best = 0, fallback = 0;
  for (int pass = 0; pass < 2 && best == 0; ++pass) {
    for (int d = 1; d <= 16; ++d) {
      if (KT % d != 0 || (KT / d) % 8 != 0 || KT / d > 128) continue;
      if (gemv5_smem_for(n, shallow, KT / d, 2, kMaxRows) > 227 * 1024) continue;
      const size_t smem = gemv5_smem_for(n, shallow, KT / d, 1, 8);
      if (split_override > 0) {
        if (d == split_override) best = d;
        continue;
      }
      if (pass == 0 && smem > kThreePerSm) continue;
      if (fallback == 0) fallback = d;  // the smallest allowed in this pass
      if (static_cast<int64_t>(CB) * d <= static_cast<int64_t>(sms) * 3) best = d;
    }
    if (best == 0) best = fallback;
  }
  if (best == 0) {
    *why = "exl3_b200: no cluster split of this input width";
    return false;
  }
  p.kt = KT;
  p.kc = best;
  p.kr = KT / best;
  p.stages = gemv5_smem_for(n, deep, p.kr, row_groups, p.rows) <= kThreePerSm ? deep : shallow;
  p.xp_bytes = static_cast<int64_t>(p.kr) * row_groups * 256;
  p.grid = CB * best;
  p.contrib_max = 1;
  return true;
}

cudaError_t launch_gemv5(const GemvParams& p, int n, int row_groups, bool imma, cudaStream_t st, bool pdl) {
  if (row_groups == 1) return imma ? launch5_k<1, true>(p, n, st, pdl) : launch5_k<1, false>(p, n, st, pdl);
  if (row_groups == 2) return imma ? launch5_k<2, true>(p, n, st, pdl) : launch5_k<2, false>(p, n, st, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace exl3
