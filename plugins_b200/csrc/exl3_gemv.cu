// exl3_gemv.cu -- the EXL3 decode GEMV for 1..16 rows (sm_100a).
//
// Computes, per the reference (plugins/sushi_ds41/src/sushi/exl3/project_rows.zig:170-308, the multi-row kernel,
// and expert_exl3.zig:490-566, the scalar definition):
//   xp = f16(H128(x * suh) / sqrt(128))            per 128-block of the input     (fused prologue)
//   inner[c] = sum_k xp[k] W_hat[k, c]             f32 accumulation                (main loop)
//   y = H128(inner) / sqrt(128) * svh              per 128-block of the output     (epilogue)
//
// Design (B200):
//  * one launch per linear.  The work is the grid of (output 128-column block, 16-row k slab) units -- 8 tiles,
//    contiguous in the pack layout; it is ordered segment-major, then by k-chunk (KR slabs), then column block,
//    then slab, and split into equal contiguous shares over a persistent grid (CTAs per SM fixed), so every shape
//    fills all 148 SMs with equal work;
//  * a CTA's units go round-robin to its 4 warps; each warp prefetches its own units with 16-byte cp.async into a
//    private 4-stage ring.  The weights need nothing from the previous kernel, so the rings fill before
//    griddepcontrol.wait;
//  * the prologue then rotates just the input slabs the share touches into shared memory, in the fragment order of
//    the MMA's B operand (no separate prepare launch);
//  * each tile is decoded in registers: lane t's eight windows ARE the A fragment of W^T, so a tile is one MMA
//    (mul1 byte sums on dp4a, or on the tensor pipe as a u8 IMMA), f32 accumulation;
//  * at the end of a (segment, chunk, column block) run the warps' partials are summed in warp order; a column
//    block split over CTAs or chunks gets a fixed slot per (chunk, contributor), and its last contributor adds
//    them in a fixed order (deterministic), applies the output Hadamard and svh and stores y.
#include <cuda_runtime.h>

#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace exl3 {

constexpr int kWarps = 4;    // warps per CTA; a CTA's units go round-robin to its warps
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;   // stages (units) per warp ring
constexpr int kRedStride = 132;
constexpr int kMaxChunks = 128;  // k-chunks of one linear (in_features <= 128 * 1024)
constexpr int kMaxContrib = 512; // partial slots summed for one column block

// ------------------------------------------------------------------ unit walking

// Position of a unit in the segment / chunk / column-block / slab order.
struct UnitPos {
  int s, c, cb, t;  // segment, chunk, column block within the segment, slab within the chunk
};

struct Walker {
  const GemvParams* p;
  UnitPos pos;
  __device__ __forceinline__ int seg_cbs(int s) const {  // column blocks of segment s
    int lo = p->seg_cb[0], hi = p->seg_cb[1];
#pragma unroll
    for (int t = 1; t < kMaxSegments; ++t)
      if (t == s) {
        lo = p->seg_cb[t];
        hi = p->seg_cb[t + 1];
      }
    return hi - lo;
  }
  __device__ __forceinline__ int seg_base(int s) const {
    int v = p->seg_cb[0];
#pragma unroll
    for (int t = 1; t <= kMaxSegments; ++t)
      if (t == s) v = p->seg_cb[t];
    return v;
  }
  __device__ __forceinline__ void seek(uint32_t u) {
    const int KT = p->kt, KR = p->kr;
    int s = 0;
#pragma unroll
    for (int t = 1; t < kMaxSegments; ++t)
      if (t < p->nseg && static_cast<int>(u) >= p->seg_cb[t] * KT) s = t;
    const uint32_t local = u - static_cast<uint32_t>(seg_base(s) * KT);
    const uint32_t blk = static_cast<uint32_t>(seg_cbs(s) * KR);
    pos.s = s;
    pos.c = static_cast<int>(local / blk);
    const uint32_t rem = local % blk;
    pos.cb = static_cast<int>(rem / KR);
    pos.t = static_cast<int>(rem % KR);
  }
  __device__ __forceinline__ void step() {
    if (++pos.t == p->kr) {
      pos.t = 0;
      if (++pos.cb == seg_cbs(pos.s)) {
        pos.cb = 0;
        if (++pos.c == p->kc) {
          pos.c = 0;
          ++pos.s;
        }
      }
    }
  }
  __device__ __forceinline__ int global_cb() const { return seg_base(pos.s) + pos.cb; }
  __device__ __forceinline__ int slab() const { return pos.c * p->kr + pos.t; }
  __device__ __forceinline__ int block_index() const { return pos.s * p->kc + pos.c; }  // (segment, chunk)
};

struct Partition {
  uint64_t U, G;
  __device__ __forceinline__ uint32_t start(uint32_t c) const { return static_cast<uint32_t>(U * c / G); }
  __device__ __forceinline__ uint32_t owner(uint32_t u) const {  // the CTA whose share holds unit u
    return static_cast<uint32_t>(((static_cast<uint64_t>(u) + 1) * G + U - 1) / U) - 1u;
  }
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ------------------------------------------------------------------ the kernel

// Release of this CTA's prior writes (ordered before it by the caller's barrier) at GPU scope, then an atomic add.
__device__ __forceinline__ uint32_t release_add(uint32_t* ctr) {
  __threadfence();
  return atomicAdd(ctr, 1u);
}

template <int N, int RG, bool IMMA>
__global__ void __launch_bounds__(kThreads, RG == 1 ? kGemvCtasPerSm : 2) gemv_kernel(GemvParams p) {
  constexpr uint32_t kTileBytes = 2u * N;            // 2n bytes
  constexpr uint32_t kUnitBytes = 8u * kTileBytes;   // one unit: 8 tiles, contiguous in the pack layout
  constexpr uint32_t kSlabX = RG * 256u;             // activation fragments of one slab
  constexpr uint32_t W = kWarps;

  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  const int rows = p.rows;
  uint8_t* xps = smem;                                                  // [span][KR][RG][32][8 B]
  uint8_t* ring = smem + p.xp_bytes + warp * (kStages * kUnitBytes);   // this warp's ring
  float* red = reinterpret_cast<float*>(smem + p.xp_bytes + W * kStages * kUnitBytes);  // [W][rows][kRedStride]
  volatile int* s_last = reinterpret_cast<volatile int*>(red + W * rows * kRedStride);
  uint32_t* s_own = reinterpret_cast<uint32_t*>(red + W * rows * kRedStride) + 4;  // [kc] first contributor per chunk
  uint32_t* s_cnt = s_own + kMaxChunks;                                              // [kc] contributors per chunk
  uint32_t* s_list = s_cnt + kMaxChunks;                          // [kMaxContrib] slot offsets of one block's partials

  const int KT = p.kt, KR = p.kr;
  const size_t OT = static_cast<size_t>(p.out_features / 16);
  const Partition part{static_cast<uint64_t>(p.out_features / 128) * KT, gridDim.x};
  const uint32_t cta = blockIdx.x;
  const uint32_t u0 = part.start(cta), u1 = part.start(cta + 1);
  const uint32_t nunits = u1 - u0;
  const uint32_t mine = nunits > warp ? (nunits - warp + W - 1u) / W : 0u;  // units u0 + warp + W i
  const uint8_t* trellis = reinterpret_cast<const uint8_t*>(p.trellis);

  pdl_launch_dependents();  // the next launch may be scheduled; it waits for this grid to finish

  // ---- weight prefetch (independent of the previous kernel): this warp's units, one unit per stage
  Walker iw{&p, {}};
  iw.seek(u0 + warp);
  auto advance = [&](Walker& wk) {  // the next unit of this warp: W slabs on
    if (wk.pos.t + static_cast<int>(W) < KR) {
      wk.pos.t += W;
    } else {
#pragma unroll 1
      for (uint32_t k = 0; k < W; ++k) wk.step();
    }
  };
  auto issue = [&](uint32_t i) {  // unit i of this warp into stage i % kStages; iw is at that unit
    const uint8_t* src = trellis + (static_cast<size_t>(iw.slab()) * OT + static_cast<size_t>(iw.global_cb()) * 8u) * kTileBytes;
    uint8_t* dst = ring + (i % kStages) * kUnitBytes;
#pragma unroll
    for (uint32_t ch = lane; ch < kUnitBytes / 16u; ch += 32u) cp_async16(dst + ch * 16u, src + ch * 16u);
    advance(iw);
  };
#pragma unroll 1
  for (uint32_t i = 0; i + 1 < static_cast<uint32_t>(kStages); ++i) {
    if (i < mine) issue(i);
    cp_async_commit();
  }

  // ---- activations: wait for the previous kernel, then rotate the slabs this share touches
  pdl_wait();
  Walker pw{&p, {}};
  pw.seek(u0);
  const int blk_first = pw.block_index();
  {
    Walker lw2{&p, {}};
    lw2.seek(nunits ? u1 - 1 : u0);
    const int nblk = lw2.block_index() - blk_first + 1;
    uint4* z = reinterpret_cast<uint4*>(xps);
    const uint32_t nz = static_cast<uint32_t>(nblk) * KR * kSlabX / 16u;
    for (uint32_t i = tid; i < nz; i += kThreads) z[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    const int per_blk = (KR / 8) * rows;  // jobs: (block, 128-wide input block in the chunk, row)
    const int jobs = nblk * per_blk;
    __half* xh = reinterpret_cast<__half*>(xps);
    for (int job = warp; job < jobs; job += W) {
      const int b = job / per_blk, rem = job % per_blk;
      const int h = rem / rows, row = rem % rows;
      const int blk = blk_first + b;
      const int s = blk / p.kc, c = blk % p.kc;
      const int k0 = (c * KR + h * 8) * 16;  // first input element of this 128-block
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const size_t k = static_cast<size_t>(k0) + lane + 32 * i;
        const float xv = load_act(p.x, static_cast<size_t>(p.row0 + row) * p.x_row_stride + k, p.x_dtype);
        v[i] = p.prepared ? xv : xv * f16_bits_to_float(p.suh[static_cast<size_t>(s) * p.in_features + k]);
      }
      if (!p.prepared) {
        fwht128_warp(v, lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] *= kHadScale;
      }
      const int rg = row >> 3, g = row & 7;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kk_all = lane + 32 * i;  // 0..127 within the block
        const int t = h * 8 + (kk_all >> 4), kk = kk_all & 15;
        int q, e;
        if (IMMA) {
          q = kk >> 2;
          e = kk & 3;
        } else {
          q = (kk & 7) >> 1;
          e = (kk & 1) | ((kk >> 3) << 1);
        }
        const size_t at = ((static_cast<size_t>(b) * KR + t) * RG + rg) * 128 + (g * 4 + q) * 4 + e;
        xh[at] = __float2half_rn(v[i]);
      }
    }
    __syncthreads();
  }

  // ---- main loop: runs of one (segment, chunk, column block), each ending in the block epilogue
  LaneWin<N> lwin;
  lwin.init(lane);
  ImmaIndicator ind;
  ind.init(lane);
  const uint32_t g = lane >> 2, q = lane & 3u;

  uint32_t i = 0;  // this warp's next unit (its stage counter)
  uint32_t u = u0;
#pragma unroll 1
  while (u < u1) {
    const UnitPos run = pw.pos;
    const uint32_t run_end = min(u1, u + static_cast<uint32_t>(KR - run.t));
    const uint8_t* xrun = xps + (static_cast<size_t>(pw.block_index() - blk_first) * KR) * kSlabX;
    float acc[8][RG][4];
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int r = 0; r < RG; ++r)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][r][e] = 0.0f;

    const uint32_t first = u + ((warp + W - (u - u0) % W) % W);
#pragma unroll 1
    for (uint32_t my = first; my < run_end; my += W, ++i) {
      cp_async_wait<kStages - 2>();
      __syncwarp();
      const uint32_t* tw = reinterpret_cast<const uint32_t*>(ring + (i % kStages) * kUnitBytes);
      const uint8_t* xs = xrun + static_cast<size_t>(run.t + static_cast<int>(my - u)) * kSlabX;
      uint32_t b0[RG], b1[RG];
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const uint2 xv = reinterpret_cast<const uint2*>(xs + r * 256)[lane];
        b0[r] = xv.x;
        b1[r] = xv.y;
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        uint32_t w[8], a[4];
        tile_codewords<N>(tw + t * (kTileBytes / 4u), lwin, w);
        if constexpr (IMMA) decode_afrag_imma(w, ind, a);
        else decode_afrag_dp4a(w, a);
#pragma unroll
        for (int r = 0; r < RG; ++r) mma_16816(acc[t][r], a, b0[r], b1[r]);
      }
      __syncwarp();
      if (i + kStages - 1 < mine) issue(i + kStages - 1);
      cp_async_commit();
    }

    // ---- block epilogue: the warps' partials, summed in warp order
    float* rw = red + warp * rows * kRedStride;
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const int col = 16 * t + static_cast<int>(g), row = 8 * r + 2 * static_cast<int>(q);
        if (row < rows) {
          rw[row * kRedStride + col] = acc[t][r][0];
          rw[row * kRedStride + col + 8] = acc[t][r][2];
        }
        if (row + 1 < rows) {
          rw[(row + 1) * kRedStride + col] = acc[t][r][1];
          rw[(row + 1) * kRedStride + col + 8] = acc[t][r][3];
        }
      }
    __syncthreads();
    for (int idx = tid; idx < rows * 128; idx += kThreads) {
      const int row = idx >> 7, col = idx & 127;
      float v = 0.0f;
#pragma unroll
      for (uint32_t w2 = 0; w2 < W; ++w2) v += red[(w2 * rows + row) * kRedStride + col];
      red[row * kRedStride + col] = v;
    }
    __syncthreads();

    Walker rw2{&p, run};
    const int s = run.s, cbl = run.cb, cbg = rw2.global_cb();
    const int cbs = rw2.seg_cbs(s);
    const uint32_t useg = static_cast<uint32_t>(rw2.seg_base(s) * KT);
    // contributors to this column block, per chunk: the first owner and the count (one division per thread)
    if (tid < static_cast<uint32_t>(p.kc)) {
      const uint32_t f = useg + static_cast<uint32_t>((static_cast<int>(tid) * cbs + cbl) * KR);
      const uint32_t o0 = part.owner(f);
      s_own[tid] = o0;
      s_cnt[tid] = part.owner(f + KR - 1) - o0 + 1u;
    }
    __syncthreads();
    uint32_t total = 0;
    for (int c = 0; c < p.kc; ++c) total += s_cnt[c];
    bool fin = total == 1u;
    if (!fin) {
      const size_t pair = static_cast<size_t>(rw2.seg_base(s)) * p.kc + static_cast<size_t>(run.c) * cbs + cbl;
      float* slot = p.partials + ((pair * p.contrib_max + (cta - s_own[run.c])) * rows) * 128;
      for (int idx = tid; idx < rows * 128; idx += kThreads) slot[idx] = red[(idx >> 7) * kRedStride + (idx & 127)];
      __syncthreads();
      if (tid == 0) *s_last = (release_add(&p.counters[cbg]) + 1u == total) ? 1 : 0;
      __syncthreads();
      fin = *s_last != 0;
      if (fin) {
        __threadfence();  // acquire: the other contributors' slots
        // the contributions in their fixed order (chunk, then contributor), as slot offsets
        const size_t pair0 = static_cast<size_t>(rw2.seg_base(s)) * p.kc + cbl;
        if (tid == 0) {
          uint32_t k = 0;
          for (int c = 0; c < p.kc; ++c)
            for (uint32_t x = 0; x < s_cnt[c]; ++x)
              s_list[k++] = static_cast<uint32_t>((((pair0 + static_cast<size_t>(c) * cbs) * p.contrib_max + x) * rows) * 128);
        }
        __syncthreads();
        for (int idx = tid; idx < rows * 128; idx += kThreads) {
          float v = 0.0f;
          for (uint32_t k0 = 0; k0 < total; k0 += 8) {
            float part8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)  // eight independent loads in flight
              part8[k] = (k0 + k < total) ? __ldcg(p.partials + s_list[k0 + k] + idx) : 0.0f;
#pragma unroll
            for (int k = 0; k < 8; ++k)
              if (k0 + k < total) v += part8[k];
          }
          red[(idx >> 7) * kRedStride + (idx & 127)] = v;
        }
        if (tid == 0) p.counters[cbg] = 0u;  // ready for the next launch
        __syncthreads();
      }
    }
    if (fin) {
      const int seg_c0 = rw2.seg_base(s) * 128;
      const int seg_w = cbs * 128;
      for (int row = static_cast<int>(warp); row < rows; row += W) {
        const size_t grow = static_cast<size_t>(p.row0 + row);
        const size_t ybase = p.nseg == 1 ? grow * p.y_row_stride
                                         : static_cast<size_t>(p.rows_total) * seg_c0 + grow * seg_w - seg_c0;
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = red[row * kRedStride + lane + 32 * k];
        if (!p.inner_only) {
          fwht128_warp(v, lane);
#pragma unroll
          for (int k = 0; k < 4; ++k) v[k] = v[k] * kHadScale * f16_bits_to_float(p.svh[cbg * 128 + lane + 32 * k]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) store_act(p.y, ybase + static_cast<size_t>(cbg) * 128 + lane + 32 * k, v[k], p.y_dtype);
      }
    }
    __syncthreads();
    // next run: slab 0 of the next (column block, chunk, segment)
    pw.pos.t = KR - 1;
    pw.step();
    u = run_end;
  }
  cp_async_wait<0>();  // no copy outlives the CTA
}

// ------------------------------------------------------------------ host launch

template <int N, int RG, bool IMMA>
static size_t gemv_smem_bytes(size_t xp_bytes, int rows) {
  return xp_bytes + static_cast<size_t>(kWarps) * kStages * 8u * 2u * N +
         static_cast<size_t>(kWarps) * rows * kRedStride * 4 + 16 + (2 * kMaxChunks + kMaxContrib) * 4;
}

template <int N, int RG, bool IMMA>
static cudaError_t launch_gemv_t(const GemvParams& p, unsigned grid, cudaStream_t st, bool pdl) {
  auto kern = gemv_kernel<N, RG, IMMA>;
  const size_t smem = gemv_smem_bytes<N, RG, IMMA>(p.xp_bytes, p.rows);
  static KernelSetup setup;
  if (cudaError_t e = kernel_setup(setup, kern, kThreads, smem); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int RG, bool IMMA>
static cudaError_t launch_gemv_k(const GemvParams& p, int n, unsigned grid, cudaStream_t st, bool pdl) {
  cudaError_t e = cudaErrorInvalidValue;
  with_rate(n, [&](auto N) { e = launch_gemv_t<decltype(N)::value, RG, IMMA>(p, grid, st, pdl); });
  return e;
}

// Host copy of the kernel's partition arithmetic.
static uint32_t host_start(uint64_t U, uint64_t G, uint32_t c) { return static_cast<uint32_t>(U * c / G); }
static uint32_t host_owner(uint64_t U, uint64_t G, uint32_t u) {
  return static_cast<uint32_t>(((static_cast<uint64_t>(u) + 1) * G + U - 1) / U) - 1u;
}

bool gemv_geometry(GemvParams& p, int sms, int row_groups, size_t partial_capacity_floats, const char** why) {
  const int KT = p.in_features / 16;
  const int CB = p.out_features / 128;
  // chunk: the largest divisor of KT that is a multiple of 8 and at most 64 slabs (1024 inputs)
  int KR = 8;
  for (int d = 64; d >= 8; d -= 8)
    if (KT % d == 0) {
      KR = d;
      break;
    }
  p.kt = KT;
  p.kr = KR;
  p.kc = KT / KR;
  if (p.kc > kMaxChunks) {
    *why = "exl3_b200: in_features too large for the decode GEMV";
    return false;
  }
  const uint64_t U = static_cast<uint64_t>(CB) * KT;
  // persistent grid, but no share below 32 units (256 tiles): small layers are latency-bound, and fewer shares mean
  // fewer partials to fix up.  G depends on the shape only, so a row's sum order does not depend on the row count.
  uint64_t G = static_cast<uint64_t>(sms) * kGemvCtasPerSm;
  if (G > U / 32) G = U / 32;
  if (G < 1) G = 1;
  // blocks (segment, chunk) a share can span, and contributors per (segment, chunk, column block)
  auto block_of = [&](uint32_t u) {
    int s = 0;
    for (int t = 1; t < p.nseg; ++t)
      if (u >= static_cast<uint64_t>(p.seg_cb[t]) * KT) s = t;
    const uint64_t local = u - static_cast<uint64_t>(p.seg_cb[s]) * KT;
    const uint64_t blk = static_cast<uint64_t>(p.seg_cb[s + 1] - p.seg_cb[s]) * KR;
    return s * p.kc + static_cast<int>(local / blk);
  };
  int span = 1;
  for (uint32_t c = 0; c < G; ++c) {
    const uint32_t a = host_start(U, G, c), b = host_start(U, G, c + 1);
    if (b > a) {
      const int sp = block_of(b - 1) - block_of(a) + 1;
      if (sp > span) span = sp;
    }
  }
  int cmax = 1;
  for (int s = 0; s < p.nseg; ++s) {
    const int cbs = p.seg_cb[s + 1] - p.seg_cb[s];
    for (int c = 0; c < p.kc; ++c)
      for (int cb = 0; cb < cbs; ++cb) {
        const uint32_t f = static_cast<uint32_t>(p.seg_cb[s] * KT + (c * cbs + cb) * KR);
        const int n = static_cast<int>(host_owner(U, G, f + KR - 1) - host_owner(U, G, f)) + 1;
        if (n > cmax) cmax = n;
      }
  }
  p.contrib_max = cmax;
  if (static_cast<int64_t>(cmax) * p.kc > kMaxContrib) {
    *why = "exl3_b200: too many split partials per column block";
    return false;
  }
  p.xp_bytes = static_cast<int64_t>(span) * KR * row_groups * 256;
  if (p.xp_bytes > 112 * 1024) {
    *why = "exl3_b200: the input is too wide for one decode-GEMV launch";
    return false;
  }
  const size_t need = static_cast<size_t>(CB) * p.kc * cmax * static_cast<size_t>(p.rows) * 128;
  if (need > partial_capacity_floats) {
    *why = "exl3_b200: the layer needs more split partials than the workspace holds";
    return false;
  }
  p.grid = static_cast<int32_t>(G);
  return true;
}

cudaError_t launch_gemv(const GemvParams& p, int n, int row_groups, bool imma, cudaStream_t st, bool pdl) {
  if (p.cw_mask || p.mcg) return cudaErrorInvalidValue;  // narrowed windows and mcg take the cluster-split GEMV
  const unsigned grid = static_cast<unsigned>(p.grid);
  if (row_groups == 1) return imma ? launch_gemv_k<1, true>(p, n, grid, st, pdl) : launch_gemv_k<1, false>(p, n, grid, st, pdl);
  if (row_groups == 2) return imma ? launch_gemv_k<2, true>(p, n, grid, st, pdl) : launch_gemv_k<2, false>(p, n, grid, st, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace exl3
