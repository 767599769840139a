// exl3_gemv6.cu -- the EXL3 decode GEMV as a persistent, work-balanced kernel (sm_100a), 1..8 rows.
//
// The same three steps as the cluster-split GEMV (exl3_gemv5.cu; the reference's multi-row kernel,
// plugins/sushi_ds41/src/sushi/exl3/project_rows.zig:170-308, and the scalar definition, expert_exl3.zig:490-566):
//   xp = f16(H128(x * suh) / sqrt(128))            per 128-block of the input     (prepare launch)
//   inner[c] = sum_k xp[k] W_hat[k, c]             f32 accumulation                (main loop)
//   y = H128(inner) / sqrt(128) * svh              per 128-block of the output     (epilogue)
//
// Two launches chained with programmatic dependent launch (one, for 1..4 rows split into runs of <= kXiSlabs slabs):
//   prepare -- x of the launch's rows rotated once, per segment (each segment of a stacked weight has its own suh),
//              into MMA B-fragment order in global memory (L2-resident: every CTA reads it); with 1..4 rows and short
//              runs each CTA instead rotates just the 128-input blocks its run covers into shared memory, while its
//              first weights stream in (the same arithmetic, so the same bits: a launch saves the prepare launch's
//              ~2 us and spends ~2 % more issue per row);
//   GEMV    -- a persistent grid over the weight's 128-column blocks ("units", all segments in order).  The work is
//              cut for V = 3 x SMs virtual CTAs: whole units go round-robin while every virtual CTA gets one, then
//              the remaining units' 16-row slabs, laid end to end, are cut into one equal run per virtual CTA
//              (stream-K), so every CTA streams the same bytes and the grid ends together whatever the shape.  The
//              real CTAs (as many as fit on the SMs: V with one row group, fewer with two) take the virtual ones
//              round-robin; the sums depend on V only, so 1 to 16 rows give every row the same bits.  A CTA's four warps take a run's slabs round-robin,
//              each through its own deep cp.async ring (weights prefetched before griddepcontrol.wait, so the stream
//              overlaps the prepare launch); lane t's windows ARE the A fragment of W^T, decoded in registers into
//              mma.sync m16n8k16 against the fragment-order x.  A unit that two or more runs share is finished by
//              the run that completes it last (a per-unit counter, reset by that run): it adds the runs' partials in
//              run order and applies the output rotation -- the order of every sum is fixed by the shape and the
//              grid, never by timing.
#include <cuda_fp16.h>
#include <cstdlib>
#include <cuda_runtime.h>

#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace exl3 {

namespace {

constexpr int kW6 = 4;            // warps per CTA
constexpr int kT6 = kW6 * 32;
constexpr int kRed6 = 132;        // row stride of the reduction buffer (floats)
constexpr int kMinRun6 = 32;      // slabs: the shortest run a CTA takes (eight per warp)
constexpr int kPart6 = 16 * 128;  // floats of one run's partial of a unit (up to 16 rows)
constexpr int kVirt6 = 3;         // virtual CTAs per SM: the work split
constexpr int kXiSlabs = 136;     // in-CTA rotation: the most slabs one piece of a run covers (17 input blocks)
constexpr int kXiRows = 4;        // in-CTA rotation: the rows its shared-memory layout holds
constexpr int kXiTake = 1;        // in-CTA rotation: the most rows that take it (measured: from two rows on, the
                                  // prepare launch is faster: config 2's gate|up 35.9 against 37.9 us at two rows)
constexpr int kXiBatch = 4;       // in-CTA rotation: a warp's jobs whose loads are in flight together

template <int N>  // n halfwords per tile (16 x bits per weight)
constexpr int stages6() { return N <= 32 ? 16 : (N <= 64 ? 12 : (N <= 80 ? 10 : 8)); }
// With the prepared input, each ring slot also carries its unit's x fragments (RG x 256 bytes): the deepest ring that
// still keeps 3 CTAs per SM (one row group) or 2 (two) beside the reduction buffer.
template <int N, int RG, bool XI>
constexpr int stages6x() {
  if (XI) return stages6<N>();
  constexpr int budget = RG == 1 ? 76672 : 115584;  // dynamic shared memory per CTA at 3 (2) CTAs per SM
  constexpr int fit = (budget / kW6 - 8 * RG * kRed6 * 4) / (16 * N + 256 * RG);
  return stages6<N>() < fit ? stages6<N>() : fit;
}

__device__ __forceinline__ void cp_async16_6(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit6() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait6() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// x -> xf[s][t][rg][128 halfs]: row 8 rg + g's input 16 t + kk at half (g * 4 + kk / 4) * 4 + kk % 4 of group rg
// of slab t (the IMMA decode's k order).  Grid (in / 128, nseg), 32 x 8 RG threads: warp r is row r (zeros past the
// launch's rows).
template <int RG>
__global__ void __launch_bounds__(256 * RG) gemv6_prep_kernel(GemvParams p, __half* __restrict__ xf) {
  pdl_launch_dependents();  // the GEMV may start streaming weights; it reads xf only after this grid completes
  pdl_wait();               // x comes from the previous kernel
  const int blk = blockIdx.x, s = blockIdx.y;
  const uint32_t lane = threadIdx.x & 31u, r = threadIdx.x >> 5, rg = r >> 3, g = r & 7u;
  const int KT = p.in_features / 16;
  const int k0 = blk * 128;
  float v[4];
  if (static_cast<int>(r) < p.rows) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      v[i] = load_act(p.x, static_cast<size_t>(p.row0 + r) * p.x_row_stride + k0 + lane + 32 * i, p.x_dtype);
    if (!p.prepared) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        v[i] *= f16_bits_to_float(p.suh[static_cast<size_t>(s) * p.in_features + k0 + lane + 32 * i]);
      fwht128_warp(v, lane);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] *= kHadScale;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = 0.0f;
  }
  __half* dst = xf + static_cast<size_t>(s) * KT * RG * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kin = static_cast<int>(lane) + 32 * i;
    const int t = blk * 8 + (kin >> 4), kk = kin & 15;
    dst[(static_cast<size_t>(t) * RG + rg) * 128 + (g * 4 + (kk >> 2)) * 4 + (kk & 3)] = __float2half_rn(v[i]);
  }
}

template <int N, int RG, int ST, bool XI>
__global__ void __launch_bounds__(kT6, RG == 1 ? 3 : 2) gemv6_kernel(GemvParams p, const __half* __restrict__ xf,
                                                                    float* __restrict__ part, uint32_t* __restrict__ done) {
  static_assert(!XI || RG == 1, "in-CTA rotation is for one row group");
  constexpr int kRedRows = XI ? kXiRows : 8 * RG;
  constexpr uint32_t kTileBytes = 2u * N;
  constexpr uint32_t kUnitBytes = 8u * kTileBytes;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_last;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  uint8_t* ring = smem + warp * (ST * kUnitBytes);
  float* red = reinterpret_cast<float*>(smem + kW6 * ST * kUnitBytes);  // [kW6][kRedRows][kRed6]
  // XI: the run piece's rotated x, [slab][rows 0..3][16 halfs] (the first half of a slab's fragments)
  __half* xbuf = reinterpret_cast<__half*>(smem + kW6 * ST * kUnitBytes + kW6 * kRedRows * kRed6 * 4);
  // !XI: this warp's ring of the units' x fragments (slot i beside weight slot i: RG x 32 uint2 each)
  uint2* xring = reinterpret_cast<uint2*>(smem + kW6 * ST * kUnitBytes + kW6 * kRedRows * kRed6 * 4) +
                 static_cast<size_t>(warp) * ST * RG * 32;
  const int KT = p.in_features / 16, CB = p.out_features / 128, rows = p.rows;
  const size_t OT = static_cast<size_t>(p.out_features / 16);
  const size_t slab_stride = OT * kTileBytes;  // bytes from one slab's unit to the next
  const uint8_t* tr = reinterpret_cast<const uint8_t*>(p.trellis);

  pdl_launch_dependents();
  // the split: V virtual CTAs; virtual CTA v takes whole units v, v + V, ... below dp, then its run [r0, r1) of the
  // remaining units' slabs laid end to end
  const int V = p.grid;
  const int dp = CB / V * V;
  const int64_t work = static_cast<int64_t>(CB - dp) * KT;
  int64_t run = (work + V - 1) / V;
  run = (run < kMinRun6 ? kMinRun6 : run + 3) & ~int64_t{3};

  LaneWin<N> lwin;
  lwin.init(lane);
  ImmaIndicator ind;
  ind.init(lane);
  const uint32_t g = lane >> 2, q = lane & 3u;
  bool waited = false;
  int vc = static_cast<int>(blockIdx.x);
  int next = vc;
  int64_t r0 = static_cast<int64_t>(vc) * run;
  int64_t r1 = r0 + run < work ? r0 + run : work;
  for (int64_t at = r0;;) {
    int cb, su = 0, k0 = 0, k1 = KT;
    if (next < dp) {
      cb = next;
      next += V;
    } else if (at < r1) {
      su = static_cast<int>(at / KT);
      k0 = static_cast<int>(at - static_cast<int64_t>(su) * KT);
      k1 = static_cast<int>(r1 - at < KT - k0 ? k0 + (r1 - at) : KT);
      at += k1 - k0;
      cb = dp + su;
    } else {
      vc += static_cast<int>(gridDim.x);  // this CTA's next virtual CTA
      if (vc >= V) break;
      next = vc;
      r0 = static_cast<int64_t>(vc) * run;
      r1 = r0 + run < work ? r0 + run : work;
      at = r0;
      continue;
    }
    // segment of this column block
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegments; ++i)
      if (i < p.nseg && cb >= p.seg_cb[i]) s = i;
    int seg_lo = p.seg_cb[0], seg_hi = p.seg_cb[1];
#pragma unroll
    for (int i = 1; i < kMaxSegments; ++i)
      if (i == s) {
        seg_lo = p.seg_cb[i];
        seg_hi = p.seg_cb[i + 1];
      }

    // this warp's slabs: k0 + warp, k0 + warp + 4, ... (k0 and k1 are multiples of four)
    const uint32_t nk = static_cast<uint32_t>(k1 - k0);
    const uint32_t mine = nk > warp ? (nk - warp + kW6 - 1) / kW6 : 0u;
    const uint8_t* src0 = tr + (static_cast<size_t>(k0 + static_cast<int>(warp)) * OT + static_cast<size_t>(cb) * 8u) * kTileBytes;
    // the ring's next slot and source advance by one unit per issue (no per-unit division or 64-bit multiply)
    const uint8_t* src_next = src0;
    const size_t src_step = static_cast<size_t>(kW6) * slab_stride;
    uint32_t slot_next = 0, issued = 0, slot_use = 0;
    // !XI: the prepared fragments of this warp's units (RG x 256 bytes each, kW6 slabs apart), copied into the x
    // ring with their weights once the prepare launch is complete
    const uint8_t* xsrc0 = reinterpret_cast<const uint8_t*>(xf + (static_cast<size_t>(s) * KT + k0 + warp) * RG * 128);
    const uint8_t* xsrc_next = xsrc0;
    constexpr size_t kXStep = static_cast<size_t>(kW6) * RG * 256;
    auto issue = [&]() {
      if (issued < mine) {
        uint8_t* dst = ring + slot_next * kUnitBytes;
#pragma unroll
        for (uint32_t ch = lane; ch < kUnitBytes / 16u; ch += 32u) cp_async16_6(dst + ch * 16u, src_next + ch * 16u);
        src_next += src_step;
        if constexpr (!XI) {
          if (waited && lane < 16u * RG)
            cp_async16_6(reinterpret_cast<uint8_t*>(xring + slot_next * RG * 32) + lane * 16u, xsrc_next + lane * 16u);
          xsrc_next += kXStep;
        }
      }
      ++issued;
      slot_next = slot_next + 1u == static_cast<uint32_t>(ST) ? 0u : slot_next + 1u;
    };
#pragma unroll 1
    for (uint32_t i = 0; i + 1 < static_cast<uint32_t>(ST); ++i) {
      issue();
      cp_async_commit6();
    }
    if (!waited) {  // the prepared x (and, for the stream, nothing else) comes from the prepare launch
      pdl_wait();
      waited = true;
      if (p.tp && blockIdx.x == 0 && tid == 0) {  // the slot's size, for this rank's gather (same on every rank)
        p.tp->meta[p.tp_slot * 4 + 0] = p.tp_meta_cb;
        p.tp->meta[p.tp_slot * 4 + 1] = p.tp_meta_bytes;
      }
      if constexpr (!XI) {
        // the x fragments of the units issued before the wait, into their slots (loads batched, then stores)
        const int pre = static_cast<int>(mine < static_cast<uint32_t>(ST - 1) ? mine : static_cast<uint32_t>(ST - 1));
        const int total = pre * RG * 16;  // uint4s: slot u holds RG x 16 of them, slots contiguous
        for (int base = static_cast<int>(lane); base < total; base += 32 * 8) {
          uint4 v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int idx = base + 32 * u;
            if (idx < total)
              v[u] = __ldcg(reinterpret_cast<const uint4*>(xsrc0 + static_cast<size_t>(idx / (RG * 16)) * kXStep) +
                            idx % (RG * 16));
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int idx = base + 32 * u;
            if (idx < total) reinterpret_cast<uint4*>(xring)[idx] = v[u];
          }
        }
        __syncwarp();
      }
    }
    // x fragments of slab t, row group rg: 32 uint2 at xf + ((s KT + t) RG + rg) 128 halfs; XI: 16 uint2 per slab of
    // xbuf, lanes of rows past the launch's reading zero
    const uint2* xs;
    bool live = true;
    if constexpr (XI) {
      const int b0 = k0 >> 3, nb = ((k1 - 1) >> 3) - b0 + 1;
      // eight of the warp's jobs at a time: their loads are issued before the first rotation (same bits)
      for (int base = static_cast<int>(warp); base < nb * rows; base += kXiBatch * kW6) {
        float v[kXiBatch][4];
#pragma unroll
        for (int u = 0; u < kXiBatch; ++u) {
          const int j = base + u * kW6;
          if (j >= nb * rows) continue;  // (warp-uniform)
          const int blk = b0 + j / rows, r = j % rows, kb = blk * 128;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[u][i] = load_act(p.x, static_cast<size_t>(p.row0 + r) * p.x_row_stride + kb + lane + 32 * i, p.x_dtype);
            if (!p.prepared)
              v[u][i] *= f16_bits_to_float(p.suh[static_cast<size_t>(s) * p.in_features + kb + lane + 32 * i]);
          }
        }
#pragma unroll
        for (int u = 0; u < kXiBatch; ++u) {
          const int j = base + u * kW6;
          if (j >= nb * rows) continue;
          const int blk = b0 + j / rows, r = j % rows;
          if (!p.prepared) {
            fwht128_warp(v[u], lane);
#pragma unroll
            for (int i = 0; i < 4; ++i) v[u][i] *= kHadScale;
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int kin = static_cast<int>(lane) + 32 * i;
            const int t = (blk - b0) * 8 + (kin >> 4), kk = kin & 15;
            xbuf[t * 64 + (r * 4 + (kk >> 2)) * 4 + (kk & 3)] = __float2half_rn(v[u][i]);
          }
        }
      }
      __syncthreads();
      xs = reinterpret_cast<const uint2*>(xbuf) + (k0 + static_cast<int>(warp) - 8 * b0) * 16 + lane;
      live = static_cast<int>(g) < rows;
    } else {
      xs = nullptr;  // (the x ring)
    }
    auto xload = [&](uint32_t i) -> uint2 { return live ? xs[static_cast<size_t>(kW6) * i * 16] : make_uint2(0u, 0u); };
    uint2 xn[RG];
#pragma unroll
    for (int r = 0; r < RG; ++r) xn[r] = (XI && mine > 0) ? xload(0) : make_uint2(0u, 0u);

    float acc[8][RG][4];
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int r = 0; r < RG; ++r)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][r][e] = 0.0f;
#pragma unroll 1
    for (uint32_t i = 0; i < mine; ++i) {
      cp_async_wait6<ST - 2>();
      __syncwarp();
      uint2 xv[RG];
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        if constexpr (XI) {
          xv[r] = xn[r];
          if (i + 1 < mine) xn[r] = xload(i + 1);
        } else {
          xv[r] = xring[(slot_use * RG + r) * 32 + lane];
        }
      }
      const uint32_t* tw = reinterpret_cast<const uint32_t*>(ring + slot_use * kUnitBytes);
      slot_use = slot_use + 1u == static_cast<uint32_t>(ST) ? 0u : slot_use + 1u;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        uint32_t w[8], a[4];
        tile_codewords<N>(tw + t * (kTileBytes / 4u), lwin, w);
        decode_afrag_imma<true>(w, ind, a);
#pragma unroll
        for (int r = 0; r < RG; ++r) mma_16816(acc[t][r], a, xv[r].x, xv[r].y);
      }
      __syncwarp();
      issue();
      cp_async_commit6();
    }
    cp_async_wait6<0>();

    // the warps' partials, summed in warp order
    float* rw = red + warp * kRedRows * kRed6;
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const int col = 16 * t + static_cast<int>(g), row = 8 * r + 2 * static_cast<int>(q);
        if (row < kRedRows) {  // (XI: rows 4..7 are zero)
          rw[row * kRed6 + col] = acc[t][r][0];
          rw[(row + 1) * kRed6 + col] = acc[t][r][1];
          rw[row * kRed6 + col + 8] = acc[t][r][2];
          rw[(row + 1) * kRed6 + col + 8] = acc[t][r][3];
        }
      }
    __syncthreads();
    const bool whole = k0 == 0 && k1 == KT;
    const int64_t u0 = static_cast<int64_t>(su) * KT;  // the unit's first slab in the runs' numbering
    for (int idx = static_cast<int>(tid); idx < rows * 128; idx += kT6) {
      const int at2 = (idx >> 7) * kRed6 + (idx & 127);
      float v = red[at2];
#pragma unroll
      for (int w2 = 1; w2 < kW6; ++w2) v += red[w2 * kRedRows * kRed6 + at2];
      if (whole) red[at2] = v;
      else __stcg(part + (static_cast<size_t>(vc) * 2 + (r0 >= u0 ? 0 : 1)) * kPart6 + idx, v);
    }
    if (!whole) {
      // runs first .. last cover this unit; the one that completes it adds the partials in run order (run c keeps
      // its partial of the unit its run starts in at end 0, of the unit it ends in at end 1)
      const int first = static_cast<int>(u0 / run), last = static_cast<int>((u0 + KT - 1) / run);
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const uint32_t prior = atomicAdd(done + cb, 1u);
        s_last = static_cast<int>(prior) == last - first;
        if (s_last) done[cb] = 0u;  // zero for the next launch
      }
      __syncthreads();
      if (!s_last) continue;
      __threadfence();
      if (XI || rows <= 2) {
        // one or two rows: each thread's element is the sum of the runs' partials in run order (few loads each)
        for (int idx = static_cast<int>(tid); idx < rows * 128; idx += kT6) {
          float v = 0.0f;
          for (int c = first; c <= last; ++c) {
            const int end = static_cast<int64_t>(c) * run >= u0 ? 0 : 1;
            v += __ldcg(part + (static_cast<size_t>(c) * 2 + end) * kPart6 + idx);
          }
          red[(idx >> 7) * kRed6 + (idx & 127)] = v;
        }
      } else {
        // the runs' partials, in run order: as many as the (now idle) rings hold at a time are copied into shared memory
        // together (cp.async, so none of their latency is paid per run), then added into red element by element
        float* stage = reinterpret_cast<float*>(smem);  // the CTA's rings
        const int per = rows * 128;                                                // floats of one run's partial
        const int chunk = static_cast<int>(kW6 * ST * kUnitBytes / 4u) / per;      // runs per pass
        for (int ca = first; ca <= last; ca += chunk) {
          const int cn = last - ca + 1 < chunk ? last - ca + 1 : chunk;
          for (int q4 = static_cast<int>(tid); q4 < cn * per / 4; q4 += kT6) {
            const int c = ca + q4 / (per / 4), e4 = q4 % (per / 4);
            const int end = static_cast<int64_t>(c) * run >= u0 ? 0 : 1;
            cp_async16_6(stage + static_cast<size_t>(q4) * 4,
                         part + (static_cast<size_t>(c) * 2 + end) * kPart6 + static_cast<size_t>(e4) * 4);
          }
          cp_async_commit6();
          cp_async_wait6<0>();
          __syncthreads();
          for (int idx = static_cast<int>(tid); idx < per; idx += kT6) {
            const int at = (idx >> 7) * kRed6 + (idx & 127);
            float v = ca == first ? 0.0f : red[at];
            for (int c = 0; c < cn; ++c) v += stage[c * per + idx];
            red[at] = v;
          }
          __syncthreads();
        }
      }
    }
    __syncthreads();
    // epilogue: one warp per row
    const int seg_c0 = seg_lo * 128, seg_w = (seg_hi - seg_lo) * 128;
    for (int row = static_cast<int>(warp); row < rows; row += kW6) {
      const size_t grow = static_cast<size_t>(p.row0 + row);
      const size_t ybase = p.nseg == 1 ? grow * p.y_row_stride
                                       : static_cast<size_t>(p.rows_total) * seg_c0 + grow * seg_w - seg_c0;
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = red[row * kRed6 + lane + 32 * k];
      if (!p.inner_only) {
        fwht128_warp(v, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = v[k] * kHadScale * f16_bits_to_float(p.svh[cb * 128 + lane + 32 * k]);
      }
      if (p.tp) {
        // column-parallel exchange: the row's 128 outputs through a staging row in the (idle) ring, then 16-byte
        // stores into this step's slot of every rank (the step's gather publishes them)
        const TpDev& tp = *p.tp;
        const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(tp.step);
        const size_t esize = p.y_dtype == kF32 ? 4 : 2;
        const size_t slot_off = (static_cast<size_t>(step & 1u) * tp.slots + p.tp_slot) * tp.slot_bytes;
        int64_t tot = p.tp_total[0], c0 = p.tp_col0[0], sb = p.tp_seg_base[0];
#pragma unroll
        for (int i = 1; i < kMaxSegments; ++i)
          if (i == s) {
            tot = p.tp_total[i];
            c0 = p.tp_col0[i];
            sb = p.tp_seg_base[i];
          }
        uint8_t* stage = smem + warp * 512u;
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) store_act(stage, lane + 32 * k, v[k], p.y_dtype);
        __syncwarp();
        const int64_t col = c0 + (static_cast<int64_t>(cb) * 128 - seg_c0);  // first gathered column of this block
        const size_t at = static_cast<size_t>(sb + static_cast<int64_t>(p.row0 + row) * tot + col) * esize;
        if (lane * 16u < 128u * esize) {
          const uint4 chunk = reinterpret_cast<const uint4*>(stage)[lane];
          for (int q2 = 0; q2 < tp.world; ++q2) reinterpret_cast<uint4*>(tp.y[q2] + slot_off + at)[lane] = chunk;
        }
        __syncwarp();
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) store_act(p.y, ybase + static_cast<size_t>(cb) * 128 + lane + 32 * k, v[k], p.y_dtype);
      }
    }
    __syncthreads();
  }
}

template <int N, int RG, bool XI>
cudaError_t launch6_t(const GemvParams& p, int sms, __half* xf, float* part, uint32_t* done, cudaStream_t st) {
  constexpr int ST = stages6x<N, RG, XI>();
  auto kern = gemv6_kernel<N, RG, ST, XI>;
  const size_t smem = static_cast<size_t>(kW6) * ST * 8u * 2u * N +
                      static_cast<size_t>(kW6) * (XI ? kXiRows : 8 * RG) * kRed6 * 4 +
                      (XI ? kXiSlabs * 128 : static_cast<size_t>(kW6) * ST * RG * 256);
  static KernelSetup setup;
  int per_sm = 0;  // resident CTAs per SM (at most kVirt6): the persistent grid is exactly one wave
  if (cudaError_t e = kernel_setup(setup, kern, kT6, smem, false, &per_sm, kVirt6); e != cudaSuccess) return e;
  GemvParams q = p;
  q.grid = sms * kVirt6;  // the virtual CTAs the work is cut for
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sms * per_sm));
  cfg.blockDim = dim3(kT6);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, q, static_cast<const __half*>(xf), part, done);
}

template <int RG, bool XI>
cudaError_t launch6_k(const GemvParams& p, int n, int sms, __half* xf, float* part, uint32_t* done, cudaStream_t st) {
  cudaError_t e = cudaErrorInvalidValue;
  with_rate(n, [&](auto N) { e = launch6_t<decltype(N)::value, RG, XI>(p, sms, xf, part, done, st); });
  return e;
}

// The kernel's run length for V virtual CTAs, and whether every unit is split (no whole units round-robin).
void split6(const GemvParams& p, int sms, int64_t* run, bool* all_runs) {
  const int V = sms * kVirt6, CB = p.out_features / 128, KT = p.in_features / 16;
  const int dp = CB / V * V;
  const int64_t work = static_cast<int64_t>(CB - dp) * KT;
  int64_t r = (work + V - 1) / V;
  *run = (r < kMinRun6 ? kMinRun6 : r + 3) & ~int64_t{3};
  *all_runs = dp == 0;
}

}  // namespace

size_t gemv6_scratch_bytes(const GemvParams& p, int sms) {
  const size_t xf = static_cast<size_t>(p.nseg) * p.in_features * 32;  // [nseg][in/16][2][128 halfs]
  const size_t parts = static_cast<size_t>(sms) * kVirt6 * 2 * kPart6 * 4;
  return ((xf + 255) & ~size_t{255}) + parts;
}

size_t gemv_prep_bytes(const GemvParams& p, int row_groups) {
  return static_cast<size_t>(p.nseg) * (p.in_features / 16) * row_groups * 256;
}

cudaError_t launch_gemv_prep(const GemvParams& p, int row_groups, void* xf, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.in_features / 128), static_cast<unsigned>(p.nseg));
  cfg.blockDim = dim3(256 * row_groups);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  __half* dst = static_cast<__half*>(xf);
  return row_groups == 1 ? cudaLaunchKernelEx(&cfg, gemv6_prep_kernel<1>, p, dst)
                         : cudaLaunchKernelEx(&cfg, gemv6_prep_kernel<2>, p, dst);
}

bool gemv6_prefers(const GemvParams& p) {
  const int cb = p.out_features / 128;
  const int64_t slabs = static_cast<int64_t>(cb) * (p.in_features / 16);
  return slabs >= kGemv6MinSlabs || (p.in_features >= 8192 && slabs >= kGemv6MinSlabsDeep) ||
         (cb <= kGemv6NarrowCb && slabs >= kGemv6NarrowSlabs);
}

cudaError_t launch_gemv6(const GemvParams& p, int n, int sms, void* scratch, uint32_t* counters, cudaStream_t st) {
  if (p.cw_mask || p.mcg) return cudaErrorInvalidValue;  // narrowed windows and mcg take the cluster-split GEMV
  if (p.rows < 1 || p.rows > 16) return cudaErrorInvalidValue;
  const int rg = p.rows <= 8 ? 1 : 2;
  __half* xf = static_cast<__half*>(scratch);
  const size_t xf_bytes = static_cast<size_t>(p.nseg) * p.in_features * 32;
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + ((xf_bytes + 255) & ~size_t{255}));
  int64_t run = 0;
  bool all_runs = false;
  split6(p, sms, &run, &all_runs);
  // measurement override: EXL3_GEMV_XI = the most rows that rotate in-CTA (0 .. kXiRows)
  int xi_rows = kXiTake;
  if (const char* e = getenv("EXL3_GEMV_XI")) xi_rows = atoi(e) < kXiRows ? atoi(e) : kXiRows;
  if (p.rows <= xi_rows && all_runs && run <= kXiSlabs - 8)  // each CTA rotates its runs' inputs itself
    return launch6_k<1, true>(p, n, sms, xf, part, counters, st);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.in_features / 128), static_cast<unsigned>(p.nseg));
  cfg.blockDim = dim3(256 * rg);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = rg == 1 ? cudaLaunchKernelEx(&cfg, gemv6_prep_kernel<1>, p, xf)
                          : cudaLaunchKernelEx(&cfg, gemv6_prep_kernel<2>, p, xf);
  if (e != cudaSuccess) return e;
  return rg == 1 ? launch6_k<1, false>(p, n, sms, xf, part, counters, st)
                 : launch6_k<2, false>(p, n, sms, xf, part, counters, st);
}

}  // namespace exl3
