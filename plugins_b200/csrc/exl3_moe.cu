// exl3_moe.cu -- routed SwiGLU experts (the reference's swiglu seam, plugins/turboexl3_ds41/plugin.zig:267-283;
// SX/root.zig:32-167; the decode chain of SX/expert_exl3_kernels.zig:2274-2650).
//
// Per (row r, top-k slot k), e = inds[r, k]:
//   g = gate_e(x_r), u = up_e(x_r)                        (EXL3 linears: prepare, decode GEMV, finish)
//   g = min(g, limit), u = clamp(u, -limit, limit)        when limit > 0   (MID_SOURCE's CLAMP_LIMIT)
//   h = silu(g) * u
//   y_r = sum_k score[r, k] * down_e(h)                   f32, k order (REDUCE_SOURCE)
//
// B200 plan, five launches chained with programmatic dependent launch, rows in passes of 512 / topk:
//   1. route    -- one CTA: a stable counting sort of the slots by expert (deterministic; each slot placed by its
//                  own thread, its position kept for the combine), cut into chunks of at most 8 slots of one expert
//                  (the MMA's N), the active chunk list on the device;
//   2. prepare  -- each chunk's rows rotated for gate and for up (suh, 128-wide Hadamard, f16) into B-fragment order;
//   3. gate|up  -- a persistent decode GEMV over (chunk, 128-column block of the intermediate) units that streams
//                  the expert's gate and up tiles together (both contiguous per k slab), accumulates both, and in
//                  the epilogue applies both finishes, the clamp, SwiGLU and the down projection's prepare (its
//                  128-wide input block is exactly this column block), writing the down GEMV's B fragments;
//   4. down     -- the same GEMV over (chunk, 128-column block of the hidden size), finishing to f32 per slot;
//   5. combine  -- y_r = sum_k score * d in k order, in x's dtype.
// Work split: every unit's k range is cut into the same runs in every call (at most kMaxRuns runs of about 128 slabs,
// set by the input width alone).  Whole units go round-robin over the persistent grid while every CTA gets one
// (neighbouring CTAs stream the same expert's k slabs together); the remaining units' runs, laid end to end, are cut
// into one equal range per CTA, so every CTA streams about the same bytes however few experts a call touches.  Each
// warp sums a run's slabs from zero in its MMA accumulators and adds the run to its running total in run order; a
// unit's value is the warps' totals in warp order.  A unit that two or more CTAs share is finished by the CTA that
// completes it last (a per-unit counter): it continues each warp's total of the first CTA's runs with the later
// runs, one by one in run order, then sums the warps -- the same sums a whole unit makes.  So the order of every
// sum is fixed by the input width and the tile layout, never by the routing, the grid or timing: a slot's output
// has the same bytes whatever other rows and experts share the call (the reference checks its expert kernels for
// this row invariance, plugins/turboexl3_ds41/src/exl3/selfcheck.zig:755-851).
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>
#include <new>

#include "exl3_common.cuh"
#include "exl3_internal.h"
#include "exl3_moe.h"

namespace exl3 {

namespace {

constexpr int kMaxTopK = 32;       // the reference's REDUCE_MAX_TOPK (SX/expert_exl3_kernels.zig:2593)
constexpr int kMaxSlots = 512;     // (row, k) slots per pass: a pass takes kMaxSlots / topk rows
constexpr int kChunkRows = 8;      // slots per chunk: the MMA's N
constexpr int kWarpsM = 4;
constexpr int kStagesM = 4;
constexpr int kRedStrideM = 132;
constexpr int kMaxRuns = 8;         // runs per unit at most (the partial slots a CTA may need)

// A unit's run length in slabs for kt slabs of input: about 128 (32 per warp), a multiple of four, at most kMaxRuns
// runs (the last one shorter).  Measured on config 4's banks (256 experts, 32 tokens, top-8): runs of about 32 slabs
// 1641 us, 64 slabs 1340 us, 128 slabs 1177 us -- fewer runs mean fewer flushes of the accumulators and fewer units
// shared between CTAs (their partials and the last CTA's fix-up).
constexpr int kRunSlabs = 128;
__host__ __device__ constexpr int moe_run_slabs(int kt) {
  const int r = (kt + kRunSlabs - 1) / kRunSlabs < kMaxRuns ? (kt + kRunSlabs - 1) / kRunSlabs : kMaxRuns;
  return ((kt + r - 1) / r + 3) & ~3;
}
constexpr int kPrepChunks = 48;     // prepare: chunk columns of the grid
constexpr int kCombineRows = 64;    // combine: row columns of the grid
constexpr int kIntsM = 5 * kMaxSlots + 64;  // the route's ints: order, chunk_e/s/n, pos, nchunks, bad

struct MoeParams {
  // banks: trellis [E][in/16][out/16][n], suh [E][in], svh [E][out]
  const uint16_t *g_tr, *g_suh, *g_svh;
  const uint16_t *u_tr, *u_suh, *u_svh;
  const uint16_t *d_tr, *d_suh, *d_svh;
  int32_t experts, hidden, inter;
  // column-parallel experts (every rank holds a column slice of every expert): inter_full is the down input's width
  // and inter_off the first column of this rank's gate/up slice in it; hidden_out the down bank's (sliced) output
  // width.  A single-device call has inter_full = inter, inter_off = 0, hidden_out = hidden.
  int32_t inter_full, inter_off, hidden_out;
  uint8_t* hp_dst[8];  // every rank's down-input buffer (same layout as hp) when hp_world > 0
  int32_t hp_world;
  int32_t max_cb;     // column blocks the unit_done array holds per chunk
  uint32_t cw_mask_gu, cw_mask_d;  // gate|up's and down's narrowed codeword window masks (0: the full 16 bits)
  int32_t mcg_gu, mcg_d;           // gate|up's and down's codebook is mcg (else mul1)
  const void* x;      // [rows][hidden]
  int32_t x_dtype;
  const void* inds;   // [rows][topk]
  int32_t inds_u32;
  const float* scores;  // [rows][topk] f32
  void* y;            // [rows][hidden], in y_dtype (x's dtype or f32)
  int32_t y_dtype;
  int32_t rows, topk, row0;  // this pass: rows row0 .. row0 + rows - 1 of the call
  float limit;
  // scratch
  int32_t* order;      // [kMaxSlots] slot ids sorted by expert (stable)
  int32_t* pos;        // [kMaxSlots] slot id -> its position in `order` (-1: absent)
  int32_t* chunk_e;    // [kMaxSlots] chunk -> expert
  int32_t* chunk_s;    // [kMaxSlots] chunk -> first position in `order`
  int32_t* chunk_n;    // [kMaxSlots] chunk -> slots
  int32_t* nchunks;    // [1]
  int32_t* bad;        // [1] an expert index out of range was seen
  uint8_t* xg;         // [chunk][hidden/16][256 B] gate-prepared rows
  uint8_t* xu;         // [chunk][hidden/16][256 B] up-prepared rows
  uint8_t* hp;         // [chunk][inter/16][256 B] down-prepared rows
  float* dout;         // [kMaxSlots][hidden] down outputs per slot (position in `order`)
  float* part;         // [grid][P runs][4 warps][2 weights][8][128] sums of the units a CTA shares with others: slots
                       // 0 .. P - 2 the runs of a unit it joins after its first run, P - 1 the warps' totals of the
                       // unit it starts but does not finish
  int32_t* unit_done;  // [2 launches][kMaxSlots * max CB] runs finished per unit (each reset by its unit's last run)
  // the shared expert folded into the combine (exl3_swiglu_shared): y = RN(RN(routed) + g), g = shared or, gated,
  // RN(RN(sigmoid(logit)) * shared); RN rounds to x's dtype (y_dtype == x_dtype)
  const void* shared;       // [rows][hidden] in x's dtype, or null (no fold)
  const void* sh_logit;     // [rows] in x's dtype, or null
  const void* sh_gate_vec;  // [hidden] in x's dtype: logit = RN(x . gate_vec), or null
  const void* sigtab;       // [65536] in x's dtype (16-bit activations), or null: sigmoid in f32, rounded
};

__device__ __forceinline__ int slot_expert(const MoeParams& p, int slot) {
  const int r = slot / p.topk, k = slot % p.topk;
  const size_t at = static_cast<size_t>(p.row0 + r) * p.topk + k;
  return p.inds_u32 ? static_cast<int>(static_cast<const uint32_t*>(p.inds)[at]) : static_cast<const int32_t*>(p.inds)[at];
}

// fragment position (IMMA order) of input element kk (0..15) of row g in a slab: halves
__device__ __forceinline__ int frag_half(int g, int kk) { return (g * 4 + (kk >> 2)) * 4 + (kk & 3); }

// ---------------------------------------------------------------- 1. route

// Block-wide exclusive scan of one int per thread (1024 threads); *total receives the sum.
__device__ int scan_excl_1024(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += y;
    }
    s_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  *total = s_warp[31];
  return x - v + (warp > 0 ? s_warp[warp - 1] : 0);
}

// One CTA of 1024 threads.  Slot s (< S <= kMaxSlots) of expert e goes to position off[e] + (the slots before s of
// expert e): a stable counting sort, every slot placed by its own thread.
__global__ void __launch_bounds__(1024) moe_route_kernel(MoeParams p) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int s_cnt[1024], s_off[1024], s_warp[32];
  __shared__ int16_t s_e[kMaxSlots];
  const int tid = threadIdx.x;
  const int S = p.rows * p.topk;
  const int E = p.experts;
  s_cnt[tid] = 0;
  if (tid == 0) *p.bad = 0;
  __syncthreads();
  for (int s = tid; s < S; s += blockDim.x) {
    const int e = slot_expert(p, s);
    if (e < 0 || e >= E) {
      atomicExch(p.bad, 1);
      s_e[s] = -1;
    } else {
      s_e[s] = static_cast<int16_t>(e);
      atomicAdd(&s_cnt[e], 1);
    }
  }
  __syncthreads();
  // slots and chunks before expert `tid` (both sums <= kMaxSlots: packed in one int)
  const int cnt = tid < E ? s_cnt[tid] : 0;
  const int nch = (cnt + kChunkRows - 1) / kChunkRows;
  int total;
  const int both = scan_excl_1024(cnt | (nch << 16), s_warp, &total);
  const int off = both & 0xffff, cho = both >> 16;
  s_off[tid] = off;
  for (int j = 0; j < nch; ++j) {
    p.chunk_e[cho + j] = tid;
    p.chunk_s[cho + j] = off + j * kChunkRows;
    p.chunk_n[cho + j] = min(kChunkRows, cnt - j * kChunkRows);
  }
  if (tid == 0) *p.nchunks = total >> 16;
  __syncthreads();
  for (int s = tid; s < S; s += blockDim.x) {
    const int e = s_e[s];
    int at = -1;
    if (e >= 0) {
      at = s_off[e];
      for (int s2 = 0; s2 < s; ++s2) at += s_e[s2] == e;
      p.order[at] = s;
    }
    p.pos[s] = at;
  }
  // positions past the placed slots (absent slots leave them) are marked
  for (int i = (total & 0xffff) + tid; i < S; i += blockDim.x) p.order[i] = -1;
}

// ---------------------------------------------------------------- 2. prepare gate / up inputs

// grid: (hidden/128 blocks, up to kPrepChunks); CTA (b, c) prepares block b of chunks c, c + gridDim.y, ...; warp w
// handles rows w, w+4 of a chunk
__global__ void __launch_bounds__(128) moe_prep_kernel(MoeParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int nchunks = *p.nchunks;
  for (int chunk = blockIdx.y; chunk < nchunks; chunk += gridDim.y) {
    const int e = p.chunk_e[chunk], s0 = p.chunk_s[chunk], n = p.chunk_n[chunk];
    const int blk = blockIdx.x;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const int KT = p.hidden / 16;
    for (int g = warp; g < kChunkRows; g += 4) {
      for (int which = 0; which < 2; ++which) {
        const uint16_t* suh = (which == 0 ? p.g_suh : p.u_suh) + static_cast<size_t>(e) * p.hidden;
        uint8_t* dst = (which == 0 ? p.xg : p.xu) + static_cast<size_t>(chunk) * KT * 256;
        float v[4];
        if (g < n) {
          const int row = p.order[s0 + g] / p.topk;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const size_t k = static_cast<size_t>(blk) * 128 + lane + 32 * i;
            v[i] = load_act(p.x, static_cast<size_t>(p.row0 + row) * p.hidden + k, p.x_dtype) * f16_bits_to_float(suh[k]);
          }
          fwht128_warp(v, lane);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = 0.0f;
        }
        __half* h = reinterpret_cast<__half*>(dst);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kin = lane + 32 * i;
          const int t = blk * 8 + (kin >> 4);
          h[static_cast<size_t>(t) * 128 + frag_half(g, kin & 15)] = __float2half_rn(v[i] * kHadScale);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- 3/4. the grouped decode GEMV

__device__ __forceinline__ void cp16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// PAIR: units (chunk, intermediate column block), weights gate+up, epilogue SwiGLU + down prepare.
// !PAIR: units (chunk, hidden column block), weight down, epilogue finish to f32.
template <int N, bool PAIR, int DS>
__global__ void __launch_bounds__(kWarpsM * 32, 2) moe_gemv_kernel(MoeParams p) {
  constexpr uint32_t kTileBytes = 2u * N;
  constexpr uint32_t kW = 8u * kTileBytes;                // one weight's tiles of a unit slab
  constexpr uint32_t kSlab = (PAIR ? 2u : 1u) * (kW + 256u);  // tiles + x fragments, per weight
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  uint8_t* ring = smem + warp * (kStagesM * kSlab);
  float* red = reinterpret_cast<float*>(smem + kWarpsM * kStagesM * kSlab);  // [2][W][8][stride]
  const int in_f = PAIR ? p.hidden : p.inter_full;
  const int out_f = PAIR ? p.inter : p.hidden_out;
  const int KT = in_f / 16, CB = out_f / 128;
  const size_t wstride = static_cast<size_t>(in_f / 16) * (out_f / 16) * kTileBytes;  // bytes per expert
  const uint8_t* tra = reinterpret_cast<const uint8_t*>(PAIR ? p.g_tr : p.d_tr);
  const uint8_t* trb = reinterpret_cast<const uint8_t*>(p.u_tr);
  const uint8_t* xa = PAIR ? p.xg : p.hp;
  const uint8_t* xb = p.xu;

  __shared__ int s_last;
  pdl_launch_dependents();
  pdl_wait();  // the chunk table and the prepared inputs come from the previous launches
  const int units = *p.nchunks * CB;
  LaneWin<N> lwin;
  lwin.init(lane);
  lwin.mask = spec_mask(PAIR ? p.cw_mask_gu : p.cw_mask_d);
  ImmaIndicator ind;
  ind.init(lane);
  ImmaWin<N> iwin;
  if constexpr (DS == 2) iwin.init(lane, lwin.mask);
  const uint32_t g = lane >> 2, q = lane & 3u;
  // Every unit's k range is cut the same way whatever the call: P runs of L slabs (the last run shorter), a warp's
  // slabs of a run summed from zero in its MMA accumulators, the warp's runs added in run order, then the warps in
  // warp order.  Whole units go round-robin while every CTA gets one (dp of them); the remaining units' runs, laid
  // end to end, are cut into one equal range [R0, R1) per CTA.
  const int G = static_cast<int>(gridDim.x);
  const int L = moe_run_slabs(KT), P = (KT + L - 1) / L, Lw = L / kWarpsM;
  const int dp = units / G * G;
  const int64_t sk_runs = static_cast<int64_t>(units - dp) * P;
  const int64_t per = sk_runs > 0 ? (sk_runs + G - 1) / G : 1;
  const int64_t R0 = static_cast<int64_t>(blockIdx.x) * per;
  const int64_t R1 = R0 + per < sk_runs ? R0 + per : sk_runs;
  int32_t* done = p.unit_done + (PAIR ? 0 : kMaxSlots * static_cast<int64_t>(p.max_cb));
  constexpr int kPart = (PAIR ? 2 : 1) * 8 * 128;  // one warp's sums of a unit: [weight][row][column]

  int next = static_cast<int>(blockIdx.x);
  for (int64_t at = R0;;) {
    int unit, su = 0, ra = 0, rb = P;  // this item: runs ra .. rb - 1 of the unit
    if (next < dp) {
      unit = next;
      next += G;
    } else if (at < R1) {
      su = static_cast<int>(at / P);
      ra = static_cast<int>(at - static_cast<int64_t>(su) * P);
      rb = static_cast<int>(R1 - at < P - ra ? ra + (R1 - at) : P);
      at += rb - ra;
      unit = dp + su;
    } else {
      break;
    }
    const int k0 = ra * L, k1 = rb * L < KT ? rb * L : KT;
    const int chunk = unit / CB, cb = unit % CB;
    const int e = p.chunk_e[chunk], s0 = p.chunk_s[chunk], nrow = p.chunk_n[chunk];
    const uint8_t* wa = tra + e * wstride + static_cast<size_t>(cb) * 8u * kTileBytes;
    const uint8_t* wb = trb + e * wstride + static_cast<size_t>(cb) * 8u * kTileBytes;
    const uint8_t* xca = xa + static_cast<size_t>(chunk) * KT * 256;
    const uint8_t* xcb = xb + static_cast<size_t>(chunk) * KT * 256;
    const size_t rowstride = static_cast<size_t>(CB) * 8u * kTileBytes;  // bytes between k slabs
    // this warp's slabs of the item: k0 + warp, k0 + warp + 4, ... (k0 and k1 are multiples of four); every run
    // gives each warp L / 4 of them (the unit's last run fewer: it ends the item)
    const uint32_t nk = static_cast<uint32_t>(k1 - k0);
    const uint32_t mine = nk > warp ? (nk - warp + kWarpsM - 1) / kWarpsM : 0u;
    auto issue = [&](uint32_t i) {
      if (i >= mine) return;
      const uint32_t t = static_cast<uint32_t>(k0) + warp + kWarpsM * i;
      uint8_t* dst = ring + (i % kStagesM) * kSlab;
#pragma unroll
      for (uint32_t c = lane; c < kW / 16u; c += 32u) cp16(dst + c * 16u, wa + t * rowstride + c * 16u);
      if (lane < 16u) cp16(dst + kW + lane * 16u, xca + static_cast<size_t>(t) * 256 + lane * 16u);
      if constexpr (PAIR) {
        uint8_t* d2 = dst + kW + 256u;
#pragma unroll
        for (uint32_t c = lane; c < kW / 16u; c += 32u) cp16(d2 + c * 16u, wb + t * rowstride + c * 16u);
        if (lane < 16u) cp16(d2 + kW + lane * 16u, xcb + static_cast<size_t>(t) * 256 + lane * 16u);
      }
    };
    for (uint32_t i = 0; i + 1 < static_cast<uint32_t>(kStagesM); ++i) {
      issue(i);
      cp_commit();
    }
    float acc[PAIR ? 2 : 1][8][4];
#pragma unroll
    for (int w2 = 0; w2 < (PAIR ? 2 : 1); ++w2)
#pragma unroll
      for (int t = 0; t < 8; ++t)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[w2][t][c] = 0.0f;
    // run r's sums of this warp leave the accumulators: into the warp's running total in shared memory when this CTA
    // holds the unit from its first run, else into this CTA's slot for run r in global memory (the unit's last CTA
    // adds them in run order); no barrier, the ring keeps streaming
    auto flush = [&](int r) {
      // (ra > 0) this CTA's slot for run r: its offset in the CTA's range, below P - 1
      const int64_t slot = ra > 0 ? static_cast<int64_t>(su) * P + r - R0 : 0;
      float* gw = p.part + ((static_cast<size_t>(blockIdx.x) * P + static_cast<size_t>(slot)) * kWarpsM + warp) * kPart;
#pragma unroll
      for (int w2 = 0; w2 < (PAIR ? 2 : 1); ++w2) {
        float* rw = red + (w2 * kWarpsM + warp) * 8 * kRedStrideM;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int row = 2 * static_cast<int>(q) + (c & 1), col = 16 * t + static_cast<int>(g) + 8 * (c >> 1);
            if (ra == 0) {
              float& tot = rw[row * kRedStrideM + col];
              tot = r == 0 ? acc[w2][t][c] : tot + acc[w2][t][c];
            } else {
              __stcg(gw + w2 * 1024 + row * 128 + col, acc[w2][t][c]);
            }
            acc[w2][t][c] = 0.0f;
          }
        }
      }
    };
    int run = ra, left = Lw;
    for (uint32_t i = 0; i < mine; ++i) {
      cp_wait<kStagesM - 2>();
      __syncwarp();
      const uint8_t* st = ring + (i % kStagesM) * kSlab;
#pragma unroll
      for (int w2 = 0; w2 < (PAIR ? 2 : 1); ++w2) {
        const uint8_t* sw = st + w2 * (kW + 256u);
        const uint2 xv = reinterpret_cast<const uint2*>(sw + kW)[lane];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          uint32_t a[4];  // (mul1 pairs packed on the FMA pipe: measured 2.5 % faster)
          decode_tile_imma<N, DS, true>(reinterpret_cast<const uint32_t*>(sw) + t * (kTileBytes / 4u), lwin, iwin, ind, a);
          mma_16816(acc[w2][t], a, xv.x, xv.y);
        }
      }
      __syncwarp();
      issue(i + kStagesM - 1);
      cp_commit();
      if (--left == 0 && i + 1 < mine) {
        flush(run++);
        left = Lw;
      }
    }
    cp_wait<0>();
    flush(run);  // the item's last run (rb - 1)
    __half* stage = reinterpret_cast<__half*>(smem);  // warp 0's ring, drained: the down-input block's staging (2 KiB)
    __syncthreads();
    if (ra == 0 && rb == P) {
      // a whole unit: the warps' totals in warp order
      for (int idx = tid; idx < kPart; idx += kWarpsM * 32) {
        const int w2 = idx / 1024, row = (idx / 128) % 8, col = idx % 128;
        float v = 0.0f;
#pragma unroll
        for (int w3 = 0; w3 < kWarpsM; ++w3) v += red[((w2 * kWarpsM + w3) * 8 + row) * kRedStrideM + col];
        red[((w2 * kWarpsM) * 8 + row) * kRedStrideM + col] = v;
      }
    } else {
      // a unit shared with other CTAs: CTAs cf .. cl of the grid hold its runs; cf, which holds runs 0 .. j0, keeps
      // every warp's total of them in its slot P - 1, the others each run in its own slot; the last to finish adds
      // each warp's runs in run order onto that total, then the warps in warp order -- the sums a whole unit makes
      if (ra == 0)
        for (int idx = tid; idx < kWarpsM * kPart; idx += kWarpsM * 32) {
          const int w3 = idx / kPart, w2 = (idx % kPart) / 1024, row = (idx / 128) % 8, col = idx % 128;
          __stcg(p.part + (static_cast<size_t>(blockIdx.x) * P + P - 1) * kWarpsM * kPart + idx,
                 red[((w2 * kWarpsM + w3) * 8 + row) * kRedStrideM + col]);
        }
      const int64_t u0 = static_cast<int64_t>(su) * P;  // the unit's first run in the ranges' numbering
      const int cf = static_cast<int>(u0 / per), cl = static_cast<int>((u0 + P - 1) / per);
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const int prior = atomicAdd(done + unit, 1);
        s_last = prior == cl - cf;
        if (s_last) done[unit] = 0;  // ready for the next call
      }
      __syncthreads();
      if (!s_last) continue;
      __threadfence();
      const int j0 = static_cast<int>((static_cast<int64_t>(cf) + 1) * per - 1 - u0);  // < P - 1: cf ends inside
      for (int idx = tid; idx < kPart; idx += kWarpsM * 32) {
        const int w2 = idx / 1024, row = (idx / 128) % 8, col = idx % 128;
        float v = 0.0f;
        for (int w3 = 0; w3 < kWarpsM; ++w3) {
          float tw = __ldcg(p.part + ((static_cast<size_t>(cf) * P + P - 1) * kWarpsM + w3) * kPart + idx);
          for (int r = j0 + 1; r < P; ++r) {
            const int64_t R = u0 + r, c = R / per;
            tw += __ldcg(p.part + ((static_cast<size_t>(c) * P + static_cast<size_t>(R - c * per)) * kWarpsM + w3) *
                                      kPart + idx);
          }
          v += tw;
        }
        red[((w2 * kWarpsM) * 8 + row) * kRedStrideM + col] = v;
      }
    }
    if constexpr (PAIR)  // rows of the chunk beyond its slots stay zero in the down input
      for (int v = static_cast<int>(tid); v < 128; v += kWarpsM * 32) reinterpret_cast<uint4*>(stage)[v] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    // epilogue: one warp per slot row
    for (int row = static_cast<int>(warp); row < nrow; row += kWarpsM) {
      float va[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) va[i] = red[row * kRedStrideM + lane + 32 * i];
      fwht128_warp(va, lane);
      const size_t ce = static_cast<size_t>(cb) * 128;
      if constexpr (PAIR) {
        float vb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) vb[i] = red[((kWarpsM * 8) + row) * kRedStrideM + lane + 32 * i];
        fwht128_warp(vb, lane);
        float h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const size_t c = ce + lane + 32 * i;
          float gv = va[i] * kHadScale * f16_bits_to_float(p.g_svh[static_cast<size_t>(e) * p.inter + c]);
          float uv = vb[i] * kHadScale * f16_bits_to_float(p.u_svh[static_cast<size_t>(e) * p.inter + c]);
          if (p.limit > 0.0f) {
            gv = fminf(gv, p.limit);
            uv = fminf(fmaxf(uv, -p.limit), p.limit);
          }
          const float sig = 1.0f / (1.0f + __expf(-gv));
          h[i] = gv * sig * uv *
                 f16_bits_to_float(p.d_suh[static_cast<size_t>(e) * p.inter_full + p.inter_off + c]);
        }
        fwht128_warp(h, lane);
        __half* dst = stage;  // this block's 8 slabs of the down input, [8][128 halfs]
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kin = lane + 32 * i;
          dst[(kin >> 4) * 128 + frag_half(row, kin & 15)] = __float2half_rn(h[i] * kHadScale);
        }
      } else {
        float* dst = p.dout + static_cast<size_t>(s0 + row) * p.hidden_out;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const size_t c = ce + lane + 32 * i;
          dst[c] = va[i] * kHadScale * f16_bits_to_float(p.d_svh[static_cast<size_t>(e) * p.hidden_out + c]);
        }
      }
    }
    if constexpr (PAIR) {
      // the staged block (rows past the chunk's slots zero) -> the down input of this rank, or of every rank, with
      // 16-byte stores: slabs (inter_off / 128 + cb) * 8 .. + 7 of the chunk, contiguous
      __syncthreads();
      const size_t at = (static_cast<size_t>(chunk) * (p.inter_full / 16) + (p.inter_off / 128 + cb) * 8) * 256;
      const uint4* src = reinterpret_cast<const uint4*>(stage);
      if (p.hp_world > 0) {
        for (int q2 = 0; q2 < p.hp_world; ++q2)
          for (int v = static_cast<int>(tid); v < 128; v += kWarpsM * 32)
            reinterpret_cast<uint4*>(p.hp_dst[q2] + at)[v] = src[v];
      } else {
        for (int v = static_cast<int>(tid); v < 128; v += kWarpsM * 32) reinterpret_cast<uint4*>(p.hp + at)[v] = src[v];
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- 5. combine

__device__ __forceinline__ float round_act(float v, int32_t dt) {
  if (dt == kF16) return __half2float(__float2half_rn(v));
  if (dt == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}

__device__ __forceinline__ uint16_t act_bits16(float v, int32_t dt) {
  return dt == kF16 ? __half_as_ushort(__float2half_rn(v)) : __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// The shared gate of row `row` as sigmoid(logit) in x's dtype (SX/root.zig:50-68: MLX's sigmoid of the logit's
// 16-bit pattern where the host gives its table).  With a gate vector every CTA of the row sums x . gate_vec in the
// same fixed order (each thread a strided run, then the warps in order), so all agree; every thread must call it.
__device__ float shared_gate(const MoeParams& p, int row, float* s_red) {
  float logit;
  if (p.sh_logit) {
    logit = load_act(p.sh_logit, static_cast<size_t>(row), p.x_dtype);
  } else {
    float part = 0.0f;
    for (int d = static_cast<int>(threadIdx.x); d < p.hidden; d += 128)
      part += load_act(p.x, static_cast<size_t>(row) * p.hidden + d, p.x_dtype) * load_act(p.sh_gate_vec, d, p.x_dtype);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xFFFFFFFFu, part, o);
    __syncthreads();  // s_red is free (the previous row's readers are past it)
    if ((threadIdx.x & 31u) == 0) s_red[threadIdx.x >> 5] = part;
    __syncthreads();
    logit = round_act(((s_red[0] + s_red[1]) + s_red[2]) + s_red[3], p.x_dtype);
  }
  if (p.sigtab)
    return load_act(p.sigtab, act_bits16(logit, p.x_dtype), p.x_dtype);
  return round_act(1.0f / (1.0f + expf(-logit)), p.x_dtype);
}

// grid: (ceil(hidden/512), up to kCombineRows), 128 threads of four columns each; y[r] = sum_k score[r,k] *
// dout[pos(r,k)], k in order; with a shared expert, y[r] = RN(RN(that sum) + g) (exl3_swiglu_shared)
__global__ void __launch_bounds__(128) moe_combine_kernel(MoeParams p) {
  __shared__ float s_red[4];
  pdl_wait();
  pdl_launch_dependents();
  const size_t c = (static_cast<size_t>(blockIdx.x) * 128 + threadIdx.x) * 4;
  const bool live = c < static_cast<size_t>(p.hidden_out);  // (a multiple of 128: c + 3 < hidden_out when live)
  const bool gated = p.shared && (p.sh_logit || p.sh_gate_vec);
  for (int r = blockIdx.y; r < p.rows; r += gridDim.y) {
    const float sig = gated ? shared_gate(p, p.row0 + r, s_red) : 1.0f;
    if (!live) continue;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int k = 0; k < p.topk; ++k) {
      const int pos = p.pos[r * p.topk + k];
      if (pos >= 0) {
        const float sc = p.scores[static_cast<size_t>(p.row0 + r) * p.topk + k];
        const float4 d = *reinterpret_cast<const float4*>(p.dout + static_cast<size_t>(pos) * p.hidden_out + c);
        acc[0] += sc * d.x;
        acc[1] += sc * d.y;
        acc[2] += sc * d.z;
        acc[3] += sc * d.w;
      }
    }
    const size_t at = static_cast<size_t>(p.row0 + r) * p.hidden_out + c;
    if (p.shared) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float sh = load_act(p.shared, at + j, p.x_dtype);
        const float g = gated ? round_act(sig * sh, p.x_dtype) : sh;
        acc[j] = round_act(acc[j], p.y_dtype) + g;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) store_act(p.y, at + j, acc[j], p.y_dtype);
  }
}

// ---------------------------------------------------------------- host

struct MoeScratch {
  bool ready = false;
  uint8_t* base = nullptr;
  size_t bytes = 0;
  int hidden = 0, inter = 0;
  int sms = 0;
};
constexpr int kMaxDev = 64;
std::mutex g_moe_mu;
MoeScratch g_moe[kMaxDev];

constexpr int kMaxCtasPerSm = 4;

// The fixed part of the workspace (its offsets depend only on the reserved width and the SM count, so the per-unit
// counters, zeroed once at allocation and reset by each unit's last run, stay in place from call to call): the
// route's ints, unit_done, the runs' partials.  The per-call arrays follow.
size_t fixed_bytes(int width, int sms) {
  const size_t ints = kIntsM;
  const size_t done = 2 * static_cast<size_t>(kMaxSlots) * (width / 128);
  const size_t part = static_cast<size_t>(sms) * kMaxCtasPerSm * kMaxRuns * kWarpsM * 1024;
  return (ints + done + part) * 4;
}

// The routing of a call through one expert (the shared expert's linears as a one-expert bank): kMaxSlots i32 zeros
// then kMaxSlots f32 ones, at the end of the workspace.
constexpr size_t kOneExpertBytes = 2 * static_cast<size_t>(kMaxSlots) * 4;

size_t scratch_bytes(int width, int sms) {
  const size_t xs = 2 * static_cast<size_t>(kMaxSlots) * (width / 16) * 256;
  const size_t hs = static_cast<size_t>(kMaxSlots) * (width / 16) * 256;
  const size_t ds = static_cast<size_t>(kMaxSlots) * width * 4;
  return fixed_bytes(width, sms) + xs + hs + ds + 4 * 256 + kOneExpertBytes;
}

exl3_verdict refuse_m(int32_t code, const char* why) { return {code, why}; }

// The most CTAs per SM the grouped GEMV's persistent grid may take (it takes what fits, up to this): kMaxCtasPerSm,
// or EXL3_MOE_CTAS (1..kMaxCtasPerSm) for measurements.
int moe_ctas_per_sm() {
  static const int v = [] {
    const char* e = getenv("EXL3_MOE_CTAS");
    const int n = e ? atoi(e) : kMaxCtasPerSm;
    return n >= 1 && n <= kMaxCtasPerSm ? n : kMaxCtasPerSm;
  }();
  return v;
}

template <int N, bool PAIR, int DS>
cudaError_t launch_moe_gemv(const MoeParams& p, int sms, cudaStream_t st) {
  auto kern = moe_gemv_kernel<N, PAIR, DS>;
  constexpr size_t slab = (PAIR ? 2u : 1u) * (8u * 2u * N + 256u);
  const size_t smem = kWarpsM * kStagesM * slab + (PAIR ? 2 : 1) * kWarpsM * 8 * kRedStrideM * 4;
  static KernelSetup setup;
  int per_sm = 0;  // resident CTAs per SM: the persistent grid is exactly one wave
  if (cudaError_t e = kernel_setup(setup, kern, kWarpsM * 32, smem, false, &per_sm, moe_ctas_per_sm()); e != cudaSuccess)
    return e;
  // the grid's partial slots ([grid][P][4 warps][kPart]) must fit the workspace's (sized for kMaxCtasPerSm CTAs per
  // SM of kMaxRuns slots of 1024 floats): at most 2 CTAs per SM for gate|up at kMaxRuns runs
  const int kt = (PAIR ? p.hidden : p.inter_full) / 16;
  const int runs = (kt + moe_run_slabs(kt) - 1) / moe_run_slabs(kt);
  const int fit = kMaxCtasPerSm * kMaxRuns * 1024 / (runs * (PAIR ? 2048 : 1024));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms * (per_sm < fit ? per_sm : fit));
  cfg.blockDim = dim3(kWarpsM * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool PAIR>
cudaError_t launch_moe_gemv_k(const MoeParams& p, int n, int sms, cudaStream_t st) {
  cudaError_t e = cudaErrorInvalidValue;
  with_rate_decode(n, PAIR ? p.cw_mask_gu : p.cw_mask_d, (PAIR ? p.mcg_gu : p.mcg_d) != 0, [&](auto N, auto DS) {
    e = launch_moe_gemv<decltype(N)::value, PAIR, decltype(DS)::value>(p, sms, st);
  });
  return e;
}

template <typename Kern>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, const MoeParams& p, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

bool bank_ok(const exl3_weight* w, int in_f, int out_f) {
  return w && w->size == sizeof(exl3_weight) && w->trellis && w->suh && w->svh && w->nseg == 1 &&
         w->in_features == in_f && w->out_features == out_f && exl3::rate_served_n(w->n) &&
         (reinterpret_cast<uintptr_t>(w->trellis) & 15u) == 0;
}

}  // namespace

exl3_verdict moe_reserve(int device, int in_features, int out_features) {
  if (device < 0 || device >= kMaxDev) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: device index out of range");
  // a bank is either gate/up (hidden -> inter) or down (inter -> hidden): reserve for the larger of each dim
  std::lock_guard<std::mutex> lk(g_moe_mu);
  MoeScratch& s = g_moe[device];
  const int hidden = in_features > out_features ? in_features : out_features;
  const int inter = in_features < out_features ? in_features : out_features;
  const int nh = hidden > s.hidden ? hidden : s.hidden, ni = inter > s.inter ? inter : s.inter;
  // inter may exceed hidden in another model: size both dims for the larger
  const int m = nh > ni ? nh : ni;
  if (s.ready && m <= s.hidden) return {EXL3_OK, nullptr};
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  if (s.base) {
    cudaDeviceSynchronize();
    cudaFree(s.base);
    s.base = nullptr;
  }
  cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, device);
  const size_t need = scratch_bytes(m, s.sms);
  bool ok = cudaMalloc(&s.base, need) == cudaSuccess && cudaMemset(s.base, 0, need) == cudaSuccess;
  if (ok) {
    std::vector<float> ones(kMaxSlots, 1.0f);
    ok = cudaMemcpy(s.base + need - kOneExpertBytes / 2, ones.data(), kOneExpertBytes / 2, cudaMemcpyHostToDevice) ==
         cudaSuccess;
  }
  if (prev >= 0) cudaSetDevice(prev);
  if (!ok) {
    s.ready = false;
    return refuse_m(EXL3_TOO_LARGE, "exl3_b200: MoE workspace allocation failed");
  }
  s.bytes = need;
  s.hidden = m;
  s.inter = m;
  s.ready = true;
  return {EXL3_OK, nullptr};
}

namespace {

// What the combine folds in (exl3_swiglu_shared); all null for a plain routed call.
struct SharedFold {
  const void* shared = nullptr;
  const void* logit = nullptr;
  const void* gate_vec = nullptr;
  const void* sigtab = nullptr;
};

exl3_verdict moe_swiglu_impl(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                             const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores, int limit,
                             const SharedFold& fold, void* stream, exl3_tensor* out, bool verify_rows = false);

}  // namespace

exl3_verdict moe_swiglu(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down, const exl3_tensor* x,
                        const exl3_tensor* inds, const exl3_tensor* scores, const exl3_swiglu_opts* opts, void* stream,
                        exl3_tensor* out) {
  if (opts && opts->size != sizeof(exl3_swiglu_opts)) return refuse_m(EXL3_FAILED, "exl3_b200: bad swiglu options");
  return moe_swiglu_impl(gate, up, down, x, inds, scores, opts ? opts->limit : 0, SharedFold{}, stream, out,
                         opts && opts->verify_rows);
}

exl3_verdict moe_swiglu_shared(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                               const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores,
                               const exl3_shared_swiglu* opts, void* stream, exl3_tensor* out) {
  if (!opts || opts->size != sizeof(exl3_shared_swiglu)) return refuse_m(EXL3_FAILED, "exl3_b200: bad shared-expert options");
  if (!x || !out || x->ndim != 3 || out->ndim != 3) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (x [B, S, D])");
  if (out->dtype != x->dtype) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Dtype (out is x's dtype)");
  const bool linears = opts->gate || opts->up || opts->down;
  if (linears == (opts->shared != nullptr))
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: the shared expert's three linears or its output, one of the two");
  if (opts->logit && opts->gate_vec) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: the shared gate's logit or its vector, not both");
  if (opts->sigtab && x->dtype == EXL3_F32)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Dtype (a sigmoid table is for 16-bit activations)");
  const int hidden = static_cast<int>(x->shape[2]);
  const int64_t rows = x->shape[0] * x->shape[1];
  SharedFold fold;
  fold.shared = opts->shared ? opts->shared : out->data;
  fold.logit = opts->logit;
  fold.gate_vec = opts->gate_vec;
  fold.sigtab = opts->sigtab;
  if (linears) {
    if (!opts->gate || !opts->up || !opts->down) return refuse_m(EXL3_FAILED, "exl3_b200: the shared expert needs gate, up and down");
    const exl3_weight* sg = opts->gate;
    if (sg->groups != 1 || opts->up->groups != 1 || opts->down->groups != 1)
      return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (the shared expert's linears are one group each)");
    if (sg->in_features != hidden || opts->down->out_features != hidden)
      return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (the shared expert reads and writes D)");
    const int dev = sg->device;
    uint8_t* k1 = nullptr;
    {
      std::lock_guard<std::mutex> lk(g_moe_mu);
      if (dev >= 0 && dev < kMaxDev && g_moe[dev].ready) k1 = g_moe[dev].base + g_moe[dev].bytes - kOneExpertBytes;
    }
    if (!k1) return refuse_m(EXL3_FAILED, "exl3_b200: no MoE workspace on the shared expert's device");
    // the shared expert first, into out (one expert, score 1, kMaxSlots rows a call), then the routed call reads it
    const size_t es = x->dtype == EXL3_F32 ? 4 : 2;
    for (int64_t r0 = 0; r0 < rows; r0 += kMaxSlots) {
      const int64_t rc = rows - r0 < kMaxSlots ? rows - r0 : kMaxSlots;
      exl3_tensor xc = *x, oc = *out, ic{}, sc{};
      xc.data = static_cast<uint8_t*>(x->data) + static_cast<size_t>(r0) * hidden * es;
      oc.data = static_cast<uint8_t*>(out->data) + static_cast<size_t>(r0) * hidden * es;
      xc.shape[0] = oc.shape[0] = 1;
      xc.shape[1] = oc.shape[1] = rc;
      ic.data = k1;
      ic.dtype = EXL3_I32;
      sc.data = k1 + kOneExpertBytes / 2;
      sc.dtype = EXL3_F32;
      ic.ndim = sc.ndim = 3;
      ic.shape[0] = sc.shape[0] = 1;
      ic.shape[1] = sc.shape[1] = rc;
      ic.shape[2] = sc.shape[2] = 1;
      exl3_verdict v = moe_swiglu_impl(opts->gate, opts->up, opts->down, &xc, &ic, &sc, 0, SharedFold{}, stream, &oc);
      if (v.code != EXL3_OK) return v;
    }
  }
  return moe_swiglu_impl(gate, up, down, x, inds, scores, opts->limit, fold, stream, out);
}

namespace {

exl3_verdict moe_swiglu_impl(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                             const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores, int limit,
                             const SharedFold& fold, void* stream, exl3_tensor* out, bool verify_rows) {
  if (!gate || !up || !down || !x || !inds || !scores || !out) return refuse_m(EXL3_FAILED, "exl3_b200: bad arguments");
  if (limit < 0 || limit > 128) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: InvalidExl3Clamp");
  if (x->ndim != 3 || inds->ndim != 3 || scores->ndim != 3 || out->ndim != 3)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (x [B, S, D], inds / scores [B, S, K])");
  const int hidden = static_cast<int>(x->shape[2]);
  const int64_t rows = x->shape[0] * x->shape[1];
  const int topk = static_cast<int>(inds->shape[2]);
  if (inds->shape[0] != x->shape[0] || inds->shape[1] != x->shape[1] || topk <= 0 || topk > kMaxTopK)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (inds)");
  for (int i = 0; i < 3; ++i)
    if (scores->shape[i] != inds->shape[i] || out->shape[i] != x->shape[i])
      return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (scores / out)");
  if (x->dtype != EXL3_F16 && x->dtype != EXL3_BF16 && x->dtype != EXL3_F32) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Dtype (x)");
  if (inds->dtype != EXL3_I32 && inds->dtype != EXL3_U32) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Dtype (inds)");
  if (scores->dtype != EXL3_F32) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Dtype (scores are f32)");
  if (out->dtype != x->dtype && out->dtype != EXL3_F32)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Dtype (out is x's dtype or f32)");
  const int inter = gate->out_features;
  const int experts = gate->groups;
  if (hidden <= 0 || hidden % 128 != 0 || inter <= 0 || inter % 128 != 0)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (hidden and intermediate are multiples of 128)");
  if (!bank_ok(gate, hidden, inter) || !bank_ok(up, hidden, inter) || !bank_ok(down, inter, hidden))
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (banks: gate/up [E, hidden -> inter], down [E, inter -> hidden])");
  if (up->groups != experts || down->groups != experts || experts < 1 || experts > 1024)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: the banks hold different expert counts");
  if (gate->n != up->n) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: gate and up banks at different rates");
  if ((gate->flags ^ up->flags) & (EXL3_WEIGHT_WINDOW_MASK | EXL3_WEIGHT_MCG))
    return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: gate and up banks with different codeword windows or codebooks");
  if (gate->device != up->device || gate->device != down->device) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: banks on different devices");
  if (rows == 0) return {EXL3_OK, nullptr};
  const int dev = gate->device;
  // prompt widths: the tensor-core path where a prefill workspace serves the banks (the decode chain with verify_rows)
  if (!verify_rows && !fold.shared && rows * topk >= kPrefillMinSlots && out->dtype == x->dtype &&
      moe_prefill_serves(dev, experts, hidden, inter, rows * topk))
    return moe_prefill_run(gate, up, down, x, inds, scores, static_cast<float>(limit), stream, out);
  MoeScratch* sc = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_moe_mu);
    if (dev >= 0 && dev < kMaxDev && g_moe[dev].ready && g_moe[dev].hidden >= hidden && g_moe[dev].inter >= inter)
      sc = &g_moe[dev];
  }
  if (!sc) return refuse_m(EXL3_FAILED, "exl3_b200: no MoE workspace for these banks (load them with exl3_load_bank)");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != dev) cudaSetDevice(dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MoeParams p{};
  p.g_tr = gate->trellis; p.g_suh = gate->suh; p.g_svh = gate->svh;
  p.u_tr = up->trellis; p.u_suh = up->suh; p.u_svh = up->svh;
  p.d_tr = down->trellis; p.d_suh = down->suh; p.d_svh = down->svh;
  p.experts = experts; p.hidden = hidden; p.inter = inter;
  p.inter_full = inter; p.inter_off = 0; p.hidden_out = hidden;
  p.x = x->data; p.x_dtype = x->dtype;
  p.inds = inds->data; p.inds_u32 = inds->dtype == EXL3_U32;
  p.scores = static_cast<const float*>(scores->data);
  p.y = out->data; p.y_dtype = out->dtype; p.topk = topk; p.limit = static_cast<float>(limit);
  p.shared = fold.shared;
  p.sh_logit = fold.logit;
  p.sh_gate_vec = fold.gate_vec;
  p.sigtab = fold.sigtab;
  int32_t* ints = reinterpret_cast<int32_t*>(sc->base);
  p.order = ints;
  p.chunk_e = ints + kMaxSlots;
  p.chunk_s = ints + 2 * kMaxSlots;
  p.chunk_n = ints + 3 * kMaxSlots;
  p.pos = ints + 4 * kMaxSlots;
  p.nchunks = ints + 5 * kMaxSlots;
  p.bad = ints + 5 * kMaxSlots + 1;
  p.max_cb = sc->hidden / 128;
  p.cw_mask_gu = window_mask(flags_window_bits(gate->flags));
  p.cw_mask_d = window_mask(flags_window_bits(down->flags));
  p.mcg_gu = (gate->flags & EXL3_WEIGHT_MCG) ? 1 : 0;
  p.mcg_d = (down->flags & EXL3_WEIGHT_MCG) ? 1 : 0;
  p.unit_done = ints + kIntsM;
  p.part = reinterpret_cast<float*>(p.unit_done + 2 * static_cast<size_t>(kMaxSlots) * p.max_cb);
  uint8_t* cur = sc->base + fixed_bytes(sc->hidden, sc->sms);
  const size_t xs = static_cast<size_t>(kMaxSlots) * (hidden / 16) * 256;
  p.xg = cur; cur += xs;
  p.xu = cur; cur += xs;
  p.hp = cur; cur += static_cast<size_t>(kMaxSlots) * (inter / 16) * 256;
  p.dout = reinterpret_cast<float*>(cur);
  cudaError_t err = cudaSuccess;
  const int pass_rows = kMaxSlots / topk;  // every expert a pass touches is read once per pass
  for (int64_t r0 = 0; r0 < rows && err == cudaSuccess; r0 += pass_rows) {
    p.row0 = static_cast<int32_t>(r0);
    p.rows = static_cast<int32_t>(rows - r0 < pass_rows ? rows - r0 : pass_rows);
    const int S = p.rows * topk;
    err = launch_pdl(moe_route_kernel, dim3(1), dim3(1024), p, st);
    if (err == cudaSuccess)
      err = launch_pdl(moe_prep_kernel, dim3(hidden / 128, S < kPrepChunks ? S : kPrepChunks), dim3(128), p, st);
    if (err == cudaSuccess) err = launch_moe_gemv_k<true>(p, gate->n, sc->sms, st);
    if (err == cudaSuccess) err = launch_moe_gemv_k<false>(p, down->n, sc->sms, st);
    if (err == cudaSuccess)
      err = launch_pdl(moe_combine_kernel, dim3((hidden + 511) / 512, p.rows < kCombineRows ? p.rows : kCombineRows),
                       dim3(128), p, st);
  }
  if (prev >= 0 && prev != dev) cudaSetDevice(prev);
  if (err != cudaSuccess) return refuse_m(EXL3_FAILED, "exl3_b200: MoE launch failed");
  return {EXL3_OK, nullptr};
}

}  // namespace

// ================================================================ column-parallel experts over NVLink peer memory
//
// Every rank holds a column slice of every expert: gate/up output columns [r inter/W, (r+1) inter/W) and down output
// columns [r hidden/W, (r+1) hidden/W) (down's input is the whole intermediate), so each rank streams exactly 1/W of the
// distinct experts' bytes whatever the routing.  A call (every rank brings T tokens with K slots each):
//   in     -- each rank's x, inds, scores rows into every rank's gathered block (rows [rank T, rank T + T));
//   wait 0 -- a one-CTA launch (the copies' launch has completed) advances the step word, releases done[0][rank] on
//             every rank once and waits (bounded) until every rank's rows are in;
//   route, prepare, gate|up GEMV on all W T rows -- the same slot order and chunk table on every rank (deterministic);
//             the gate|up epilogue stores its blocks of the down input into every rank's down-input buffer;
//   sync 1 -- this rank's gate|up is complete: release done[1][rank] on every rank, wait for every rank's (bounded);
//   down GEMV over this rank's output columns (the whole down input is local now), combine -> ycol [W T][hidden/W];
//   out    -- each owner's T rows of ycol into its output block (columns [rank hidden/W, ...));
//   final  -- its first CTA releases done[2][rank] once (the out launch has completed); every rank's columns are in
//             (bounded); the T rows to the caller's out.
// One copy of each buffer suffices: a rank writes a peer's buffers of call s + 1 only after passing a wait of call
// s + 1 that the peer releases after it finished reading them in call s.  Every wait gives up after one second with
// EXL3_ERR_EP_TIMEOUT; the done words only grow, so graph replays need nothing reset.

struct CpxDev {
  uint8_t* buf[8];      // every rank's exchange buffer
  uint32_t* step;       // this rank's step word
  uint32_t* arrive;     // [3] (unused: each phase publishes once, from the launch that waits for it)
  int32_t world, rank, tokens, topk, hidden, hidden_out, esize;
  int64_t off_x, off_inds, off_scores, off_hp, off_y, off_done;
  uint64_t* trace;      // the phase timeline ring, or null: 0 in begins, 1 its copies done, 2 every rank's rows seen,
                        // 3 gate|up done, 4 every rank's gate|up seen, 5 down and combine done, 6 every rank's
                        // columns seen, 7 copied out
};

namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys_m(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t* cpx_done(const CpxDev& d, int q, int phase) {
  return reinterpret_cast<uint32_t*>(d.buf[q] + d.off_done) + phase * d.world;
}

// Threads 0..world-1 of the CTA wait (one second at most) until every rank's done[phase] word holds `step`.
__device__ void cpx_wait_all(const CpxDev& d, int phase, uint32_t step, uint32_t* err) {
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if (threadIdx.x < static_cast<uint32_t>(d.world)) {
    const uint32_t* f = cpx_done(d, d.rank, phase) + threadIdx.x;
    if (static_cast<int32_t>(ld_acquire_sys_m(f) - step) < 0) {
      const uint64_t t0 = global_timer_ns();
      while (static_cast<int32_t>(ld_acquire_sys_m(f) - step) < 0) {
        if (global_timer_ns() - t0 > 1000000000ull) {
          s_fail = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (s_fail && threadIdx.x == 0) atomicOr(err, kErrEpTimeout);
}

__device__ void cpx_release(const CpxDev& d, int phase, uint32_t step) {
  asm volatile("fence.sc.sys;" ::: "memory");
  for (int q = 0; q < d.world; ++q) {
    uint32_t* f = cpx_done(d, q, phase) + d.rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(step) : "memory");
  }
}

__device__ void copy16(uint8_t* dst, const uint8_t* src, size_t bytes, size_t t0, size_t stride) {
  for (size_t w = t0; w < bytes / 16; w += stride)
    reinterpret_cast<uint4*>(dst)[w] = reinterpret_cast<const uint4*>(src)[w];
}

// grid (world, c): this rank's rows into block `rank` of every rank's gathered x / inds / scores
__global__ void __launch_bounds__(256) cpx_in_kernel(const CpxDev* dp, const uint8_t* __restrict__ x,
                                                     const int32_t* __restrict__ inds, const float* __restrict__ scores) {
  pdl_wait();  // every launch before this one in the stream is complete (programmatic dependent launch)
  pdl_launch_dependents();
  const CpxDev& d = *dp;
  const int q = blockIdx.x;
  if (q == 0 && blockIdx.y == 0 && threadIdx.x == 0)
    trace_at(d.trace, *reinterpret_cast<const volatile uint32_t*>(d.step) + 1u, 0);
  const size_t xrow = static_cast<size_t>(d.hidden) * d.esize;
  const size_t t0 = static_cast<size_t>(blockIdx.y) * blockDim.x + threadIdx.x, stride = static_cast<size_t>(gridDim.y) * blockDim.x;
  copy16(d.buf[q] + d.off_x + static_cast<size_t>(d.rank) * d.tokens * xrow, x, d.tokens * xrow, t0, stride);
  const int n = d.tokens * d.topk;
  int32_t* qi = reinterpret_cast<int32_t*>(d.buf[q] + d.off_inds) + static_cast<size_t>(d.rank) * n;
  float* qs = reinterpret_cast<float*>(d.buf[q] + d.off_scores) + static_cast<size_t>(d.rank) * n;
  for (size_t i = t0; i < static_cast<size_t>(n); i += stride) {
    qi[i] = inds[i];
    qs[i] = scores[i];
  }
}

// After this rank's copies into every rank (the previous launch, complete): advance the step word, publish phase 0
// -- one system-scope fence for all of the launch's stores -- and wait (bounded) for every rank's.
__global__ void cpx_in_publish_kernel(const CpxDev* dp, uint32_t* err) {
  pdl_wait();  // the copies' launch is complete: its stores are performed
  pdl_launch_dependents();
  const CpxDev& d = *dp;
  __shared__ uint32_t s_step;
  if (threadIdx.x == 0) {
    const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(d.step) + 1u;
    trace_at(d.trace, step, 1);
    *d.step = step;
    cpx_release(d, 0, step);
    s_step = step;
  }
  __syncthreads();
  cpx_wait_all(d, 0, s_step, err);
  if (threadIdx.x == 0) trace_at(d.trace, s_step, 2);
}

// After this rank's gate|up (the previous launch, complete): publish it, wait for every rank's.
__global__ void cpx_sync_kernel(const CpxDev* dp, uint32_t* err) {
  pdl_wait();  // the gate|up launch is complete: its stores into every rank are performed
  pdl_launch_dependents();
  const CpxDev& d = *dp;
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(d.step);
  if (threadIdx.x == 0) {
    trace_at(d.trace, step, 3);
    cpx_release(d, 1, step);
  }
  cpx_wait_all(d, 1, step, err);
  if (threadIdx.x == 0) trace_at(d.trace, step, 4);
}

// grid (world, c): owner q's T rows of ycol [W T][hidden_out] -> its output block, columns [rank hidden_out, ...)
__global__ void __launch_bounds__(256) cpx_out_kernel(const CpxDev* dp, const uint8_t* __restrict__ ycol) {
  pdl_wait();
  pdl_launch_dependents();
  const CpxDev& d = *dp;
  const int q = blockIdx.x;
  if (q == 0 && blockIdx.y == 0 && threadIdx.x == 0)
    trace_at(d.trace, *reinterpret_cast<const volatile uint32_t*>(d.step), 5);
  const size_t seg = static_cast<size_t>(d.hidden_out) * d.esize;  // bytes of one row's column slice
  const size_t words = seg / 16;
  for (size_t w = static_cast<size_t>(blockIdx.y) * blockDim.x + threadIdx.x; w < d.tokens * words;
       w += static_cast<size_t>(gridDim.y) * blockDim.x) {
    const size_t r = w / words, c = w % words;
    const uint4* src = reinterpret_cast<const uint4*>(ycol + (static_cast<size_t>(q) * d.tokens + r) * seg);
    uint4* dst = reinterpret_cast<uint4*>(d.buf[q] + d.off_y + r * d.hidden * d.esize + d.rank * seg);
    dst[c] = src[c];
  }
}

// After the out copies (the previous launch, complete): CTA 0 publishes phase 2 (one system-scope fence for all of
// them); every rank's columns of this rank's rows are in (bounded), then they go to the caller's out
__global__ void __launch_bounds__(256) cpx_final_kernel(const CpxDev* dp, uint8_t* __restrict__ out, uint32_t* err) {
  pdl_wait();  // the out copies' launch is complete: its stores are performed
  pdl_launch_dependents();
  const CpxDev& d = *dp;
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(d.step);
  if (blockIdx.x == 0 && threadIdx.x == 0) cpx_release(d, 2, step);
  cpx_wait_all(d, 2, step, err);
  if (blockIdx.x == 0 && threadIdx.x == 0) trace_at(d.trace, step, 6);
  const size_t bytes = static_cast<size_t>(d.tokens) * d.hidden * d.esize;
  copy16(out, d.buf[d.rank] + d.off_y, bytes, static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x,
         static_cast<size_t>(gridDim.x) * blockDim.x);
  __syncthreads();
  if (threadIdx.x == 0) trace_last(d.trace, step, 7);
}

}  // namespace

}  // namespace exl3

struct exl3_cpx {
  int device = -1, world = 0, rank = 0, tokens = 0, topk = 0, hidden = 0, inter = 0, dtype = 0, esize = 2;
  int chunks = 0;
  uint8_t* base = nullptr;
  size_t bytes = 0;
  int64_t off_ycol = 0;
  uint8_t* peer[8] = {};
  exl3::CpxDev host{};
  exl3::CpxDev* dev = nullptr;
  bool connected = false;
};

namespace exl3 {

namespace {
struct CpxScope {
  int prev = -1;
  explicit CpxScope(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
    else prev = -1;
  }
  ~CpxScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

}  // namespace exl3

extern "C" {

exl3_verdict exl3_cpx_create(int32_t device, int32_t world, int32_t rank, int32_t tokens, int32_t topk, int32_t hidden,
                             int32_t inter, int32_t dtype, exl3_cpx** out, uint8_t* ipc_handle) {
  using namespace exl3;
  if (!out || !ipc_handle) return refuse_m(EXL3_FAILED, "exl3_cpx_create: bad arguments");
  *out = nullptr;
  if (world < 1 || world > 8 || rank < 0 || rank >= world) return refuse_m(EXL3_UNSUPPORTED, "exl3_cpx_create: 1..8 ranks");
  if (tokens < 1 || topk < 1 || topk > kMaxTopK || static_cast<int64_t>(world) * tokens * topk > kMaxSlots)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_cpx_create: every rank's tokens x slots at most 512 in all");
  if (hidden % (128 * world) != 0 || inter % (128 * world) != 0)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_cpx_create: hidden and intermediate split into 128-column blocks per rank");
  if (dtype != EXL3_F16 && dtype != EXL3_BF16 && dtype != EXL3_F32) return refuse_m(EXL3_UNSUPPORTED, "exl3_cpx_create: an activation dtype");
  CpxScope scope(device);
  exl3_cpx* e = new (std::nothrow) exl3_cpx;
  if (!e) return refuse_m(EXL3_FAILED, "exl3_cpx_create: out of host memory");
  e->device = device, e->world = world, e->rank = rank, e->tokens = tokens, e->topk = topk, e->hidden = hidden;
  e->inter = inter, e->dtype = dtype, e->esize = dtype == EXL3_F32 ? 4 : 2;
  const int64_t rows = static_cast<int64_t>(world) * tokens;
  e->chunks = static_cast<int>(rows * topk);  // at most one chunk per slot
  auto up = [](int64_t v) { return (v + 255) & ~int64_t{255}; };
  int64_t at = 0;
  CpxDev& h = e->host;
  h.off_x = at; at = up(at + rows * hidden * e->esize);
  h.off_inds = at; at = up(at + rows * topk * 4);
  h.off_scores = at; at = up(at + rows * topk * 4);
  h.off_hp = at; at = up(at + static_cast<int64_t>(e->chunks) * (inter / 16) * 256);
  h.off_y = at; at = up(at + static_cast<int64_t>(tokens) * hidden * e->esize);
  h.off_done = at; at = up(at + 3 * 8 * 4);
  const int64_t off_local = at; at = up(at + 64);  // step, arrive[3]
  e->off_ycol = at; at = up(at + rows * (hidden / world) * e->esize);
  e->bytes = static_cast<size_t>(at);
  bool ok = cudaMalloc(&e->base, e->bytes) == cudaSuccess && cudaMemset(e->base, 0, e->bytes) == cudaSuccess;
  cudaIpcMemHandle_t hd;
  ok = ok && cudaIpcGetMemHandle(&hd, e->base) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  if (!ok) {
    if (e->base) cudaFree(e->base);
    delete e;
    return refuse_m(EXL3_TOO_LARGE, "exl3_cpx_create: exchange buffer allocation failed");
  }
  memcpy(ipc_handle, &hd, 64);
  e->peer[rank] = e->base;
  h.step = reinterpret_cast<uint32_t*>(e->base + off_local);
  h.arrive = h.step + 4;
  h.world = world, h.rank = rank, h.tokens = tokens, h.topk = topk, h.hidden = hidden;
  h.hidden_out = hidden / world, h.esize = e->esize;
  h.trace = trace_alloc();
  *out = e;
  return {EXL3_OK, nullptr};
}

exl3_verdict exl3_cpx_connect(exl3_cpx* e, const uint8_t* ipc_handles) {
  using namespace exl3;
  if (!e || !ipc_handles || e->connected) return refuse_m(EXL3_FAILED, "exl3_cpx_connect: bad arguments");
  CpxScope scope(e->device);
  bool ok = true;
  for (int q = 0; q < e->world && ok; ++q) {
    if (q == e->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handles + 64 * q, 64);
    void* p = nullptr;
    ok = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    e->peer[q] = static_cast<uint8_t*>(p);
  }
  for (int q = 0; q < e->world; ++q) e->host.buf[q] = e->peer[q];
  ok = ok && cudaMalloc(&e->dev, sizeof(CpxDev)) == cudaSuccess &&
       cudaMemcpy(e->dev, &e->host, sizeof(CpxDev), cudaMemcpyHostToDevice) == cudaSuccess;
  if (!ok) return refuse_m(EXL3_FAILED, "exl3_cpx_connect: opening a peer's exchange buffer failed");
  e->connected = true;
  return {EXL3_OK, nullptr};
}

void exl3_cpx_destroy(exl3_cpx* e) {
  if (!e) return;
  exl3::CpxScope scope(e->device);
  cudaDeviceSynchronize();
  for (int q = 0; q < e->world; ++q)
    if (q != e->rank && e->peer[q]) cudaIpcCloseMemHandle(e->peer[q]);
  if (e->dev) cudaFree(e->dev);
  if (e->base) cudaFree(e->base);
  if (e->host.trace) cudaFree(e->host.trace);
  delete e;
}

exl3_verdict exl3_cpx_trace(exl3_cpx* e, uint64_t* out) {
  using namespace exl3;
  if (!e || !e->connected || !out) return refuse_m(EXL3_FAILED, "exl3_cpx_trace: bad arguments");
  if (!e->host.trace) return refuse_m(EXL3_UNSUPPORTED, "exl3_cpx_trace: the exchange was created without EXL3_TRACE=1");
  CpxScope scope(e->device);
  return trace_copy(e->host.trace, e->host.step, out) ? exl3_verdict{EXL3_OK, nullptr}
                                                      : refuse_m(EXL3_FAILED, "exl3_cpx_trace: copy failed");
}

exl3_verdict exl3_swiglu_cp(exl3_cpx* e, const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                            const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores,
                            const exl3_swiglu_opts* opts, void* stream, exl3_tensor* out) {
  using namespace exl3;
  if (!e || !e->connected || !gate || !up || !down || !x || !inds || !scores || !out)
    return refuse_m(EXL3_FAILED, "exl3_swiglu_cp: bad arguments");
  if (opts && opts->size != sizeof(exl3_swiglu_opts)) return refuse_m(EXL3_FAILED, "exl3_b200: bad swiglu options");
  const int limit = opts ? opts->limit : 0;
  if (limit < 0 || limit > 128) return refuse_m(EXL3_UNSUPPORTED, "exl3_b200: InvalidExl3Clamp");
  const int W = e->world, T = e->tokens, K = e->topk, hidden = e->hidden, inter = e->inter;
  if (x->ndim != 2 || x->shape[0] != T || x->shape[1] != hidden || x->dtype != e->dtype || out->ndim != 2 ||
      out->shape[0] != T || out->shape[1] != hidden || out->dtype != e->dtype)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_swiglu_cp: x and out [T, hidden] in the exchange's dtype");
  if (inds->ndim != 2 || inds->shape[0] != T || inds->shape[1] != K || inds->dtype != EXL3_I32 || scores->ndim != 2 ||
      scores->shape[0] != T || scores->shape[1] != K || scores->dtype != EXL3_F32)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_swiglu_cp: inds i32 and scores f32 [T, K]");
  if (reinterpret_cast<uintptr_t>(x->data) % 16 || reinterpret_cast<uintptr_t>(out->data) % 16)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_swiglu_cp: x and out on 16-byte boundaries");
  const int islice = inter / W, hslice = hidden / W;
  const int experts = gate->groups;
  if (!bank_ok(gate, hidden, islice) || !bank_ok(up, hidden, islice) || !bank_ok(down, inter, hslice) ||
      up->groups != experts || down->groups != experts || experts < 1 || experts > 1024 || gate->n != up->n ||
      ((gate->flags ^ up->flags) & (EXL3_WEIGHT_WINDOW_MASK | EXL3_WEIGHT_MCG)))
    return refuse_m(EXL3_UNSUPPORTED,
                    "exl3_swiglu_cp: banks gate/up [E, hidden -> inter/W], down [E, inter -> hidden/W], one rate and window for gate and up");
  if (gate->device != e->device || up->device != e->device || down->device != e->device)
    return refuse_m(EXL3_UNSUPPORTED, "exl3_swiglu_cp: banks on the exchange's device");
  MoeScratch* sc = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_moe_mu);
    const int dev = e->device;
    if (dev >= 0 && dev < kMaxDev && g_moe[dev].ready && g_moe[dev].hidden >= hidden && g_moe[dev].inter >= hidden)
      sc = &g_moe[dev];
  }
  if (!sc) return refuse_m(EXL3_FAILED, "exl3_swiglu_cp: no MoE workspace for these banks (load them with exl3_load_bank)");
  CpxScope scope(e->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* err = device_error_ptr();
  if (!err) return refuse_m(EXL3_FAILED, "exl3_swiglu_cp: no device error word");
  const CpxDev& h = e->host;
  MoeParams p{};
  p.g_tr = gate->trellis; p.g_suh = gate->suh; p.g_svh = gate->svh;
  p.u_tr = up->trellis; p.u_suh = up->suh; p.u_svh = up->svh;
  p.d_tr = down->trellis; p.d_suh = down->suh; p.d_svh = down->svh;
  p.experts = experts; p.hidden = hidden; p.inter = islice;
  p.inter_full = inter; p.inter_off = e->rank * islice; p.hidden_out = hslice;
  p.x = e->base + h.off_x; p.x_dtype = e->dtype;
  p.inds = e->base + h.off_inds; p.inds_u32 = 0;
  p.scores = reinterpret_cast<const float*>(e->base + h.off_scores);
  p.y = e->base + e->off_ycol; p.y_dtype = e->dtype; p.topk = K; p.limit = static_cast<float>(limit);
  p.row0 = 0; p.rows = W * T;
  int32_t* ints = reinterpret_cast<int32_t*>(sc->base);
  p.order = ints;
  p.chunk_e = ints + kMaxSlots;
  p.chunk_s = ints + 2 * kMaxSlots;
  p.chunk_n = ints + 3 * kMaxSlots;
  p.pos = ints + 4 * kMaxSlots;
  p.nchunks = ints + 5 * kMaxSlots;
  p.bad = ints + 5 * kMaxSlots + 1;
  p.max_cb = sc->hidden / 128;
  p.cw_mask_gu = window_mask(flags_window_bits(gate->flags));
  p.cw_mask_d = window_mask(flags_window_bits(down->flags));
  p.mcg_gu = (gate->flags & EXL3_WEIGHT_MCG) ? 1 : 0;
  p.mcg_d = (down->flags & EXL3_WEIGHT_MCG) ? 1 : 0;
  p.unit_done = ints + kIntsM;
  p.part = reinterpret_cast<float*>(p.unit_done + 2 * static_cast<size_t>(kMaxSlots) * p.max_cb);
  uint8_t* cur = sc->base + fixed_bytes(sc->hidden, sc->sms);
  const size_t xs = static_cast<size_t>(kMaxSlots) * (hidden / 16) * 256;
  p.xg = cur; cur += xs;
  p.xu = cur; cur += xs;
  cur += static_cast<size_t>(kMaxSlots) * (sc->hidden / 16) * 256;  // (the local down input lives in the exchange)
  p.dout = reinterpret_cast<float*>(cur);
  p.hp = e->base + h.off_hp;
  for (int q = 0; q < W; ++q) p.hp_dst[q] = e->peer[q] + h.off_hp;
  p.hp_world = W;
  const int S = W * T * K;
  const int copy = W >= 148 ? 1 : (148 + W - 1) / W;
  const CpxDev* dv = e->dev;
  cudaError_t er = launch_pdl_k(cpx_in_kernel, dim3(W, copy), dim3(256), st, dv, static_cast<const uint8_t*>(x->data),
                                static_cast<const int32_t*>(inds->data), static_cast<const float*>(scores->data));
  if (er == cudaSuccess) er = launch_pdl_k(cpx_in_publish_kernel, dim3(1), dim3(32), st, dv, err);
  if (er == cudaSuccess) er = launch_pdl(moe_route_kernel, dim3(1), dim3(1024), p, st);
  if (er == cudaSuccess)
    er = launch_pdl(moe_prep_kernel, dim3(hidden / 128, S < kPrepChunks ? S : kPrepChunks), dim3(128), p, st);
  if (er == cudaSuccess) er = launch_moe_gemv_k<true>(p, gate->n, sc->sms, st);
  if (er == cudaSuccess) er = launch_pdl_k(cpx_sync_kernel, dim3(1), dim3(32), st, dv, err);
  if (er == cudaSuccess) er = launch_moe_gemv_k<false>(p, down->n, sc->sms, st);
  if (er == cudaSuccess)
    er = launch_pdl(moe_combine_kernel, dim3((hslice + 511) / 512, p.rows < kCombineRows ? p.rows : kCombineRows),
                    dim3(128), p, st);
  if (er == cudaSuccess)
    er = launch_pdl_k(cpx_out_kernel, dim3(W, copy), dim3(256), st, dv,
                      static_cast<const uint8_t*>(e->base + e->off_ycol));
  if (er == cudaSuccess)
    er = launch_pdl_k(cpx_final_kernel, dim3(16), dim3(256), st, dv, static_cast<uint8_t*>(out->data), err);
  return er == cudaSuccess ? exl3_verdict{EXL3_OK, nullptr} : refuse_m(EXL3_FAILED, "exl3_swiglu_cp: launch failed");
}

}  // extern "C"
