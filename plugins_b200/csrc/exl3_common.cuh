// exl3_common.cuh -- device helpers shared by the EXL3 kernels (sm_100a).
//
// Format (the reference's, restated): a 16x16 weight tile is a tail-biting bitstream of n = 16K halfwords; weight p
// of the stream reads the 16-bit window ending at bit floor((p+1) n / 16), MSB-first over little-endian u32 words
// (plugins/sushi_ds41/src/sushi/exl3/expert_exl3.zig:313-336); the window's state s decodes through the mul1 codebook
// to f16 RN((1024 + bytesum(s * 0x83DCD12D)) * f16(0x1EEE) + f16(0xC931)) (expert_exl3.zig:275-284); stream position
// p lands at row-major tile slot tensorCorePerm[p] (expert_exl3.zig:379-398).  That permutation is the m16n8k16 MMA
// operand order: lane t of a warp owns stream positions 8t..8t+7, i.e. k-rows {2(t%4), +1, +8, +9} at output
// columns t/4 and t/4 + 8 -- exactly the A fragment of W^T (rows = output columns, cols = k).
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "exl3_windows.h"

namespace exl3 {

constexpr uint32_t kMul1Mult = 0x83DCD12Du;
constexpr uint32_t kHalfInv = 0x1EEEu;   // f16(0x1EEE)
constexpr uint32_t kHalfBias = 0xC931u;  // f16(0xC931)
constexpr float kHadScale = 0.08838834764831845f;

// Error bits a kernel ORs into the device error word (read back by exl3_device_error()).
enum : uint32_t {
  kErrWaitTimeout = 1u << 0,   // a bounded mbarrier wait gave up
  kErrBadShape = 1u << 1,      // a launch saw a shape its host validation should have refused
  kErrEpOverflow = 1u << 2,    // an expert-parallel dispatch had more rows for one peer than its capacity
  kErrTpTimeout = 1u << 3,     // a column-parallel gather gave up waiting for a peer's columns
  kErrEpTimeout = 1u << 4,     // a peer expert-parallel exchange gave up waiting for a peer's rows
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ mbarrier + bulk copy (TMA, 1-D)

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for `parity` with a wall-clock bound (about two seconds).  Returns false after the bound; the caller records
// kErrWaitTimeout and leaves its loop, so a lost arrival can never hang the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > 2000000000ull) return false;
  }
}

// cp.async.bulk global -> shared (this CTA), completion counted on `bar` in bytes.  `bytes` and both addresses are
// multiples of 16.  The L2 hint marks streamed weights evict-first so they do not push activations out of L2.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------ programmatic dependent launch

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Exclusive scan of one int per thread over the CTA (blockDim.x a multiple of 32, at most 1024); *total receives the
// sum.  s_warp: 32 ints of shared memory, reusable when the call returns.
__device__ __forceinline__ int cta_scan_excl(int v, int* s_warp, int* total) {
  const int lane = static_cast<int>(threadIdx.x & 31u), warp = static_cast<int>(threadIdx.x >> 5);
  const int nw = static_cast<int>(blockDim.x >> 5);
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += y;
    }
    if (lane < nw) s_warp[lane] = w;
  }
  __syncthreads();
  *total = s_warp[nw - 1];
  const int r = x - v + (warp > 0 ? s_warp[warp - 1] : 0);
  __syncthreads();
  return r;
}

// ------------------------------------------------------------------ tile decode

// The 64 stream bits of a tile ending at lane t's last window end E = 8 (t+1) K, as (hi, lo).  `words` is the tile's
// u32 view (n/2 words), read circularly.  Word offsets and the funnel shift depend only on the lane, so callers
// compute a LaneWindows once and reuse it for every tile.
template <int K>
struct LaneWindows {
  uint32_t o0, o1, o2;  // word offsets (c-2, c-1, c) mod n/2
  uint32_t sh;          // right funnel shift (wraps: 0 when E is word-aligned)
  __device__ __forceinline__ void init(uint32_t lane) {
    constexpr uint32_t nw = 8u * K;  // n/2 u32 words per tile
    const uint32_t e = 8u * (lane + 1u) * K;
    const uint32_t c = (e - 1u) >> 5;
    o2 = c % nw;
    o1 = (c + nw - 1u) % nw;
    o0 = (c + nw - 2u) % nw;
    sh = (0u - e) & 31u;
  }
};

// Eight codeword windows of lane t (stream positions 8t..8t+7), low 16 bits of each result.
template <int K>
__device__ __forceinline__ void lane_codewords(const uint32_t* tile_words, const LaneWindows<K>& lw, uint32_t (&w)[8]) {
  static_assert(K >= 1 && K <= 6, "8 windows must fit 64 bits");
  uint32_t vlo, vhi;
  if constexpr ((8 * K) % 32 == 0) {
    // E is always word-aligned (K = 4): two plain words.
    vlo = tile_words[lw.o2];
    vhi = tile_words[lw.o1];
  } else {
    const uint32_t a = tile_words[lw.o0], b = tile_words[lw.o1], c = tile_words[lw.o2];
    vlo = __funnelshift_r(c, b, lw.sh);
    vhi = __funnelshift_r(b, a, lw.sh);
  }
  if constexpr (K == 4) {
    // windows j and j+4 are the high and low halves of one 32-bit funnel
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t s = (3 - j) * 4;  // shift of window j+4
      const uint32_t c = s == 0 ? vlo : __funnelshift_r(vlo, vhi, s);
      w[j] = c >> 16;
      w[j + 4] = c & 0xFFFFu;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t s = (7 - j) * K;  // the window is bits [s, s + 16) of (vhi:vlo)
      uint32_t v;
      if (s >= 32) v = vhi >> (s - 32);
      else if (s + 16 <= 32) v = vlo >> s;
      else v = __funnelshift_r(vlo, vhi, s);
      w[j] = v & 0xFFFFu;
    }
  }
}

// A tile of N halfwords (N = 16 x bits per weight; half-bit rates included): whole-bit rates take the extraction
// above, half-bit rates the general rule of exl3_windows.h (the same windows: both follow the bitstream rule).  NW
// (a narrowed codeword window, lw.mask): the general rule at every rate, each window masked.
template <int N, bool NW = false>
__device__ __forceinline__ void tile_codewords(const uint32_t* tile_words, const LaneWin<N>& lw, uint32_t (&w)[8]) {
  if constexpr (N % 16 == 0 && !NW) {
    LaneWindows<N / 16> lk;
    lk.o0 = lw.o0;
    lk.o1 = lw.o1;
    lk.o2 = lw.o2;
    lk.sh = lw.sh;
    lane_codewords<N / 16>(tile_words, lk, w);
  } else {
    lane_windows<N, NW>(tile_words, lw, w);
  }
}

// mul1 of a pair of codewords: f16x2 (lo = cw_a, hi = cw_b) with exactly one rounding, as the reference.
__device__ __forceinline__ uint32_t mul1_pair_dp4a(uint32_t cw_a, uint32_t cw_b) {
  // unsigned byte sums (the int overload of __dp4a sums signed bytes)
  const uint32_t sa = __dp4a(cw_a * kMul1Mult, 0x01010101u, 0x6400u);
  const uint32_t sb = __dp4a(cw_b * kMul1Mult, 0x01010101u, 0x6400u);
  const uint32_t h = __byte_perm(sa, sb, 0x5410);
  const uint32_t inv2 = kHalfInv | (kHalfInv << 16), bias2 = kHalfBias | (kHalfBias << 16);
  uint32_t out;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(h), "r"(inv2), "r"(bias2));
  return out;
}

// Two decoded byte sums (f16 bits of 1024 + bytesum in the low halves) -> f16x2 (lo, hi) through the mul1 affine.
// Both halves are below 2^16, so the packing is exact either way: a byte permute (ALU pipe) or hi * 65536 + lo (an
// integer multiply-add, FMA pipe).  Which is faster depends on which pipe the rest of the kernel loads: measured on
// B200, the multiply-add for the deep-ring decode GEMVs and the grouped expert GEMV, the permute elsewhere.
template <bool kPackFma = false>
__device__ __forceinline__ uint32_t mul1_pack_affine(uint32_t h_lo16, uint32_t h_hi16) {
  uint32_t h;
  if constexpr (kPackFma) asm("mad.lo.u32 %0, %1, 65536, %2;" : "=r"(h) : "r"(h_hi16), "r"(h_lo16));
  else h = __byte_perm(h_lo16, h_hi16, 0x5410);
  const uint32_t inv2 = kHalfInv | (kHalfInv << 16), bias2 = kHalfBias | (kHalfBias << 16);
  uint32_t out;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(h), "r"(inv2), "r"(bias2));
  return out;
}

// The m16n8k16 A fragment of W^T for this lane's eight positions, via dp4a byte sums:
// reg0 = (j0, j1) [col g, k 2q..2q+1], reg1 = (j4, j5) [col g+8], reg2 = (j2, j3) [col g, k 2q+8..], reg3 = (j6, j7).
__device__ __forceinline__ void decode_afrag_dp4a(const uint32_t (&w)[8], uint32_t (&a)[4]) {
  a[0] = mul1_pair_dp4a(w[0], w[1]);
  a[1] = mul1_pair_dp4a(w[4], w[5]);
  a[2] = mul1_pair_dp4a(w[2], w[3]);
  a[3] = mul1_pair_dp4a(w[6], w[7]);
}

// The same weights through the tensor pipe: the byte sums of 128 hash products per m16n8k32 u8 IMMA (A = products,
// B = group indicator, C = 0x6400).  Lane (g, q) then holds column g's weights at k = 4q, 4q+2, 4q+1, 4q+3 (d0..d3),
// so the main MMA's logical k' = 2q + e maps to physical 4q + e and k' = 2q + 8 + e to 4q + 2 + e; the activation
// fragment is then x[4q .. 4q+3], one 8-byte load.
__device__ __forceinline__ void imma_bytesum(const uint32_t (&x)[4], uint32_t b0, uint32_t b1, uint32_t (&d)[4]) {
  int c = 0x6400;
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(x[0]), "r"(x[1]), "r"(x[2]), "r"(x[3]), "r"(b0), "r"(b1), "r"(c), "r"(c), "r"(c), "r"(c));
}

struct ImmaIndicator {
  uint32_t b0, b1;
  __device__ __forceinline__ void init(uint32_t lane) {
    const uint32_t g = lane >> 2, q = lane & 3u;
    b0 = (q == g) ? 0x01010101u : 0u;        // k-group q of column g
    b1 = (q + 4u == g) ? 0x01010101u : 0u;   // k-group q + 4 of column g
  }
};

template <bool kPackFma = false>
__device__ __forceinline__ void decode_afrag_imma(const uint32_t (&w)[8], const ImmaIndicator& ind,
                                                  uint32_t (&a)[4]) {
  uint32_t x0[4], x1[4], d0[4], d1[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    x0[j] = w[j] * kMul1Mult;
    x1[j] = w[j + 4] * kMul1Mult;
  }
  imma_bytesum(x0, ind.b0, ind.b1, d0);
  imma_bytesum(x1, ind.b0, ind.b1, d1);
  a[0] = mul1_pack_affine<kPackFma>(d0[0], d0[2]);  // col g,   k' 2q..2q+1   <- phys 4q, 4q+1
  a[1] = mul1_pack_affine<kPackFma>(d1[0], d1[2]);  // col g+8
  a[2] = mul1_pack_affine<kPackFma>(d0[1], d0[3]);  // col g,   k' 2q+8..     <- phys 4q+2, 4q+3
  a[3] = mul1_pack_affine<kPackFma>(d1[1], d1[3]);  // col g+8
}

// ------------------------------------------------------------------ the mcg codebook

constexpr uint32_t kMcgMult = 0xCBAC1FEDu;

// mcg of a pair of codewords (plugins/sushi_ds41/src/sushi/exl3/expert_exl3.zig:267-273 decodeMcg): each codeword's
// product, masked and flipped, is a pair of f16 halves whose sum is the weight.  The halves are normal with biased
// exponents 12..15, so their f32 sum is exact and its single f16 rounding is the f16x2 add's (the same bits for all
// 65,536 codewords).  Out: f16x2, lo = cw_a's weight, hi = cw_b's.
__device__ __forceinline__ uint32_t mcg_pair(uint32_t cw_a, uint32_t cw_b) {
  const uint32_t pa = ((cw_a * kMcgMult) & 0x8FFF8FFFu) ^ 0x3B603B60u;
  const uint32_t pb = ((cw_b * kMcgMult) & 0x8FFF8FFFu) ^ 0x3B603B60u;
  const uint32_t lo = __byte_perm(pa, pb, 0x5410), hi = __byte_perm(pa, pb, 0x7632);
  uint32_t out;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(out) : "r"(lo), "r"(hi));
  return out;
}

// ------------------------------------------------------------------ one tile's A fragment, by decode spec
//
// DS: 0 = mul1 at the full 16-bit window, 1 = mul1 at a narrowed window (lw.mask), 2 = mcg (any window: lw.mask).

template <int N, int DS, bool kPackFma = false>
__device__ __forceinline__ void decode_tile_imma(const uint32_t* tile_words, const LaneWin<N>& lw,
                                                 const ImmaWin<N>& iw, const ImmaIndicator& ind, uint32_t (&a)[4]) {
  uint32_t w[8];
  if constexpr (DS == 2) {
    // the tensor-pipe order: this lane's k = 4q .. 4q + 3 come from two neighbours' windows (exl3_windows.h)
    imma_windows<N>(tile_words, iw, w);
    a[0] = mcg_pair(w[0], w[1]);  // column g,     k 4q, 4q + 1
    a[1] = mcg_pair(w[2], w[3]);  // column g + 8
    a[2] = mcg_pair(w[4], w[5]);  // column g,     k 4q + 2, 4q + 3
    a[3] = mcg_pair(w[6], w[7]);  // column g + 8
  } else {
    tile_codewords<N, DS == 1>(tile_words, lw, w);
    decode_afrag_imma<kPackFma>(w, ind, a);
  }
}

template <int N, int DS>
__device__ __forceinline__ void decode_tile_natural(const uint32_t* tile_words, const LaneWin<N>& lw, uint32_t (&a)[4]) {
  uint32_t w[8];
  tile_codewords<N, DS != 0>(tile_words, lw, w);
  if constexpr (DS == 2) {
    a[0] = mcg_pair(w[0], w[1]);
    a[1] = mcg_pair(w[4], w[5]);
    a[2] = mcg_pair(w[2], w[3]);
    a[3] = mcg_pair(w[6], w[7]);
  } else {
    decode_afrag_dp4a(w, a);
  }
}

// D[16 x 8] += A[16 x 16] (f16) * B[16 x 8] (f16), f32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------ 128-wide Hadamard in one warp

// v[i] holds element lane + 32 i of a 128-vector; returns H128 v (unnormalised Sylvester order: sign (-1)^popcount).
__device__ __forceinline__ void fwht128_warp(float (&v)[4], uint32_t lane) {
#pragma unroll
  for (uint32_t bit = 1; bit <= 16; bit <<= 1) {
    const bool lower = (lane & bit) == 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float p = __shfl_xor_sync(0xFFFFFFFFu, v[i], bit);
      v[i] = lower ? v[i] + p : p - v[i];
    }
  }
  const float s0 = v[0] + v[1], s1 = v[0] - v[1], s2 = v[2] + v[3], s3 = v[2] - v[3];
  v[0] = s0 + s2;
  v[1] = s1 + s3;
  v[2] = s0 - s2;
  v[3] = s1 - s3;
}

// ------------------------------------------------------------------ activation dtypes

enum DType : int32_t { kF16 = 0, kBF16 = 1, kF32 = 2 };

__device__ __forceinline__ float load_act(const void* p, size_t i, int32_t dt) {
  if (dt == kF16) return __half2float(static_cast<const __half*>(p)[i]);
  if (dt == kBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_act(void* p, size_t i, float v, int32_t dt) {
  if (dt == kF16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else if (dt == kBF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<float*>(p)[i] = v;
}

// 32 bytes to a 32-byte aligned global address (sm_100's 256-bit store): a lane writes a whole L2 sector.
__device__ __forceinline__ void st_global_v8(void* dst, const uint32_t (&r)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(r[0]), "r"(r[1]), "r"(r[2]),
               "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ float f16_bits_to_float(uint16_t b) { return __half2float(__ushort_as_half(b)); }

}  // namespace exl3
