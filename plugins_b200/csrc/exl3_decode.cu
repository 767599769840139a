// exl3_decode.cu -- decode a trellis to the dense W_hat (f16 bits, row-major [in][out]).
//
// The GPU side of the reference's bit-exact decode checks (plugins/turboexl3_ds41/src/exl3/selfcheck.zig:861-930,
// decode_table / golden_tiles, and the decmat kernels): the same in-register decode the GEMV uses, written out.
// One warp per 16x16 tile; lane t's eight weights land at rows {2(t%4), +1, +8, +9}, columns t/4 and t/4 + 8.
#include <cuda_runtime.h>

#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace exl3 {

template <int N, bool IMMA, int DS>
__global__ void __launch_bounds__(256) decode_dense_kernel(const uint16_t* __restrict__ trellis, int in_features,
                                                           int out_features, uint16_t* __restrict__ out,
                                                           uint32_t cw_mask) {
  const uint32_t lane = threadIdx.x & 31u;
  const int ot = out_features / 16;
  const size_t tiles = static_cast<size_t>(in_features / 16) * ot;
  const size_t tile = static_cast<size_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (tile >= tiles) return;  // warp-uniform
  const int tk = static_cast<int>(tile / ot), tn = static_cast<int>(tile % ot);
  const uint32_t* tw = reinterpret_cast<const uint32_t*>(trellis + tile * N);
  LaneWin<N> lw;
  lw.init(lane);
  lw.mask = cw_mask;
  uint32_t a[4];
  const uint32_t g = lane >> 2, q = lane & 3u;
  if constexpr (IMMA) {
    ImmaIndicator ind;
    ind.init(lane);
    ImmaWin<N> iw;
    if constexpr (DS == 2) iw.init(lane, cw_mask);
    decode_tile_imma<N, DS>(tw, lw, iw, ind, a);
    // a[0] = col g at k 4q, 4q+1; a[2] = col g at k 4q+2, 4q+3; a[1], a[3] = col g+8
    const int k0 = 4 * q;
    const int r = tk * 16, c = tn * 16;
    const uint32_t cols[2] = {g, g + 8};
    const uint32_t lo[2] = {a[0], a[1]}, hi[2] = {a[2], a[3]};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      out[static_cast<size_t>(r + k0 + 0) * out_features + c + cols[h]] = static_cast<uint16_t>(lo[h]);
      out[static_cast<size_t>(r + k0 + 1) * out_features + c + cols[h]] = static_cast<uint16_t>(lo[h] >> 16);
      out[static_cast<size_t>(r + k0 + 2) * out_features + c + cols[h]] = static_cast<uint16_t>(hi[h]);
      out[static_cast<size_t>(r + k0 + 3) * out_features + c + cols[h]] = static_cast<uint16_t>(hi[h] >> 16);
    }
  } else {
    decode_tile_natural<N, DS>(tw, lw, a);
    // a[0] = (j0, j1) col g k 2q..; a[1] = (j4, j5) col g+8; a[2] = (j2, j3) col g k 2q+8..; a[3] = (j6, j7)
    const int r = tk * 16, c = tn * 16;
    const int k0 = 2 * q;
    out[static_cast<size_t>(r + k0) * out_features + c + g] = static_cast<uint16_t>(a[0]);
    out[static_cast<size_t>(r + k0 + 1) * out_features + c + g] = static_cast<uint16_t>(a[0] >> 16);
    out[static_cast<size_t>(r + k0) * out_features + c + g + 8] = static_cast<uint16_t>(a[1]);
    out[static_cast<size_t>(r + k0 + 1) * out_features + c + g + 8] = static_cast<uint16_t>(a[1] >> 16);
    out[static_cast<size_t>(r + k0 + 8) * out_features + c + g] = static_cast<uint16_t>(a[2]);
    out[static_cast<size_t>(r + k0 + 9) * out_features + c + g] = static_cast<uint16_t>(a[2] >> 16);
    out[static_cast<size_t>(r + k0 + 8) * out_features + c + g + 8] = static_cast<uint16_t>(a[3]);
    out[static_cast<size_t>(r + k0 + 9) * out_features + c + g + 8] = static_cast<uint16_t>(a[3] >> 16);
  }
}

template <bool IMMA>
static cudaError_t launch_dd(const uint16_t* trellis, int in_features, int out_features, int n, uint16_t* out,
                             cudaStream_t st, uint32_t cw_mask, int mcg) {
  const size_t tiles = static_cast<size_t>(in_features / 16) * (out_features / 16);
  const dim3 grid(static_cast<unsigned>((tiles + 7) / 8)), block(256);
  const bool served = with_rate_decode(n, cw_mask, mcg != 0, [&](auto N, auto DS) {
    decode_dense_kernel<decltype(N)::value, IMMA, decltype(DS)::value>
        <<<grid, block, 0, st>>>(trellis, in_features, out_features, out, spec_mask(cw_mask));
  });
  return served ? cudaGetLastError() : cudaErrorInvalidValue;
}

cudaError_t launch_decode_dense(const uint16_t* trellis, int in_features, int out_features, int n, uint16_t* out,
                                int imma, cudaStream_t st, uint32_t cw_mask, int mcg) {
  return imma ? launch_dd<true>(trellis, in_features, out_features, n, out, st, cw_mask, mcg)
              : launch_dd<false>(trellis, in_features, out_features, n, out, st, cw_mask, mcg);
}

// ------------------------------------------------------------------ the dense effective W (reconstructPublic)
//
// W_eff[r][c] = f16( svh[c] * (H128 (suh[r] * (H128 W_hat)[r][.]))[c] ): the matrix with x @ W_eff = the linear's
// output (plugins/sushi_ds41/src/sushi/exl3/expert_exl3.zig:440-488, the dense twin of SX/linear.zig:200-224).  One
// CTA per 128 x 128 block: its 64 tiles decoded into shared memory (f32), the 128-wide Hadamard along the input for
// every column, then along the output for every row, each in one warp (butterflies in registers).

constexpr int kEffLd = 129;  // shared row stride (floats): column reads hit 32 distinct banks

template <int N, int DS>
__global__ void __launch_bounds__(256) reconstruct_public_kernel(const uint16_t* __restrict__ trellis,
                                                                 const uint16_t* __restrict__ suh,
                                                                 const uint16_t* __restrict__ svh, int in_features,
                                                                 int out_features, uint16_t* __restrict__ out,
                                                                 uint32_t cw_mask) {
  extern __shared__ float blk[];  // [128][kEffLd]
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const int rb = static_cast<int>(blockIdx.y) * 128, cb = static_cast<int>(blockIdx.x) * 128;
  const int ot = out_features / 16;
  LaneWin<N> lw;
  lw.init(lane);
  lw.mask = cw_mask;
  ImmaIndicator ind;
  ind.init(lane);
  ImmaWin<N> iw;
  if constexpr (DS == 2) iw.init(lane, cw_mask);
  const uint32_t g = lane >> 2, q = lane & 3u;
  // the block's 8 x 8 tiles, eight per warp; lane (g, q) holds columns g, g + 8 at rows 4q .. 4q + 3 of its tile
  for (int t = static_cast<int>(warp); t < 64; t += 8) {
    const int tk = rb / 16 + t / 8, tn = cb / 16 + t % 8;
    const uint32_t* tw = reinterpret_cast<const uint32_t*>(trellis + (static_cast<size_t>(tk) * ot + tn) * N);
    uint32_t a[4];
    decode_tile_imma<N, DS>(tw, lw, iw, ind, a);
    const int r0 = (t / 8) * 16 + 4 * static_cast<int>(q), c0 = (t % 8) * 16 + static_cast<int>(g);
    const uint32_t lo[2] = {a[0], a[1]}, hi[2] = {a[2], a[3]};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float* col = blk + c0 + 8 * h;
      col[(r0 + 0) * kEffLd] = f16_bits_to_float(static_cast<uint16_t>(lo[h]));
      col[(r0 + 1) * kEffLd] = f16_bits_to_float(static_cast<uint16_t>(lo[h] >> 16));
      col[(r0 + 2) * kEffLd] = f16_bits_to_float(static_cast<uint16_t>(hi[h]));
      col[(r0 + 3) * kEffLd] = f16_bits_to_float(static_cast<uint16_t>(hi[h] >> 16));
    }
  }
  __syncthreads();
  // along the input: every column's 128 rows, then row r scaled by suh[r]
  for (int c = static_cast<int>(warp); c < 128; c += 8) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = blk[(lane + 32 * i) * kEffLd + c];
    fwht128_warp(v, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      blk[(lane + 32 * i) * kEffLd + c] = v[i] * kHadScale * f16_bits_to_float(suh[rb + lane + 32 * i]);
  }
  __syncthreads();
  // along the output: every row's 128 columns, scaled by svh, rounded to f16 once
  for (int r = static_cast<int>(warp); r < 128; r += 8) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = blk[r * kEffLd + lane + 32 * i];
    fwht128_warp(v, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = cb + static_cast<int>(lane) + 32 * i;
      const float y = v[i] * kHadScale * f16_bits_to_float(svh[c]);
      out[static_cast<size_t>(rb + r) * out_features + c] = __half_as_ushort(__float2half_rn(y));
    }
  }
}

cudaError_t launch_reconstruct_public(const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh,
                                      int in_features, int out_features, int n, uint16_t* out, cudaStream_t st,
                                      uint32_t cw_mask, int mcg) {
  const dim3 grid(static_cast<unsigned>(out_features / 128), static_cast<unsigned>(in_features / 128)), block(256);
  constexpr size_t smem = 128u * kEffLd * 4u;
  cudaError_t e = cudaSuccess;
  const bool served = with_rate_decode(n, cw_mask, mcg != 0, [&](auto N, auto DS) {
    auto kern = reconstruct_public_kernel<decltype(N)::value, decltype(DS)::value>;
    static KernelSetup setup;
    e = kernel_setup(setup, kern, 256, smem);
    if (e == cudaSuccess)
      kern<<<grid, block, smem, st>>>(trellis, suh, svh, in_features, out_features, out, spec_mask(cw_mask));
  });
  if (!served) return cudaErrorInvalidValue;
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace exl3
