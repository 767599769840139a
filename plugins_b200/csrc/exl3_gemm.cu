// exl3_gemm.cu -- the prefill path of an EXL3 linear (many rows): decode once per call, contract on the
// 5th-generation tensor cores.
//
// The reference routes rows > 8 through "prep + sorted GEMM + finish" (plugins/sushi_ds41/src/sushi/linear.zig:77-100)
// and its prefill kernels decode trellis tiles into threadgroup memory ahead of the MMA
// (kernels/dsv41_prefill_dig_gemm_*.metal, header_dig_mul1h_k3.metal:1090-1166).  The math is the same three steps as
// the decode GEMV:  xp = f16(H128(x * suh) / sqrt(128)),  inner = xp . W_hat (f32),  y = H128(inner) / sqrt(128) * svh.
//
// B200 layout.  Both operands are written as "stage images": blocks of 128 rows x 64 k of f16 (16 KiB), each already
// in the UMMA K-major canonical layout with the 128-byte swizzle (row r at byte 128 r, its 16-byte chunk c at chunk
// c ^ (r % 8)).  One pipeline stage is then a handful of whole blocks that cp.async.bulk copies into shared memory
// with no tensor map and no re-layout.
//   A image: [rows/128][in/64] blocks of xp (rows padded with zeros)  -- prepare warps of images_kernel
//   B image: [cols/128][in/64] blocks of W_hat^T (row = output column) -- decode warps of images_kernel, bit-exact
// Both images come from one launch: its decode warps and prepare warps run side by side.
// The GEMM (gemm_image_kernel) is persistent, one CTA per SM, warp-specialised:
//   warp 0      producer: bulk copies of A and B blocks into a ring of stages (mbarrier tx counts)
//   warp 1      MMA issuer: tcgen05.mma kind::f16, M = 128 per A block, N = BN, K = 16, accumulators in TMEM (f32)
//   warp 2      allocates and frees the TMEM columns
//   warps 4..7  epilogue: tcgen05.ld a row's 128 accumulator columns, the output Hadamard (in registers), * svh, store
// Two TMEM accumulators alternate when they fit, so the epilogue of one tile runs under the MMAs of the next.  Every
// mbarrier wait is bounded (about two seconds); a wait that gives up sets an abort flag that every role polls, records
// kErrWaitTimeout and lets the CTA reach its TMEM release.
#include <cuda_runtime.h>

#include "exl3_common.cuh"
#include "exl3_internal.h"
#include "exl3_tc.cuh"

namespace exl3 {

using namespace tc;

// ------------------------------------------------------------------ the operand images, one launch

// consecutive column tiles of one k-row per decode warp, their loads issued together (measured on config 3's layer:
// images 39.4 / 37.5 / 36.2 us at 2 / 4 / 8)
constexpr int kDecodeTilesPerWarp = 8;

struct ImageJobs {
  // A image: xp rows [0, mp) (rows >= m written as zeros); prepared = x already holds xp
  const void* x;
  int32_t x_dtype;
  int64_t x_row_stride;
  int32_t m, mp, prepared;
  const uint16_t* suh;
  uint8_t* a_img;
  int64_t prep_jobs;     // mp * in/128 warps (prep16: mp * in/512), 0 = no A image
  int32_t prep16;        // the sixteen-per-lane prepare jobs
  // B image: trellis columns [16 tn0, 16 (tn0 + ncol_tiles))
  const uint16_t* trellis;
  int32_t out_tiles, tn0, ncol_tiles;
  uint8_t* b_img;
  int64_t decode_jobs;   // (in/16) * ncol_tiles / kDecodeTilesPerWarp warps
  int32_t in_features;
  uint32_t cw_mask;      // a narrowed codeword window's mask (0: the full 16-bit window)
};

// H128(v * suh) / sqrt(128) with sixteen elements per lane (lanes 8b .. 8b + 7 hold block b, lane 8b + p its
// elements 16p .. 16p + 15): stages h = 1 .. 8 in registers, h = 16, 32, 64 across the block's eight lanes -- the
// butterflies of rotate128 in the same stage order, so the same bytes, with 48 shuffles a block-quad instead of 80.
__device__ __forceinline__ void rotate128x16(float (&v)[16], const uint4 (&su)[2], uint32_t lane) {
  const uint32_t sw[8] = {su[0].x, su[0].y, su[0].z, su[0].w, su[1].x, su[1].y, su[1].z, su[1].w};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&sw[e]));
    v[2 * e] *= f.x, v[2 * e + 1] *= f.y;
  }
#pragma unroll
  for (int h = 1; h < 16; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if ((i & h) == 0) {
        const float a = v[i], c = v[i + h];
        v[i] = a + c;
        v[i + h] = a - c;
      }
    }
  }
#pragma unroll
  for (uint32_t bit = 1; bit <= 4; bit <<= 1) {
    const bool lower = (lane & bit) == 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float p = __shfl_xor_sync(0xFFFFFFFFu, v[i], bit);
      v[i] = lower ? v[i] + p : p - v[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] *= kHadScale;
}

// Sixteen f16 elements k0 .. k0 + 15 (k0 a multiple of 16) of one image row: two 16-byte swizzled chunks.
__device__ __forceinline__ void store_image16(uint8_t* img, int kblocks64, int row, int k0, const float (&v)[16]) {
  uint32_t h[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const __half2 t = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    h[e] = *reinterpret_cast<const uint32_t*>(&t);
  }
  uint8_t* blk = img + ((static_cast<size_t>(row) >> 7) * kblocks64 + (k0 >> 6)) * kImgBytes;
  const uint32_t r = static_cast<uint32_t>(row) & 127u, kk = static_cast<uint32_t>(k0 & 63);
  *reinterpret_cast<uint4*>(blk + image_offset(r, kk)) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(blk + image_offset(r, kk + 8u)) = make_uint4(h[4], h[5], h[6], h[7]);
}

// Prepare job: one warp per (row, 128-wide input block), lane t holding elements 4t..4t+3 (vector loads and one
// 8-byte store); the Hadamard's two low stages run in registers, the other five across lanes.
__device__ __forceinline__ void prep_job(const ImageJobs& j, int64_t job, uint32_t lane) {
  const int kblk = j.in_features / 128;
  const int row = static_cast<int>(job / kblk), b = static_cast<int>(job % kblk);
  const int k0 = b * 128 + 4 * static_cast<int>(lane);
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (row < j.m) {
    const size_t at = static_cast<size_t>(row) * j.x_row_stride + k0;
    if (j.x_dtype == kF32) {
      const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(j.x) + at);
      v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(j.x) + at);
      const uint32_t w2[2] = {u.x, u.y};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float2 f;
        if (j.x_dtype == kF16) f = __half22float2(*reinterpret_cast<const __half2*>(&w2[e]));
        else f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w2[e]));
        v[2 * e] = f.x, v[2 * e + 1] = f.y;
      }
    }
    if (!j.prepared) {
      const uint2 su = *reinterpret_cast<const uint2*>(j.suh + k0);
      const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&su.x));
      const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&su.y));
      v[0] *= s01.x, v[1] *= s01.y, v[2] *= s23.x, v[3] *= s23.y;
      const float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
      v[0] = a0 + a2, v[1] = a1 + a3, v[2] = a0 - a2, v[3] = a1 - a3;
#pragma unroll
      for (uint32_t bit = 1; bit <= 16; bit <<= 1) {
        const bool lower = (lane & bit) == 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p = __shfl_xor_sync(0xFFFFFFFFu, v[i], bit);
          v[i] = lower ? v[i] + p : p - v[i];
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] *= kHadScale;
    }
  }
  const __half2 h01 = __floats2half2_rn(v[0], v[1]), h23 = __floats2half2_rn(v[2], v[3]);
  const uint32_t r = static_cast<uint32_t>(row) & 127u;
  uint8_t* blk = j.a_img + ((static_cast<size_t>(row) >> 7) * (j.in_features / kImgK) + (k0 >> 6)) * kImgBytes;
  *reinterpret_cast<uint2*>(blk + image_offset(r, static_cast<uint32_t>(k0 & 63))) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
}

// Prepare job with sixteen elements per lane: one warp per (row, 512 inputs), lanes 8b .. 8b + 7 holding 128-block b
// (two 16-byte loads and two 16-byte stores a lane; three shuffle stages instead of five) -- the same bytes as four
// prep_job calls.  Taken when in_features is a multiple of 512 and x's rows are 16-byte aligned: the one-block jobs
// were short warps whose many waves of load latency set the prepare's time.
__device__ __forceinline__ void prep16_job(const ImageJobs& j, int64_t job, uint32_t lane) {
  const int kq = j.in_features / 512;
  const int row = static_cast<int>(job / kq);
  const int k0 = static_cast<int>(job % kq) * 512 + 16 * static_cast<int>(lane);
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = 0.f;
  if (row < j.m) {
    const size_t at = static_cast<size_t>(row) * j.x_row_stride + k0;
    if (j.x_dtype == kF32) {
      const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(j.x) + at);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float4 f = xp[c];
        v[4 * c] = f.x, v[4 * c + 1] = f.y, v[4 * c + 2] = f.z, v[4 * c + 3] = f.w;
      }
    } else {
      const uint4* xp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(j.x) + at);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 u = xp[c];
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = j.x_dtype == kF16 ? __half22float2(*reinterpret_cast<const __half2*>(&w4[e]))
                                             : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[e]));
          v[8 * c + 2 * e] = f.x, v[8 * c + 2 * e + 1] = f.y;
        }
      }
    }
    if (!j.prepared) {
      const uint4* sp = reinterpret_cast<const uint4*>(j.suh + k0);
      const uint4 su[2] = {sp[0], sp[1]};
      rotate128x16(v, su, lane);
    }
  }
  store_image16(j.a_img, j.in_features / kImgK, row, k0, v);
}

// Decode job: kDecodeTilesPerWarp consecutive 16x16 tiles of one k-row (contiguous in the trellis).  Each lane holds
// one column's four consecutive k per tile (the IMMA byte-sum order) and writes them as one 8-byte store; a warp's
// stores fill whole 32-byte sectors.
template <int N, int DS>
__device__ __forceinline__ void decode_job(const ImageJobs& j, int64_t job, uint32_t lane) {
  const int groups = j.ncol_tiles / kDecodeTilesPerWarp;
  const int tk = static_cast<int>(job / groups), tj0 = static_cast<int>(job % groups) * kDecodeTilesPerWarp;
  const uint32_t* tw =
      reinterpret_cast<const uint32_t*>(j.trellis + (static_cast<size_t>(tk) * j.out_tiles + j.tn0 + tj0) * N);
  LaneWin<N> lw;
  lw.init(lane);
  lw.mask = j.cw_mask;
  ImmaIndicator ind;
  ind.init(lane);
  ImmaWin<N> iw;
  if constexpr (DS == 2) iw.init(lane, j.cw_mask);
  uint32_t w[kDecodeTilesPerWarp][8];
  if constexpr (DS != 2) {
#pragma unroll
    for (int t = 0; t < kDecodeTilesPerWarp; ++t) tile_codewords<N, DS == 1>(tw + t * (N / 2), lw, w[t]);
  }
  const uint32_t g = lane >> 2, q = lane & 3u;
  const int kbs = j.in_features / kImgK;
  const uint32_t kin = static_cast<uint32_t>(tk & 3) * 16u + 4u * q;
#pragma unroll
  for (int t = 0; t < kDecodeTilesPerWarp; ++t) {
    uint32_t a[4];  // a[0], a[2]: column g at k 4q..4q+3; a[1], a[3]: column g + 8
    if constexpr (DS == 2) decode_tile_imma<N, 2>(tw + t * (N / 2), lw, iw, ind, a);
    else decode_afrag_imma(w[t], ind, a);
    const int tj = tj0 + t;
    const uint32_t n = static_cast<uint32_t>(tj & 7) * 16u + g;
    uint8_t* blk = j.b_img + (static_cast<size_t>(tj >> 3) * kbs + (tk >> 2)) * kImgBytes;
    *reinterpret_cast<uint2*>(blk + image_offset(n, kin)) = make_uint2(a[0], a[2]);
    *reinterpret_cast<uint2*>(blk + image_offset(n + 8u, kin)) = make_uint2(a[1], a[3]);
  }
}

// Decode warps first (the longer jobs), then prepare warps; every job is one warp.
template <int N, int DS>
__global__ void __launch_bounds__(256) images_kernel(const ImageJobs j) {
  const uint32_t lane = threadIdx.x & 31u;
  const int64_t job = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);  // warp-uniform
  if (job < j.decode_jobs) decode_job<N, DS>(j, job, lane);
  else if (job < j.decode_jobs + j.prep_jobs) {
    if (j.prep16) prep16_job(j, job - j.decode_jobs, lane);
    else prep_job(j, job - j.decode_jobs, lane);
  }
}

// ------------------------------------------------------------------ the routed experts' prefill images
//
// Rows are the call's (token, k) slots sorted by expert, each expert's rows padded to whole 128-row blocks
// (row_slot[row] = token * topk + k, or -1 for padding; m_group[row / 128] = the block's expert).  The A images hold
// the gate- and up-prepared rows (x read once per job, rotated twice), the down input's A image the SwiGLU of the
// gate|up GEMMs' outputs prepared for down; B images are each expert's decoded W_hat^T, as for a single linear.
// Padding rows are never written: a GEMM output row depends only on its own A row, and a padding row's outputs are
// neither read by the SwiGLU nor combined, so whatever its A row holds reaches no real row's bytes.

// xp = f16-ready H128(v * suh) / sqrt(128) of one warp's 128 inputs (lane t: elements 4t .. 4t + 3, su its four suh
// halves), the two low stages in registers, the other five across lanes (prep_job's arithmetic).
__device__ __forceinline__ void rotate128(float (&v)[4], uint2 su, uint32_t lane) {
  const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&su.x));
  const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&su.y));
  v[0] *= s01.x, v[1] *= s01.y, v[2] *= s23.x, v[3] *= s23.y;
  const float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
  v[0] = a0 + a2, v[1] = a1 + a3, v[2] = a0 - a2, v[3] = a1 - a3;
#pragma unroll
  for (uint32_t bit = 1; bit <= 16; bit <<= 1) {
    const bool lower = (lane & bit) == 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float p = __shfl_xor_sync(0xFFFFFFFFu, v[i], bit);
      v[i] = lower ? v[i] + p : p - v[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] *= kHadScale;
}

__device__ __forceinline__ void store_image4(uint8_t* img, int kblocks64, int row, int k0, const float (&v)[4]) {
  const __half2 h01 = __floats2half2_rn(v[0], v[1]), h23 = __floats2half2_rn(v[2], v[3]);
  uint8_t* blk = img + ((static_cast<size_t>(row) >> 7) * kblocks64 + (k0 >> 6)) * kImgBytes;
  *reinterpret_cast<uint2*>(blk + image_offset(static_cast<uint32_t>(row) & 127u, static_cast<uint32_t>(k0 & 63))) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
}

// x[i .. i + 3] as f32 (exact conversions, as load_act): one 8-byte (f16, bf16) or 16-byte (f32) load when the
// caller's rows are aligned for it (vec), else four element loads.
__device__ __forceinline__ void load_act4(const void* p, size_t i, int32_t dt, bool vec, float (&v)[4]) {
  if (vec && dt == kF32) {
    const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
  } else if (vec) {
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + i);
    float2 lo, hi;
    if (dt == kF16) {
      lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    } else {
      lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    }
    v[0] = lo.x, v[1] = lo.y, v[2] = hi.x, v[3] = hi.y;
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = load_act(p, i + q, dt);
  }
}

// One warp per (row, KB consecutive 128-input blocks), grid-stride over the call's rows (a device count).  The KB
// blocks' loads are issued before the first rotation: one block per warp left the kernel waiting on each load in turn.
template <int KB>
__global__ void __launch_bounds__(256) moe_a_images_kernel(const MoeImages j) {
  const uint32_t lane = threadIdx.x & 31u;
  const int groups = j.hidden / (128 * KB);
  const int64_t jobs = static_cast<int64_t>(*j.rows_total) * groups;
  for (int64_t job = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); job < jobs;
       job += static_cast<int64_t>(gridDim.x) * 8) {
    const int row = static_cast<int>(job / groups);
    const int slot = j.row_slot[row];
    if (slot < 0) continue;  // (warp-uniform) padding
    const int k0 = static_cast<int>(job % groups) * KB * 128 + 4 * static_cast<int>(lane);
    const size_t e = static_cast<size_t>(j.m_group[row >> 7]);
    const size_t at = static_cast<size_t>(slot / j.topk) * j.x_row_stride + k0;
    float v[KB][4];
    uint2 sg[KB], su[KB];
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      load_act4(j.x, at + b * 128, j.x_dtype, j.x_vec != 0, v[b]);
      sg[b] = *reinterpret_cast<const uint2*>(j.suh_g + e * j.hidden + k0 + b * 128);
      su[b] = *reinterpret_cast<const uint2*>(j.suh_u + e * j.hidden + k0 + b * 128);
    }
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      float vg[4] = {v[b][0], v[b][1], v[b][2], v[b][3]};
      rotate128(vg, sg[b], lane);
      store_image4(j.a_g, j.hidden / kImgK, row, k0 + b * 128, vg);
      rotate128(v[b], su[b], lane);
      store_image4(j.a_u, j.hidden / kImgK, row, k0 + b * 128, v[b]);
    }
  }
}

// The gate and up A images with sixteen elements per lane: one warp per (row, 512 inputs), grid-stride over the
// call's rows.  Taken when x's rows are 16-byte aligned (x_vec) and hidden is a multiple of 512: fewer shuffles than
// the four-per-lane form, whose rotations were bound by the shuffle rate.
__global__ void __launch_bounds__(256) moe_a_images16_kernel(const MoeImages j) {
  const uint32_t lane = threadIdx.x & 31u;
  const int groups = j.hidden / 512;
  const int64_t jobs = static_cast<int64_t>(*j.rows_total) * groups;
  for (int64_t job = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); job < jobs;
       job += static_cast<int64_t>(gridDim.x) * 8) {
    const int row = static_cast<int>(job / groups);
    const int slot = j.row_slot[row];
    if (slot < 0) continue;  // (warp-uniform) padding
    const int k0 = static_cast<int>(job % groups) * 512 + 16 * static_cast<int>(lane);
    const size_t e = static_cast<size_t>(j.m_group[row >> 7]);
    const size_t at = static_cast<size_t>(slot / j.topk) * j.x_row_stride + k0;
    float vg[16], vu[16];
    if (j.x_dtype == kF32) {
      const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(j.x) + at);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f = xp[q];
        vg[4 * q] = f.x, vg[4 * q + 1] = f.y, vg[4 * q + 2] = f.z, vg[4 * q + 3] = f.w;
      }
    } else {
      const uint4* xp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(j.x) + at);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const uint4 u = xp[q];
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 f = j.x_dtype == kF16 ? __half22float2(*reinterpret_cast<const __half2*>(&w4[c]))
                                             : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[c]));
          vg[8 * q + 2 * c] = f.x, vg[8 * q + 2 * c + 1] = f.y;
        }
      }
    }
    const uint4* sgp = reinterpret_cast<const uint4*>(j.suh_g + e * j.hidden + k0);
    const uint4* sup = reinterpret_cast<const uint4*>(j.suh_u + e * j.hidden + k0);
    const uint4 sg[2] = {sgp[0], sgp[1]}, su[2] = {sup[0], sup[1]};
#pragma unroll
    for (int i = 0; i < 16; ++i) vu[i] = vg[i];
    rotate128x16(vg, sg, lane);
    store_image16(j.a_g, j.hidden / kImgK, row, k0, vg);
    rotate128x16(vu, su, lane);
    store_image16(j.a_u, j.hidden / kImgK, row, k0, vu);
  }
}

// The down input: h = silu(g) * u of the gate|up GEMMs' f32 outputs (g, u: columns [0, inter) and [inter, 2 inter)
// of gu), clamped as the routed experts' epilogue clamps, times the down bank's suh, rotated, f16 -- one warp per
// (row, KB 128-blocks) of the rows [row_range[0], row_range[1]), loads first as above.
template <int KB>
__global__ void __launch_bounds__(256) moe_mid_images_kernel(const MoeImages j) {
  const uint32_t lane = threadIdx.x & 31u;
  const int groups = j.inter / (128 * KB);
  const int r0 = j.row_range[0];
  const int64_t jobs = static_cast<int64_t>(j.row_range[1] - r0) * groups;
  for (int64_t job = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); job < jobs;
       job += static_cast<int64_t>(gridDim.x) * 8) {
    const int row = r0 + static_cast<int>(job / groups);
    if (j.row_slot[row] < 0) continue;  // (warp-uniform) padding
    const int k0 = static_cast<int>(job % groups) * KB * 128 + 4 * static_cast<int>(lane);
    const size_t e = static_cast<size_t>(j.m_group[row >> 7]);
    const float* gr = j.gu + static_cast<size_t>(row) * j.gu_stride + k0;
    float4 g[KB], u[KB];
    uint2 sd[KB];
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      g[b] = *reinterpret_cast<const float4*>(gr + b * 128);
      u[b] = *reinterpret_cast<const float4*>(gr + j.inter + b * 128);
      sd[b] = *reinterpret_cast<const uint2*>(j.suh_d + e * j.inter + k0 + b * 128);
    }
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      const float gv[4] = {g[b].x, g[b].y, g[b].z, g[b].w}, uv0[4] = {u[b].x, u[b].y, u[b].z, u[b].w};
      float h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float gi = gv[i], ui = uv0[i];
        if (j.limit > 0.0f) {
          gi = fminf(gi, j.limit);
          ui = fminf(fmaxf(ui, -j.limit), j.limit);
        }
        const float sig = 1.0f / (1.0f + __expf(-gi));
        h[i] = gi * sig * ui;
      }
      rotate128(h, sd[b], lane);
      store_image4(j.a_d, j.inter / kImgK, row, k0 + b * 128, h);
    }
  }
}

// B images of experts e0 .. e0 + count - 1 (experts without rows skipped): expert e's decode jobs write its W_hat^T
// blocks at b_img + (e - e0) * b_group_bytes.
template <int N, int DS>
__global__ void __launch_bounds__(256) moe_b_images_kernel(ImageJobs j, int e0, int64_t jobs_per, const int32_t* counts,
                                                           int64_t tr_group, int64_t b_group_bytes) {
  const uint32_t lane = threadIdx.x & 31u;
  const int64_t job = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int e = e0 + static_cast<int>(job / jobs_per);
  if (job >= j.decode_jobs || counts[e] == 0) return;  // (warp-uniform)
  ImageJobs je = j;
  je.trellis = j.trellis + static_cast<size_t>(e) * tr_group;
  je.b_img = j.b_img + static_cast<size_t>(e - e0) * b_group_bytes;
  decode_job<N, DS>(je, job % jobs_per, lane);
}

// ------------------------------------------------------------------ the GEMM

// Orders uses of r after an earlier tcgen05.wait::ld (both asm statements are volatile, so they keep their order).
__device__ __forceinline__ void tmem_after_wait(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

template <int MS, int NS>
struct GemmShape {
  static constexpr int BM = 128 * MS, BN = 128 * NS;
  static constexpr uint32_t kStageBytes = (MS + NS) * kImgBytes;
  static constexpr int kStages = (MS + NS) == 2 ? 6 : ((MS + NS) == 3 ? 4 : 3);
  static constexpr int kAccCols = MS * BN;
  static constexpr int kAccBufs = kAccCols * 2 <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kAccCols * kAccBufs <= 256 ? 256 : 512;
  // stages, 1024-byte alignment slack, barriers, and the four epilogue warps' two svh slots of NS x 128 halves
  static constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kStageBytes + 1024 + 256 + 4 * 2 * NS * 256;
  static_assert(BN <= 256, "one MMA covers at most 256 columns");
  static_assert(kAccCols * kAccBufs <= 512, "TMEM holds 512 columns");
};

template <int MS, int NS>
__global__ void __launch_bounds__(256, 1) gemm_image_kernel(const GemmParams p) {
  using S = GemmShape<MS, NS>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* stages = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // the swizzle is anchored on 1024-byte rows
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + S::kStages * S::kStageBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* accf = empty + S::kStages;
  uint64_t* acce = accf + 2;
  uint64_t* fin = acce + 2;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(fin + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 128);
    }
    mbar_init(fin, 1);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // grouped: this launch's M blocks come from the device (the routing wrote them); MS is 1 there
  int mt0 = 0, tiles_m = p.tiles_m;
  if (p.mt_range) {
    mt0 = p.mt_range[0];
    tiles_m = p.mt_range[1] - mt0;
  }
  const int tiles = tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer
      const uint64_t pol_a = policy_evict_last(), pol_b = policy_evict_first();
      uint32_t stage = 0, phase = 0, fills = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int mb = mt0 + t % tiles_m, nb = t / tiles_m;
        const uint8_t* bimg = p.b_img + (p.m_group ? (p.m_group[mb] - p.group0) * p.b_group_bytes : 0);
        for (int kb = 0; kb < p.kb; ++kb) {
          if (!role_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          uint8_t* dst = stages + stage * S::kStageBytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
#pragma unroll
          for (int s = 0; s < MS; ++s)
            bulk_g2s(dst + s * kImgBytes, p.a_img + (static_cast<size_t>(mb * MS + s) * p.kb + kb) * kImgBytes,
                     kImgBytes, &full[stage], pol_a);
#pragma unroll
          for (int j = 0; j < NS; ++j)
            bulk_g2s(dst + (MS + j) * kImgBytes, bimg + (static_cast<size_t>(nb * NS + j) * p.kb + kb) * kImgBytes,
                     kImgBytes, &full[stage], pol_b);
          ++fills;
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // No copy may outlive the CTA: wait (bounded) for the last fill of every stage.
      const uint32_t last = fills < static_cast<uint32_t>(S::kStages) ? fills : static_cast<uint32_t>(S::kStages);
      for (uint32_t i = 1; i <= last; ++i) {
        const uint32_t f = fills - i;
        if (!mbar_wait_bounded(&full[f % S::kStages], (f / S::kStages) & 1u)) atomicOr(p.err, kErrWaitTimeout);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = umma_idesc(128, S::BN);
      uint32_t stage = 0, phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++local) {
        const int ab = S::kAccBufs == 2 ? (local & 1) : 0;
        const uint32_t aph = S::kAccBufs == 2 ? ((local >> 1) & 1) : (local & 1);
        if (!role_wait(&acce[ab], aph ^ 1u, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + static_cast<uint32_t>(ab * S::kAccCols);
        for (int kb = 0; kb < p.kb; ++kb) {
          if (!role_wait(&full[stage], phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(stages + stage * S::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < kImgK / 16; ++kk) {
            const uint64_t bdesc = sw128_desc(base + MS * kImgBytes + kk * 32);
#pragma unroll
            for (int s = 0; s < MS; ++s)
              umma_f16(d0 + s * S::BN, sw128_desc(base + s * kImgBytes + kk * 32), bdesc, idesc,
                       (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&accf[ab]);
      }
      // every MMA this thread issued has finished before TMEM is released
      umma_commit(fin);
      if (!mbar_wait_bounded(fin, 0)) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- epilogue: warp 4 + j reads TMEM lanes 32 j .. 32 j + 31
    const uint32_t wq = warp - 4;
    uint8_t* svs = stages + S::kStages * S::kStageBytes + 256 + wq * 2 * (NS * 256);  // this warp's [2][NS*128] svh
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int ab = S::kAccBufs == 2 ? (local & 1) : 0;
      const uint32_t aph = S::kAccBufs == 2 ? ((local >> 1) & 1) : (local & 1);
      const int mb = mt0 + t % tiles_m, nb = t / tiles_m;
      const int64_t sv_e = p.m_group ? static_cast<int64_t>(p.m_group[mb]) * p.svh_group : 0;
      // the tile's svh columns into this warp's shared-memory slot before the accumulator wait, so their load latency
      // hides under it instead of following the Hadamard (measured on config 3's layer: the GEMM 165 -> 161 us)
      uint8_t* svt = svs + (local & 1) * (NS * 256);
      if (!p.inner_only && lane < static_cast<uint32_t>(NS * 16)) {
        const int c = static_cast<int>(lane) / 16, q16 = static_cast<int>(lane) % 16;
        const int col0 = (nb * NS + c) * 128;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (col0 < p.ncols) {
          const uint16_t* svc = p.svh2 && col0 >= p.svh_split ? p.svh2 + sv_e + (col0 - p.svh_split)
                                                              : p.svh + sv_e + col0;
          v = __ldg(reinterpret_cast<const uint4*>(svc) + q16);
        }
        reinterpret_cast<uint4*>(svt)[lane] = v;
      }
      if (!role_wait(&accf[ab], aph, abort_flag, p.err)) break;
      tc_fence_after();
      __syncwarp();
#pragma unroll 1
      for (int s = 0; s < MS; ++s) {
        const int row = (mb * MS + s) * 128 + static_cast<int>(wq * 32 + lane);
#pragma unroll 1
        for (int c = 0; c < NS; ++c) {
          const int col0 = (nb * NS + c) * 128;
          if (col0 >= p.ncols) continue;  // warp-uniform: a ragged tile's padding columns are neither read nor stored
          float v[128];
          uint32_t rr[4][32];
          const uint32_t taddr =
              tmem + ((wq * 32u) << 16) + static_cast<uint32_t>(ab * S::kAccCols + s * S::BN + c * 128);
#pragma unroll
          for (int h = 0; h < 4; ++h) tmem_ld32(taddr + h * 32, rr[h]);  // four loads, one wait (1 % on config 3)
          tmem_wait_ld(rr[0]);
#pragma unroll
          for (int h = 1; h < 4; ++h) tmem_after_wait(rr[h]);
#pragma unroll
          for (int h = 0; h < 4; ++h)
#pragma unroll
            for (int i = 0; i < 32; ++i) v[h * 32 + i] = __uint_as_float(rr[h][i]);
          if (!p.inner_only) {
            fwht128_regs(v);
            const uint4* sv4 = reinterpret_cast<const uint4*>(svt + c * 256);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint4 u = sv4[j];
              const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
                v[j * 8 + 2 * e] *= kHadScale * f.x;
                v[j * 8 + 2 * e + 1] *= kHadScale * f.y;
              }
            }
          }
          if (row < p.m) {
            const size_t at = static_cast<size_t>(row) * p.y_row_stride + col0;
            // 32-byte stores where y allows them: with one row per thread, a 16-byte store wrote half an L2 sector
            // of 32 rows at once (measured on config 3's layer: the GEMM 172 -> 162 us)
            if (p.vec_store == 2 && p.y_dtype != kF32) {
              uint16_t* dst = static_cast<uint16_t*>(p.y) + at;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                uint32_t pk[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float lo = v[j * 16 + 2 * e], hi = v[j * 16 + 2 * e + 1];
                  if (p.y_dtype == kF16) {
                    const __half2 h2 = __floats2half2_rn(lo, hi);
                    pk[e] = *reinterpret_cast<const uint32_t*>(&h2);
                  } else {
                    const __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
                    pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
                  }
                }
                st_global_v8(dst + j * 16, pk);
              }
            } else if (p.vec_store == 2) {
              float* dst = static_cast<float*>(p.y) + at;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                uint32_t pk[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) pk[e] = __float_as_uint(v[8 * j + e]);
                st_global_v8(dst + j * 8, pk);
              }
            } else if (p.vec_store && p.y_dtype != kF32) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.y) + at);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                uint32_t pk[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float lo = v[j * 8 + 2 * e], hi = v[j * 8 + 2 * e + 1];
                  if (p.y_dtype == kF16) {
                    const __half2 h2 = __floats2half2_rn(lo, hi);
                    pk[e] = *reinterpret_cast<const uint32_t*>(&h2);
                  } else {
                    const __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
                    pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
                  }
                }
                dst[j] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              }
            } else if (p.vec_store) {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.y) + at);
#pragma unroll
              for (int j = 0; j < 32; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            } else {
#pragma unroll
              for (int i = 0; i < 128; ++i) store_act(p.y, at + i, v[i], p.y_dtype);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// ------------------------------------------------------------------ host launchers

cudaError_t launch_images(const void* x, int32_t x_dtype, int64_t x_row_stride, int m, int mp, const uint16_t* suh,
                          int prepared, uint8_t* a_img, const uint16_t* trellis, int in_features, int out_features,
                          int col0, int ncols, int n, uint8_t* b_img, cudaStream_t st, uint32_t cw_mask, int mcg) {
  if (in_features % 128 != 0 || !rate_served_n(n)) return cudaErrorInvalidValue;
  ImageJobs j{};
  j.in_features = in_features;
  j.cw_mask = spec_mask(cw_mask);
  if (a_img) {
    if (mp % 128 != 0 || m > mp) return cudaErrorInvalidValue;
    const size_t vec = x_dtype == kF32 ? 16 : 8;  // four elements per vector load
    if (reinterpret_cast<uintptr_t>(x) % vec != 0 || (x_row_stride * (x_dtype == kF32 ? 4 : 2)) % vec != 0)
      return cudaErrorInvalidValue;
    j.x = x, j.x_dtype = x_dtype, j.x_row_stride = x_row_stride;
    j.m = m, j.mp = mp, j.prepared = prepared, j.suh = suh, j.a_img = a_img;
    const size_t xsz = x_dtype == kF32 ? 4 : 2;
    j.prep16 = in_features % 512 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 && (x_row_stride * xsz) % 16 == 0 &&
               (prepared || reinterpret_cast<uintptr_t>(suh) % 16 == 0);
    j.prep_jobs = static_cast<int64_t>(mp) * (in_features / (j.prep16 ? 512 : 128));
  }
  if (b_img) {
    if (col0 % 128 != 0 || ncols % 128 != 0) return cudaErrorInvalidValue;
    j.trellis = trellis, j.out_tiles = out_features / 16, j.tn0 = col0 / 16, j.ncol_tiles = ncols / 16;
    j.b_img = b_img;
    j.decode_jobs = static_cast<int64_t>(in_features / 16) * (ncols / 16) / kDecodeTilesPerWarp;
  }
  const int64_t warps = j.prep_jobs + j.decode_jobs;
  if (warps == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((warps + 7) / 8)), block(256);
  const bool served = with_rate_decode(n, b_img ? cw_mask : 0u, b_img && mcg, [&](auto N, auto DS) {
    images_kernel<decltype(N)::value, decltype(DS)::value><<<grid, block, 0, st>>>(j);
  });
  return served ? cudaGetLastError() : cudaErrorInvalidValue;
}

cudaError_t launch_moe_a_images(const MoeImages& j, int sms, cudaStream_t st) {
  if (j.hidden % 128 != 0) return cudaErrorInvalidValue;
  const bool suh16 = reinterpret_cast<uintptr_t>(j.suh_g) % 16 == 0 && reinterpret_cast<uintptr_t>(j.suh_u) % 16 == 0;
  if (j.hidden % 512 == 0 && j.x_vec && suh16) moe_a_images16_kernel<<<sms * 8, 256, 0, st>>>(j);
  else if (j.hidden % 512 == 0) moe_a_images_kernel<4><<<sms * 8, 256, 0, st>>>(j);
  else moe_a_images_kernel<1><<<sms * 8, 256, 0, st>>>(j);
  return cudaGetLastError();
}

cudaError_t launch_moe_mid_images(const MoeImages& j, int sms, cudaStream_t st) {
  if (j.inter % 128 != 0) return cudaErrorInvalidValue;
  if (j.inter % 512 == 0) moe_mid_images_kernel<4><<<sms * 8, 256, 0, st>>>(j);
  else moe_mid_images_kernel<1><<<sms * 8, 256, 0, st>>>(j);
  return cudaGetLastError();
}

cudaError_t launch_moe_b_images(const uint16_t* trellis, int in_features, int out_features, int n, int e0, int count,
                                const int32_t* counts, uint8_t* b_img, int64_t b_group_bytes, cudaStream_t st,
                                uint32_t cw_mask, int mcg) {
  if (in_features % 128 != 0 || out_features % 128 != 0 || !rate_served_n(n) || count < 1) return cudaErrorInvalidValue;
  ImageJobs j{};
  j.in_features = in_features;
  j.cw_mask = spec_mask(cw_mask);
  j.trellis = trellis, j.out_tiles = out_features / 16, j.tn0 = 0, j.ncol_tiles = out_features / 16;
  j.b_img = b_img;
  const int64_t per = static_cast<int64_t>(in_features / 16) * (out_features / 16) / kDecodeTilesPerWarp;
  j.decode_jobs = per * count;
  const int64_t tr_group = static_cast<int64_t>(in_features / 16) * (out_features / 16) * n;
  const dim3 grid(static_cast<unsigned>((j.decode_jobs + 7) / 8)), block(256);
  const bool served = with_rate_decode(n, cw_mask, mcg != 0, [&](auto N, auto DS) {
    moe_b_images_kernel<decltype(N)::value, decltype(DS)::value>
        <<<grid, block, 0, st>>>(j, e0, per, counts, tr_group, b_group_bytes);
  });
  return served ? cudaGetLastError() : cudaErrorInvalidValue;
}

template <int MS, int NS>
static cudaError_t launch_gemm_t(const GemmParams& p, int sms, cudaStream_t st) {
  using S = GemmShape<MS, NS>;
  if (p.tiles_m * 128 * MS < p.m) return cudaErrorInvalidValue;
  if ((p.mt_range || p.m_group) && MS != 1) return cudaErrorInvalidValue;
  static KernelSetup setup;
  if (cudaError_t e = kernel_setup(setup, gemm_image_kernel<MS, NS>, 256, S::kSmemBytes); e != cudaSuccess) return e;
  const int tiles = p.tiles_m * p.tiles_n;  // (grouped: an upper bound; the kernel reads the launch's blocks)
  const int grid = tiles < sms ? tiles : sms;
  gemm_image_kernel<MS, NS><<<grid, 256, S::kSmemBytes, st>>>(p);
  return cudaGetLastError();
}

int gemm_block_m(int shape) { return shape == 2 || shape == 3 ? 256 : 128; }
int gemm_block_n(int shape) { return shape == 1 || shape == 3 ? 256 : 128; }

cudaError_t launch_gemm_image(const GemmParams& p, int shape, int sms, cudaStream_t st) {
  switch (shape) {
    case 0: return launch_gemm_t<1, 1>(p, sms, st);
    case 1: return launch_gemm_t<1, 2>(p, sms, st);
    case 2: return launch_gemm_t<2, 1>(p, sms, st);
    case 3: return launch_gemm_t<2, 2>(p, sms, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace exl3
