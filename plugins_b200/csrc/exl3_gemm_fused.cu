// exl3_gemm_fused.cu -- the prefill GEMM with W_hat^T decoded inside it (sm_100a): no B image.
//
// gemm_image_kernel (exl3_gemm.cu) reads W_hat^T from an operand image that a decode launch wrote: two bytes per
// weight written to HBM and read back, against the trellis' 2-6 bits.  Where a block's rows are one expert's (the routed
// experts' prefill, whose experts hold a few dozen rows each: the default there) or every row fits one tile (a dense
// call of up to 256 rows, on request), each B block is needed by one tile only, so this kernel decodes it straight into
// the shared-memory stage the tensor core reads, in the same 128-byte-swizzled K-major layout, with the same
// arithmetic (the bytes of a tile are those of the image path).  768 threads, warp-specialised:
//   warp 0       A producer: bulk copies of the A image blocks of each k-step (mbarrier tx count)
//   warp 1       MMA issuer: tcgen05.mma kind::f16, M = 128 per A block, N = BN, K = 16, f32 accumulators in TMEM
//   warp 2       allocates and frees the TMEM columns
//   warps 4..7   epilogue: per 128-column block, the 32-point Hadamards of four 32-column chunks in registers and back
//                into TMEM, then the two cross-chunk stages 8 columns of each chunk at a time (so the 128-point output
//                Hadamard needs 32 registers, not 128), * svh, 16-byte stores
//   warps 8..23  decoders: four per k-row, each streams NS x 2 consecutive tiles of every k-step through a cp.async ring
//                (about 48 KB in flight per SM), decodes them in registers (window extraction, IMAD hash, IMMA byte sums, the mul1
//                affine) and writes their A-fragment pairs as 8-byte stores into the stage's B block, then fences the
//                writes for the async proxy and arrives on the stage's full barrier (with the A producer's arrival and
//                its bytes, seventeen arrivals per phase)
// Every wait is bounded (role_wait: two seconds, then an abort flag every role polls and kErrWaitTimeout); each role
// drains what it issued before the CTA frees its TMEM.
#include <cuda_runtime.h>

#include "exl3_common.cuh"
#include "exl3_internal.h"
#include "exl3_tc.cuh"

namespace exl3 {

using namespace tc;

namespace {

constexpr int kDecodeWarps = 16;  // warps 8 .. 23
constexpr int kDecWarp0 = 8;
constexpr int kFusedThreads = (kDecWarp0 + kDecodeWarps) * 32;
constexpr int kDecPerRow = kDecodeWarps / 4;  // decode warps per k-row of a k-step

template <int N, int MS, int NS>
struct FusedShape {
  static constexpr int BN = 128 * NS;
  static constexpr int kTilesPerWarp = NS * 8 / kDecPerRow;              // one k-row's consecutive tiles per k-step
  static constexpr uint32_t kSlotBytes = kTilesPerWarp * 2u * N;         // their trellis bytes
  // trellis ring slots per decode warp: about 48 KB in flight per SM (the HBM latency times the decode's rate),
  // 4 to 16 slots
  static constexpr int kTrFit = static_cast<int>(49152u / (kDecodeWarps * kSlotBytes));
  static constexpr int kTrStages = kTrFit < 4 ? 4 : (kTrFit > 16 ? 16 : kTrFit);
  static constexpr uint32_t kRingBytes = kDecodeWarps * kTrStages * kSlotBytes;
  static constexpr uint32_t kStageBytes = (MS + NS) * kImgBytes;
  static constexpr int kFit = static_cast<int>((232448u - 2048u - kRingBytes) / kStageBytes);
  static constexpr int kStages = kFit < 4 ? kFit : 4;
  static constexpr int kAccCols = MS * BN;
  static constexpr int kAccBufs = kAccCols * 2 <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kAccCols * kAccBufs <= 256 ? 256 : 512;
  static constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kStageBytes + kRingBytes + 1024 + 256;
  static_assert(kStages >= 2, "two stages at least");
  static_assert(kSlotBytes % 16 == 0, "16-byte copies");
};

__device__ __forceinline__ void cp_async16_f(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_commit_f() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int K>
__device__ __forceinline__ void cp_wait_f() { asm volatile("cp.async.wait_group %0;" ::"n"(K) : "memory"); }

// In-register 32-point Hadamard (Sylvester order, unnormalised): the first five stages of the 128-point one.
__device__ __forceinline__ void fwht32_regs(float (&v)[32]) {
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if ((i & h) == 0) {
        const float a = v[i], b = v[i + h];
        v[i] = a + b;
        v[i + h] = a - b;
      }
    }
  }
}

// A lane-uniform bounded wait: lane 0 polls, the warp follows its answer.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag, uint32_t* err,
                                          uint32_t lane) {
  int ok = 0;
  if (lane == 0) ok = role_wait(bar, parity, abort_flag, err) ? 1 : 0;
  return __shfl_sync(0xFFFFFFFFu, ok, 0) != 0;
}

template <int N, int MS, int NS>
__global__ void __launch_bounds__(kFusedThreads, 1) gemm_fused_kernel(const GemmParams p) {
  using S = FusedShape<N, MS, NS>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* stages = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // the swizzle is anchored on 1024-byte rows
  uint8_t* rings = stages + S::kStages * S::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(rings + S::kRingBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* accf = empty + S::kStages;
  uint64_t* acce = accf + 2;
  uint64_t* fin = acce + 2;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(fin + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1 + kDecodeWarps);
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
  int mt0 = 0, tiles_m = p.tiles_m;  // grouped: this launch's M blocks come from the device (the routing wrote them)
  if (p.mt_range) {
    mt0 = p.mt_range[0];
    tiles_m = p.mt_range[1] - mt0;
  }
  const int tiles = tiles_m * p.tiles_n;
  // output tile t's M and N blocks.  Grouped launches walk an M block's N blocks together: the CTAs of one wave then
  // share its A rows through L2 (read from HBM once, not once per N block) and an expert's trellis columns are read
  // by its M blocks in the same wave.  Plain launches walk the M blocks first (A is small and stays in L2).
  const bool n_inner = p.m_group != nullptr;
  auto tile_mb = [&](int t) { return mt0 + (n_inner ? t / p.tiles_n : t % tiles_m); };
  auto tile_nb = [&](int t) { return n_inner ? t % p.tiles_n : t / tiles_m; };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- A producer
      const uint64_t pol_a = policy_evict_last();
      uint32_t stage = 0, phase = 0, fills = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int mb = tile_mb(t);
        for (int kb = 0; kb < p.kb; ++kb) {
          if (!role_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) {
            ok = false;
            break;
          }
          uint8_t* dst = stages + stage * S::kStageBytes;
          mbar_arrive_expect_tx(&full[stage], MS * kImgBytes);
#pragma unroll
          for (int s = 0; s < MS; ++s)
            bulk_g2s(dst + s * kImgBytes, p.a_img + (static_cast<size_t>(mb * MS + s) * p.kb + kb) * kImgBytes,
                     kImgBytes, &full[stage], pol_a);
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
  } else if (warp >= 4 && warp < 8) {
    // ---------------- epilogue: warp 4 + j reads TMEM lanes 32 j .. 32 j + 31
    const uint32_t wq = warp - 4;
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int ab = S::kAccBufs == 2 ? (local & 1) : 0;
      const uint32_t aph = S::kAccBufs == 2 ? ((local >> 1) & 1) : (local & 1);
      if (!role_wait(&accf[ab], aph, abort_flag, p.err)) break;
      tc_fence_after();
      const int mb = tile_mb(t), nb = tile_nb(t);
      const int64_t sv_e = p.m_group ? static_cast<int64_t>(p.m_group[mb]) * p.svh_group : 0;
#pragma unroll 1
      for (int s = 0; s < MS; ++s) {
        const int row = (mb * MS + s) * 128 + static_cast<int>(wq * 32 + lane);
#pragma unroll 1
        for (int c = 0; c < NS; ++c) {
          const int col0 = (nb * NS + c) * 128;
          if (col0 >= p.ncols) continue;  // warp-uniform: a ragged tile's padding columns are neither read nor stored
          const uint32_t tb =
              tmem + ((wq * 32u) << 16) + static_cast<uint32_t>(ab * S::kAccCols + s * S::BN + c * 128);
          if (!p.inner_only) {
            // the Hadamard's five low stages, per 32-column chunk, back into TMEM
#pragma unroll 1
            for (int j = 0; j < 4; ++j) {
              uint32_t r[32];
              tmem_ld32(tb + j * 32, r);
              tmem_wait_ld(r);
              float v[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
              fwht32_regs(v);
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
              tmem_st32(tb + j * 32, r);
            }
            tmem_wait_st();
          }
          const uint16_t* svc = p.svh2 && col0 >= p.svh_split ? p.svh2 + sv_e + (col0 - p.svh_split)
                                                              : p.svh + sv_e + col0;
          const size_t at = static_cast<size_t>(row) * p.y_row_stride + col0;
#pragma unroll 1
          for (int i0 = 0; i0 < 32; i0 += 8) {
            uint32_t r[4][8];
#pragma unroll
            for (int j = 0; j < 4; ++j) tmem_ld8(tb + j * 32 + i0, r[j]);
#pragma unroll
            for (int j = 0; j < 4; ++j) tmem_wait_ld8(r[j]);
            float o[4][8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float x0 = __uint_as_float(r[0][i]), x1 = __uint_as_float(r[1][i]);
              const float x2 = __uint_as_float(r[2][i]), x3 = __uint_as_float(r[3][i]);
              if (p.inner_only) {
                o[0][i] = x0, o[1][i] = x1, o[2][i] = x2, o[3][i] = x3;
              } else {
                // the two cross-chunk stages (h = 32, then 64), in the 128-point transform's order
                const float a0 = x0 + x1, a1 = x0 - x1, a2 = x2 + x3, a3 = x2 - x3;
                o[0][i] = a0 + a2, o[2][i] = a0 - a2, o[1][i] = a1 + a3, o[3][i] = a1 - a3;
              }
            }
            if (!p.inner_only) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(svc + j * 32 + i0));
                const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
                  o[j][2 * e] *= kHadScale * f.x;
                  o[j][2 * e + 1] *= kHadScale * f.y;
                }
              }
            }
            if (row < p.m) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const size_t aj = at + j * 32 + i0;
                if (p.vec_store && p.y_dtype != kF32) {
                  uint32_t pk[4];
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    if (p.y_dtype == kF16) {
                      const __half2 h2 = __floats2half2_rn(o[j][2 * e], o[j][2 * e + 1]);
                      pk[e] = *reinterpret_cast<const uint32_t*>(&h2);
                    } else {
                      const __nv_bfloat162 b2 = __floats2bfloat162_rn(o[j][2 * e], o[j][2 * e + 1]);
                      pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
                    }
                  }
                  *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.y) + aj) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                } else if (p.vec_store == 2) {
                  uint32_t pk[8];  // eight f32 columns: one 32-byte store, a whole L2 sector
#pragma unroll
                  for (int e = 0; e < 8; ++e) pk[e] = __float_as_uint(o[j][e]);
                  st_global_v8(static_cast<float*>(p.y) + aj, pk);
                } else if (p.vec_store) {
                  float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.y) + aj);
                  dst[0] = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
                  dst[1] = make_float4(o[j][4], o[j][5], o[j][6], o[j][7]);
                } else {
#pragma unroll
                  for (int i = 0; i < 8; ++i) store_act(p.y, aj + i, o[j][i], p.y_dtype);
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[ab]);
    }
  } else if (warp >= kDecWarp0) {
    // ---------------- decoders: warp dw takes k-row kk of every k-step, tile columns hf * kTilesPerWarp .. + that
    const uint32_t dw = warp - kDecWarp0, kk = dw / kDecPerRow, hf = dw % kDecPerRow;
    constexpr int kTrStages = S::kTrStages;
    uint8_t* ring = rings + dw * (kTrStages * S::kSlotBytes);
    LaneWin<N> lw;
    lw.init(lane);
    ImmaIndicator ind;
    ind.init(lane);
    const uint32_t g = lane >> 2, q = lane & 3u;
    const int kbn = p.kb;
    const int my_tiles = tiles > static_cast<int>(blockIdx.x)
                             ? (tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                                   static_cast<int>(gridDim.x)
                             : 0;
    const int items = my_tiles * kbn;  // this CTA's (tile, k-step) pairs, in the order every role walks them
    // the issue cursor: its tile, k-step, ring slot and the tile's first trellis tile of this warp (advanced per issue,
    // no division per k-step)
    int it_t = static_cast<int>(blockIdx.x), it_kb = 0, issued = 0;
    uint32_t it_slot = 0;
    const uint16_t* it_base = nullptr;
    auto tile_base = [&](int t) {
      const int mb = tile_mb(t), nb = tile_nb(t);
      const uint16_t* tr = p.trellis + (p.m_group ? static_cast<int64_t>(p.m_group[mb] - p.group0) * p.tr_group : 0);
      const int tn = p.tn0 + nb * NS * 8 + static_cast<int>(hf) * S::kTilesPerWarp;
      return tr + (static_cast<size_t>(kk) * p.out_tiles + tn) * N;  // k-step 0's tiles; + kb 4 out_tiles N per step
    };
    if (items > 0) it_base = tile_base(it_t);
    const size_t kstep_halfs = static_cast<size_t>(4) * p.out_tiles * N;
    auto issue = [&]() {
      if (issued < items) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(it_base + static_cast<size_t>(it_kb) * kstep_halfs);
        uint8_t* dst = ring + it_slot * S::kSlotBytes;
        for (uint32_t c = lane; c < S::kSlotBytes / 16u; c += 32u) cp_async16_f(dst + c * 16u, src + c * 16u);
        ++issued;
        if (++it_kb == kbn) {
          it_kb = 0;
          it_t += static_cast<int>(gridDim.x);
          if (issued < items) it_base = tile_base(it_t);
        }
        it_slot = it_slot + 1u == static_cast<uint32_t>(kTrStages) ? 0u : it_slot + 1u;
      }
    };
#pragma unroll 1
    for (int i = 0; i + 1 < kTrStages; ++i) {
      issue();
      cp_commit_f();
    }
    // this lane's image offset in the stage for its first tile.  A warp's tiles never straddle a 128-column block
    // (kTilesPerWarp divides 8) and every tile row of the lane has row & 7 == g, so tile t's two rows sit t * 2048
    // and t * 2048 + 1024 bytes further: the swizzle is computed once, not twice per tile.
    static_assert(8 % S::kTilesPerWarp == 0, "a warp's tiles stay inside one 128-column block");
    const uint32_t t0 = hf * S::kTilesPerWarp;
    const uint32_t lane_off = (t0 >> 3) * kImgBytes + (t0 & 7u) * 2048u + image_offset(g, kk * 16u + 4u * q);
    // Two k-steps per iteration where three stages or more let the MMA drain one while the decoders fill two: the
    // waits, fences, arrivals and ring cursors are paid once per eight tiles instead of four, and the two k-steps'
    // decodes interleave (measured on B200: the routed experts' prefill at config 4's banks 3.46 -> 3.19 ms a call).
    constexpr bool kPair = S::kStages >= 3;
    uint32_t stage = 0, phase = 0, slot_use = 0;
    auto decode_item = [&](const uint32_t* tw, uint32_t st) {
      uint8_t* bst = stages + st * S::kStageBytes + MS * kImgBytes + lane_off;
#pragma unroll
      for (int t = 0; t < S::kTilesPerWarp; ++t) {
        uint32_t w[8], a[4];
        tile_codewords<N>(tw + t * (N / 2), lw, w);
        // a[0], a[2]: column g at k 4q .. 4q + 3; a[1], a[3]: column g + 8.  The f16 pairs are packed on the FMA
        // pipe: the window extraction loads the ALU pipe (measured on B200: 2 % on the routed experts' prefill).
        decode_afrag_imma<true>(w, ind, a);
        *reinterpret_cast<uint2*>(bst + t * 2048u) = make_uint2(a[0], a[2]);
        *reinterpret_cast<uint2*>(bst + t * 2048u + 1024u) = make_uint2(a[1], a[3]);
      }
    };
    auto next_stage = [](uint32_t& st, uint32_t& ph) {
      if (++st == static_cast<uint32_t>(S::kStages)) {
        st = 0;
        ph ^= 1u;
      }
    };
    auto next_slot = [](uint32_t sl) { return sl + 1u == static_cast<uint32_t>(kTrStages) ? 0u : sl + 1u; };
#pragma unroll 1
    for (int i = 0; i < items; i += kPair ? 2 : 1) {
      const bool two = kPair && i + 1 < items;  // (warp-uniform)
      // item i's trellis words (and item i + 1's) have landed: one commit group per item, kTrStages - 1 ahead
      cp_wait_f<kPair ? kTrStages - 3 : kTrStages - 2>();
      __syncwarp();
      uint32_t stage2 = stage, phase2 = phase;
      next_stage(stage2, phase2);
      if (!warp_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, lane)) break;
      if (two && !warp_wait(&empty[stage2], phase2 ^ 1u, abort_flag, p.err, lane)) break;
      const uint32_t slot2 = next_slot(slot_use);
      decode_item(reinterpret_cast<const uint32_t*>(ring + slot_use * S::kSlotBytes), stage);
      if (two) decode_item(reinterpret_cast<const uint32_t*>(ring + slot2 * S::kSlotBytes), stage2);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full[stage]);
        if (two) mbar_arrive(&full[stage2]);
      }
      issue();
      cp_commit_f();
      if (kPair) {
        issue();
        cp_commit_f();
        slot_use = next_slot(slot2);
        stage = stage2;
        phase = phase2;
      } else {
        slot_use = slot2;
      }
      next_stage(stage, phase);
    }
    cp_wait_f<0>();  // no copy outlives the CTA
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

template <int N, int MS, int NS>
cudaError_t launch_fused_t(const GemmParams& p, int sms, cudaStream_t st) {
  using S = FusedShape<N, MS, NS>;
  if (!p.trellis || p.n != N || p.tiles_m * 128 * MS < p.m) return cudaErrorInvalidValue;
  if ((p.mt_range || p.m_group) && MS != 1) return cudaErrorInvalidValue;
  static KernelSetup setup;
  if (cudaError_t e = kernel_setup(setup, gemm_fused_kernel<N, MS, NS>, kFusedThreads, S::kSmemBytes); e != cudaSuccess)
    return e;
  const int tiles = p.tiles_m * p.tiles_n;  // (grouped: an upper bound; the kernel reads the launch's blocks)
  const int grid = tiles < sms ? tiles : sms;
  gemm_fused_kernel<N, MS, NS><<<grid, kFusedThreads, S::kSmemBytes, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_fused(const GemmParams& p, int shape, int sms, cudaStream_t st) {
  cudaError_t e = cudaErrorInvalidValue;
  with_rate(p.n, [&](auto N) {
    constexpr int n = decltype(N)::value;
    switch (shape) {
      case 0: e = launch_fused_t<n, 1, 1>(p, sms, st); break;
      case 1: e = launch_fused_t<n, 1, 2>(p, sms, st); break;
      case 2: e = launch_fused_t<n, 2, 1>(p, sms, st); break;
      case 3: e = launch_fused_t<n, 2, 2>(p, sms, st); break;
      default: break;
    }
  });
  return e;
}

}  // namespace exl3
