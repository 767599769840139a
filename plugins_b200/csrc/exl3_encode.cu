// exl3_encode.cu -- trellis encoder: target tiles (already Hadamard-rotated and scaled to the codebook's unit
// variance) -> EXL3 mul1 bitstreams in the pack layout [in/16][out/16][n].
//
// The reference has no encoder (plugins/turboexl3_ds41/NOTICE:30-32: no exllamav3 code is shipped), so this is the
// build's own: a tail-biting greedy search, one thread per tile.  Pass 1 walks the 256 stream positions choosing each
// weight's K fresh bits to minimise the squared error of its mul1 value, starting from an all-zero wrap; pass 2 starts
// from the wrap bits pass 1 ended with and forces the last weights' fresh bits to equal them, so the stream is
// consistent around the tail.  Decoding is defined for any bitstream, so the encoder's quality does not enter the
// parity checks; it only has to be deterministic and reasonable.
#include <cuda_runtime.h>

#include "exl3_common.cuh"

namespace exl3 {

__device__ __forceinline__ float mul1_value(uint32_t state) {
  const uint32_t x = state * kMul1Mult;
  const uint32_t s = __dp4a(x, 0x01010101u, 0x6400u);  // unsigned byte sum
  const __half h = __ushort_as_half(static_cast<uint16_t>(s));
  const __half r = __hfma(h, __ushort_as_half(static_cast<uint16_t>(kHalfInv)), __ushort_as_half(static_cast<uint16_t>(kHalfBias)));
  return __half2float(r);
}

__device__ __forceinline__ uint32_t tc_perm(uint32_t p) {
  const uint32_t t = p >> 3, j = p & 7u;
  const uint32_t r0 = (t & 3u) * 2u;
  const uint32_t rows[4] = {r0, r0 + 1u, r0 + 8u, r0 + 9u};
  return rows[j & 3u] * 16u + (t >> 2) + (j < 4u ? 0u : 8u);
}

template <int K>
__device__ uint32_t greedy_pass(const float (&tgt)[256], uint32_t prefix, bool force, uint32_t* bits /* [8K] words */) {
  constexpr uint32_t total = 256u * K, wrap = 16u - K;
  for (uint32_t i = 0; i < 8u * K; ++i) bits[i] = 0u;
  uint32_t win = prefix;  // low (16 - K) bits: the stream bits before weight 0's fresh bits
  for (uint32_t p = 0; p < 256u; ++p) {
    const uint32_t base = (win << K) & 0xFFFFu;
    float best = 3.4e38f;
    uint32_t bestv = 0u;
    for (uint32_t v = 0; v < (1u << K); ++v) {
      if (force && (p + 1u) * K > total - wrap) {
        bool agree = true;
        for (uint32_t i = 0; i < K; ++i) {
          const uint32_t b = p * K + i;  // stream bit of v's bit (K-1-i)
          if (b >= total - wrap) {
            const uint32_t want = (prefix >> (total - 1u - b)) & 1u;
            if (((v >> (K - 1u - i)) & 1u) != want) agree = false;
          }
        }
        if (!agree) continue;
      }
      const float d = mul1_value(base | v) - tgt[p];
      const float e = d * d;
      if (e < best) {
        best = e;
        bestv = v;
      }
    }
    win = base | bestv;
    for (uint32_t i = 0; i < K; ++i) {
      const uint32_t b = p * K + i;
      const uint32_t bit = (bestv >> (K - 1u - i)) & 1u;
      bits[b >> 5] |= bit << (31u - (b & 31u));
    }
  }
  return win & ((1u << wrap) - 1u);  // the last (16 - K) stream bits
}

template <int K>
__global__ void __launch_bounds__(64) encode_kernel(const float* __restrict__ target, int in_features, int out_features,
                                                    uint16_t* __restrict__ trellis) {
  const int ot = out_features / 16;
  const size_t tiles = static_cast<size_t>(in_features / 16) * ot;
  const size_t tile = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (tile >= tiles) return;
  const int tk = static_cast<int>(tile / ot), tn = static_cast<int>(tile % ot);
  float tgt[256];
  for (uint32_t p = 0; p < 256u; ++p) {
    const uint32_t slot = tc_perm(p);
    tgt[p] = target[static_cast<size_t>(tk * 16 + slot / 16) * out_features + tn * 16 + slot % 16];
  }
  uint32_t bits[8 * K];
  const uint32_t prefix = greedy_pass<K>(tgt, 0u, false, bits);
  greedy_pass<K>(tgt, prefix, true, bits);
  uint16_t* out = trellis + tile * (16 * K);
  for (uint32_t m = 0; m < 8u * K; ++m) {
    out[2 * m] = static_cast<uint16_t>(bits[m] & 0xFFFFu);
    out[2 * m + 1] = static_cast<uint16_t>(bits[m] >> 16);
  }
}

cudaError_t launch_encode(const float* target, int in_features, int out_features, int n, uint16_t* trellis,
                          cudaStream_t st) {
  const size_t tiles = static_cast<size_t>(in_features / 16) * (out_features / 16);
  const dim3 grid(static_cast<unsigned>((tiles + 63) / 64)), block(64);
  if (n % 16 != 0) return cudaErrorInvalidValue;  // the encoder searches whole-bit trellises only
  switch (n / 16) {
    case 1: encode_kernel<1><<<grid, block, 0, st>>>(target, in_features, out_features, trellis); break;
    case 2: encode_kernel<2><<<grid, block, 0, st>>>(target, in_features, out_features, trellis); break;
    case 3: encode_kernel<3><<<grid, block, 0, st>>>(target, in_features, out_features, trellis); break;
    case 4: encode_kernel<4><<<grid, block, 0, st>>>(target, in_features, out_features, trellis); break;
    case 5: encode_kernel<5><<<grid, block, 0, st>>>(target, in_features, out_features, trellis); break;
    case 6: encode_kernel<6><<<grid, block, 0, st>>>(target, in_features, out_features, trellis); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace exl3
