// exl3_windows.h -- a lane's eight trellis windows of a tile, for any rate of n halfwords per tile (n even, 16..96).
//
// The bitstream rule (SX/expert_exl3.zig:180-245 bitEnd, :317-336 unpackTile): stream position p of a tile reads the
// 16-bit window ending at bit floor((p + 1) n / 16), tail-biting over the tile's 16 n bits, MSB-first in
// little-endian u32 words.  Lane t of a warp decodes positions 8t .. 8t + 7 (the m16n8k16 A fragment of W^T).  With n
// even, 8t n / 16 = t n / 2 is whole, so lane t's windows end at t n / 2 + floor((j + 1) n / 16): the lane's last
// window ends at E = (t + 1) n / 2, and window j sits s_j = n / 2 - floor((j + 1) n / 16) bits below it -- the same
// shifts for every lane.  The 64 bits below E hold all eight windows while s_0 + 16 <= 64, i.e. n <= 96.
// For n = 16 K this is the integer-rate rule (s_j = (7 - j) K).
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define EXL3_HD __host__ __device__ __forceinline__
#else
#define EXL3_HD inline
#endif

namespace exl3 {

template <int N>
struct LaneWin {
  static_assert(N % 2 == 0 && N >= 16 && N <= 96, "n even, 16..96");
  uint32_t o0, o1, o2;  // word offsets (c - 2, c - 1, c) mod n/2 of the u32 words around E
  uint32_t sh;          // right funnel shift that brings E to a word boundary (0 when E is word-aligned)
  uint32_t mask = 0xFFFFu;  // the codeword: the low w bits of the 16-bit window (w = 8..16, a narrowed window)
  EXL3_HD void init(uint32_t lane) {
    constexpr uint32_t nw = N / 2;  // u32 words per tile
    const uint32_t e = (lane + 1u) * (N / 2);
    const uint32_t c = (e - 1u) >> 5;
    o2 = c % nw;
    o1 = (c + nw - 1u) % nw;
    o0 = (c + nw - 2u) % nw;
    sh = (0u - e) & 31u;
  }
};

EXL3_HD uint32_t funnel_r(uint32_t lo, uint32_t hi, uint32_t s) {  // (hi:lo) >> s, s < 32
#if defined(__CUDA_ARCH__)
  return __funnelshift_r(lo, hi, s);
#else
  return s == 0 ? lo : (lo >> s) | (hi << (32u - s));
#endif
}

// Lane t's eight codewords (low 16 bits of each; with MASKED, the low w bits: lw.mask) from the tile's u32 words.
template <int N, bool MASKED = false>
EXL3_HD void lane_windows(const uint32_t* tile_words, const LaneWin<N>& lw, uint32_t (&w)[8]) {
  const uint32_t a = tile_words[lw.o0], b = tile_words[lw.o1], c = tile_words[lw.o2];
  const uint32_t vlo = funnel_r(c, b, lw.sh), vhi = funnel_r(b, a, lw.sh);  // the 64 bits below E
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int j = 0; j < 8; ++j) {
    const int s = N / 2 - ((j + 1) * N) / 16;  // compile-time per j
    uint32_t v;
    if (s >= 32) v = vhi >> (s - 32);
    else if (s + 16 <= 32) v = vlo >> s;
    else v = funnel_r(vlo, vhi, static_cast<uint32_t>(s));
    w[j] = v & (MASKED ? lw.mask : 0xFFFFu);
  }
}

// The codewords a lane needs when its MMA operand is in the tensor-pipe byte-sum order (lane (g, q) holding column g's
// and g + 8's weights at k = 4q .. 4q + 3) and the codebook decodes per codeword (no byte sums to carry them across
// lanes): the windows of lanes (g, 2q mod 4) and (g, 2q + 1 mod 4) at positions jb, jb + 1, jb + 4, jb + 5 (jb = 0 for
// q < 2, else 2) -- the natural fragment's (k 2q', 2q' + 1) and (k 2q' + 8, 2q' + 9) pairs that cover k = 4q .. 4q + 3.
template <int N>
struct ImmaWin {
  LaneWin<N> src[2];
  uint32_t sh[2][4];  // per source lane, per window: its shift below that lane's window end E (in the 64 bits below E)
  EXL3_HD void init(uint32_t lane, uint32_t mask) {
    const uint32_t g = lane >> 2, q = lane & 3u, jb = q < 2u ? 0u : 2u;
    const uint32_t js[4] = {jb, jb + 1u, jb + 4u, jb + 5u};
    for (int i = 0; i < 2; ++i) {
      src[i].init(4u * g + ((2u * q + static_cast<uint32_t>(i)) & 3u));
      src[i].mask = mask;
      for (int k = 0; k < 4; ++k) sh[i][k] = N / 2 - ((js[k] + 1u) * N) / 16;
    }
  }
};

// w[0..3]: the first source lane's windows jb, jb + 1, jb + 4, jb + 5; w[4..7] the second's; each masked (src mask).
template <int N>
EXL3_HD void imma_windows(const uint32_t* tile_words, const ImmaWin<N>& iw, uint32_t (&w)[8]) {
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int i = 0; i < 2; ++i) {
    const LaneWin<N>& lw = iw.src[i];
    const uint32_t a = tile_words[lw.o0], b = tile_words[lw.o1], c = tile_words[lw.o2];
    const uint64_t v = (static_cast<uint64_t>(funnel_r(b, a, lw.sh)) << 32) | funnel_r(c, b, lw.sh);
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
    for (int k = 0; k < 4; ++k) w[4 * i + k] = static_cast<uint32_t>(v >> iw.sh[i][k]) & lw.mask;
  }
}

}  // namespace exl3
