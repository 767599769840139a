/*
 * exl3_oracle.c -- CPU restatement of the reference's EXL3 (mul1 codebook) trellis decode + matmul.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, `__graft_entry__.smoke()` and the
 * `cpu_baseline` / `--impl reference` legs of bench.py compare against.  Nothing in the product path
 * (plugins_b200/, include/) links, loads or calls it.
 *
 * Every function follows a reference function; paths are relative to the reference project root:
 *   SX = plugins/sushi_ds41/src/sushi/exl3/   (the in-tree EXL3 module, API-compatible with turboexl3)
 *   TX = plugins/turboexl3_ds41/src/exl3/      (the ds41 lane's host decoder and golden-plane generator)
 *
 * Floating point follows the reference's order of operations: f32 accumulation in the reference's loop
 * order, f16 rounding (round-to-nearest-even) exactly where the reference rounds, and a fused multiply-add
 * only where the reference writes @mulAdd.  Build with -ffp-contract=off so the compiler adds no other
 * contraction.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

#define TILE 16
#define TILE_VALUES 256
#define HAD_DIM 128
/* SX/expert_exl3.zig:7 HAD_SCALE (1/sqrt(128) as an f32 literal). */
static const float HAD_SCALE = 0.08838834764831845f;
/* SX/expert_exl3.zig:11 MUL1_MULT. */
#define MUL1_MULT 0x83DCD12Du

/* ---------------------------------------------------------------- f16 <-> f32 / f64 (IEEE binary16, RNE) */

float exl3o_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int shift = 0;
            while ((m & 0x400u) == 0) { m <<= 1; shift++; }
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 + 1 - shift) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t exl3o_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t a = x & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (a > 0x7F800000u ? (0x200u | ((a >> 13) & 0x3FFu)) : 0u));
    if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 rounds to inf */
    if (a < 0x38800000u) {                                   /* below 2^-14: f16 subnormal or zero */
        if (a < 0x33000000u) return (uint16_t)sign;          /* below 2^-25 */
        uint32_t e = a >> 23;
        uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e; /* value * 2^24 = m * 2^(e-126) */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t r = a - 0x38000000u;
    r = (r + 0x0FFFu + ((r >> 13) & 1u)) >> 13;
    return (uint16_t)(sign | r);
}

/* Correctly rounded f64 -> f16 (used where the reference rounds an exact f64 once, TX/kernels.zig:967-975). */
uint16_t exl3o_f64_to_f16(double d) {
    uint64_t x;
    memcpy(&x, &d, 8);
    uint16_t sign = (uint16_t)((x >> 48) & 0x8000u);
    uint64_t a = x & 0x7FFFFFFFFFFFFFFFull;
    if (a >= 0x7FF0000000000000ull) return (uint16_t)(sign | 0x7C00u | (a > 0x7FF0000000000000ull ? 0x200u : 0u));
    double ad;
    memcpy(&ad, &a, 8);
    if (ad >= 65520.0) return (uint16_t)(sign | 0x7C00u);
    /* scale so the f16 ulp becomes 1: ulp = 2^(e-10) for normals, 2^-24 for subnormals */
    int e2;
    frexp(ad, &e2); /* ad = f * 2^e2, f in [0.5, 1) -> exponent e = e2 - 1 */
    int e = e2 - 1;
    if (ad == 0.0) return sign;
    if (e < -14) e = -14;
    double scaled = ldexp(ad, 10 - e); /* exact */
    double q = nearbyint(scaled);      /* default rounding mode: ties to even */
    double v = ldexp(q, e - 10);
    float vf = (float)v; /* exact: an f16 value */
    return (uint16_t)(sign | exl3o_f32_to_f16(vf));
}

/* ---------------------------------------------------------------- rate (SX/expert_exl3.zig:180-245) */

/* One past the last bit of weight t's codeword window: floor((t+1) * n / 16). SX/expert_exl3.zig:207-209 */
uint32_t exl3o_bit_end(uint32_t n, uint32_t t) { return ((t + 1u) * n) >> 4; }

/* Admitted packed dims: even, 16..128. SX/expert_exl3.zig:240-245 kFromPackedDim */
int exl3o_rate_admitted(uint32_t n) { return (n % 2u == 0u) && n >= 16u && n <= 128u; }

/* ---------------------------------------------------------------- codebook (SX/expert_exl3.zig:275-284) */

/* decodeMul1: f16 = RN_f16(fma_f32((1024 + bytesum(cw * MUL1_MULT)), f16(0x1EEE), f16(0xC931))) */
uint16_t exl3o_decode_mul1(uint16_t cw) {
    uint32_t mixed = (uint32_t)cw * MUL1_MULT;
    uint32_t s = (mixed & 0xFFu) + ((mixed >> 8) & 0xFFu) + ((mixed >> 16) & 0xFFu) + (mixed >> 24);
    float h = exl3o_f16_to_f32((uint16_t)(0x6400u + s));
    float inv = exl3o_f16_to_f32(0x1EEE);
    float bias = exl3o_f16_to_f32(0xC931);
    return exl3o_f32_to_f16(fmaf(h, inv, bias));
}

/* mul1Decode (TX/kernels.zig:967-975): the same value through an exact f64 product, rounded once. */
uint16_t exl3o_decode_mul1_f64(uint16_t state) {
    uint32_t x = (uint32_t)state * MUL1_MULT;
    uint32_t s = (x & 0xFFu) + ((x >> 8) & 0xFFu) + ((x >> 16) & 0xFFu) + (x >> 24);
    double k_inv = (double)exl3o_f16_to_f32(0x1EEE);
    double k_bias = (double)exl3o_f16_to_f32(0xC931);
    return exl3o_f64_to_f16((double)(1024u + s) * k_inv + k_bias);
}

void exl3o_mul1_table(uint16_t *out /* [65536] */) {
    for (uint32_t s = 0; s < 65536u; s++) out[s] = exl3o_decode_mul1((uint16_t)s);
}

/* MCG codebook (SX/expert_exl3.zig:267-273); kept for the KAT that pins the window masking. */
uint16_t exl3o_decode_mcg(uint16_t cw) {
    uint32_t mixed = (uint32_t)cw * 0xCBAC1FEDu;
    uint32_t pair = 0x3B603B60u ^ (mixed & 0x8FFF8FFFu);
    float lo = exl3o_f16_to_f32((uint16_t)pair);
    float hi = exl3o_f16_to_f32((uint16_t)(pair >> 16));
    return exl3o_f32_to_f16(lo + hi);
}

/* ---------------------------------------------------------------- unpack (SX/expert_exl3.zig:313-336) */

static inline uint32_t word_u32(const uint16_t *words, uint32_t index) {
    return (uint32_t)words[index * 2u] | ((uint32_t)words[index * 2u + 1u] << 16);
}

/* unpackTile: 256 16-bit codewords; tail-biting windows, MSB-first over little-endian u32 words. */
void exl3o_unpack_tile(const uint16_t *words, uint32_t n, uint16_t *out /* [256] */) {
    uint32_t word_count = n / 2u;
    uint32_t total = TILE * n;
    for (uint32_t thread = 0; thread < 128u; thread++) {
        uint32_t e0 = exl3o_bit_end(n, thread * 2u);
        uint32_t e1 = exl3o_bit_end(n, thread * 2u + 1u);
        uint32_t bit0 = e0 + total - 16u;
        uint32_t bit2 = e1 + total;
        uint32_t index0 = bit0 / 32u;
        uint32_t index1 = (bit2 - 1u) / 32u;
        uint32_t shift = (index1 + 1u) * 32u - bit2;
        uint64_t merged = ((uint64_t)word_u32(words, index0 % word_count) << 32) | (uint64_t)word_u32(words, index1 % word_count);
        uint32_t funnel = (uint32_t)(merged >> shift);
        uint32_t fresh = e1 - e0;
        out[thread * 2u] = (uint16_t)((funnel >> fresh) & 0xFFFFu);
        out[thread * 2u + 1u] = (uint16_t)(funnel & 0xFFFFu);
    }
}

/* The bit-by-bit definition the reference's own test checks unpackTile against (SX/expert_exl3.zig:1051-1066). */
uint16_t exl3o_codeword_by_definition(const uint16_t *words, uint32_t n, uint32_t slot) {
    uint32_t cw = 0;
    for (uint32_t bit = 0; bit < 16u; bit++) {
        uint32_t at = ((slot + 1u) * n / 16u + 16u * n - 16u + bit) % (16u * n);
        uint32_t v = (words[2u * (at / 32u) + (1u - (at % 32u) / 16u)] >> (15u - at % 16u)) & 1u;
        cw = (cw << 1) | v;
    }
    return (uint16_t)cw;
}

/* ---------------------------------------------------------------- permutation (SX/expert_exl3.zig:379-398) */

void exl3o_tensor_core_perm(uint32_t *out /* [256] */) {
    for (uint32_t thread = 0; thread < 32u; thread++) {
        uint32_t row0 = (thread % 4u) * 2u, row1 = row0 + 1u, row2 = row0 + 8u, row3 = row0 + 9u;
        uint32_t col0 = thread / 4u, col1 = col0 + 8u;
        uint32_t base = thread * 8u;
        out[base + 0] = row0 * 16u + col0;
        out[base + 1] = row1 * 16u + col0;
        out[base + 2] = row2 * 16u + col0;
        out[base + 3] = row3 * 16u + col0;
        out[base + 4] = row0 * 16u + col1;
        out[base + 5] = row1 * 16u + col1;
        out[base + 6] = row2 * 16u + col1;
        out[base + 7] = row3 * 16u + col1;
    }
}

static uint32_t g_perm[256];
static int g_perm_ready = 0;
static uint16_t g_mul1[65536];
static int g_mul1_ready = 0;

static void ensure_tables(void) {
    if (!g_perm_ready) {
        exl3o_tensor_core_perm(g_perm);
        g_perm_ready = 1;
    }
    if (!g_mul1_ready) {
        exl3o_mul1_table(g_mul1);
        g_mul1_ready = 1;
    }
}

/* Call once before threads use the decoders (builds the perm and the mul1 table). */
void exl3o_init(void) { ensure_tables(); }

/* decodeTile, mul1, window w (8..16): W_hat tile, f16 bits, row-major [16][16] (SX/expert_exl3.zig:338-357). */
void exl3o_decode_tile(const uint16_t *words, uint32_t n, uint32_t window_bits, uint16_t *out /* [256] */) {
    ensure_tables();
    uint16_t cw[TILE_VALUES];
    exl3o_unpack_tile(words, n, cw);
    uint16_t mask = (uint16_t)((1u << window_bits) - 1u);
    for (uint32_t i = 0; i < TILE_VALUES; i++) out[g_perm[i]] = g_mul1[cw[i] & mask];
}

/* The same with the MCG codebook (only for the window-masking KAT). */
void exl3o_decode_tile_mcg(const uint16_t *words, uint32_t n, uint32_t window_bits, uint16_t *out) {
    ensure_tables();
    uint16_t cw[TILE_VALUES];
    exl3o_unpack_tile(words, n, cw);
    uint16_t mask = (uint16_t)((1u << window_bits) - 1u);
    for (uint32_t i = 0; i < TILE_VALUES; i++) out[g_perm[i]] = exl3o_decode_mcg((uint16_t)(cw[i] & mask));
}

/* One tile at codebook `cb` (0 mul1, 1 mcg) and window `window_bits` (SX/expert_exl3.zig decodeTile with a Decode). */
static void decode_tile_cb(const uint16_t *words, uint32_t n, uint32_t window_bits, int cb, uint16_t *out) {
    if (cb == 1) exl3o_decode_tile_mcg(words, n, window_bits, out);
    else exl3o_decode_tile(words, n, window_bits, out);
}

/* ---------------------------------------------------------------- Hadamard (SX/expert_exl3.zig:400-414) */

void exl3o_hadamard128(float *values /* [128] */) {
    float tmp[HAD_DIM];
    for (uint32_t r = 0; r < HAD_DIM; r++) {
        float acc = 0.0f;
        for (uint32_t k = 0; k < HAD_DIM; k++) {
            float e = (__builtin_popcount(r & k) % 2 == 0) ? HAD_SCALE : -HAD_SCALE;
            acc += e * values[k];
        }
        tmp[r] = acc;
    }
    memcpy(values, tmp, sizeof tmp);
}

/* ---------------------------------------------------------------- reconstruct (SX/expert_exl3.zig:416-488) */

/* reconstructInner: W_hat f16 bits [in][out] row-major, codeword window `window_bits` (8..16). */
void exl3o_reconstruct_inner_w(const uint16_t *trellis, uint32_t in_features, uint32_t out_features, uint32_t n,
                               uint32_t window_bits, int codebook, uint16_t *out);
void exl3o_reconstruct_inner(const uint16_t *trellis, uint32_t in_features, uint32_t out_features, uint32_t n,
                             uint16_t *out) {
    exl3o_reconstruct_inner_w(trellis, in_features, out_features, n, 16, 0, out);
}
/* codebook 0 mul1, 1 mcg; window_bits 8..16 */
void exl3o_reconstruct_inner_w(const uint16_t *trellis, uint32_t in_features, uint32_t out_features, uint32_t n,
                               uint32_t window_bits, int codebook, uint16_t *out) {
    uint32_t in_tiles = in_features / TILE, out_tiles = out_features / TILE;
    uint16_t tile[TILE_VALUES];
    for (uint32_t tk = 0; tk < in_tiles; tk++) {
        for (uint32_t tn = 0; tn < out_tiles; tn++) {
            size_t off = ((size_t)tk * out_tiles + tn) * n;
            decode_tile_cb(trellis + off, n, window_bits, codebook, tile);
            for (uint32_t r = 0; r < TILE; r++)
                memcpy(out + (size_t)(tk * TILE + r) * out_features + tn * TILE, tile + r * TILE, TILE * 2);
        }
    }
}

/* reconstruct (TX/kernels.zig:1009-1024) also returns each weight's trellis state. */
void exl3o_reconstruct_states(const uint16_t *trellis, uint32_t in_features, uint32_t out_features, uint32_t n,
                              uint16_t *w, uint16_t *states) {
    ensure_tables();
    uint32_t n_i = in_features / TILE, n_j = out_features / TILE;
    uint16_t st[TILE_VALUES];
    for (uint32_t ti = 0; ti < n_i; ti++) {
        for (uint32_t tj = 0; tj < n_j; tj++) {
            exl3o_unpack_tile(trellis + ((size_t)ti * n_j + tj) * n, n, st);
            for (uint32_t p = 0; p < TILE_VALUES; p++) {
                uint32_t pos = g_perm[p];
                size_t at = (size_t)(ti * 16u + pos / 16u) * out_features + tj * 16u + pos % 16u;
                w[at] = g_mul1[st[p]];
                if (states) states[at] = st[p];
            }
        }
    }
}

/* reconstructPublic: the dense effective W (f16 bits) [in][out]. */
int exl3o_reconstruct_public(const uint16_t *trellis, const uint16_t *suh, const uint16_t *svh, uint32_t in_features,
                             uint32_t out_features, uint32_t n, uint16_t *out) {
    size_t count = (size_t)in_features * out_features;
    uint16_t *inner = (uint16_t *)malloc(count * 2);
    float *w = (float *)malloc(count * 4);
    if (!inner || !w) {
        free(inner);
        free(w);
        return -1;
    }
    exl3o_reconstruct_inner(trellis, in_features, out_features, n, inner);
    for (size_t i = 0; i < count; i++) w[i] = exl3o_f16_to_f32(inner[i]);
    float vec[HAD_DIM];
    for (uint32_t rb = 0; rb < in_features; rb += HAD_DIM) {
        for (uint32_t col = 0; col < out_features; col++) {
            for (uint32_t r = 0; r < HAD_DIM; r++) vec[r] = w[(size_t)(rb + r) * out_features + col];
            exl3o_hadamard128(vec);
            for (uint32_t r = 0; r < HAD_DIM; r++) w[(size_t)(rb + r) * out_features + col] = vec[r];
        }
    }
    for (uint32_t r = 0; r < in_features; r++) {
        float s = exl3o_f16_to_f32(suh[r]);
        for (uint32_t c = 0; c < out_features; c++) w[(size_t)r * out_features + c] *= s;
    }
    for (uint32_t cb = 0; cb < out_features; cb += HAD_DIM) {
        for (uint32_t r = 0; r < in_features; r++) {
            float *row = w + (size_t)r * out_features + cb;
            exl3o_hadamard128(row);
        }
    }
    for (uint32_t c = 0; c < out_features; c++) {
        float s = exl3o_f16_to_f32(svh[c]);
        for (uint32_t r = 0; r < in_features; r++) w[(size_t)r * out_features + c] *= s;
    }
    for (size_t i = 0; i < count; i++) out[i] = exl3o_f32_to_f16(w[i]);
    free(inner);
    free(w);
    return 0;
}

/* ---------------------------------------------------------------- the scalar linear (SX/expert_exl3.zig:490-566) */

/* prepareInput: xp = f16(H128(f16(x) * suh)) per 128-block. */
void exl3o_prepare_input(const float *x, const uint16_t *suh, uint32_t in_features, float *out) {
    for (uint32_t i = 0; i < in_features; i++)
        out[i] = exl3o_f16_to_f32(exl3o_f32_to_f16(x[i])) * exl3o_f16_to_f32(suh[i]);
    for (uint32_t b = 0; b < in_features; b += HAD_DIM) {
        exl3o_hadamard128(out + b);
        for (uint32_t i = 0; i < HAD_DIM; i++) out[b + i] = exl3o_f16_to_f32(exl3o_f32_to_f16(out[b + i]));
    }
}

/* innerGemv over the output tiles [tn0, tn1): tk outer, tn inner, f32 sums, then one f16 rounding. */
static void inner_gemv_range(const uint16_t *trellis, const float *xp, uint32_t in_features, uint32_t out_features,
                             uint32_t n, uint32_t tn0, uint32_t tn1, float *out) {
    uint32_t in_tiles = in_features / TILE, out_tiles = out_features / TILE;
    uint16_t tile[TILE_VALUES];
    for (uint32_t c = tn0 * TILE; c < tn1 * TILE; c++) out[c] = 0.0f;
    for (uint32_t tk = 0; tk < in_tiles; tk++) {
        for (uint32_t tn = tn0; tn < tn1; tn++) {
            exl3o_decode_tile(trellis + ((size_t)tk * out_tiles + tn) * n, n, 16, tile);
            uint32_t xb = tk * TILE, yb = tn * TILE;
            for (uint32_t r = 0; r < TILE; r++) {
                float xv = xp[xb + r];
                for (uint32_t c = 0; c < TILE; c++) out[yb + c] += xv * exl3o_f16_to_f32(tile[r * TILE + c]);
            }
        }
    }
    for (uint32_t c = tn0 * TILE; c < tn1 * TILE; c++) out[c] = exl3o_f16_to_f32(exl3o_f32_to_f16(out[c]));
}

void exl3o_inner_gemv(const uint16_t *trellis, const float *xp, uint32_t in_features, uint32_t out_features,
                      uint32_t n, float *out) {
    inner_gemv_range(trellis, xp, in_features, out_features, n, 0, out_features / TILE, out);
}

/* finishOutput: y = f16(H128(inner) * svh) per 128-block. */
void exl3o_finish_output(const float *inner, const uint16_t *svh, uint32_t out_features, float *out) {
    memcpy(out, inner, (size_t)out_features * 4);
    for (uint32_t b = 0; b < out_features; b += HAD_DIM) exl3o_hadamard128(out + b);
    for (uint32_t c = 0; c < out_features; c++)
        out[c] = exl3o_f16_to_f32(exl3o_f32_to_f16(out[c] * exl3o_f16_to_f32(svh[c])));
}

/* project: the whole linear, scalar.  `threads` > 1 splits innerGemv's output tiles over OpenMP threads;
 * every output keeps the single-thread sum order, so the result is the same bits at any thread count. */
int exl3o_project(const float *x, const uint16_t *trellis, const uint16_t *suh, const uint16_t *svh,
                  uint32_t in_features, uint32_t out_features, uint32_t n, int threads, float *out) {
    ensure_tables();
    float *xp = (float *)malloc((size_t)in_features * 4);
    float *inner = (float *)malloc((size_t)out_features * 4);
    if (!xp || !inner) {
        free(xp);
        free(inner);
        return -1;
    }
    exl3o_prepare_input(x, suh, in_features, xp);
    uint32_t out_tiles = out_features / TILE;
    if (threads <= 1) {
        inner_gemv_range(trellis, xp, in_features, out_features, n, 0, out_tiles, inner);
    } else {
#pragma omp parallel for num_threads(threads) schedule(static)
        for (int t = 0; t < threads; t++) {
            uint32_t a = (uint32_t)((uint64_t)out_tiles * t / threads);
            uint32_t b = (uint32_t)((uint64_t)out_tiles * (t + 1) / threads);
            if (b > a) inner_gemv_range(trellis, xp, in_features, out_features, n, a, b, inner);
        }
    }
    exl3o_finish_output(inner, svh, out_features, out);
    free(xp);
    free(inner);
    return 0;
}

/* ---------------------------------------------------------------- f32 truth (SX/linear.zig:121-197) */

/* Host.project (SX/linear.zig:178-197): no intermediate f16 rounding anywhere; rows are independent. */
int exl3o_host_project_w(const float *x, const uint16_t *trellis, const uint16_t *suh, const uint16_t *svh,
                         uint32_t rows, uint32_t in_features, uint32_t out_features, uint32_t n, uint32_t window_bits,
                         int codebook, int threads, float *out);
int exl3o_host_project(const float *x, const uint16_t *trellis, const uint16_t *suh, const uint16_t *svh,
                       uint32_t rows, uint32_t in_features, uint32_t out_features, uint32_t n, int threads,
                       float *out) {
    return exl3o_host_project_w(x, trellis, suh, svh, rows, in_features, out_features, n, 16, 0, threads, out);
}
/* The same at a codeword window (8..16 bits) and codebook (0 mul1, 1 mcg). */
int exl3o_host_project_w(const float *x, const uint16_t *trellis, const uint16_t *suh, const uint16_t *svh,
                         uint32_t rows, uint32_t in_features, uint32_t out_features, uint32_t n, uint32_t window_bits,
                         int codebook, int threads, float *out) {
    ensure_tables();
    uint32_t in_tiles = in_features / TILE, out_tiles = out_features / TILE;
    float *sc = (float *)malloc((size_t)rows * in_features * 4);
    if (!sc) return -1;
    for (uint32_t r = 0; r < rows; r++) {
        float *s = sc + (size_t)r * in_features;
        for (uint32_t i = 0; i < in_features; i++) s[i] = x[(size_t)r * in_features + i] * exl3o_f16_to_f32(suh[i]);
        for (uint32_t b = 0; b < in_features; b += HAD_DIM) exl3o_hadamard128(s + b);
    }
    int nt = threads < 1 ? 1 : threads;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int t = 0; t < nt; t++) {
        uint32_t a = (uint32_t)((uint64_t)out_tiles * t / nt);
        uint32_t b = (uint32_t)((uint64_t)out_tiles * (t + 1) / nt);
        uint16_t tile[TILE_VALUES];
        float wf[TILE_VALUES];
        for (uint32_t r = 0; r < rows; r++)
            for (uint32_t c = a * TILE; c < b * TILE; c++) out[(size_t)r * out_features + c] = 0.0f;
        for (uint32_t tk = 0; tk < in_tiles; tk++) {
            for (uint32_t tn = a; tn < b; tn++) {
                decode_tile_cb(trellis + ((size_t)tk * out_tiles + tn) * n, n, window_bits, codebook, tile);
                for (uint32_t i = 0; i < TILE_VALUES; i++) wf[i] = exl3o_f16_to_f32(tile[i]);
                for (uint32_t r = 0; r < rows; r++) {
                    const float *s = sc + (size_t)r * in_features + tk * TILE;
                    float *o = out + (size_t)r * out_features + tn * TILE;
                    for (uint32_t rr = 0; rr < TILE; rr++)
                        for (uint32_t c = 0; c < TILE; c++) o[c] += s[rr] * wf[rr * TILE + c];
                }
            }
        }
    }
    for (uint32_t r = 0; r < rows; r++) {
        float *o = out + (size_t)r * out_features;
        for (uint32_t b = 0; b < out_features; b += HAD_DIM) exl3o_hadamard128(o + b);
        for (uint32_t c = 0; c < out_features; c++) o[c] *= exl3o_f16_to_f32(svh[c]);
    }
    free(sc);
    return 0;
}

/* ---------------------------------------------------------------- routed SwiGLU truth (SX/root.zig:116-167,
 * SX/expert_exl3_kernels.zig:2274-2420): per (row, k) slot, expert e = inds[row*topk+k]:
 *   g = gate_e(x_row), u = up_e(x_row)             (f32 truth linears, as Host.project)
 *   g = min(g, limit), u = clamp(u, -limit, limit) when limit > 0   (MID_SOURCE's CLAMP_LIMIT)
 *   h = silu(g) * u
 *   y_row = sum_k score[row, k] * down_e(h)        (REDUCE_SOURCE: f32 score-weighted sum)
 * Banks are stacked on the expert axis: trellis [E][in/16][out/16][n], suh [E][in], svh [E][out]. */
int exl3o_moe_truth_w(const float *x, const int32_t *inds, const float *scores, uint32_t rows, uint32_t topk,
                      const uint16_t *g_tr, const uint16_t *g_suh, const uint16_t *g_svh, uint32_t g_n,
                      const uint16_t *u_tr, const uint16_t *u_suh, const uint16_t *u_svh, uint32_t u_n,
                      const uint16_t *d_tr, const uint16_t *d_suh, const uint16_t *d_svh, uint32_t d_n,
                      uint32_t gu_window, uint32_t d_window, int gu_cb, int d_cb, uint32_t hidden, uint32_t inter,
                      float limit, int threads, float *y);
int exl3o_moe_truth(const float *x, const int32_t *inds, const float *scores, uint32_t rows, uint32_t topk,
                    const uint16_t *g_tr, const uint16_t *g_suh, const uint16_t *g_svh, uint32_t g_n,
                    const uint16_t *u_tr, const uint16_t *u_suh, const uint16_t *u_svh, uint32_t u_n,
                    const uint16_t *d_tr, const uint16_t *d_suh, const uint16_t *d_svh, uint32_t d_n,
                    uint32_t hidden, uint32_t inter, float limit, int threads, float *y) {
    return exl3o_moe_truth_w(x, inds, scores, rows, topk, g_tr, g_suh, g_svh, g_n, u_tr, u_suh, u_svh, u_n, d_tr,
                             d_suh, d_svh, d_n, 16, 16, 0, 0, hidden, inter, limit, threads, y);
}
/* The same with gate/up and down at codeword windows (8..16 bits) and codebooks (0 mul1, 1 mcg). */
int exl3o_moe_truth_w(const float *x, const int32_t *inds, const float *scores, uint32_t rows, uint32_t topk,
                      const uint16_t *g_tr, const uint16_t *g_suh, const uint16_t *g_svh, uint32_t g_n,
                      const uint16_t *u_tr, const uint16_t *u_suh, const uint16_t *u_svh, uint32_t u_n,
                      const uint16_t *d_tr, const uint16_t *d_suh, const uint16_t *d_svh, uint32_t d_n,
                      uint32_t gu_window, uint32_t d_window, int gu_cb, int d_cb, uint32_t hidden, uint32_t inter,
                      float limit, int threads, float *y) {
    size_t gate_words = (size_t)(hidden / 16) * (inter / 16) * g_n;
    size_t up_words = (size_t)(hidden / 16) * (inter / 16) * u_n;
    size_t down_words = (size_t)(inter / 16) * (hidden / 16) * d_n;
    float *g = (float *)malloc((size_t)inter * 4);
    float *u = (float *)malloc((size_t)inter * 4);
    float *d = (float *)malloc((size_t)hidden * 4);
    if (!g || !u || !d) {
        free(g);
        free(u);
        free(d);
        return -1;
    }
    for (uint32_t r = 0; r < rows; r++) {
        float *yr = y + (size_t)r * hidden;
        for (uint32_t c = 0; c < hidden; c++) yr[c] = 0.0f;
        for (uint32_t k = 0; k < topk; k++) {
            uint32_t e = (uint32_t)inds[r * topk + k];
            const float *xr = x + (size_t)r * hidden;
            exl3o_host_project_w(xr, g_tr + e * gate_words, g_suh + (size_t)e * hidden, g_svh + (size_t)e * inter, 1,
                                 hidden, inter, g_n, gu_window, gu_cb, threads, g);
            exl3o_host_project_w(xr, u_tr + e * up_words, u_suh + (size_t)e * hidden, u_svh + (size_t)e * inter, 1,
                               hidden, inter, u_n, gu_window, gu_cb, threads, u);
            for (uint32_t i = 0; i < inter; i++) {
                float gv = g[i], uv = u[i];
                if (limit > 0.0f) {
                    gv = gv < limit ? gv : limit;
                    uv = uv < -limit ? -limit : (uv > limit ? limit : uv);
                }
                float sig = 1.0f / (1.0f + expf(-gv));
                g[i] = gv * sig * uv;
            }
            exl3o_host_project_w(g, d_tr + e * down_words, d_suh + (size_t)e * inter, d_svh + (size_t)e * hidden, 1,
                                 inter, hidden, d_n, d_window, d_cb, threads, d);
            float w = scores[r * topk + k];
            for (uint32_t c = 0; c < hidden; c++) yr[c] += w * d[c];
        }
    }
    free(g);
    free(u);
    free(d);
    return 0;
}

/* ---------------------------------------------------------------- golden planes (TX/kernels.zig:1026-1045) */

uint64_t exl3o_splitmix64(uint64_t *state) {
    *state += 0x9E3779B97F4A7C15ull;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* synthPlane: the little-endian int16 view of splitmix64(seed) outputs, `count` halfwords (a multiple of 4). */
void exl3o_synth_plane(uint64_t seed, size_t count, uint16_t *out) {
    uint64_t s = seed;
    for (size_t i = 0; i < count; i += 4) {
        uint64_t z = exl3o_splitmix64(&s);
        for (int j = 0; j < 4; j++) out[i + j] = (uint16_t)(z >> (16 * j));
    }
}
