// exl3_moe_prefill.cu -- the routed SwiGLU experts at prompt widths on the 5th-generation tensor cores.
//
// The reference runs wide expert calls as expert-sorted windows through a decode-to-threadgroup GEMM
// (plugins/sushi_ds41/src/sushi/exl3/expert_exl3_kernels.zig:2955-3029 moePrefill, :1413-1465 innerGemmSorted,
// :1302 gemmWindowTable).  Here a call of many (token, k) slots runs as:
//   route     -- slots counted per expert, each expert's rows padded to whole 128-row blocks and laid out in expert
//                order (the row of a slot is fixed by an atomic cursor: a row's output depends only on its own input
//                and its expert's weights, never on its neighbours, so any placement gives the same bytes);
//   A images  -- every row's x prepared for gate and for up (x * suh, the 128-wide Hadamard, f16), in the UMMA
//                canonical 128-byte-swizzled layout of the prefill GEMM (exl3_gemm.cu);
//   per group of experts: their gate and up W_hat^T decoded to B images; the grouped tcgen05 GEMMs (one 128-row block
//                of one expert per M tile) with the output Hadamard and svh in the epilogue, f32 out; the SwiGLU
//                (the routed experts' clamp) prepared for down into the down input's A image; down's B images; the
//                grouped down GEMM, f32 per row;
//   combine   -- y[t] = sum_k score[t, k] * row(t, k), k in order, in x's dtype.
// The images and GEMMs are the prefill linear's (exl3_gemm.cu), with a per-block expert for the B image and svh.
#include <cuda_runtime.h>

#include <cstdlib>

#include <cstdint>
#include <mutex>

#include "../../include/exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_internal.h"
#include "exl3_moe.h"

namespace exl3 {

namespace {

constexpr int kGroupExperts = 32;  // experts whose B images are decoded at once (the images' memory)

struct Prefill {
  bool ready = false;
  uint8_t* base = nullptr;
  size_t bytes = 0;
  int experts = 0, hidden = 0, inter = 0, max_slots = 0, rows_max = 0, sms = 0;
  int32_t *counts, *cursor, *base_row, *m_group, *row_slot, *pos, *rows_total;
  int32_t* ranges;  // [groups][2]: each group of experts' rows
  int32_t* blocks;  // [groups][2]: the same as 128-row blocks (the GEMMs' device range)
  int32_t* all;     // [4]: every block {0, blocks} and every row {0, rows} of the call (the one-pass form)
  uint8_t *a_g, *a_u, *a_d, *b_g, *b_u, *b_d;
  float* gu;   // [rows_max][2 inter] f32; the down GEMM's output reuses it ([rows_max][hidden])
  int64_t gu_stride;
};

constexpr int kMaxDev = 64;
std::mutex g_pf_mu;
Prefill g_pf[kMaxDev];

size_t align256(size_t v) { return (v + 255) & ~size_t{255}; }

// The layout of a workspace for `experts` experts of hidden x inter, max_slots slots; returns its bytes.
size_t layout(Prefill& f, uint8_t* b) {
  const int E = f.experts, groups = (E + kGroupExperts - 1) / kGroupExperts;
  f.rows_max = f.max_slots + E * 127;
  f.rows_max = (f.rows_max + 127) / 128 * 128;
  const size_t R = static_cast<size_t>(f.rows_max);
  f.gu_stride = 2 * static_cast<int64_t>(f.inter) > f.hidden ? 2 * static_cast<int64_t>(f.inter) : f.hidden;
  size_t at = 0;
  auto take = [&](size_t n) {
    uint8_t* p = b ? b + at : nullptr;
    at += align256(n);
    return p;
  };
  f.counts = reinterpret_cast<int32_t*>(take(4 * static_cast<size_t>(E)));
  f.cursor = reinterpret_cast<int32_t*>(take(4 * static_cast<size_t>(E)));
  f.base_row = reinterpret_cast<int32_t*>(take(4 * static_cast<size_t>(E + 1)));
  f.m_group = reinterpret_cast<int32_t*>(take(4 * (R / 128)));
  f.row_slot = reinterpret_cast<int32_t*>(take(4 * R));
  f.pos = reinterpret_cast<int32_t*>(take(4 * static_cast<size_t>(f.max_slots)));
  f.rows_total = reinterpret_cast<int32_t*>(take(4));
  f.ranges = reinterpret_cast<int32_t*>(take(8 * static_cast<size_t>(groups)));
  f.blocks = reinterpret_cast<int32_t*>(take(8 * static_cast<size_t>(groups)));
  f.all = reinterpret_cast<int32_t*>(take(16));
  f.a_g = take(R * f.hidden * 2);
  f.a_u = take(R * f.hidden * 2);
  f.a_d = take(R * f.inter * 2);
  const size_t bimg = static_cast<size_t>(f.hidden) * f.inter * 2;  // one expert's W_hat^T, f16
  const size_t ge = E < kGroupExperts ? E : kGroupExperts;            // a group's experts at most
  f.b_g = take(ge * bimg);
  f.b_u = take(ge * bimg);
  f.b_d = take(ge * bimg);
  f.gu = reinterpret_cast<float*>(take(R * static_cast<size_t>(f.gu_stride) * 4));
  return at;
}

// counts[e] += slots routed to e (indices outside the bank count nowhere)
__global__ void pf_count_kernel(const void* inds, int inds_u32, int64_t slots, int experts, int32_t* counts) {
  for (int64_t s = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; s < slots;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = inds_u32 ? static_cast<int>(static_cast<const uint32_t*>(inds)[s]) : static_cast<const int32_t*>(inds)[s];
    if (e >= 0 && e < experts) atomicAdd(counts + e, 1);
  }
}

// One CTA: each expert's first padded row (whole 128-row blocks), the blocks' experts, the padding rows' marks, the
// rows of every group of kGroupExperts experts, the call's padded rows.
__global__ void __launch_bounds__(1024) pf_layout_kernel(Prefill f, int experts) {
  __shared__ int s_warp[32];
  __shared__ int s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  for (int e0 = 0; e0 < experts; e0 += 1024) {
    const int e = e0 + static_cast<int>(threadIdx.x);
    const int padded = e < experts ? (f.counts[e] + 127) / 128 * 128 : 0;
    int total = 0;
    const int ex = cta_scan_excl(padded, s_warp, &total);
    const int start = s_carry + ex;
    if (e < experts) {
      f.base_row[e] = start;
      f.cursor[e] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_carry += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    f.base_row[experts] = s_carry;
    *f.rows_total = s_carry;
  }
  __syncthreads();
  // per expert: its blocks' expert, its padding rows
  for (int e = static_cast<int>(threadIdx.x >> 5); e < experts; e += 32) {
    const int b0 = f.base_row[e], b1 = f.base_row[e + 1], c = f.counts[e];
    for (int r = b0 + static_cast<int>(threadIdx.x & 31u); r < b1; r += 32) {
      if ((r & 127) == 0) f.m_group[r >> 7] = e;
      if (r >= b0 + c) f.row_slot[r] = -1;
    }
  }
  const int groups = (experts + kGroupExperts - 1) / kGroupExperts;
  for (int g = static_cast<int>(threadIdx.x); g < groups; g += blockDim.x) {
    const int e1 = (g + 1) * kGroupExperts < experts ? (g + 1) * kGroupExperts : experts;
    f.ranges[2 * g] = f.base_row[g * kGroupExperts];
    f.ranges[2 * g + 1] = f.base_row[e1];
  }
}

// Each slot's row: its expert's first row + its place among the expert's slots.
__global__ void pf_place_kernel(Prefill f, const void* inds, int inds_u32, int64_t slots, int experts) {
  for (int64_t s = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; s < slots;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = inds_u32 ? static_cast<int>(static_cast<const uint32_t*>(inds)[s]) : static_cast<const int32_t*>(inds)[s];
    int r = -1;
    if (e >= 0 && e < experts) {
      r = f.base_row[e] + atomicAdd(f.cursor + e, 1);
      f.row_slot[r] = static_cast<int32_t>(s);
    }
    f.pos[s] = r;
  }
}

// The group's M blocks [ranges[0] / 128, ranges[1] / 128), as the GEMM's device range.
__global__ void pf_blocks_kernel(const int32_t* ranges, int32_t* mt) {
  mt[0] = ranges[0] / 128;
  mt[1] = ranges[1] / 128;
}

// The call's whole range: blocks {0, rows / 128}, rows {0, rows} (rows: the padded total the layout wrote).
__global__ void pf_all_kernel(const int32_t* rows_total, int32_t* all) {
  all[0] = 0;
  all[1] = *rows_total / 128;
  all[2] = 0;
  all[3] = *rows_total;
}

// y[t] = sum_k score[t, k] * out[pos(t, k)], k in order; grid (hidden / 512, up to 65535 token columns), 128 threads
// of four columns.  Up to eight slots a token: their rows are loaded together, then summed in k order (one load in
// flight per thread had left the kernel waiting on each in turn).
__global__ void __launch_bounds__(128) pf_combine_kernel(const float* out, int64_t stride, const int32_t* pos,
                                                         const float* scores, int64_t rows, int topk, int hidden,
                                                         void* y, int32_t y_dtype) {
  constexpr int kBatch = 8;
  const int c = (static_cast<int>(blockIdx.x) * 128 + static_cast<int>(threadIdx.x)) * 4;
  if (c >= hidden) return;
  for (int64_t t = blockIdx.y; t < rows; t += gridDim.y) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < topk; k0 += kBatch) {
      float4 d[kBatch];
      float sc[kBatch];
      int r[kBatch];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        r[i] = k0 + i < topk ? pos[t * topk + k0 + i] : -1;
        sc[i] = r[i] >= 0 ? scores[t * topk + k0 + i] : 0.f;
        if (r[i] >= 0) d[i] = *reinterpret_cast<const float4*>(out + static_cast<size_t>(r[i]) * stride + c);
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        if (r[i] < 0) continue;
        acc[0] += sc[i] * d[i].x;
        acc[1] += sc[i] * d[i].y;
        acc[2] += sc[i] * d[i].z;
        acc[3] += sc[i] * d[i].w;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) store_act(y, static_cast<size_t>(t) * hidden + c + i, acc[i], y_dtype);
  }
}

}  // namespace

exl3_verdict moe_prefill_reserve(int device, int experts, int hidden, int inter, int max_slots, uint64_t* bytes) {
  if (device < 0 || device >= kMaxDev) return {EXL3_UNSUPPORTED, "exl3_b200: device index out of range"};
  std::lock_guard<std::mutex> lk(g_pf_mu);
  Prefill& f = g_pf[device];
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  if (f.base) {
    cudaDeviceSynchronize();
    cudaFree(f.base);
    f = Prefill{};
  }
  if (bytes) *bytes = 0;
  if (max_slots == 0) {
    if (prev >= 0) cudaSetDevice(prev);
    return {EXL3_OK, nullptr};
  }
  if (experts < 1 || experts > 1024 || hidden <= 0 || hidden % 128 || inter <= 0 || inter % 128 || max_slots < 0 ||
      max_slots > (1 << 22)) {
    if (prev >= 0) cudaSetDevice(prev);
    return {EXL3_UNSUPPORTED, "exl3_b200: BadExl3Shape (prefill workspace: experts 1..1024, hidden and intermediate "
                              "multiples of 128, at most 2^22 slots)"};
  }
  f.experts = experts, f.hidden = hidden, f.inter = inter, f.max_slots = max_slots;
  cudaDeviceGetAttribute(&f.sms, cudaDevAttrMultiProcessorCount, device);
  const size_t need = layout(f, nullptr);
  const bool ok = cudaMalloc(&f.base, need) == cudaSuccess && cudaMemset(f.base, 0, need) == cudaSuccess;
  if (prev >= 0) cudaSetDevice(prev);
  if (!ok) {
    if (f.base) cudaFree(f.base);
    f = Prefill{};
    return {EXL3_TOO_LARGE, "exl3_b200: the prefill workspace does not fit"};
  }
  layout(f, f.base);
  f.bytes = need;
  f.ready = true;
  if (bytes) *bytes = need;
  return {EXL3_OK, nullptr};
}

bool moe_prefill_serves(int device, int experts, int hidden, int inter, int64_t slots) {
  if (device < 0 || device >= kMaxDev) return false;
  std::lock_guard<std::mutex> lk(g_pf_mu);
  const Prefill& f = g_pf[device];
  return f.ready && experts <= f.experts && hidden <= f.hidden && inter <= f.inter && slots <= f.max_slots;
}

exl3_verdict moe_prefill_run(const exl3_weight* gate, const exl3_weight* up, const exl3_weight* down,
                             const exl3_tensor* x, const exl3_tensor* inds, const exl3_tensor* scores, float limit,
                             void* stream, exl3_tensor* out) {
  const int dev = gate->device;
  Prefill f;
  {
    std::lock_guard<std::mutex> lk(g_pf_mu);
    f = g_pf[dev];
  }
  const int E = gate->groups, hidden = gate->in_features, inter = gate->out_features;
  const int64_t rows = x->shape[0] * x->shape[1];
  const int topk = static_cast<int>(inds->shape[2]);
  const int64_t slots = rows * topk;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != dev) cudaSetDevice(dev);
  cudaError_t err = cudaSuccess;
  auto ok = [&](cudaError_t e) {
    if (err == cudaSuccess) err = e;
    return err == cudaSuccess;
  };
  Prefill ff = f;  // this call's view: the real expert count
  const uint32_t cw_gu = window_mask(flags_window_bits(gate->flags)), cw_d = window_mask(flags_window_bits(down->flags));
  const int mcg_gu = (gate->flags & EXL3_WEIGHT_MCG) ? 1 : 0, mcg_d = (down->flags & EXL3_WEIGHT_MCG) ? 1 : 0;
  const int inds_u32 = inds->dtype == EXL3_U32;
  const int threads = 256, blocks = f.sms * 4;
  // route
  ok(cudaMemsetAsync(f.counts, 0, 4 * static_cast<size_t>(E), st));
  pf_count_kernel<<<blocks, threads, 0, st>>>(inds->data, inds_u32, slots, E, f.counts);
  ok(cudaGetLastError());
  pf_layout_kernel<<<1, 1024, 0, st>>>(ff, E);
  ok(cudaGetLastError());
  pf_place_kernel<<<blocks, threads, 0, st>>>(ff, inds->data, inds_u32, slots, E);
  ok(cudaGetLastError());
  // A images of gate and up (every row)
  MoeImages mi{};
  mi.row_slot = f.row_slot, mi.m_group = f.m_group, mi.rows_total = f.rows_total, mi.topk = topk;
  mi.x = x->data, mi.x_dtype = x->dtype, mi.x_row_stride = hidden, mi.hidden = hidden, mi.inter = inter;
  {
    const size_t esz = x->dtype == EXL3_F32 ? 4 : 2;
    // (hidden is a multiple of 128, so every row starts as aligned as x)
    mi.x_vec = reinterpret_cast<uintptr_t>(x->data) % (4 * esz) == 0 ? 1 : 0;
    if (reinterpret_cast<uintptr_t>(x->data) % 16 != 0) mi.x_vec = 0;  // the sixteen-per-lane form's 16-byte loads
  }
  mi.suh_g = gate->suh, mi.suh_u = up->suh, mi.suh_d = down->suh;
  mi.a_g = f.a_g, mi.a_u = f.a_u, mi.a_d = f.a_d;
  mi.gu = f.gu, mi.gu_stride = f.gu_stride, mi.limit = limit;
  if (err == cudaSuccess) ok(launch_moe_a_images(mi, f.sms, st));
  // the full mul1 window: W_hat^T decoded inside the GEMMs, all experts in one pass (gate, up, the SwiGLU into down's
  // A image, down); EXL3_GEMM_FUSED=0 keeps the image form for measurement
  const char* fz = getenv("EXL3_GEMM_FUSED");
  const bool fused = !cw_gu && !cw_d && !mcg_gu && !mcg_d && !(fz && atoi(fz) == 0);
  if (fused && err == cudaSuccess) {
    pf_all_kernel<<<1, 1, 0, st>>>(f.rows_total, f.all);
    ok(cudaGetLastError());
    for (int w = 0; w < 2 && err == cudaSuccess; ++w) {
      const exl3_weight* wt = w == 0 ? gate : up;
      GemmParams gp{};
      gp.a_img = w == 0 ? f.a_g : f.a_u;
      gp.svh = wt->svh;
      gp.y = f.gu + (w == 0 ? 0 : inter);
      gp.y_dtype = kF32;
      gp.y_row_stride = f.gu_stride;
      gp.m = f.rows_max;
      gp.ncols = inter;
      gp.tiles_m = f.rows_max / 128;
      gp.tiles_n = inter % 256 == 0 ? inter / 256 : inter / 128;
      gp.kb = hidden / 64;
      gp.vec_store = store_width(f.gu, f.gu_stride * 4);
      gp.err = device_error_ptr();
      gp.mt_range = f.all;
      gp.m_group = f.m_group;
      gp.group0 = 0;
      gp.svh_group = inter;
      gp.trellis = wt->trellis;
      gp.tr_group = static_cast<int64_t>(hidden / 16) * (inter / 16) * wt->n;
      gp.out_tiles = inter / 16;
      gp.tn0 = 0;
      gp.n = wt->n;
      ok(launch_gemm_fused(gp, inter % 256 == 0 ? 1 : 0, f.sms, st));
    }
    mi.row_range = f.all + 2;
    if (err == cudaSuccess) ok(launch_moe_mid_images(mi, f.sms, st));
    GemmParams gd{};
    gd.a_img = f.a_d;
    gd.svh = down->svh;
    gd.y = f.gu;  // the gate|up outputs are consumed: down's rows overwrite them
    gd.y_dtype = kF32;
    gd.y_row_stride = f.gu_stride;
    gd.m = f.rows_max;
    gd.ncols = hidden;
    gd.tiles_m = f.rows_max / 128;
    gd.tiles_n = hidden % 256 == 0 ? hidden / 256 : hidden / 128;
    gd.kb = inter / 64;
    gd.vec_store = store_width(f.gu, f.gu_stride * 4);
    gd.err = device_error_ptr();
    gd.mt_range = f.all;
    gd.m_group = f.m_group;
    gd.group0 = 0;
    gd.svh_group = hidden;
    gd.trellis = down->trellis;
    gd.tr_group = static_cast<int64_t>(inter / 16) * (hidden / 16) * down->n;
    gd.out_tiles = hidden / 16;
    gd.tn0 = 0;
    gd.n = down->n;
    if (err == cudaSuccess) ok(launch_gemm_fused(gd, hidden % 256 == 0 ? 1 : 0, f.sms, st));
  }
  // per group of experts: B images, the gate and up GEMMs, the SwiGLU into down's A image, down's B images and GEMM
  const int groups = fused ? 0 : (E + kGroupExperts - 1) / kGroupExperts;
  const int64_t bimg = static_cast<int64_t>(hidden) * inter * 2;
  for (int g = 0; g < groups && err == cudaSuccess; ++g) {
    const int e0 = g * kGroupExperts, cnt = E - e0 < kGroupExperts ? E - e0 : kGroupExperts;
    int32_t* mtg = f.blocks + 2 * g;
    pf_blocks_kernel<<<1, 1, 0, st>>>(f.ranges + 2 * g, mtg);
    ok(cudaGetLastError());
    ok(launch_moe_b_images(gate->trellis, hidden, inter, gate->n, e0, cnt, f.counts, f.b_g, bimg, st, cw_gu, mcg_gu));
    ok(launch_moe_b_images(up->trellis, hidden, inter, up->n, e0, cnt, f.counts, f.b_u, bimg, st, cw_gu, mcg_gu));
    for (int w = 0; w < 2 && err == cudaSuccess; ++w) {
      GemmParams gp{};
      gp.a_img = w == 0 ? f.a_g : f.a_u;
      gp.b_img = w == 0 ? f.b_g : f.b_u;
      gp.svh = w == 0 ? gate->svh : up->svh;
      gp.y = f.gu + (w == 0 ? 0 : inter);
      gp.y_dtype = kF32;
      gp.y_row_stride = f.gu_stride;
      gp.m = f.rows_max;
      gp.ncols = inter;
      gp.tiles_m = f.rows_max / 128;
      gp.tiles_n = inter % 256 == 0 ? inter / 256 : inter / 128;
      gp.kb = hidden / 64;
      gp.vec_store = store_width(f.gu, f.gu_stride * 4);
      gp.err = device_error_ptr();
      gp.mt_range = mtg;
      gp.m_group = f.m_group;
      gp.group0 = e0;
      gp.b_group_bytes = bimg;
      gp.svh_group = inter;
      ok(launch_gemm_image(gp, inter % 256 == 0 ? 1 : 0, f.sms, st));
    }
    mi.row_range = f.ranges + 2 * g;
    if (err == cudaSuccess) ok(launch_moe_mid_images(mi, f.sms, st));
    ok(launch_moe_b_images(down->trellis, inter, hidden, down->n, e0, cnt, f.counts, f.b_d, bimg, st, cw_d, mcg_d));
    GemmParams gd{};
    gd.a_img = f.a_d;
    gd.b_img = f.b_d;
    gd.svh = down->svh;
    gd.y = f.gu;  // the gate|up outputs of these rows are consumed: down's rows overwrite them
    gd.y_dtype = kF32;
    gd.y_row_stride = f.gu_stride;
    gd.m = f.rows_max;
    gd.ncols = hidden;
    gd.tiles_m = f.rows_max / 128;
    gd.tiles_n = hidden % 256 == 0 ? hidden / 256 : hidden / 128;
    gd.kb = inter / 64;
    gd.vec_store = store_width(f.gu, f.gu_stride * 4);
    gd.err = device_error_ptr();
    gd.mt_range = mtg;
    gd.m_group = f.m_group;
    gd.group0 = e0;
    gd.b_group_bytes = bimg;
    gd.svh_group = hidden;
    if (err == cudaSuccess) ok(launch_gemm_image(gd, hidden % 256 == 0 ? 1 : 0, f.sms, st));
  }
  if (err == cudaSuccess) {
    const dim3 cg(static_cast<unsigned>((hidden + 511) / 512), static_cast<unsigned>(rows < 65535 ? rows : 65535));
    pf_combine_kernel<<<cg, 128, 0, st>>>(f.gu, f.gu_stride, f.pos, static_cast<const float*>(scores->data), rows,
                                          topk, hidden, out->data, out->dtype);
    ok(cudaGetLastError());
  }
  if (prev >= 0 && prev != dev) cudaSetDevice(prev);
  if (err != cudaSuccess) return {EXL3_FAILED, "exl3_b200: MoE prefill launch failed"};
  return {EXL3_OK, nullptr};
}

}  // namespace exl3
