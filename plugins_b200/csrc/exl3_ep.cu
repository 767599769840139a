// exl3_ep.cu -- expert parallelism for the routed experts: the dispatch and combine either side of the two NCCL
// all-to-alls (the all-to-alls themselves are the caller's: torch.distributed or ncclSend/ncclRecv).
//
// Rank r of `world` owns experts [r E/world, (r+1) E/world) of every bank (plus, when a shared expert is used, the
// shared expert as local expert E/world: its slots stay on the token's own rank).  A dispatch buffer holds one block per peer,
// each [C + 1][D] in x's dtype:
//   rows 0 .. C-1   token rows routed to that peer's experts, in slot order (token-major, k minor);
//   row C           metadata: 32-bit word j (j < C) = the peer-local expert of row j, -1 for an empty row.
// Every block has the same size, so the exchange is an equal-split all_to_all_single and a step needs no counts on the
// host (graph-capturable).  After the exchange the owner unpacks the metadata rows into swiglu's expert indices (score
// 1 for every row, -1 for the metadata rows themselves) and runs its bank on all received rows with an f32 output; the
// second all-to-all returns those rows, and the source combines out[t] = sum_k score[t][k] * back[slot(t, k)] in k
// order (f32), plus an optional shared expert's f32 rows -- the order and arithmetic of the single-GPU combine.
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace {

using exl3::kF16;
using exl3::kBF16;
using exl3::kF32;

constexpr int kMaxEpCapacity = 2048;  // rows per peer block

__device__ __forceinline__ int read_index(const void* inds, int u32, size_t i) {
  return u32 ? static_cast<int>(static_cast<const uint32_t*>(inds)[i]) : static_cast<const int32_t*>(inds)[i];
}

// Grid (world, copy CTAs): CTA (d, c) lists the slots routed to peer d (its thread 0, in slot order) and copies every
// c-th of their token rows; CTA (d, 0) also writes the metadata row and the slots' return positions.  A slot whose
// expert is `experts` with `shared` set goes to this rank's own block (the shared expert, held by every rank at local
// index experts / world); other experts outside the bank are absent (CTA (0, 0) marks them).  Slots beyond the
// capacity are dropped and flagged.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const void* __restrict__ x, int32_t esize, int tokens,
                                                          int topk, int hidden, const void* __restrict__ inds,
                                                          int inds_u32, int experts, int world, int rank, int shared,
                                                          int cap, uint8_t* __restrict__ send,
                                                          int32_t* __restrict__ back_slot, uint32_t* err) {
  __shared__ int s_tok[kMaxEpCapacity];
  __shared__ int s_count;
  const int d = blockIdx.x;
  const bool head = blockIdx.y == 0;
  const int per = experts / world;
  const size_t row_bytes = static_cast<size_t>(hidden) * esize;
  uint8_t* block = send + static_cast<size_t>(d) * (cap + 1) * row_bytes;
  int32_t* meta = reinterpret_cast<int32_t*>(block + static_cast<size_t>(cap) * row_bytes);
  // the slots routed to peer d in slot order: a CTA-wide stable compaction, 256 slots at a time
  __shared__ int s_warp[32];
  __shared__ int s_over;
  if (threadIdx.x == 0) s_over = 0;
  int base = 0;
  const int nslots = tokens * topk;
  for (int s0 = 0; s0 < nslots; s0 += static_cast<int>(blockDim.x)) {
    const int s = s0 + static_cast<int>(threadIdx.x);
    int flag = 0, local = 0;
    if (s < nslots) {
      const int e = read_index(inds, inds_u32, s);
      int dest = -1;
      if (e >= 0 && e < experts) {
        dest = e / per;
        local = e - dest * per;
      } else if (shared && e == experts) {
        dest = rank;
        local = per;
      } else if (head && d == 0) {
        back_slot[s] = -1;
      }
      flag = dest == d;
    }
    int total;
    const int pos = exl3::cta_scan_excl(flag, s_warp, &total);
    if (flag) {
      const int j = base + pos;
      if (j < cap) {
        s_tok[j] = s / topk;
        if (head) {
          meta[j] = local;
          back_slot[s] = d * (cap + 1) + j;
        }
      } else {
        if (head) back_slot[s] = -1;
        s_over = 1;
      }
    }
    base += total;
  }
  if (head) {
    for (int i = (base < cap ? base : cap) + static_cast<int>(threadIdx.x); i < cap; i += static_cast<int>(blockDim.x))
      meta[i] = -1;
  }
  __syncthreads();
  if (head && threadIdx.x == 0 && s_over) atomicOr(err, exl3::kErrEpOverflow);
  if (threadIdx.x == 0) s_count = base < cap ? base : cap;
  __syncthreads();
  const int n = s_count;
  const size_t words = row_bytes / 16;  // rows are whole 16-byte vectors (hidden % 128 == 0)
  for (int j = static_cast<int>(blockIdx.y); j < n; j += static_cast<int>(gridDim.y)) {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) + s_tok[j] * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(block + static_cast<size_t>(j) * row_bytes);
    for (size_t w = threadIdx.x; w < words; w += blockDim.x) dst[w] = src[w];
  }
}

// Received blocks -> swiglu's per-row expert index (topk 1) and score 1; metadata rows get -1 (skipped).
__global__ void __launch_bounds__(256) ep_unpack_kernel(const uint8_t* __restrict__ recv, int32_t esize, int hidden,
                                                        int cap, int32_t* __restrict__ inds,
                                                        float* __restrict__ scores) {
  const int d = blockIdx.x;
  const size_t row_bytes = static_cast<size_t>(hidden) * esize;
  const int32_t* meta =
      reinterpret_cast<const int32_t*>(recv + (static_cast<size_t>(d) * (cap + 1) + cap) * row_bytes);
  for (int j = threadIdx.x; j <= cap; j += blockDim.x) {
    const size_t at = static_cast<size_t>(d) * (cap + 1) + j;
    inds[at] = j < cap ? meta[j] : -1;
    scores[at] = 1.0f;
  }
}

// out[t] = sum_k score[t][k] * back[slot(t, k)] (k order, f32), + shared[t] when given.
__global__ void __launch_bounds__(128) ep_combine_kernel(const float* __restrict__ back,
                                                         const int32_t* __restrict__ back_slot,
                                                         const float* __restrict__ scores, int topk, int hidden,
                                                         const float* __restrict__ shared, void* __restrict__ out,
                                                         int32_t out_dtype) {
  const int t = blockIdx.y;
  const size_t c = static_cast<size_t>(blockIdx.x) * 128 + threadIdx.x;
  float acc = 0.0f;
  for (int k = 0; k < topk; ++k) {
    const int pos = back_slot[static_cast<size_t>(t) * topk + k];
    if (pos >= 0) acc += scores[static_cast<size_t>(t) * topk + k] * back[static_cast<size_t>(pos) * hidden + c];
  }
  if (shared) acc += shared[static_cast<size_t>(t) * hidden + c];
  exl3::store_act(out, static_cast<size_t>(t) * hidden + c, acc, out_dtype);
}

exl3_verdict refuse(int32_t code, const char* why) { return {code, why}; }

int32_t esize_of(int32_t dt) { return dt == EXL3_F32 ? 4 : 2; }
bool act_dtype(int32_t dt) { return dt == EXL3_F16 || dt == EXL3_BF16 || dt == EXL3_F32; }

struct Dev {
  int prev = -1;
  explicit Dev(const void* p) {
    cudaPointerAttributes a{};
    cudaGetDevice(&prev);
    if (cudaPointerGetAttributes(&a, p) == cudaSuccess && a.type == cudaMemoryTypeDevice && a.device != prev)
      cudaSetDevice(a.device);
    else
      prev = -1;
  }
  ~Dev() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" {

exl3_verdict exl3_ep_dispatch(const exl3_tensor* x, const exl3_tensor* inds, int32_t experts, int32_t world,
                              int32_t rank, int32_t shared, void* stream, exl3_tensor* send, exl3_tensor* back_slot) {
  if (!x || !inds || !send || !back_slot) return refuse(EXL3_FAILED, "exl3_ep_dispatch: bad arguments");
  if (x->ndim != 2 || inds->ndim != 2 || send->ndim != 3 || back_slot->ndim != 2)
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: x [T, D], inds [T, K], send [world, C + 1, D], back_slot [T, K]");
  const int64_t tokens = x->shape[0], hidden = x->shape[1], topk = inds->shape[1];
  const int64_t cap = send->shape[1] - 1;
  if (!act_dtype(x->dtype) || send->dtype != x->dtype)
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: x is f16, bf16 or f32 and send has x's dtype");
  if (inds->dtype != EXL3_I32 && inds->dtype != EXL3_U32) return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: inds are i32 or u32");
  if (back_slot->dtype != EXL3_I32) return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: back_slot is i32");
  if (inds->shape[0] != tokens || back_slot->shape[0] != tokens || back_slot->shape[1] != topk || topk < 1 || topk > 32)
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: inds and back_slot are [T, K], K <= 32");
  if (world < 1 || experts < world || experts % world != 0)
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: the experts split evenly over the ranks");
  if (rank < 0 || rank >= world) return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: rank out of range");
  if (send->shape[0] != world || send->shape[2] != hidden || hidden % 128 != 0)
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: send is [world, C + 1, D], D a multiple of 128");
  if (cap < 1 || cap > kMaxEpCapacity || 4 * cap > hidden * esize_of(x->dtype))
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: capacity C is 1 .. 2048 and its metadata fits one row");
  if (tokens * topk > (1 << 20)) return refuse(EXL3_TOO_LARGE, "exl3_ep_dispatch: too many slots");
  if (tokens == 0) return {EXL3_OK, nullptr};
  if (!x->data || !inds->data || !send->data || !back_slot->data) return refuse(EXL3_FAILED, "exl3_ep_dispatch: bad tensors");
  if (reinterpret_cast<uintptr_t>(x->data) % 16 != 0 || reinterpret_cast<uintptr_t>(send->data) % 16 != 0)
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_dispatch: x and send start on 16-byte boundaries");
  Dev dev(send->data);
  uint32_t* err = exl3::device_error_ptr();
  if (!err) return refuse(EXL3_FAILED, "exl3_ep_dispatch: no device error word");
  // copy CTAs per peer: about 148 CTAs in all, at least one per peer
  const int copy = world >= 148 ? 1 : (148 + world - 1) / world;
  ep_dispatch_kernel<<<dim3(world, copy), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x->data, esize_of(x->dtype), static_cast<int>(tokens), static_cast<int>(topk), static_cast<int>(hidden),
      inds->data, inds->dtype == EXL3_U32, experts, world, rank, shared ? 1 : 0, static_cast<int>(cap),
      static_cast<uint8_t*>(send->data), static_cast<int32_t*>(back_slot->data), err);
  if (cudaGetLastError() != cudaSuccess) return refuse(EXL3_FAILED, "exl3_ep_dispatch: launch failed");
  return {EXL3_OK, nullptr};
}

exl3_verdict exl3_ep_unpack(const exl3_tensor* recv, void* stream, exl3_tensor* inds, exl3_tensor* scores) {
  if (!recv || !inds || !scores || recv->ndim != 3 || inds->ndim != 3 || scores->ndim != 3)
    return refuse(EXL3_FAILED, "exl3_ep_unpack: recv [world, C + 1, D], inds and scores [world, C + 1, 1]");
  const int64_t world = recv->shape[0], rows = recv->shape[1], hidden = recv->shape[2];
  if (!act_dtype(recv->dtype) || inds->dtype != EXL3_I32 || scores->dtype != EXL3_F32)
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_unpack: recv in an activation dtype, inds i32, scores f32");
  for (const exl3_tensor* t : {inds, scores})
    if (t->shape[0] != world || t->shape[1] != rows || t->shape[2] != 1)
      return refuse(EXL3_UNSUPPORTED, "exl3_ep_unpack: inds and scores are [world, C + 1, 1]");
  if (rows < 2 || rows - 1 > kMaxEpCapacity || hidden % 128 != 0) return refuse(EXL3_UNSUPPORTED, "exl3_ep_unpack: bad block");
  if (world == 0) return {EXL3_OK, nullptr};
  Dev dev(recv->data);
  ep_unpack_kernel<<<static_cast<unsigned>(world), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(recv->data), esize_of(recv->dtype), static_cast<int>(hidden),
      static_cast<int>(rows - 1), static_cast<int32_t*>(inds->data), static_cast<float*>(scores->data));
  if (cudaGetLastError() != cudaSuccess) return refuse(EXL3_FAILED, "exl3_ep_unpack: launch failed");
  return {EXL3_OK, nullptr};
}

exl3_verdict exl3_ep_combine(const exl3_tensor* back, const exl3_tensor* back_slot, const exl3_tensor* scores,
                             const exl3_tensor* shared, void* stream, exl3_tensor* out) {
  if (!back || !back_slot || !scores || !out) return refuse(EXL3_FAILED, "exl3_ep_combine: bad arguments");
  if (back->ndim != 3 || back->dtype != EXL3_F32) return refuse(EXL3_UNSUPPORTED, "exl3_ep_combine: back is f32 [world, C + 1, D]");
  if (out->ndim != 2 || !act_dtype(out->dtype)) return refuse(EXL3_UNSUPPORTED, "exl3_ep_combine: out is [T, D] f16, bf16 or f32");
  const int64_t tokens = out->shape[0], hidden = out->shape[1];
  if (back->shape[2] != hidden || hidden % 128 != 0) return refuse(EXL3_UNSUPPORTED, "exl3_ep_combine: back and out differ in D");
  if (back_slot->ndim != 2 || back_slot->dtype != EXL3_I32 || back_slot->shape[0] != tokens ||
      scores->ndim != 2 || scores->dtype != EXL3_F32 || scores->shape[0] != tokens || scores->shape[1] != back_slot->shape[1])
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_combine: back_slot i32 and scores f32, both [T, K]");
  const bool has_shared = shared && shared->data;
  if (has_shared && (shared->ndim != 2 || shared->dtype != EXL3_F32 || shared->shape[0] != tokens || shared->shape[1] != hidden))
    return refuse(EXL3_UNSUPPORTED, "exl3_ep_combine: shared is f32 [T, D]");
  if (tokens == 0) return {EXL3_OK, nullptr};
  Dev dev(out->data);
  ep_combine_kernel<<<dim3(static_cast<unsigned>(hidden / 128), static_cast<unsigned>(tokens)), 128, 0,
                      static_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(back->data), static_cast<const int32_t*>(back_slot->data),
      static_cast<const float*>(scores->data), static_cast<int>(back_slot->shape[1]), static_cast<int>(hidden),
      has_shared ? static_cast<const float*>(shared->data) : nullptr, out->data, out->dtype);
  if (cudaGetLastError() != cudaSuccess) return refuse(EXL3_FAILED, "exl3_ep_combine: launch failed");
  return {EXL3_OK, nullptr};
}

}  // extern "C"
