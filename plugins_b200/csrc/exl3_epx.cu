// exl3_epx.cu -- the expert-parallel exchange over NVLink peer memory: the two all-to-alls of a routed-expert step
// done by this library's own kernels, with no collective library in the step (one process per GPU).
//
// Every rank holds, in its own HBM, mapped into the other ranks with CUDA IPC:
//   recv   [2 parities][world][C + 1][D] (x's dtype)  rows other ranks routed to this rank's experts, block q from q;
//   back   [2 parities][world][C + 1][D] f32          this rank's slots' expert outputs, block q computed by rank q;
//   done   [2 phases][world] u32                      per rank q: the last step whose dispatch (phase 0) or return
//                                                     (phase 1) q has published here;
//   step   u32                                        this rank's step counter;
//   arrive [2 phases] u32                             CTAs of this rank's dispatch that have finished (phase 0);
//   used   [world] i32                                this step's rows from each source (receive -> return).
// A step: exl3_epx_dispatch (the dispatch -- the layout of exl3_ep_dispatch -- writes block `rank` of every peer's
// recv directly; each CTA arrives; the last CTA to arrive advances the step word), exl3_epx_receive (its first CTA
// releases done[0][rank] = step on every rank -- one system-scope fence after the dispatch launch completed -- then
// every CTA waits, bounded, until every rank's done[0] holds the step; copies recv into the caller's fixed buffer and
// unpacks swiglu's indices), the caller's swiglu on that buffer (f32 out), exl3_epx_return (block q of the output
// straight into rank q's back, block `rank`; then a one-CTA launch releases done[1][rank] on every rank),
// exl3_epx_combine (waits for every rank's done[1], then sum_k score * back[slot] in k order).  Parity = step & 1: a rank dispatches step s + 2
// into a peer only after its step s + 1 combine saw that peer's step s + 1 return, which the peer issued after its
// step s receive copied recv out, so the two copies of recv and back never race.  The done words only grow; nothing
// is reset, and graph replays need no host work.  Every wait is bounded (one second): a missing peer sets
// EXL3_ERR_EP_TIMEOUT and the kernel returns.
#include <cuda_runtime.h>

#include <cstring>
#include <new>

#include "../../include/exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxCap = 2048;

struct EpxDev {
  uint8_t* recv[kMaxRanks];
  float* back[kMaxRanks];
  uint32_t* done[kMaxRanks];  // [2][world]
  uint32_t* step;
  uint32_t* arrive;  // [2]
  int32_t* used;     // [world] this step's rows from each source (the receive writes, the return reads)
  int32_t world, rank, cap, hidden, esize;
  uint64_t* trace;   // the phase timeline ring, or null: 0 dispatch begins, 1 its copies done, 2 every rank's dispatch
                     // seen, 3 received, 4 return begins (the caller's swiglu done), 5 its copies done, 6 every
                     // rank's return seen, 7 combined
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Every rank's done[phase] word for this step, waited for by threads [0, world) of the CTA (bounded); true if all.
__device__ bool wait_all(const EpxDev& d, int phase, uint32_t step, uint32_t* err) {
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if (threadIdx.x < static_cast<uint32_t>(d.world)) {
    const uint32_t* f = d.done[d.rank] + phase * d.world + threadIdx.x;
    if (static_cast<int32_t>(ld_acquire_sys(f) - step) < 0) {
      const uint64_t t0 = exl3::global_timer_ns();
      while (static_cast<int32_t>(ld_acquire_sys(f) - step) < 0) {
        if (exl3::global_timer_ns() - t0 > 1000000000ull) {
          s_fail = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (s_fail && threadIdx.x == 0) atomicOr(err, exl3::kErrEpTimeout);
  return s_fail == 0;
}

// Releases done[phase][rank] = step on every rank: one system-scope fence for every store this rank made before it
// (the copies of a launch that has completed), then a release store per rank.
__device__ void publish(const EpxDev& d, int phase, uint32_t step) {
  asm volatile("fence.sc.sys;" ::: "memory");
  for (int q = 0; q < d.world; ++q) {
    uint32_t* f = d.done[q] + phase * d.world + d.rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(step) : "memory");
  }
}

// The end of the dispatch's copies, run by every CTA: it arrives; the last CTA to arrive (every CTA has read the
// step word by then) resets the count and advances the step word.  The release waits for the launch boundary.
__device__ void arrive_and_advance(const EpxDev& d, uint32_t step) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t total = gridDim.x * gridDim.y;
    uint32_t prior;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prior) : "l"(d.arrive) : "memory");
    s_last = prior == total - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    d.arrive[0] = 0u;
    *d.step = step;
    exl3::trace_at(d.trace, step, 1);
  }
}

__device__ __forceinline__ int read_index(const void* inds, int u32, size_t i) {
  return u32 ? static_cast<int>(static_cast<const uint32_t*>(inds)[i]) : static_cast<const int32_t*>(inds)[i];
}

// Grid (world, copy CTAs), as exl3_ep_dispatch, but block d goes to block `rank` of peer d's recv (this parity).
__global__ void __launch_bounds__(256) epx_dispatch_kernel(const EpxDev* dp, const void* __restrict__ x, int tokens,
                                                           int topk, const void* __restrict__ inds, int inds_u32,
                                                           int experts, int shared, int32_t* __restrict__ back_slot,
                                                           uint32_t* err) {
  __shared__ int s_tok[kMaxCap];
  __shared__ int s_count;
  exl3::pdl_wait();  // every launch before this one in the stream is complete (programmatic dependent launch)
  exl3::pdl_launch_dependents();
  const EpxDev& d = *dp;
  const int dst = blockIdx.x, cap = d.cap;
  const bool head = blockIdx.y == 0;
  const int per = experts / d.world;
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(d.step) + 1u;  // this launch's step
  if (dst == 0 && head && threadIdx.x == 0) exl3::trace_at(d.trace, step, 0);
  const size_t row_bytes = static_cast<size_t>(d.hidden) * d.esize;
  const size_t block_bytes = static_cast<size_t>(cap + 1) * row_bytes;
  uint8_t* block = d.recv[dst] + (static_cast<size_t>(step & 1u) * d.world + d.rank) * block_bytes;
  int32_t* meta = reinterpret_cast<int32_t*>(block + static_cast<size_t>(cap) * row_bytes);
  // the slots routed to peer dst in slot order: a CTA-wide stable compaction, 256 slots at a time
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
        dest = d.rank;
        local = per;
      } else if (head && dst == 0) {
        back_slot[s] = -1;
      }
      flag = dest == dst;
    }
    int total;
    const int pos = exl3::cta_scan_excl(flag, s_warp, &total);
    if (flag) {
      const int j = base + pos;
      if (j < cap) {
        s_tok[j] = s / topk;
        if (head) {
          meta[j] = local;
          back_slot[s] = dst * (cap + 1) + j;
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
  const size_t words = row_bytes / 16;
  for (int j = static_cast<int>(blockIdx.y); j < n; j += static_cast<int>(gridDim.y)) {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) + s_tok[j] * row_bytes);
    uint4* out = reinterpret_cast<uint4*>(block + static_cast<size_t>(j) * row_bytes);
    for (size_t w = threadIdx.x; w < words; w += blockDim.x) out[w] = src[w];
  }
  arrive_and_advance(d, step);
}

// After every rank's dispatch: recv (this parity) -> the caller's fixed buffer; CTA (q, 0) also unpacks block q's
// metadata into swiglu's indices (metadata rows -1) and scores (1).
__global__ void __launch_bounds__(256) epx_receive_kernel(const EpxDev* dp, uint8_t* __restrict__ xbuf,
                                                          int32_t* __restrict__ inds, float* __restrict__ scores,
                                                          uint32_t* err) {
  exl3::pdl_wait();  // the dispatch launch is complete: its stores are performed
  exl3::pdl_launch_dependents();
  const EpxDev& d = *dp;
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(d.step);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) publish(d, 0, step);  // this rank's dispatch is done
  wait_all(d, 0, step, err);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) exl3::trace_at(d.trace, step, 2);
  const int q = blockIdx.x, cap = d.cap;
  const size_t row_bytes = static_cast<size_t>(d.hidden) * d.esize;
  const size_t block_bytes = static_cast<size_t>(cap + 1) * row_bytes;
  const uint8_t* src = d.recv[d.rank] + (static_cast<size_t>(step & 1u) * d.world + q) * block_bytes;
  uint8_t* dst = xbuf + static_cast<size_t>(q) * block_bytes;
  const int32_t* meta = reinterpret_cast<const int32_t*>(src + static_cast<size_t>(cap) * row_bytes);
  if (blockIdx.y == 0) {
    for (int j = threadIdx.x; j <= cap; j += blockDim.x) {
      const size_t at = static_cast<size_t>(q) * (cap + 1) + j;
      inds[at] = j < cap ? meta[j] : -1;
      scores[at] = 1.0f;
    }
  }
  // the rows rank q sent are the block's first n (the dispatch compacts them; the rest carry metadata -1): only those
  // are copied here and returned after swiglu
  int n = 0;
  for (int j0 = 0; j0 < cap; j0 += static_cast<int>(blockDim.x)) {
    const int j = j0 + static_cast<int>(threadIdx.x);
    n += __syncthreads_count(j < cap && meta[j] >= 0);
  }
  if (blockIdx.y == 0 && threadIdx.x == 0) d.used[q] = n;
  const size_t words = static_cast<size_t>(n) * row_bytes / 16;  // the token rows (the metadata row stays)
  for (size_t w = static_cast<size_t>(blockIdx.y) * blockDim.x + threadIdx.x; w < words;
       w += static_cast<size_t>(gridDim.y) * blockDim.x)
    reinterpret_cast<uint4*>(dst)[w] = reinterpret_cast<const uint4*>(src)[w];
  __syncthreads();
  if (threadIdx.x == 0) exl3::trace_last(d.trace, step, 3);
}

// The swiglu output's block q (rows rank q sent) -> block `rank` of rank q's back (this parity).
__global__ void __launch_bounds__(256) epx_return_kernel(const EpxDev* dp, const float* __restrict__ ys) {
  exl3::pdl_wait();
  exl3::pdl_launch_dependents();
  const EpxDev& d = *dp;
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(d.step);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) exl3::trace_at(d.trace, step, 4);
  const int q = blockIdx.x, cap = d.cap;
  const size_t block_floats = static_cast<size_t>(cap + 1) * d.hidden;
  const float* src = ys + static_cast<size_t>(q) * block_floats;
  float* dst = d.back[q] + (static_cast<size_t>(step & 1u) * d.world + d.rank) * block_floats;
  const size_t words = static_cast<size_t>(d.used[q]) * d.hidden / 4;  // the rows rank q sent this step
  for (size_t w = static_cast<size_t>(blockIdx.y) * blockDim.x + threadIdx.x; w < words;
       w += static_cast<size_t>(gridDim.y) * blockDim.x)
    reinterpret_cast<float4*>(dst)[w] = reinterpret_cast<const float4*>(src)[w];
}

// After the return's copies (the previous launch, complete): release them to every rank, once.
__global__ void epx_publish_return_kernel(const EpxDev* dp) {
  exl3::pdl_wait();  // the return launch is complete: its stores are performed
  exl3::pdl_launch_dependents();
  const EpxDev& d = *dp;
  if (threadIdx.x == 0) {
    const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(d.step);
    exl3::trace_at(d.trace, step, 5);
    publish(d, 1, step);
  }
}

// After every rank's return: out[t] = sum_k score * back[slot(t, k)] in k order (f32), this parity.
__global__ void __launch_bounds__(128) epx_combine_kernel(const EpxDev* dp, const int32_t* __restrict__ back_slot,
                                                          const float* __restrict__ scores, int topk,
                                                          void* __restrict__ out, int32_t out_dtype, uint32_t* err) {
  exl3::pdl_wait();
  exl3::pdl_launch_dependents();
  const EpxDev& d = *dp;
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(d.step);
  wait_all(d, 1, step, err);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) exl3::trace_at(d.trace, step, 6);
  const float* back = d.back[d.rank] + static_cast<size_t>(step & 1u) * d.world * (d.cap + 1) * d.hidden;
  const int t = blockIdx.y;
  const size_t c = static_cast<size_t>(blockIdx.x) * 128 + threadIdx.x;
  float acc = 0.0f;
  for (int k = 0; k < topk; ++k) {
    const int pos = back_slot[static_cast<size_t>(t) * topk + k];
    if (pos >= 0) acc += scores[static_cast<size_t>(t) * topk + k] * back[static_cast<size_t>(pos) * d.hidden + c];
  }
  exl3::store_act(out, static_cast<size_t>(t) * d.hidden + c, acc, out_dtype);
  __syncthreads();
  if (threadIdx.x == 0) exl3::trace_last(d.trace, step, 7);
}

exl3_verdict refuse(int32_t code, const char* why) { return {code, why}; }
bool act_dtype(int32_t dt) { return dt == EXL3_F16 || dt == EXL3_BF16 || dt == EXL3_F32; }

}  // namespace

struct exl3_epx {
  int device = -1, world = 0, rank = 0, cap = 0, hidden = 0, dtype = 0, esize = 2;
  uint8_t* base = nullptr;
  size_t recv_bytes = 0, back_bytes = 0;
  uint8_t* peer[kMaxRanks] = {};
  EpxDev* dev = nullptr;
  uint64_t* trace = nullptr;  // the phase timeline ring (EXL3_TRACE=1 at create), or null
  bool connected = false;
};

namespace {
struct DevScope {
  int prev = -1;
  explicit DevScope(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
    else prev = -1;
  }
  ~DevScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

extern "C" {

exl3_verdict exl3_epx_create(int32_t device, int32_t world, int32_t rank, int32_t cap, int32_t hidden, int32_t dtype,
                             exl3_epx** out, uint8_t* ipc_handle) {
  if (!out || !ipc_handle) return refuse(EXL3_FAILED, "exl3_epx_create: bad arguments");
  *out = nullptr;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return refuse(EXL3_UNSUPPORTED, "exl3_epx_create: 1..8 ranks");
  if (cap < 1 || cap > kMaxCap || hidden < 128 || hidden % 128 != 0 || !act_dtype(dtype))
    return refuse(EXL3_UNSUPPORTED, "exl3_epx_create: capacity 1..2048, hidden a multiple of 128, an activation dtype");
  const int esize = dtype == EXL3_F32 ? 4 : 2;
  if (4 * cap > hidden * esize) return refuse(EXL3_UNSUPPORTED, "exl3_epx_create: the metadata does not fit one row");
  DevScope scope(device);
  exl3_epx* e = new (std::nothrow) exl3_epx;
  if (!e) return refuse(EXL3_FAILED, "exl3_epx_create: out of host memory");
  e->device = device, e->world = world, e->rank = rank, e->cap = cap, e->hidden = hidden, e->dtype = dtype;
  e->esize = esize;
  e->recv_bytes = 2u * world * static_cast<size_t>(cap + 1) * hidden * esize;
  e->back_bytes = 2u * world * static_cast<size_t>(cap + 1) * hidden * 4;
  const size_t total = e->recv_bytes + e->back_bytes + 256 + 256;
  bool ok = cudaMalloc(&e->base, total) == cudaSuccess;
  ok = ok && cudaMemset(e->base, 0, total) == cudaSuccess;
  cudaIpcMemHandle_t h;
  ok = ok && cudaIpcGetMemHandle(&h, e->base) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  if (!ok) {
    if (e->base) cudaFree(e->base);
    delete e;
    return refuse(EXL3_TOO_LARGE, "exl3_epx_create: exchange buffer allocation failed");
  }
  memcpy(ipc_handle, &h, 64);
  e->peer[rank] = e->base;
  e->trace = exl3::trace_alloc();
  *out = e;
  return {EXL3_OK, nullptr};
}

exl3_verdict exl3_epx_connect(exl3_epx* e, const uint8_t* ipc_handles) {
  if (!e || !ipc_handles || e->connected) return refuse(EXL3_FAILED, "exl3_epx_connect: bad arguments");
  DevScope scope(e->device);
  bool ok = true;
  for (int q = 0; q < e->world && ok; ++q) {
    if (q == e->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handles + 64 * q, 64);
    void* p = nullptr;
    ok = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    e->peer[q] = static_cast<uint8_t*>(p);
  }
  EpxDev host{};
  for (int q = 0; q < e->world; ++q) {
    host.recv[q] = e->peer[q];
    host.back[q] = e->peer[q] ? reinterpret_cast<float*>(e->peer[q] + e->recv_bytes) : nullptr;
    host.done[q] = e->peer[q] ? reinterpret_cast<uint32_t*>(e->peer[q] + e->recv_bytes + e->back_bytes) : nullptr;
  }
  host.step = reinterpret_cast<uint32_t*>(e->base + e->recv_bytes + e->back_bytes + 256);
  host.arrive = host.step + 4;
  host.used = reinterpret_cast<int32_t*>(host.step + 8);
  host.world = e->world, host.rank = e->rank, host.cap = e->cap, host.hidden = e->hidden, host.esize = e->esize;
  host.trace = e->trace;
  ok = ok && cudaMalloc(&e->dev, sizeof host) == cudaSuccess &&
       cudaMemcpy(e->dev, &host, sizeof host, cudaMemcpyHostToDevice) == cudaSuccess;
  if (!ok) return refuse(EXL3_FAILED, "exl3_epx_connect: opening a peer's exchange buffer failed");
  e->connected = true;
  return {EXL3_OK, nullptr};
}

void exl3_epx_destroy(exl3_epx* e) {
  if (!e) return;
  DevScope scope(e->device);
  cudaDeviceSynchronize();
  for (int q = 0; q < e->world; ++q)
    if (q != e->rank && e->peer[q]) cudaIpcCloseMemHandle(e->peer[q]);
  if (e->dev) cudaFree(e->dev);
  if (e->base) cudaFree(e->base);
  if (e->trace) cudaFree(e->trace);
  delete e;
}

exl3_verdict exl3_epx_dispatch(exl3_epx* e, const exl3_tensor* x, const exl3_tensor* inds, int32_t experts,
                               int32_t shared, void* stream, exl3_tensor* back_slot) {
  if (!e || !e->connected || !x || !inds || !back_slot) return refuse(EXL3_FAILED, "exl3_epx_dispatch: bad arguments");
  if (x->ndim != 2 || inds->ndim != 2 || back_slot->ndim != 2 || x->dtype != e->dtype || x->shape[1] != e->hidden)
    return refuse(EXL3_UNSUPPORTED, "exl3_epx_dispatch: x [T, D] in the exchange's dtype, inds and back_slot [T, K]");
  if ((inds->dtype != EXL3_I32 && inds->dtype != EXL3_U32) || back_slot->dtype != EXL3_I32 ||
      inds->shape[0] != x->shape[0] || back_slot->shape[0] != x->shape[0] || back_slot->shape[1] != inds->shape[1] ||
      inds->shape[1] < 1 || inds->shape[1] > 33)
    return refuse(EXL3_UNSUPPORTED, "exl3_epx_dispatch: inds i32/u32 and back_slot i32, both [T, K], K <= 33");
  if (experts < e->world || experts % e->world != 0) return refuse(EXL3_UNSUPPORTED, "exl3_epx_dispatch: the experts split evenly over the ranks");
  if (x->shape[0] == 0) return {EXL3_OK, nullptr};
  if (reinterpret_cast<uintptr_t>(x->data) % 16 != 0) return refuse(EXL3_UNSUPPORTED, "exl3_epx_dispatch: x on a 16-byte boundary");
  DevScope scope(e->device);
  uint32_t* err = exl3::device_error_ptr();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int copy = e->world >= 148 ? 1 : (148 + e->world - 1) / e->world;
  const cudaError_t le = exl3::launch_pdl_k(epx_dispatch_kernel, dim3(e->world, copy), dim3(256), st,
                                            static_cast<const EpxDev*>(e->dev), static_cast<const void*>(x->data),
                                            static_cast<int>(x->shape[0]), static_cast<int>(inds->shape[1]),
                                            static_cast<const void*>(inds->data), inds->dtype == EXL3_U32 ? 1 : 0,
                                            static_cast<int>(experts), shared ? 1 : 0,
                                            static_cast<int32_t*>(back_slot->data), err);
  return (err && le == cudaSuccess) ? exl3_verdict{EXL3_OK, nullptr}
                                                    : refuse(EXL3_FAILED, "exl3_epx_dispatch: launch failed");
}

exl3_verdict exl3_epx_receive(exl3_epx* e, void* stream, exl3_tensor* xbuf, exl3_tensor* inds, exl3_tensor* scores) {
  if (!e || !e->connected || !xbuf || !inds || !scores) return refuse(EXL3_FAILED, "exl3_epx_receive: bad arguments");
  const int64_t rows = static_cast<int64_t>(e->world) * (e->cap + 1);
  if (xbuf->ndim != 3 || xbuf->shape[0] != e->world || xbuf->shape[1] != e->cap + 1 || xbuf->shape[2] != e->hidden ||
      xbuf->dtype != e->dtype || inds->dtype != EXL3_I32 || scores->dtype != EXL3_F32)
    return refuse(EXL3_UNSUPPORTED, "exl3_epx_receive: xbuf [world, C + 1, D] in the exchange's dtype, inds i32, scores f32");
  int64_t ni = 1, ns = 1;
  for (int i = 0; i < inds->ndim; ++i) ni *= inds->shape[i];
  for (int i = 0; i < scores->ndim; ++i) ns *= scores->shape[i];
  if (ni != rows || ns != rows) return refuse(EXL3_UNSUPPORTED, "exl3_epx_receive: inds and scores hold world * (C + 1) rows");
  if (reinterpret_cast<uintptr_t>(xbuf->data) % 16 != 0) return refuse(EXL3_UNSUPPORTED, "exl3_epx_receive: xbuf on a 16-byte boundary");
  DevScope scope(e->device);
  uint32_t* err = exl3::device_error_ptr();
  const cudaError_t le = exl3::launch_pdl_k(epx_receive_kernel, dim3(e->world, 16), dim3(256),
                                            static_cast<cudaStream_t>(stream), static_cast<const EpxDev*>(e->dev),
                                            static_cast<uint8_t*>(xbuf->data), static_cast<int32_t*>(inds->data),
                                            static_cast<float*>(scores->data), err);
  return (err && le == cudaSuccess) ? exl3_verdict{EXL3_OK, nullptr}
                                                    : refuse(EXL3_FAILED, "exl3_epx_receive: launch failed");
}

exl3_verdict exl3_epx_return(exl3_epx* e, const exl3_tensor* ys, void* stream) {
  if (!e || !e->connected || !ys) return refuse(EXL3_FAILED, "exl3_epx_return: bad arguments");
  if (ys->ndim != 3 || ys->shape[0] != e->world || ys->shape[1] != e->cap + 1 || ys->shape[2] != e->hidden ||
      ys->dtype != EXL3_F32)
    return refuse(EXL3_UNSUPPORTED, "exl3_epx_return: ys is f32 [world, C + 1, D]");
  if (reinterpret_cast<uintptr_t>(ys->data) % 16 != 0) return refuse(EXL3_UNSUPPORTED, "exl3_epx_return: ys on a 16-byte boundary");
  DevScope scope(e->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t le = exl3::launch_pdl_k(epx_return_kernel, dim3(e->world, 16), dim3(256), st,
                                      static_cast<const EpxDev*>(e->dev), static_cast<const float*>(ys->data));
  if (le == cudaSuccess)
    le = exl3::launch_pdl_k(epx_publish_return_kernel, dim3(1), dim3(32), st, static_cast<const EpxDev*>(e->dev));
  return le == cudaSuccess ? exl3_verdict{EXL3_OK, nullptr}
                                           : refuse(EXL3_FAILED, "exl3_epx_return: launch failed");
}

exl3_verdict exl3_epx_combine(exl3_epx* e, const exl3_tensor* back_slot, const exl3_tensor* scores, void* stream,
                              exl3_tensor* out) {
  if (!e || !e->connected || !back_slot || !scores || !out) return refuse(EXL3_FAILED, "exl3_epx_combine: bad arguments");
  if (out->ndim != 2 || out->shape[1] != e->hidden || !act_dtype(out->dtype) || back_slot->ndim != 2 ||
      back_slot->dtype != EXL3_I32 || back_slot->shape[0] != out->shape[0] || scores->ndim != 2 ||
      scores->dtype != EXL3_F32 || scores->shape[0] != out->shape[0] || scores->shape[1] != back_slot->shape[1])
    return refuse(EXL3_UNSUPPORTED, "exl3_epx_combine: out [T, D], back_slot i32 and scores f32 [T, K]");
  if (out->shape[0] == 0) return {EXL3_OK, nullptr};
  DevScope scope(e->device);
  uint32_t* err = exl3::device_error_ptr();
  const cudaError_t le = exl3::launch_pdl_k(epx_combine_kernel, dim3(e->hidden / 128, static_cast<unsigned>(out->shape[0])),
                                            dim3(128), static_cast<cudaStream_t>(stream),
                                            static_cast<const EpxDev*>(e->dev),
                                            static_cast<const int32_t*>(back_slot->data),
                                            static_cast<const float*>(scores->data),
                                            static_cast<int>(back_slot->shape[1]), out->data,
                                            static_cast<int32_t>(out->dtype), err);
  return (err && le == cudaSuccess) ? exl3_verdict{EXL3_OK, nullptr}
                                                    : refuse(EXL3_FAILED, "exl3_epx_combine: launch failed");
}

exl3_verdict exl3_epx_trace(exl3_epx* e, uint64_t* out) {
  if (!e || !e->connected || !out) return refuse(EXL3_FAILED, "exl3_epx_trace: bad arguments");
  if (!e->trace) return refuse(EXL3_UNSUPPORTED, "exl3_epx_trace: the exchange was created without EXL3_TRACE=1");
  DevScope scope(e->device);
  const uint32_t* step = reinterpret_cast<const uint32_t*>(e->base + e->recv_bytes + e->back_bytes + 256);
  return exl3::trace_copy(e->trace, step, out) ? exl3_verdict{EXL3_OK, nullptr}
                                               : refuse(EXL3_FAILED, "exl3_epx_trace: copy failed");
}

}  // extern "C"
