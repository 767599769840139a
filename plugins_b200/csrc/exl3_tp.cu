// exl3_tp.cu -- column-parallel linears with the all-gather fused into the decode GEMV (one process per GPU).
//
// Every rank holds an exchange buffer in its own HBM, mapped into the other ranks with CUDA IPC:
//   y region    [2 parities][slots][slot_bytes]  gathered outputs, one slot per column-parallel linear of a step;
//   done        [world] u32                      per rank: the last step whose columns it has published here;
//   meta        [slots][4] u32                   per slot: its gathered bytes (written by the GEMV);
//   step        u32                              this rank's step counter.
// A step is exl3_tp_begin (step += 1 on the device), the column-parallel GEMVs (exl3_matmul_tp: each cluster leader
// stores its 128 output columns into the slot of EVERY rank over NVLink, plain stores), and exl3_tp_gather: one
// thread fences at system scope and releases done[rank] = step on every rank (the step's stores of this rank, all
// launches at once), then the slots' CTAs wait (acquire) until every rank's done holds the step and copy the slots
// out.  One system-scope release per step, not per launch: measured, a release per GEMV launch cost more than the
// launch.  Parity = step & 1: a rank starts step s+1 only after its gather saw every rank publish step s, and a rank
// publishes step s+1 only after its own step-s gather finished, so the two copies of the slots never race.  The done
// words only grow, so nothing is reset between steps and a CUDA graph of whole steps replays as is.  Every wait is
// bounded (one second): a missing peer sets EXL3_ERR_TP_TIMEOUT in the device error word and the kernel returns.
#include <cuda_runtime.h>

#include <cstring>
#include <new>

#include "../../include/exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_internal.h"

struct exl3_tp {
  int device = -1, world = 0, rank = 0, slots = 0, max_cb = 0;
  int64_t slot_bytes = 0;
  uint8_t* base = nullptr;  // local exchange buffer
  size_t y_bytes = 0, flag_bytes = 0;
  uint8_t* peer[exl3::kMaxTpRanks] = {};  // every rank's buffer as mapped here (peer[rank] = base)
  exl3::TpDev* dev = nullptr;             // device copy of the table
  uint64_t* trace = nullptr;              // the phase timeline ring (EXL3_TRACE=1 at create), or null
  bool connected = false;
};

namespace {

constexpr size_t kMetaBytes = 16;  // per slot

exl3_verdict refuse(int32_t code, const char* why) { return {code, why}; }

uint32_t* meta_of(uint8_t* base, size_t y_bytes, size_t flag_bytes) {
  return reinterpret_cast<uint32_t*>(base + y_bytes + flag_bytes);
}

__global__ void tp_begin_kernel(uint32_t* step, uint64_t* trace) {
  exl3::pdl_wait();  // the previous step's gather has read the step word
  exl3::pdl_launch_dependents();
  if (threadIdx.x == 0) {
    const uint32_t s = *step + 1u;
    *step = s;
    exl3::trace_at(trace, s, 0);
  }
}

// This rank's columns of the step, published to every rank: a system-scope fence (the GEMVs before this kernel in
// stream order wrote them), then done[rank] = step on every rank.
__global__ void tp_publish_kernel(const exl3::TpDev* tp) {
  exl3::pdl_wait();  // the step's GEMVs are complete: their stores are performed
  exl3::pdl_launch_dependents();
  if (threadIdx.x != 0) return;
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(tp->step);
  exl3::trace_at(tp->trace, step, 1);
  asm volatile("fence.sc.sys;" ::: "memory");
  for (int q = 0; q < tp->world; ++q) {
    uint32_t* f = tp->flag[q] + tp->rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(step) : "memory");
  }
}

// One CTA per slot: wait (bounded) until every rank published the step, then copy the slot to out.
__global__ void __launch_bounds__(256) tp_gather_kernel(const uint8_t* __restrict__ y, const uint32_t* done,
                                                        const uint32_t* meta, const uint32_t* step_p, int world,
                                                        int slots, int64_t slot_bytes, int slot0,
                                                        uint8_t* __restrict__ out, uint32_t* err, uint64_t* trace) {
  __shared__ int s_fail;
  exl3::pdl_wait();
  exl3::pdl_launch_dependents();
  const int slot = slot0 + static_cast<int>(blockIdx.x);
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(step_p);
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if (threadIdx.x < static_cast<uint32_t>(world)) {
    const uint32_t* f = done + threadIdx.x;
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (static_cast<int32_t>(v - step) < 0) {
      const uint64_t t0 = exl3::global_timer_ns();
      while (true) {
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if (static_cast<int32_t>(v - step) >= 0) break;
        if (exl3::global_timer_ns() - t0 > 1000000000ull) {
          s_fail = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (s_fail && threadIdx.x == 0) atomicOr(err, exl3::kErrTpTimeout);
  if (blockIdx.x == 0 && threadIdx.x == 0) exl3::trace_at(trace, step, 2);
  const uint32_t nbytes = meta[slot * 4 + 1];
  const uint8_t* src = y + (static_cast<size_t>(step & 1u) * slots + slot) * slot_bytes;
  uint8_t* dst = out + static_cast<size_t>(blockIdx.x) * slot_bytes;
  const uint32_t n16 = nbytes / 16u;
  for (uint32_t i = threadIdx.x; i < n16; i += blockDim.x)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  for (uint32_t i = n16 * 16u + threadIdx.x; i < nbytes; i += blockDim.x) dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) exl3::trace_last(trace, step, 3);
}

}  // namespace

namespace exl3 {
const TpDev* tp_device(const exl3_tp* tp) { return tp && tp->connected ? tp->dev : nullptr; }
int tp_device_index(const exl3_tp* tp) { return tp ? tp->device : -1; }
int tp_max_cb(const exl3_tp* tp) { return tp ? tp->max_cb : 0; }
int tp_slots(const exl3_tp* tp) { return tp ? tp->slots : 0; }
int64_t tp_slot_bytes(const exl3_tp* tp) { return tp ? tp->slot_bytes : 0; }
}  // namespace exl3

extern "C" {

exl3_verdict exl3_tp_create(int32_t device, int32_t world, int32_t rank, int32_t slots, int64_t slot_bytes,
                            int32_t max_cb, exl3_tp** out, uint8_t* ipc_handle) {
  if (!out || !ipc_handle) return refuse(EXL3_FAILED, "exl3_tp_create: bad arguments");
  *out = nullptr;
  if (world < 1 || world > exl3::kMaxTpRanks || rank < 0 || rank >= world)
    return refuse(EXL3_UNSUPPORTED, "exl3_tp_create: 1..8 ranks");
  if (slots < 1 || slots > 4096 || slot_bytes < 16 || slot_bytes % 16 != 0 || max_cb < 1 || max_cb > 65536)
    return refuse(EXL3_UNSUPPORTED, "exl3_tp_create: slots 1..4096, slot_bytes a multiple of 16, max_cb 1..65536");
  int prev = -1;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return refuse(EXL3_FAILED, "exl3_tp_create: bad device");
  exl3_tp* tp = new (std::nothrow) exl3_tp;
  if (!tp) return refuse(EXL3_FAILED, "exl3_tp_create: out of host memory");
  tp->device = device;
  tp->world = world;
  tp->rank = rank;
  tp->slots = slots;
  tp->max_cb = max_cb;
  tp->slot_bytes = slot_bytes;
  tp->trace = exl3::trace_alloc();
  tp->y_bytes = 2u * static_cast<size_t>(slots) * slot_bytes;
  tp->flag_bytes = 256;  // done[world]
  const size_t total = tp->y_bytes + tp->flag_bytes + static_cast<size_t>(slots) * kMetaBytes + 256;
  bool ok = cudaMalloc(&tp->base, total) == cudaSuccess;
  ok = ok && cudaMemset(tp->base + tp->y_bytes, 0, total - tp->y_bytes) == cudaSuccess;
  cudaIpcMemHandle_t h;
  ok = ok && cudaIpcGetMemHandle(&h, tp->base) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  if (prev >= 0) cudaSetDevice(prev);
  if (!ok) {
    if (tp->base) cudaFree(tp->base);
    if (tp->trace) cudaFree(tp->trace);
    delete tp;
    return refuse(EXL3_TOO_LARGE, "exl3_tp_create: exchange buffer allocation failed");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handles");
  memcpy(ipc_handle, &h, 64);
  tp->peer[rank] = tp->base;
  *out = tp;
  return {EXL3_OK, nullptr};
}

exl3_verdict exl3_tp_connect(exl3_tp* tp, const uint8_t* ipc_handles) {
  if (!tp || !ipc_handles || tp->connected) return refuse(EXL3_FAILED, "exl3_tp_connect: bad arguments");
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(tp->device);
  bool ok = true;
  for (int q = 0; q < tp->world && ok; ++q) {
    if (q == tp->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handles + 64 * q, 64);
    void* p = nullptr;
    ok = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    tp->peer[q] = static_cast<uint8_t*>(p);
  }
  exl3::TpDev host{};
  for (int q = 0; q < tp->world; ++q) {
    host.y[q] = tp->peer[q];
    host.flag[q] = tp->peer[q] ? reinterpret_cast<uint32_t*>(tp->peer[q] + tp->y_bytes) : nullptr;
  }
  host.meta = meta_of(tp->base, tp->y_bytes, tp->flag_bytes);
  host.step = reinterpret_cast<uint32_t*>(tp->base + tp->y_bytes + tp->flag_bytes +
                                          static_cast<size_t>(tp->slots) * kMetaBytes);
  host.world = tp->world;
  host.rank = tp->rank;
  host.slots = tp->slots;
  host.max_cb = tp->max_cb;
  host.slot_bytes = tp->slot_bytes;
  host.trace = tp->trace;
  ok = ok && cudaMalloc(&tp->dev, sizeof host) == cudaSuccess &&
       cudaMemcpy(tp->dev, &host, sizeof host, cudaMemcpyHostToDevice) == cudaSuccess;
  if (prev >= 0) cudaSetDevice(prev);
  if (!ok) return refuse(EXL3_FAILED, "exl3_tp_connect: opening a peer's exchange buffer failed");
  tp->connected = true;
  return {EXL3_OK, nullptr};
}

void exl3_tp_destroy(exl3_tp* tp) {
  if (!tp) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(tp->device);
  cudaDeviceSynchronize();
  for (int q = 0; q < tp->world; ++q)
    if (q != tp->rank && tp->peer[q]) cudaIpcCloseMemHandle(tp->peer[q]);
  if (tp->dev) cudaFree(tp->dev);
  if (tp->base) cudaFree(tp->base);
  if (tp->trace) cudaFree(tp->trace);
  if (prev >= 0) cudaSetDevice(prev);
  delete tp;
}

exl3_verdict exl3_tp_begin(exl3_tp* tp, void* stream) {
  if (!tp || !tp->connected) return refuse(EXL3_FAILED, "exl3_tp_begin: not a connected exchange");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != tp->device) cudaSetDevice(tp->device);
  uint32_t* step = reinterpret_cast<uint32_t*>(tp->base + tp->y_bytes + tp->flag_bytes +
                                               static_cast<size_t>(tp->slots) * kMetaBytes);
  const bool ok = exl3::launch_pdl_k(tp_begin_kernel, dim3(1), dim3(32), static_cast<cudaStream_t>(stream), step,
                                     tp->trace) == cudaSuccess;
  if (prev >= 0 && prev != tp->device) cudaSetDevice(prev);
  return ok ? exl3_verdict{EXL3_OK, nullptr} : refuse(EXL3_FAILED, "exl3_tp_begin: launch failed");
}

exl3_verdict exl3_tp_gather(exl3_tp* tp, int32_t slot0, int32_t nslots, void* stream, void* out) {
  if (!tp || !tp->connected || !out) return refuse(EXL3_FAILED, "exl3_tp_gather: bad arguments");
  if (slot0 < 0 || nslots < 1 || slot0 + nslots > tp->slots) return refuse(EXL3_UNSUPPORTED, "exl3_tp_gather: slot range");
  if (reinterpret_cast<uintptr_t>(out) % 16 != 0) return refuse(EXL3_UNSUPPORTED, "exl3_tp_gather: out on a 16-byte boundary");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != tp->device) cudaSetDevice(tp->device);
  uint32_t* err = exl3::device_error_ptr();
  const uint32_t* done = reinterpret_cast<const uint32_t*>(tp->base + tp->y_bytes);
  const uint32_t* meta = meta_of(tp->base, tp->y_bytes, tp->flag_bytes);
  const uint32_t* step = reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(meta) +
                                                           static_cast<size_t>(tp->slots) * kMetaBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool ok = exl3::launch_pdl_k(tp_publish_kernel, dim3(1), dim3(32), st,
                               static_cast<const exl3::TpDev*>(tp->dev)) == cudaSuccess;
  ok = ok && err &&
       exl3::launch_pdl_k(tp_gather_kernel, dim3(nslots), dim3(256), st, static_cast<const uint8_t*>(tp->base), done,
                          meta, step, tp->world, tp->slots, tp->slot_bytes, slot0, static_cast<uint8_t*>(out), err,
                          tp->trace) == cudaSuccess;
  if (prev >= 0 && prev != tp->device) cudaSetDevice(prev);
  return ok ? exl3_verdict{EXL3_OK, nullptr} : refuse(EXL3_FAILED, "exl3_tp_gather: launch failed");
}

exl3_verdict exl3_tp_trace(exl3_tp* tp, uint64_t* out) {
  if (!tp || !tp->connected || !out) return refuse(EXL3_FAILED, "exl3_tp_trace: bad arguments");
  if (!tp->trace) return refuse(EXL3_UNSUPPORTED, "exl3_tp_trace: the exchange was created without EXL3_TRACE=1");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != tp->device) cudaSetDevice(tp->device);
  const uint32_t* step = reinterpret_cast<const uint32_t*>(tp->base + tp->y_bytes + tp->flag_bytes +
                                                           static_cast<size_t>(tp->slots) * kMetaBytes);
  const bool ok = exl3::trace_copy(tp->trace, step, out);
  if (prev >= 0 && prev != tp->device) cudaSetDevice(prev);
  return ok ? exl3_verdict{EXL3_OK, nullptr} : refuse(EXL3_FAILED, "exl3_tp_trace: copy failed");
}

}  // extern "C"
