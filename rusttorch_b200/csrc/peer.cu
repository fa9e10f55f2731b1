// peer.cu — the global sum's exchange between GPUs over peer memory.
//
// With one process per GPU, each rank holds an f64 partial of a sharded sum
// (rtc_sum_device of its shard) and every rank needs the total.  That is an
// 8-byte all-reduce, and its cost is latency alone: each rank writes its
// partial into a slot on every rank's GPU (stores through CUDA IPC mappings,
// over NVLink / NVSwitch), raises a generation number beside it, waits until
// every rank's slot on its own GPU carries the current generation, and adds
// the slots in rank order (so every rank gets the same bits).  One kernel of
// one thread; no NCCL call, no host round trip.
//
// Slot array layout on every rank: [2][world] {value, generation}, indexed by
// the generation's parity.  A rank cannot run two generations ahead of
// another (its call g + 1 needs every rank's g + 1 value, written only after
// that rank has finished reading generation g), so the slots of generation
// g + 1 never overwrite values a slower rank still has to read.
//
// Every wait is bounded: after the limit the kernel raises the library's
// wait-timeout flag (reported by rtc_synchronize), writes NaN and returns, so
// a rank that never arrives costs the others an error, not a hung GPU.
#include "../../include/rusttorch_cuda.h"
#include "rt_abi_util.h"
#include "rt_internal.h"
#include "rt_tma.cuh"

#include <cmath>
#include <cstring>

using namespace rt;

namespace {

struct __align__(16) PeerSlot {
  double value;
  unsigned long long gen;
};

struct PeerPtrs {
  PeerSlot* p[RTC_PEER_MAX_RANKS];
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void peer_allreduce_kernel(const double* local, PeerPtrs slots, int world, int rank,
                                      unsigned long long gen, double* out, int* err,
                                      unsigned long long limit_ns) {
  const int par = (int)(gen & 1ull);
  const double v = *local;
  // my value into my slot on every rank, then (after a system-scope fence,
  // so no rank sees the generation before the value) the generation
  for (int p = 0; p < world; p++) {
    volatile PeerSlot* dst = slots.p[p] + par * world + rank;
    dst->value = v;
  }
  __threadfence_system();
  for (int p = 0; p < world; p++) {
    volatile PeerSlot* dst = slots.p[p] + par * world + rank;
    dst->gen = gen;
  }
  // every rank's value in my own slots
  volatile PeerSlot* mine = slots.p[rank] + par * world;
  const unsigned long long t0 = global_ns();
  for (int q = 0; q < world; q++) {
    while (mine[q].gen != gen) {
      if (global_ns() - t0 > limit_ns) {
        atomicExch(err, 1);
        *out = __longlong_as_double(0x7ff8000000000000ll);
        return;
      }
      __nanosleep(64);
    }
  }
  __threadfence_system();
  double s = 0.0;
  for (int q = 0; q < world; q++) s = s + mine[q].value;   // rank order
  *out = s;
}

}  // namespace

extern "C" rtc_result rtc_ipc_handle(int device, const void* dev_ptr, void* handle_out) {
  RTC_OP_RANGE();
  if (!dev_ptr || !handle_out) return invalid_argument("pointer", "must not be null");
  DeviceScope scope(device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return backend_error("cudaIpcGetMemHandle", e);
  static_assert(sizeof(h) == RTC_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof h);
  return ok();
}

extern "C" rtc_result rtc_ipc_open(int device, const void* handle, void** dev_ptr_out) {
  RTC_OP_RANGE();
  if (!handle || !dev_ptr_out) return invalid_argument("pointer", "must not be null");
  DeviceScope scope(device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return backend_error("cudaIpcOpenMemHandle", e);
  return ok();
}

extern "C" rtc_result rtc_ipc_close(int device, void* dev_ptr) {
  RTC_OP_RANGE();
  if (!dev_ptr) return invalid_argument("dev_ptr", "must not be null");
  DeviceScope scope(device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return backend_error("cudaIpcCloseMemHandle", e);
  return ok();
}

extern "C" size_t rtc_peer_slot_bytes(int world) {
  return world < 1 ? 0 : 2 * (size_t)world * sizeof(PeerSlot);
}

extern "C" rtc_result rtc_peer_allreduce_sum_f64(int device, const double* local,
                                                 void* const* slots, int world, int rank,
                                                 unsigned long long generation, double* out) {
  RTC_OP_RANGE();
  if (!local || !slots || !out) return invalid_argument("pointer", "must not be null");
  if (world < 1 || world > RTC_PEER_MAX_RANKS)
    return invalid_argument("world", "must be in 1.." + std::to_string(RTC_PEER_MAX_RANKS));
  if (rank < 0 || rank >= world) return invalid_argument("rank", "must be in 0..world-1");
  if (generation == 0) return invalid_argument("generation", "must be at least 1");
  PeerPtrs ptrs{};
  for (int p = 0; p < world; p++) {
    if (!slots[p]) return invalid_argument("slots", "every rank's slot array is needed");
    if (reinterpret_cast<uintptr_t>(slots[p]) % alignof(PeerSlot))
      return invalid_argument("slots", "must be 16-byte aligned");
    ptrs.p[p] = static_cast<PeerSlot*>(slots[p]);
  }
  DeviceScope scope(device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  int* err = wait_timeout_flag(device);
  if (!err) return backend_error("wait-timeout flag", cudaErrorUnknown);
  const unsigned long long limit_ns = 2000000000ull;   // 2 s
  peer_allreduce_kernel<<<1, 1, 0, thread_stream()>>>(local, ptrs, world, rank, generation, out,
                                                      err, limit_ns);
  return launched(cudaGetLastError(), "peer all-reduce");
}
