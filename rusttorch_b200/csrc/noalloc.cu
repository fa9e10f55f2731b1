// noalloc.cu — rtc_sum_device_noalloc: the device-side sum without any
// device-memory allocation.
//
// rtc_sum_device takes the per-block partial sums of its two-kernel
// reduction from the stream-ordered pool (cudaMallocAsync).  Some callers may
// not allocate at all: a host application whose framework allocator has
// already reserved the GPU's memory, a latency-critical loop that must not
// risk an allocation's synchronisation or its out-of-memory failure, or a
// plugin whose host forbids it by policy.  For them the partials live in
// the fixed array below, part of the library's device image, which every GPU
// that loads the library keeps until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents; nothing in it has to start at zero, because each call writes
// every partial it later reads.  Calls whose work overlaps on the GPU (two
// streams, or two threads) race on it: issue them in one stream, or use
// rtc_sum_device.
#include "rt_abi_util.h"

#include <mutex>
#include <vector>

namespace rt {
namespace {

// Room for this many per-block partials.  The reduction launches at most
// eight blocks per SM (stats_max_parts), so 2048 covers any GPU with up to
// 256 SMs; B200 uses 1184.
constexpr int kNoAllocMaxParts = 2048;

static __device__ __align__(256) StatsPart g_noalloc_parts[kNoAllocMaxParts];

// Device address of g_noalloc_parts per device.  In host code the symbol's
// name is only a host-side stand-in, so the address is looked up once per
// device with that device current, on the first call there, and kept.  A
// device reset (cudaDeviceReset, or the primary context reset by the host
// application) invalidates it: the library must not be used on a device
// after that device has been reset.
std::mutex g_mu;
std::vector<StatsPart*> g_addr;

cudaError_t scratch_address(int device, StatsPart** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if ((size_t)device >= g_addr.size()) g_addr.resize(device + 1, nullptr);
  if (!g_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_parts);
    if (e != cudaSuccess) return e;
    g_addr[device] = static_cast<StatsPart*>(p);
  }
  *out = g_addr[device];
  return cudaSuccess;
}

}  // namespace
}  // namespace rt

using namespace rt;

extern "C" rtc_result rtc_sum_device_noalloc(const rtc_tensor* x, double* device_out) {
  RTC_OP_RANGE();
  TRY(check_desc(x, "input"));
  if (!device_out) return invalid_argument("device_out", "must not be null");
  TRY(require_f32(x, "sum"));
  if (x->device < 0)
    return invalid_argument("device", "rtc_sum_device_noalloc needs a device tensor");
  DeviceScope scope(x->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaStream_t s = thread_stream();
  if (x->numel == 0) return launched(cudaMemsetAsync(device_out, 0, sizeof(double), s), "sum");
  const int nparts = stats_num_parts(x->device, x->numel);
  if (nparts > kNoAllocMaxParts)
    return invalid_argument("input", "needs " + std::to_string(nparts) +
                                         " partial sums; rtc_sum_device_noalloc holds at most " +
                                         std::to_string(kNoAllocMaxParts) +
                                         " (use rtc_sum_device)");
  StatsPart* parts = nullptr;
  cudaError_t e = scratch_address(x->device, &parts);
  if (e != cudaSuccess) return backend_error("cudaGetSymbolAddress", e);
  return launched(launch_stats(cf(x), x->numel, parts, nparts, nullptr, s, device_out), "sum");
}
