// tma_util.cu — host side of the TMA kernels: tensor-map encoding through
// the driver entry point (no link-time dependency on libcuda) and the
// device flag that bounded waits raise.
#include "rt_internal.h"
#include "rt_tma.cuh"

#include <cudaTypedefs.h>

#include <mutex>
#include <vector>

namespace rt {
namespace {

__device__ int g_wait_timeouts;

std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
bool g_encode_looked_up = false;
std::vector<int*> g_flag;

}  // namespace

bool encode_tensor_map_f32(CUtensorMap* tm, const void* base, int rank, const uint64_t* dims,
                           const uint64_t* strides_bytes, const uint32_t* box) {
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_encode_looked_up) {
      g_encode_looked_up = true;
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
              cudaSuccess &&
          q == cudaDriverEntryPointSuccess)
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  if (!g_encode) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; i++) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  const CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank,
                              const_cast<void*>(base), d, st, b, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int* wait_timeout_flag(int device) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (device < 0) return nullptr;
  if ((size_t)device >= g_flag.size()) g_flag.resize(device + 1, nullptr);
  if (!g_flag[device]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_wait_timeouts) != cudaSuccess) return nullptr;
    g_flag[device] = static_cast<int*>(p);
  }
  return g_flag[device];
}

int take_wait_timeouts(int device) {
  if (!wait_timeout_flag(device)) return 0;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(int)) != cudaSuccess) return 0;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(int));
  }
  return v;
}

namespace {

// One thread waits (50 ms at most) on an mbarrier that nothing arrives on,
// exactly as a consumer whose tile never lands would, and takes the same
// exit: it raises the device flag and returns.
__global__ void bounded_wait_probe_kernel(int* err) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  mbar_fence_init();
  if (!mbar_wait_for(&bar, 0, 50ull * 1000 * 1000)) atomicExch(err, 1);
}

}  // namespace

cudaError_t launch_bounded_wait_probe(int device, cudaStream_t s) {
  int* err = wait_timeout_flag(device);
  if (!err) return cudaErrorInvalidValue;
  bounded_wait_probe_kernel<<<1, 1, 0, s>>>(err);
  return cudaGetLastError();
}

}  // namespace rt
