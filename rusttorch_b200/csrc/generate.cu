// generate.cu — seeded synthetic inputs on the device.
//
// Element i of a stream is a pure function of (seed, offset + i): splitmix64
// of the counter, then
//   uniform: lo + (hi - lo) * u,  u = (z >> 40) * 2^-24 in [0, 1)
//   normal : mean + std * sqrt(-2 ln u1) cos(2 pi u2), two 26-bit uniforms
//            taken from the same 64-bit draw, evaluated in double.
// The uniform stream is bit-identical to the host generator the tests use;
// the normal stream can differ in the last bit of a double only where CUDA's
// and glibc's log/cos differ, which almost never survives the cast to float.
#include "rt_internal.h"

#include <algorithm>

namespace rt {

namespace {

__device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(kThreads)
fill_kernel(float* out, size_t n, uint64_t seed, uint64_t offset, float a, float b, int normal) {
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    const uint64_t z = splitmix64_at(seed, offset + i);
    float v;
    if (!normal) {
      const double u = (double)(z >> 40) * 0x1p-24;
      v = (float)((double)a + ((double)b - (double)a) * u);
    } else {
      const double u1 = ((double)(z >> 38) + 0.5) * 0x1p-26;
      const double u2 = (double)((z >> 12) & 0x3FFFFFFULL) * 0x1p-26;
      const double r = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
      v = (float)((double)a + (double)b * r);
    }
    out[i] = v;
  }
}

}  // namespace

cudaError_t launch_fill(float* out, size_t n, uint64_t seed, uint64_t offset, float a, float b,
                        int normal, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned grid = (unsigned)std::max<size_t>(
      1, std::min<size_t>((n + kThreads - 1) / kThreads, (size_t)sm_count(dev) * 16));
  fill_kernel<<<grid, kThreads, 0, s>>>(out, n, seed, offset, a, b, normal);
  return cudaGetLastError();
}

}  // namespace rt
