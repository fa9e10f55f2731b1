// probe.cu — bandwidth probes (diagnostics; no counterpart in the reference).
//
// They measure what the streaming kernels of this library are measured
// against: how fast one B200 can READ HBM (the global and per-lane
// reductions only read), in two forms, beside a plain copy and the sizing
// variants of the small fused add->mul_scalar map.
//
//  mode 0  read, 16-byte loads (LDG.128) with U loads in flight per thread;
//          p0 = threads per block, p1 = U (4, 8 or 16), p2 = blocks per SM;
//          layout: grid-stride.
//  mode 1  the same with one contiguous range per block.
//  mode 2  read through a cp.async.bulk ring (global -> shared, no
//          multicast): one thread per CTA keeps p1 slots of p0 bytes in
//          flight; p2 CTAs per SM; nothing else touches the data.
//  mode 3  the same ring with all 256 threads folding every slot out of
//          shared memory (f32 adds), as a reduction consumer would.
//  mode 4  copy with 16-byte loads and stores (src -> dst), p0/p1/p2 as mode 0.
//  mode 5  add->mul_scalar map (the product's map kernel template) with
//          U = p1 and p2 blocks per SM (p2 = 0: one wave of resident blocks,
//          p2 < 0: enough blocks to cover the tensor once) over
//          a = src, b = src + bytes/2 (bytes/2 each), out = dst.
//  mode 6  the same map with one contiguous balanced range per block,
//          p2 blocks per SM (0: one wave).
//  mode 8  the last-axis sum of src viewed as [bytes/4/p0, p0] (cfg3's
//          sum_dim(1) for p0 = 16384) into dst by the four-lanes-per-warp
//          kernel with p1 warps per CTA.
//  mode 9  the dim-0 sum of src viewed as [bytes/4/p0, p0] (cfg4's
//          broadcast_add_backward onto [1, C] for p0 = 4096) into dst by the
//          TMA strip kernel with p1 % 1000 columns per CTA, p2 / 100 rows per
//          tile and p2 % 100 ring stages (p1 >= 1000: the kernel that takes
//          the width at run time even for 16 and 32 columns).
//  mode 7  the global sum/max/min kernel (reduce.cu) in the shape p0
//          threads, p1 loads in flight per thread, p2 blocks per SM (0: as
//          many as stay resident), over bytes/4 floats of src; p2 >= 100:
//          the grid-stride pipelined kernel with p2 - 100 blocks per SM.
//
// Every mbarrier wait is bounded (rt_tma.cuh); a ring that gives up raises
// the library's wait-timeout flag (reported by rtc_synchronize), waits
// (bounded again) for its own copies in flight and returns.
#include "../../include/rusttorch_cuda.h"
#include "rt_abi_util.h"
#include "rt_internal.h"
#include "rt_map.cuh"
#include "rt_ops.cuh"
#include "rt_tma.cuh"

#include <algorithm>

namespace rt {
namespace {

__device__ float g_probe_sink[4];   // written only if a fold hits 1234.5
constexpr int kProbeParts = 4096;
__device__ StatsPart g_probe_parts[kProbeParts];
__device__ double g_probe_sum;

template <int U>
__global__ void probe_read_kernel(const float4* x, size_t n4, int contiguous, float* sink) {
  float acc = 0.0f;
  size_t i, stride, end;
  if (contiguous) {
    const size_t per = (n4 + gridDim.x - 1) / gridDim.x;
    i = (size_t)blockIdx.x * per + threadIdx.x;
    end = min(n4, (size_t)(blockIdx.x + 1) * per);
    stride = blockDim.x;
  } else {
    i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    stride = (size_t)gridDim.x * blockDim.x;
    end = n4;
  }
  for (; i + (U - 1) * stride < end; i += U * stride) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++) v[u] = __ldcs(x + i + u * stride);
#pragma unroll
    for (int u = 0; u < U; u++) acc += (v[u].x + v[u].y) + (v[u].z + v[u].w);
  }
  for (; i < end; i += stride) {
    const float4 v = __ldcs(x + i);
    acc += (v.x + v.y) + (v.z + v.w);
  }
  if (acc == 1234.5f) sink[0] = acc;   // keeps the loads alive
}

template <int U>
__global__ void probe_copy_kernel(const float4* x, float4* y, size_t n4) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (U - 1) * stride < n4; i += U * stride) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++) v[u] = __ldcs(x + i + u * stride);
#pragma unroll
    for (int u = 0; u < U; u++) __stcs(y + i + u * stride, v[u]);
  }
  for (; i < n4; i += stride) __stcs(y + i, __ldcs(x + i));
}

constexpr int kRingThreads = 256;
constexpr int kMaxSlots = 16;

// CTA b reads chunks [c0, c1) of `chunk` bytes each through `slots` ring
// slots.  With FOLD every thread sums the slot's floats out of shared memory
// before the slot is refilled.
template <bool FOLD>
__global__ void __launch_bounds__(kRingThreads)
probe_ring_kernel(const char* src, size_t nchunks, unsigned chunk, int slots, float* sink,
                  int* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxSlots];
  const size_t c0 = nchunks * blockIdx.x / gridDim.x;
  const size_t c1 = nchunks * (blockIdx.x + 1) / gridDim.x;
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < slots; s++) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (!FOLD && tid != 0) return;
  if (tid == 0) {
    for (int s = 0; s < slots && c0 + s < c1; s++) {
      mbar_arrive_expect_tx(&full[s], chunk);
      bulk_load(smem + (size_t)s * chunk, src + (c0 + s) * chunk, chunk, &full[s]);
    }
  }
  float acc = 0.0f;
  size_t c = c0;
  bool gave_up = false;
  for (; c < c1; c++) {
    const size_t k = c - c0;
    const int s = (int)(k % slots);
    const unsigned parity = (unsigned)((k / slots) & 1);
    bool ok = true;
    if (FOLD || tid == 0) ok = mbar_wait(&full[s], parity);
    if (FOLD) {
      gave_up = __syncthreads_or(!ok);
    } else {
      gave_up = !ok;
    }
    if (gave_up) break;
    if (FOLD) {
      const float4* q = reinterpret_cast<const float4*>(smem + (size_t)s * chunk);
      for (unsigned j = tid; j < chunk / 16; j += kRingThreads) {
        const float4 v = q[j];
        acc += (v.x + v.y) + (v.z + v.w);
      }
      __syncthreads();
    }
    if (tid == 0 && c + slots < c1) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&full[s], chunk);
      bulk_load(smem + (size_t)s * chunk, src + (c + slots) * chunk, chunk, &full[s]);
    }
  }
  if (gave_up && tid == 0) {
    atomicExch(err, 1);
    // Wait (bounded) for every copy this CTA still has in flight.
    for (size_t d = c; d < c1 && d < c + slots; d++) {
      const size_t k = d - c0;
      mbar_wait(&full[k % slots], (unsigned)((k / slots) & 1));
    }
  }
  if (acc == 1234.5f) sink[0] = acc;
}

// The product's map (rt_map.cuh) with one contiguous, balanced range of
// float4s per block instead of a grid stride.
template <class F, int U>
__global__ void __launch_bounds__(kThreads)
map_chunk_kernel(const float* a, const float* b, float* out, size_t n4, F f) {
  const size_t lo = n4 * blockIdx.x / gridDim.x, hi = n4 * (blockIdx.x + 1) / gridDim.x;
  for (size_t base = lo + threadIdx.x; base < hi; base += (size_t)kThreads * U) {
    float4 va[U], vb[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < hi) {
        va[u] = ld4(a + 4 * j);
        vb[u] = ld4(b + 4 * j);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < hi) st4(out + 4 * j, map4(f, va[u], vb[u]));
    }
  }
}

int resident_blocks(const void* kernel, int threads, size_t smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess)
    return 1;
  return n < 1 ? 1 : n;
}

template <int U>
cudaError_t launch_map_variant(int mode, int bps, const float* a, const float* b, float* out,
                               size_t n, cudaStream_t s) {
  const OpAddMulScalar op{0.5f};
  const int sms = sm_count(current_device());
  const size_t n4 = n >> 2;
  if (mode == 5) {
    auto k = map_vec_kernel<OpAddMulScalar, 2, U>;
    size_t grid;
    if (bps > 0) grid = (size_t)bps * sms;
    else if (bps == 0) grid = (size_t)resident_blocks((const void*)k, kThreads, 0) * sms;
    else grid = (n4 + (size_t)kThreads * U - 1) / ((size_t)kThreads * U);
    In<2> in{{a, b}};
    k<<<(unsigned)std::max<size_t>(grid, 1), kThreads, 0, s>>>(in, out, n, op);
  } else {
    auto k = map_chunk_kernel<OpAddMulScalar, U>;
    const int per = bps > 0 ? bps : resident_blocks((const void*)k, kThreads, 0);
    k<<<(unsigned)(per * sms), kThreads, 0, s>>>(a, b, out, n4, op);
  }
  return cudaGetLastError();
}

cudaError_t launch_probe(int mode, const void* src, void* dst, size_t bytes, int p0, int p1,
                         int p2, cudaStream_t s) {
  const int sms = sm_count(current_device());
  float* sink = nullptr;
  cudaError_t e = cudaGetSymbolAddress((void**)&sink, g_probe_sink);
  if (e != cudaSuccess) return e;
  const size_t n4 = bytes / 16;
  if (mode == 0 || mode == 1 || mode == 4) {
    const int threads = p0 > 0 ? p0 : 256;
    const unsigned grid = (unsigned)(std::max(p2, 1) * sms);
    const float4* x = static_cast<const float4*>(src);
    const int contiguous = mode == 1;
    if (mode == 4) {
      float4* y = static_cast<float4*>(dst);
      if (p1 == 4) probe_copy_kernel<4><<<grid, threads, 0, s>>>(x, y, n4);
      else if (p1 == 8) probe_copy_kernel<8><<<grid, threads, 0, s>>>(x, y, n4);
      else probe_copy_kernel<16><<<grid, threads, 0, s>>>(x, y, n4);
    } else {
      if (p1 == 4) probe_read_kernel<4><<<grid, threads, 0, s>>>(x, n4, contiguous, sink);
      else if (p1 == 8) probe_read_kernel<8><<<grid, threads, 0, s>>>(x, n4, contiguous, sink);
      else probe_read_kernel<16><<<grid, threads, 0, s>>>(x, n4, contiguous, sink);
    }
    return cudaGetLastError();
  }
  if (mode == 2 || mode == 3) {
    const unsigned chunk = (unsigned)p0;
    const int slots = p1;
    if (chunk < 16 || chunk % 16 != 0 || slots < 1 || slots > kMaxSlots) return cudaErrorInvalidValue;
    const size_t smem = (size_t)chunk * slots;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    int* err = wait_timeout_flag(current_device());
    if (!err) return cudaErrorInvalidValue;
    const size_t nchunks = bytes / chunk;
    const unsigned grid = (unsigned)(std::max(p2, 1) * sms);
    const char* x = static_cast<const char*>(src);
    if (mode == 2) {
      cudaFuncSetAttribute(probe_ring_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      probe_ring_kernel<false><<<grid, kRingThreads, smem, s>>>(x, nchunks, chunk, slots, sink, err);
    } else {
      cudaFuncSetAttribute(probe_ring_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      probe_ring_kernel<true><<<grid, kRingThreads, smem, s>>>(x, nchunks, chunk, slots, sink, err);
    }
    return cudaGetLastError();
  }
  if (mode == 5 || mode == 6) {
    const size_t n = bytes / 8;   // elements per operand
    const float* a = static_cast<const float*>(src);
    const float* b = a + n;
    float* out = static_cast<float*>(dst);
    switch (p1) {
      case 1: return launch_map_variant<1>(mode, p2, a, b, out, n, s);
      case 2: return launch_map_variant<2>(mode, p2, a, b, out, n, s);
      case 4: return launch_map_variant<4>(mode, p2, a, b, out, n, s);
      case 8: return launch_map_variant<8>(mode, p2, a, b, out, n, s);
      default: return cudaErrorInvalidValue;
    }
  }
  if (mode == 8) {
    if (p0 <= 0 || bytes % (4 * (size_t)p0) != 0) return cudaErrorInvalidValue;
    return launch_lane_sum_variant(p1, static_cast<const float*>(src), bytes / 4 / p0, (size_t)p0,
                                   static_cast<float*>(dst), s);
  }
  if (mode == 9) {
    if (p0 <= 0 || p1 <= 0 || p2 <= 0 || bytes % (4 * (size_t)p0) != 0) return cudaErrorInvalidValue;
    bool used = false;
    e = launch_strip_tma_shape(kDimSum, static_cast<const float*>(src), 1, bytes / 4 / p0,
                               (size_t)p0, static_cast<float*>(dst), s, &used, (size_t)(p1 % 1000),
                               (size_t)(p2 / 100), p2 % 100, p1 < 1000);
    return e != cudaSuccess ? e : (used ? cudaSuccess : cudaErrorInvalidValue);
  }
  if (mode == 7) {
    StatsPart* parts = nullptr;
    double* sum = nullptr;
    e = cudaGetSymbolAddress((void**)&parts, g_probe_parts);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&sum, g_probe_sum);
    if (e != cudaSuccess) return e;
    if (p2 >= 100)   // the grid-stride pipelined kernel, p2 - 100 blocks per SM
      return launch_stats_gs_variant(p0, p1, p2 - 100, static_cast<const float*>(src), bytes / 4,
                                     parts, kProbeParts, s, sum);
    return launch_stats_variant(p0, p1, p2, static_cast<const float*>(src), bytes / 4, parts,
                                kProbeParts, s, sum);
  }
  return cudaErrorInvalidValue;
}

// The tolerance-mode primitives on the device, for comparison with their
// host build: 0 exp_fast, 1 log_fast, 2 tanh_fast, 3 rcp_cr.
__global__ void fastmath_kernel(int which, const float* x, float* out, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    float r;
    switch (which) {
      case 0: r = exp_fast(v); break;
      case 1: r = log_fast(v); break;
      case 2: r = tanh_fast(v); break;
      default: r = rcp_cr(v); break;
    }
    out[i] = r;
  }
}

}  // namespace
}  // namespace rt

using namespace rt;

extern "C" rtc_result rtc_selftest_fastmath(int which, const float* x, float* out, size_t n) {
  RTC_OP_RANGE();
  if (which < 0 || which > 3) return invalid_argument("which", "must be 0..3");
  if (n == 0) return ok();
  if (!x || !out) return invalid_argument("x/out", "must not be null");
  const unsigned grid = (unsigned)std::min<size_t>((n + 255) / 256, (size_t)sm_count(current_device()) * 16);
  fastmath_kernel<<<grid, 256, 0, thread_stream()>>>(which, x, out, n);
  return launched(cudaGetLastError(), "selftest_fastmath");
}

extern "C" rtc_result rtc_probe_stream(int mode, const void* src, void* dst, size_t bytes,
                                       int p0, int p1, int p2) {
  RTC_OP_RANGE();
  if (!src) return invalid_argument("src", "must not be null");
  if ((mode == 4 || mode == 5 || mode == 6 || mode == 8) && !dst)
    return invalid_argument("dst", "must not be null");
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u)
    return invalid_argument("src/dst", "must be 16-byte aligned");
  if (bytes % 16 != 0) return invalid_argument("bytes", "must be a multiple of 16");
  if ((mode == 0 || mode == 1 || mode == 4) && p1 != 4 && p1 != 8 && p1 != 16)
    return invalid_argument("p1", "U must be 4, 8 or 16");
  if ((mode == 2 || mode == 3) && (bytes % (size_t)(p0 > 0 ? p0 : 1) != 0))
    return invalid_argument("bytes", "must be a multiple of the chunk (p0)");
  return launched(launch_probe(mode, src, dst, bytes, p0, p1, p2, thread_stream()),
                  "probe_stream");
}
