// rt_map.cuh — the streaming map kernels shared by the elementwise,
// activation, optimizer and autograd-backward launchers.
//
// out[i] = f(in0[i], ...) over n f32 elements (or two outputs from one
// pass, for the backward ops that produce both operands' gradients).  Each
// thread moves 16-byte vectors (LDG.128 / STG.128) with U independent vectors
// per stream in flight and the streaming cache hint (.cs): every byte is
// touched once.  When any pointer is not 16-byte aligned a scalar grid-stride
// kernel gives the same results.
#pragma once
#include "rt_internal.h"
#include "rt_libm.cuh"

#include <algorithm>
#include <type_traits>

namespace rt {
namespace {

__device__ __forceinline__ float4 ld4(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st4(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

template <class F>
__device__ __forceinline__ float4 map4(const F& f, float4 a) {
  return make_float4(f(a.x), f(a.y), f(a.z), f(a.w));
}
template <class F>
__device__ __forceinline__ float4 map4(const F& f, float4 a, float4 b) {
  return make_float4(f(a.x, b.x), f(a.y, b.y), f(a.z, b.z), f(a.w, b.w));
}
template <class F>
__device__ __forceinline__ float4 map4(const F& f, float4 a, float4 b, float4 c) {
  return make_float4(f(a.x, b.x, c.x), f(a.y, b.y, c.y), f(a.z, b.z, c.z), f(a.w, b.w, c.w));
}

template <int NIN>
struct In {
  const float* p[NIN];
};

template <class F, int NIN>
__device__ __forceinline__ float apply1(const F& f, const In<NIN>& in, size_t i) {
  if constexpr (NIN == 1) return f(in.p[0][i]);
  else if constexpr (NIN == 2) return f(in.p[0][i], in.p[1][i]);
  else return f(in.p[0][i], in.p[1][i], in.p[2][i]);
}

// Vectorised map: out[i] = f(in0[i], ...).  The block's tile is U vectors per
// thread, strided by blockDim so each load instruction is fully coalesced.
template <class F, int NIN, int U>
__global__ void __launch_bounds__(kThreads) map_vec_kernel(In<NIN> in, float* out, size_t n, F f) {
  const size_t n4 = n >> 2;
  const size_t tile = (size_t)kThreads * U;
  for (size_t base = (size_t)blockIdx.x * tile + threadIdx.x; base < n4;
       base += (size_t)gridDim.x * tile) {
    float4 v[NIN][U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < n4) {
#pragma unroll
        for (int k = 0; k < NIN; k++) v[k][u] = ld4(in.p[k] + 4 * j);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < n4) {
        float4 r;
        if constexpr (NIN == 1) r = map4(f, v[0][u]);
        else if constexpr (NIN == 2) r = map4(f, v[0][u], v[1][u]);
        else r = map4(f, v[0][u], v[1][u], v[2][u]);
        st4(out + 4 * j, r);
      }
    }
  }
  // n % 4 tail elements
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const size_t i = (n4 << 2) + threadIdx.x;
    out[i] = apply1<F, NIN>(f, in, i);
  }
}

template <class F, int NIN>
__global__ void __launch_bounds__(kThreads) map_scalar_kernel(In<NIN> in, float* out, size_t n, F f) {
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads)
    out[i] = apply1<F, NIN>(f, in, i);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

// Grid for a streaming kernel: enough tiles to cover n, capped at a few
// resident waves (the kernel grid-strides beyond that).
unsigned grid_for(size_t units, size_t per_block, size_t blocks_per_sm = 32) {
  const size_t want = (units + per_block - 1) / per_block;
  const size_t cap = (size_t)sm_count(current_device()) * blocks_per_sm;
  return (unsigned)std::max<size_t>(1, std::min(want, cap));
}

// Functors that declare `static constexpr bool kLight = true` (a handful of
// instructions per element) get a deeper unroll and a larger grid: with
// little arithmetic between loads, more 16-byte loads in flight per thread
// is what raises the achieved bandwidth (relu: 0.943 -> 0.965 of peak).
template <class F, class = void>
struct is_light : std::false_type {};
template <class F>
struct is_light<F, std::void_t<decltype(F::kLight)>> : std::bool_constant<F::kLight> {};
// Functors with `static constexpr bool kHeavy = true` (the exact tanh, GELU
// and its gradient, softplus and mish: 90-200 instructions per element) take
// one vector per thread per iteration: their registers then hold one element
// group's intermediates, and the SM's many warps supply the parallelism
// (mish 5 %, softplus 2 %, GELU's gradient 9 % faster; the lighter exp-based
// ops are faster with four).
template <class F, class = void>
struct is_heavy : std::false_type {};
template <class F>
struct is_heavy<F, std::void_t<decltype(F::kHeavy)>> : std::bool_constant<F::kHeavy> {};

template <class F, int NIN>
cudaError_t launch_map(const F& f, const In<NIN>& in, float* out, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  bool vec = aligned16(out);
  for (int k = 0; k < NIN; k++) vec = vec && aligned16(in.p[k]);
  if (vec) {
    constexpr bool light = NIN == 1 && is_light<F>::value;
    constexpr bool heavy = is_heavy<F>::value;
    constexpr int U = light ? 8 : (heavy ? 1 : (NIN == 3 ? 2 : 4));
    const unsigned grid =
        grid_for(std::max<size_t>(n >> 2, 1), (size_t)kThreads * U, (light || heavy) ? 64 : 32);
    map_vec_kernel<F, NIN, U><<<grid, kThreads, 0, s>>>(in, out, n, f);
  } else {
    const unsigned grid = grid_for(n, kThreads);
    map_scalar_kernel<F, NIN><<<grid, kThreads, 0, s>>>(in, out, n, f);
  }
  return cudaGetLastError();
}


// Map for a rule with a cheap path and an expensive one that only some
// elements need (GELU in the tolerance math mode): F provides arg(x),
// needs_exact(z), fast_tanh(z), exact_tanh(z) and finish(x, t).  Every
// thread runs the cheap path on its elements; the arguments of the elements
// that need the expensive path are queued in the warp's shared memory (slot
// = the warp's running count plus the lanes below in a ballot), the whole
// warp then evaluates the queue 32 arguments at a time, and each element
// picks up its result from its slot.  So the expensive path runs on full
// warps, once per queued element, instead of on every warp that holds one
// such element (which, for inputs spread as the BASELINE configs are, is
// every warp).  Results equal F's per-element operator() bit for bit.
constexpr int kSplitU = 2;

template <class F>
__global__ void __launch_bounds__(kThreads)
map_split_kernel(const float* x, float* out, size_t n, F f) {
  __shared__ float queue[kThreads / 32][32 * 4 * kSplitU];
  const unsigned lane = threadIdx.x & 31u;
  float* wq = queue[threadIdx.x >> 5];
  const unsigned below = (1u << lane) - 1u;
  const size_t n4 = n >> 2;
  const size_t tile = (size_t)kThreads * kSplitU;
  const size_t step = (size_t)gridDim.x * tile;
  // Every lane of a warp runs the same number of iterations (the loop bound
  // is the warp's first index), so the ballots see all 32 lanes.
  const size_t warp0 = (size_t)blockIdx.x * tile + (threadIdx.x & ~31u);
  auto load = [&](size_t wbase, float4* v) {
#pragma unroll
    for (int u = 0; u < kSplitU; u++) {
      const size_t j = wbase + lane + (size_t)u * kThreads;
      v[u] = j < n4 ? ld4(x + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float4 cur[kSplitU], nxt[kSplitU];
  if (warp0 < n4) load(warp0, cur);
  for (size_t wbase = warp0; wbase < n4; wbase += step) {
    const size_t base = wbase + lane;
    float xs[4 * kSplitU], t[4 * kSplitU];
    int slot[4 * kSplitU];
#pragma unroll
    for (int u = 0; u < kSplitU; u++) {
      xs[4 * u] = cur[u].x;
      xs[4 * u + 1] = cur[u].y;
      xs[4 * u + 2] = cur[u].z;
      xs[4 * u + 3] = cur[u].w;
    }
    // the next iteration's loads are in flight during this one's arithmetic
    if (wbase + step < n4) load(wbase + step, nxt);
    int count = 0;
#pragma unroll
    for (int e = 0; e < 4 * kSplitU; e++) {
      const float z = f.arg(xs[e]);
      const bool valid = base + (size_t)(e / 4) * kThreads < n4;
      const bool need = valid && F::needs_exact(z);
      t[e] = F::fast_tanh(z);
      const unsigned m = __ballot_sync(0xffffffffu, need);
      slot[e] = need ? count + __popc(m & below) : -1;
      if (need) wq[slot[e]] = z;
      count += __popc(m);
    }
    __syncwarp();
    for (int k = (int)lane; k < count; k += 32) wq[k] = F::exact_tanh(wq[k]);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 4 * kSplitU; e++)
      if (slot[e] >= 0) t[e] = wq[slot[e]];
    __syncwarp();
#pragma unroll
    for (int u = 0; u < kSplitU; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < n4)
        st4(out + 4 * j, make_float4(F::finish(xs[4 * u], t[4 * u]),
                                     F::finish(xs[4 * u + 1], t[4 * u + 1]),
                                     F::finish(xs[4 * u + 2], t[4 * u + 2]),
                                     F::finish(xs[4 * u + 3], t[4 * u + 3])));
      cur[u] = nxt[u];
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const size_t i = (n4 << 2) + threadIdx.x;
    out[i] = f(x[i]);
  }
}

template <class F>
cudaError_t launch_map_split(const F& f, const float* x, float* out, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (aligned16(x) && aligned16(out)) {
    const unsigned grid =
        grid_for(std::max<size_t>(n >> 2, 1), (size_t)kThreads * kSplitU, 32);
    map_split_kernel<F><<<grid, kThreads, 0, s>>>(x, out, n, f);
  } else {
    In<1> in{{x}};
    map_scalar_kernel<F, 1><<<grid_for(n, kThreads), kThreads, 0, s>>>(in, out, n, f);
  }
  return cudaGetLastError();
}

// Two outputs from one pass: f returns a float2 {out0, out1}.
template <class F, int NIN>
__device__ __forceinline__ float2 apply2(const F& f, const In<NIN>& in, size_t i) {
  if constexpr (NIN == 1) return f(in.p[0][i]);
  else if constexpr (NIN == 2) return f(in.p[0][i], in.p[1][i]);
  else return f(in.p[0][i], in.p[1][i], in.p[2][i]);
}

template <class F, int NIN, int U>
__global__ void __launch_bounds__(kThreads)
map2_vec_kernel(In<NIN> in, float* out0, float* out1, size_t n, F f) {
  const size_t n4 = n >> 2;
  const size_t tile = (size_t)kThreads * U;
  for (size_t base = (size_t)blockIdx.x * tile + threadIdx.x; base < n4;
       base += (size_t)gridDim.x * tile) {
    float4 v[NIN][U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < n4) {
#pragma unroll
        for (int k = 0; k < NIN; k++) v[k][u] = ld4(in.p[k] + 4 * j);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < n4) {
        float2 r[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float* lane[NIN];
#pragma unroll
          for (int k = 0; k < NIN; k++) lane[k] = reinterpret_cast<const float*>(&v[k][u]) + e;
          if constexpr (NIN == 1) r[e] = f(*lane[0]);
          else if constexpr (NIN == 2) r[e] = f(*lane[0], *lane[1]);
          else r[e] = f(*lane[0], *lane[1], *lane[2]);
        }
        st4(out0 + 4 * j, make_float4(r[0].x, r[1].x, r[2].x, r[3].x));
        st4(out1 + 4 * j, make_float4(r[0].y, r[1].y, r[2].y, r[3].y));
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const size_t i = (n4 << 2) + threadIdx.x;
    const float2 r = apply2<F, NIN>(f, in, i);
    out0[i] = r.x;
    out1[i] = r.y;
  }
}

template <class F, int NIN>
__global__ void __launch_bounds__(kThreads)
map2_scalar_kernel(In<NIN> in, float* out0, float* out1, size_t n, F f) {
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    const float2 r = apply2<F, NIN>(f, in, i);
    out0[i] = r.x;
    out1[i] = r.y;
  }
}

template <class F, int NIN>
cudaError_t launch_map2(const F& f, const In<NIN>& in, float* out0, float* out1, size_t n,
                        cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  bool vec = aligned16(out0) && aligned16(out1);
  for (int k = 0; k < NIN; k++) vec = vec && aligned16(in.p[k]);
  if (vec) {
    constexpr int U = NIN == 3 ? 2 : 4;
    const unsigned grid = grid_for(std::max<size_t>(n >> 2, 1), (size_t)kThreads * U);
    map2_vec_kernel<F, NIN, U><<<grid, kThreads, 0, s>>>(in, out0, out1, n, f);
  } else {
    map2_scalar_kernel<F, NIN><<<grid_for(n, kThreads), kThreads, 0, s>>>(in, out0, out1, n, f);
  }
  return cudaGetLastError();
}

}  // namespace
}  // namespace rt
