// softmax.cu — softmax along a dim (rusttorch-core ops/activation.rs:92-167).
//
// Reference, per lane along `dim`:
//   m = max_by fold (NaN compares Equal), e = exp(x - m), s = sum_axis(e),
//   y = e / s
// with ndarray's sum_axis order: the eight-chain unrolled_fold when dim is the
// last axis, a sequential row-order chain otherwise — also when every axis
// after dim has length 1 (the lanes are then contiguous, but ndarray's
// minimum-stride axis is still the last one).
//
// Every exponent is x - m <= 0 (or NaN), so the exponential is
// expf_glibc_nonpos (exact math mode), which skips expf's overflow branches,
// or exp_fast_nonpos (tolerance mode, rt_fastmath.cuh): the kernels take it
// as the template parameter EXP.  Only the exponential changes between the
// modes; the sum keeps ndarray's order in both.
//
// Why m may be computed with fmaxf: the fold and fmaxf agree on every lane
// without NaN except for the sign of a zero maximum, and x - (+0) and x - (-0)
// round to the same value for every x (x - x is +0 either way), so e is
// unchanged.  A lane holding a NaN makes e, s and every output NaN under both.
//
// Last-axis kernel: one CTA per row.  The row is read once from HBM into
// shared memory (16-byte loads), exponentiated in place, the eight chains are
// summed by eight threads in exactly ndarray's order, and y is written once —
// 8 B/element of traffic, the minimum.  Rows longer than shared memory allows
// take a four-pass path through the output buffer.
#include "rt_internal.h"
#include "rt_ops.cuh"

#include <algorithm>

namespace rt {

namespace {

constexpr int kRowThreads = 256;

struct ExpExact {
  __device__ __forceinline__ static float f(float x) { return expf_glibc_nonpos(x); }
};
struct ExpTol {
  __device__ __forceinline__ static float f(float x) { return exp_fast_nonpos(x); }
};

// e / s for a lane-constant s, without a division per element: with
// r = 1/s rounded to double, (float)(e * r) equals the IEEE f32 quotient
// e/s.  Reason: e*r carries a relative error below 2^-51, while the exact
// quotient of two floats is either representable or at least 2^-49 (relative)
// away from every midpoint between floats (e - s*m is a nonzero multiple of a
// unit at most 2^-49 of s*m for a midpoint m), so rounding e*r to f32 lands
// on the same float.  Checked against IEEE division on 4.2e9 (e, s) pairs
// with e in [0, 1] (subnormals included) and s in [1, 4096].
__device__ __forceinline__ double recip_rn(float s) { return __drcp_rn((double)s); }
__device__ __forceinline__ float div_by(float e, double r) {
  return __double2float_rn(__dmul_rn((double)e, r));
}
// Largest row kept in shared memory (floats).  Larger rows use the multi-pass
// path.
constexpr size_t kMaxSmemRow = 48 * 1024;

__device__ float block_max(float v, float* red) {
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < (int)(blockDim.x >> 5) ? red[l] : -INFINITY;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  v = red[0];
  __syncthreads();
  return v;
}

// ndarray unrolled_fold over e[0..len) (shared memory), run by threads 0..7 of
// warp 0; returns the sum on thread 0.  Each chain is strictly sequential;
// its shared-memory reads are issued 16 at a time ahead of the adds.
__device__ float chain_sum8(const float* e, size_t len) {
  const int j = threadIdx.x;          // 0..7
  const size_t steps = len / 8;
  float p = 0.0f;
  size_t k = 0;
  for (; k + 16 <= steps; k += 16) {
    float b[16];
#pragma unroll
    for (int u = 0; u < 16; u++) b[u] = e[8 * (k + u) + j];
#pragma unroll
    for (int u = 0; u < 16; u++) p = fadd(p, b[u]);
  }
  for (; k < steps; k++) p = fadd(p, e[8 * k + j]);
  float q[8];
#pragma unroll
  for (int t = 0; t < 8; t++) q[t] = __shfl_sync(0xffu, p, t);
  float acc = 0.0f;
  acc = fadd(acc, fadd(q[0], q[4]));
  acc = fadd(acc, fadd(q[1], q[5]));
  acc = fadd(acc, fadd(q[2], q[6]));
  acc = fadd(acc, fadd(q[3], q[7]));
  for (size_t t = steps * 8; t < len; t++) acc = fadd(acc, e[t]);
  return acc;
}

template <class EXP>
__global__ void __launch_bounds__(kRowThreads)
softmax_row_kernel(const float* x, size_t rows, size_t len, float* out) {
  extern __shared__ __align__(16) float e[];
  __shared__ float red[kRowThreads / 32];
  __shared__ float ssum;
  const size_t row = blockIdx.x;
  const float* xr = x + row * len;
  float* yr = out + row * len;
  const bool vec = ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(yr)) & 15u) == 0 &&
                   len % 4 == 0;
  float m = -INFINITY;
  if (vec) {
    const float4* q = reinterpret_cast<const float4*>(xr);
    float4* es = reinterpret_cast<float4*>(e);
    for (size_t i = threadIdx.x; i < len / 4; i += kRowThreads) {
      const float4 v = __ldcs(q + i);
      es[i] = v;
      m = fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
  } else {
    for (size_t i = threadIdx.x; i < len; i += kRowThreads) {
      const float v = xr[i];
      e[i] = v;
      m = fmaxf(m, v);
    }
  }
  m = block_max(m, red);   // contains __syncthreads: e[] is complete
  for (size_t i = threadIdx.x; i < len; i += kRowThreads) e[i] = EXP::f(fsub(e[i], m));
  __syncthreads();
  if (threadIdx.x < 8) {
    const float s = chain_sum8(e, len);
    if (threadIdx.x == 0) ssum = s;
  }
  __syncthreads();
  const double r = recip_rn(ssum);
  if (vec) {
    const float4* es = reinterpret_cast<const float4*>(e);
    float4* q = reinterpret_cast<float4*>(yr);
    for (size_t i = threadIdx.x; i < len / 4; i += kRowThreads) {
      const float4 v = es[i];
      __stcs(q + i, make_float4(div_by(v.x, r), div_by(v.y, r), div_by(v.z, r), div_by(v.w, r)));
    }
  } else {
    for (size_t i = threadIdx.x; i < len; i += kRowThreads) yr[i] = div_by(e[i], r);
  }
}

// Rows of up to 512*VPT floats (len % 4 == 0, 16-byte aligned): 128 threads
// per row, the row held in registers (VPT float4 per thread) from the single
// load to the single store; shared memory holds only e for the eight chain
// threads.  Small CTAs let ten or more rows per SM overlap, so one row's
// sequential chain phase hides behind the other rows' memory traffic.
constexpr int kRegThreads = 128;

template <int VPT, class EXP>
__global__ void __launch_bounds__(kRegThreads)
softmax_row_reg_kernel(const float* x, size_t len, float* out) {
  extern __shared__ __align__(16) float e[];
  __shared__ float red[kRegThreads / 32];
  __shared__ float ssum;
  const size_t row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * len);
  float4* yr = reinterpret_cast<float4*>(out + row * len);
  float4* es = reinterpret_cast<float4*>(e);
  const int n4 = (int)(len / 4);
  float4 v[VPT];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int j = threadIdx.x + i * kRegThreads;
    if (j < n4) {
      v[i] = __ldcs(xr + j);
      m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
    }
  }
  m = block_max(m, red);
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int j = threadIdx.x + i * kRegThreads;
    if (j < n4) {
      v[i].x = EXP::f(fsub(v[i].x, m));
      v[i].y = EXP::f(fsub(v[i].y, m));
      v[i].z = EXP::f(fsub(v[i].z, m));
      v[i].w = EXP::f(fsub(v[i].w, m));
      es[j] = v[i];
    }
  }
  __syncthreads();
  if (threadIdx.x < 8) {
    const float s = chain_sum8(e, len);
    if (threadIdx.x == 0) ssum = s;
  }
  __syncthreads();
  const double r = recip_rn(ssum);
#pragma unroll
  for (int i = 0; i < VPT; i++) {
    const int j = threadIdx.x + i * kRegThreads;
    if (j < n4)
      __stcs(yr + j, make_float4(div_by(v[i].x, r), div_by(v[i].y, r), div_by(v[i].z, r),
                                 div_by(v[i].w, r)));
  }
}

template <int VPT, class EXP>
cudaError_t launch_row_reg(const float* x, size_t rows, size_t len, float* out, cudaStream_t s) {
  const size_t smem = len * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(softmax_row_reg_kernel<VPT, EXP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  for (size_t r0 = 0; r0 < rows; r0 += 0x7fffffffull) {
    const size_t nr = std::min<size_t>(rows - r0, 0x7fffffffull);
    softmax_row_reg_kernel<VPT, EXP><<<(unsigned)nr, kRegThreads, smem, s>>>(x + r0 * len, len,
                                                                        out + r0 * len);
  }
  return cudaGetLastError();
}

// Long rows, pass 1: m per row (block per row).
__global__ void __launch_bounds__(kRowThreads)
row_max_kernel(const float* x, size_t len, float* m_out) {
  __shared__ float red[kRowThreads / 32];
  const float* xr = x + (size_t)blockIdx.x * len;
  float m = -INFINITY;
  for (size_t i = threadIdx.x; i < len; i += kRowThreads) m = fmaxf(m, xr[i]);
  m = block_max(m, red);
  if (threadIdx.x == 0) m_out[blockIdx.x] = m;
}

// Long rows, pass 2: out = exp(x - m).
template <class EXP>
__global__ void __launch_bounds__(kRowThreads)
row_exp_kernel(const float* x, size_t len, const float* m, float* out) {
  const size_t row = blockIdx.y;
  const float mr = m[row];
  for (size_t i = (size_t)blockIdx.x * kRowThreads + threadIdx.x; i < len;
       i += (size_t)gridDim.x * kRowThreads)
    out[row * len + i] = EXP::f(fsub(x[row * len + i], mr));
}

// Long rows, pass 3: s per row, eight sequential chains (one warp per row).
__global__ void row_chain_sum_kernel(const float* e, size_t len, float* s_out) {
  const float* er = e + (size_t)blockIdx.x * len;
  if (threadIdx.x < 8) {
    const float s = chain_sum8(er, len);
    if (threadIdx.x == 0) s_out[blockIdx.x] = s;
  }
}

// Long rows, pass 4: out /= s.
__global__ void __launch_bounds__(kRowThreads)
row_div_kernel(float* out, size_t len, const float* s) {
  const size_t row = blockIdx.y;
  const double r = recip_rn(s[row]);
  for (size_t i = (size_t)blockIdx.x * kRowThreads + threadIdx.x; i < len;
       i += (size_t)gridDim.x * kRowThreads)
    out[row * len + i] = div_by(out[row * len + i], r);
}

// dim is not the last axis: one thread per (outer, inner) lane, three passes
// along len; the sum is ndarray's row-order chain res = res + e_l.
template <class EXP>
__global__ void __launch_bounds__(kThreads)
softmax_lane_kernel(const float* x, size_t outer, size_t len, size_t inner, float* out) {
  const size_t lanes = outer * inner;
  for (size_t t = (size_t)blockIdx.x * kThreads + threadIdx.x; t < lanes;
       t += (size_t)gridDim.x * kThreads) {
    const size_t o = t / inner, i = t % inner;
    const float* p = x + o * len * inner + i;
    float* q = out + o * len * inner + i;
    float m = -INFINITY;
    for (size_t l = 0; l < len; l++) m = fmaxf(m, p[l * inner]);
    float s = 0.0f;
    for (size_t l = 0; l < len; l++) {
      const float ev = EXP::f(fsub(p[l * inner], m));
      q[l * inner] = ev;
      s = fadd(s, ev);
    }
    const double r = recip_rn(s);
    for (size_t l = 0; l < len; l++) q[l * inner] = div_by(q[l * inner], r);
  }
}

template <class EXP>
cudaError_t launch_softmax_exp(const float* x, size_t outer, size_t len, size_t inner,
                               bool last_axis, float* out, cudaStream_t s) {
  if (outer == 0 || len == 0 || inner == 0) return cudaSuccess;
  // A non-last axis followed only by length-1 axes has contiguous lanes but
  // ndarray's row-order chain for the sum: short lanes take the lane kernel,
  // long ones the four-pass row path with that chain.
  const bool chain = !last_axis;
  if (inner > 1 || (chain && len < 2048)) {
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t lanes = outer * inner;
    const unsigned grid = (unsigned)std::max<size_t>(
        1, std::min<size_t>((lanes + kThreads - 1) / kThreads, (size_t)sm_count(dev) * 8));
    softmax_lane_kernel<EXP><<<grid, kThreads, 0, s>>>(x, outer, len, inner, out);
    return cudaGetLastError();
  }
  const size_t rows = outer;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  if (!chain && aligned && len % 4 == 0) {
    if (len <= 512 * 2) return launch_row_reg<2, EXP>(x, rows, len, out, s);
    if (len <= 512 * 4) return launch_row_reg<4, EXP>(x, rows, len, out, s);
    if (len <= 512 * 8) return launch_row_reg<8, EXP>(x, rows, len, out, s);
    if (len <= 512 * 16) return launch_row_reg<16, EXP>(x, rows, len, out, s);
  }
  if (!chain && len <= kMaxSmemRow) {
    const size_t smem = len * sizeof(float);
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(softmax_row_kernel<EXP>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    for (size_t r0 = 0; r0 < rows; r0 += 0x7fffffffull) {
      const size_t nr = std::min<size_t>(rows - r0, 0x7fffffffull);
      softmax_row_kernel<EXP><<<(unsigned)nr, kRowThreads, smem, s>>>(x + r0 * len, nr, len,
                                                                 out + r0 * len);
    }
    return cudaGetLastError();
  }
  // Long rows: m and s per row in stream-ordered scratch.
  float* scratch = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&scratch), 2 * rows * sizeof(float), s);
  if (e != cudaSuccess) return e;
  float* m = scratch;
  float* sm = scratch + rows;
  const unsigned gx = (unsigned)std::min<size_t>((len + kRowThreads - 1) / kRowThreads, 4096);
  for (size_t r0 = 0; r0 < rows && e == cudaSuccess; r0 += 65535) {
    const unsigned nr = (unsigned)std::min<size_t>(rows - r0, 65535);
    const float* xr = x + r0 * len;
    float* yr = out + r0 * len;
    row_max_kernel<<<nr, kRowThreads, 0, s>>>(xr, len, m + r0);
    row_exp_kernel<EXP><<<dim3(gx, nr), kRowThreads, 0, s>>>(xr, len, m + r0, yr);
    if (chain)
      e = launch_lane_chain_sum(yr, nr, len, sm + r0, s);
    else
      row_chain_sum_kernel<<<nr, 32, 0, s>>>(yr, len, sm + r0);
    row_div_kernel<<<dim3(gx, nr), kRowThreads, 0, s>>>(yr, len, sm + r0);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  const cudaError_t ef = cudaFreeAsync(scratch, s);
  return e == cudaSuccess ? ef : e;
}

}  // namespace

cudaError_t launch_softmax(const float* x, size_t outer, size_t len, size_t inner,
                           bool last_axis, float* out, cudaStream_t s) {
  return math_exact() ? launch_softmax_exp<ExpExact>(x, outer, len, inner, last_axis, out, s)
                      : launch_softmax_exp<ExpTol>(x, outer, len, inner, last_axis, out, s);
}

}  // namespace rt
