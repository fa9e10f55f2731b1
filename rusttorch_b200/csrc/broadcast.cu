// broadcast.cu — binary ops with broadcasting (core/src/ops/broadcast.rs).
//
// The reference materialises both operands at the broadcast shape
// (broadcast_tensors, :55-126) and then runs the plain op (:177-198).  Here
// the op reads each operand through per-dim strides that are 0 along
// broadcast dims, so only the output is written at full size.  The host
// collapses adjacent dims that are contiguous in both operands (a
// [4096, 4096] + [4096] bias add becomes a 2-dim plan); results are the same
// f32 operation on the same pair of values, hence bit-identical.
#include "rt_internal.h"
#include "rt_ops.cuh"

#include <algorithm>

namespace rt {

namespace {

template <class F>
__global__ void __launch_bounds__(kThreads)
bcast_kernel(const float* a, const float* b, float* out, size_t n, BcastPlan plan, F f) {
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    long long rem = (long long)i, ao = 0, bo = 0;
    for (int d = plan.nd - 1; d > 0; d--) {
      const long long c = rem % plan.shape[d];
      rem /= plan.shape[d];
      ao += c * plan.astride[d];
      bo += c * plan.bstride[d];
    }
    ao += rem * plan.astride[0];
    bo += rem * plan.bstride[0];
    out[i] = f(__ldg(a + ao), __ldg(b + bo));
  }
}

// Two collapsed dims [M, N]: no division per element.  Rows are strided
// over blockIdx.y, columns over x; float4 when a's rows are contiguous and b
// is either a contiguous row or a broadcast scalar per row.
constexpr int kRowsPerIter = 4;

template <class F, bool VEC>
__global__ void __launch_bounds__(kThreads)
bcast2_kernel(const float* a, const float* b, float* out, long long M, long long N,
              long long as0, long long as1, long long bs0, long long bs1, F f) {
  if (VEC) {
    // kRowsPerIter rows per iteration, all loads issued before any store, so
    // each thread keeps several 16-byte loads in flight.
    const long long n4 = N / 4;
    for (long long r0 = (long long)blockIdx.y * kRowsPerIter; r0 < M;
         r0 += (long long)gridDim.y * kRowsPerIter) {
      for (long long c = (long long)blockIdx.x * kThreads + threadIdx.x; c < n4;
           c += (long long)gridDim.x * kThreads) {
        float4 x[kRowsPerIter], y[kRowsPerIter];
#pragma unroll
        for (int k = 0; k < kRowsPerIter; k++) {
          const long long r = r0 + k;
          if (r < M) {
            x[k] = __ldcs(reinterpret_cast<const float4*>(a + r * as0) + c);
            if (bs1 == 0) {
              const float v = __ldg(b + r * bs0);
              y[k] = make_float4(v, v, v, v);
            } else {
              y[k] = __ldg(reinterpret_cast<const float4*>(b + r * bs0) + c);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < kRowsPerIter; k++) {
          const long long r = r0 + k;
          if (r < M)
            __stcs(reinterpret_cast<float4*>(out + r * N) + c,
                   make_float4(f(x[k].x, y[k].x), f(x[k].y, y[k].y), f(x[k].z, y[k].z),
                               f(x[k].w, y[k].w)));
        }
      }
    }
  } else {
    for (long long r = blockIdx.y; r < M; r += gridDim.y)
      for (long long c = (long long)blockIdx.x * kThreads + threadIdx.x; c < N;
           c += (long long)gridDim.x * kThreads)
        out[r * N + c] = f(__ldg(a + r * as0 + c * as1), __ldg(b + r * bs0 + c * bs1));
  }
}

template <class F>
cudaError_t launch(const F& f, const float* a, const float* b, float* out, size_t n,
                   const BcastPlan& plan, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (plan.nd <= 2) {
    const long long M = plan.nd == 2 ? plan.shape[0] : 1;
    const long long N = plan.shape[plan.nd - 1];
    const long long as0 = plan.nd == 2 ? plan.astride[0] : 0, bs0 = plan.nd == 2 ? plan.bstride[0] : 0;
    const long long as1 = plan.astride[plan.nd - 1], bs1 = plan.bstride[plan.nd - 1];
    const bool vec = as1 == 1 && (bs1 == 1 || bs1 == 0) && N % 4 == 0 && as0 % 4 == 0 &&
                     (bs1 == 0 || bs0 % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(out) |
                       (bs1 ? reinterpret_cast<uintptr_t>(b) : 0)) & 15u) == 0;
    const long long cols = vec ? N / 4 : N;
    const unsigned gx = (unsigned)std::max<long long>(
        1, std::min<long long>((cols + kThreads - 1) / kThreads, 64));
    const long long want_y = (long long)sm_count(dev) * 16 / gx + 1;
    const long long row_groups = vec ? (M + kRowsPerIter - 1) / kRowsPerIter : M;
    const unsigned gy = (unsigned)std::max<long long>(
        1, std::min<long long>(row_groups, std::min<long long>(want_y, 65535)));
    if (vec) {
      // A row-broadcast b (bs1 == 1, bs0 == 0) or column-broadcast b (bs1 == 0).
      bcast2_kernel<F, true><<<dim3(gx, gy), kThreads, 0, s>>>(a, b, out, M, N, as0, as1, bs0,
                                                               bs1, f);
    } else {
      bcast2_kernel<F, false><<<dim3(gx, gy), kThreads, 0, s>>>(a, b, out, M, N, as0, as1, bs0,
                                                                bs1, f);
    }
    return cudaGetLastError();
  }
  const unsigned grid = (unsigned)std::max<size_t>(
      1, std::min<size_t>((n + kThreads - 1) / kThreads, (size_t)sm_count(dev) * 16));
  bcast_kernel<<<grid, kThreads, 0, s>>>(a, b, out, n, plan, f);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_broadcast(BinaryOp op, const float* a, const float* b, float* out,
                             size_t n, const BcastPlan& plan, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  switch (op) {
    case kAdd: return launch(OpAdd{}, a, b, out, n, plan, s);
    case kSub: return launch(OpSub{}, a, b, out, n, plan, s);
    case kMul: return launch(OpMul{}, a, b, out, n, plan, s);
    case kDiv: return launch(OpDiv{}, a, b, out, n, plan, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace rt
