// loss.cu — rusttorch-core's loss functions (src/ops/loss.rs) for f32.
//
// Each loss is the f32 sum of per-element terms, then (f64)sum / n.  The
// reference sums mse/l1/smooth_l1 terms with ndarray's sum() (unrolled_fold:
// eight sequential chains over elements i % 8, combined at the end) and
// bce/ce terms with Iterator::sum::<f32>() (one sequential chain).  Both
// orders are reproduced exactly, so the chains are inherently serial: eight
// (or one) dependent f32 adds per element position, whatever the hardware.
//
// Two kernels: (1) every SM computes the terms (HBM-bound) into a scratch
// buffer; (2) one CTA streams that buffer through a cp.async ring while the
// chain threads fold it in order.  Kernel 2 is bound by the add latency of
// its chains (n/8 or n dependent adds), not by memory.
#include "rt_internal.h"
#include "rt_fold.cuh"
#include "rt_map.cuh"
#include "rt_ops.cuh"

namespace rt {
namespace {

// loss.rs:72-73: d = p - t; d*d
struct TermMse {
  RT_HD float operator()(float p, float t) const {
    const float d = fsub(p, t);
    return fmul(d, d);
  }
};
// loss.rs:133-134: |p - t|
struct TermL1 {
  RT_HD float operator()(float p, float t) const { return fabsf(fsub(p, t)); }
};
// loss.rs:204-213, beta as f32
struct TermSmoothL1 {
  float beta, half_beta;
  RT_HD float operator()(float p, float t) const {
    const float x = fsub(p, t);
    const float ax = fabsf(x);
    return ax < beta ? fdiv(fmul(fmul(0.5f, x), x), beta) : fsub(ax, half_beta);
  }
};
// loss.rs:289-290: pc = p.max(eps).min(1 - eps); -(t*ln(pc) + (1-t)*ln(1-pc))
// (f32::max/min return the other operand for a NaN, as fmaxf/fminf do).
struct TermBce {
  float eps, hi;
  __device__ float operator()(float p, float t) const {
    const float pc = fminf(fmaxf(p, eps), hi);
    const float a = fmul(t, logf_cr(pc));
    const float b = fmul(fsub(1.0f, t), logf_cr(fsub(1.0f, pc)));
    return -fadd(a, b);
  }
};
// loss.rs:368-369: -t * ln(p.max(eps))
struct TermCe {
  float eps;
  __device__ float operator()(float p, float t) const {
    return fmul(-t, logf_cr(fmaxf(p, eps)));
  }
};

constexpr int kOsTile = 8192;       // floats per ring stage (32 KB)
constexpr int kOsStages = 6;        // 192 KB ring
constexpr int kOsThreads = 256;

// out[0] = the ordered f32 sum of x[0..n):
//   CHAINS == 8: ndarray unrolled_fold (chains over i % 8 for the first
//                n - n % 8 elements, combined (p0+p4), (p1+p5), (p2+p6),
//                (p3+p7) onto 0, then the rest in order);
//   CHAINS == 1: init + x[0] + x[1] + ... in order.
// One CTA; x must be 16-byte aligned.
template <int CHAINS>
__global__ void __launch_bounds__(kOsThreads)
ordered_sum_kernel(const float* x, size_t n, float init, float* out) {
  extern __shared__ __align__(16) float ring[];
  const size_t lim = CHAINS == 8 ? (n / 8) * 8 : (n / 4) * 4;   // through the ring
  const size_t nst = (lim + kOsTile - 1) / kOsTile;
  const int tid = threadIdx.x;
  auto issue = [&](size_t st) {
    if (st < nst) {
      float* buf = ring + (st % kOsStages) * kOsTile;
      for (int c = tid; c < kOsTile / 4; c += kOsThreads) {
        const size_t e = st * kOsTile + 4 * (size_t)c;
        if (e + 4 <= lim) {
          const unsigned d = (unsigned)__cvta_generic_to_shared(buf + 4 * c);
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(x + e)
                       : "memory");
        }
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  for (int st = 0; st < kOsStages - 1; st++) issue(st);
  float acc = CHAINS == 8 ? 0.0f : init;
  for (size_t st = 0; st < nst; st++) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kOsStages - 2) : "memory");
    __syncthreads();
    issue(st + kOsStages - 1);
    if (tid < CHAINS) {
      const int cnt = (int)min((size_t)kOsTile, lim - st * kOsTile);
      fold_pipelined(ring + (st % kOsStages) * kOsTile + tid, CHAINS, cnt / CHAINS,
                     [&](float v) { acc = fadd(acc, v); });
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  if (tid < 32) {
    float total = acc;
    if (CHAINS == 8) {
      float q[8];
#pragma unroll
      for (int j = 0; j < 8; j++) q[j] = __shfl_sync(0xffffffffu, acc, j);
      total = 0.0f;
      total = fadd(total, fadd(q[0], q[4]));
      total = fadd(total, fadd(q[1], q[5]));
      total = fadd(total, fadd(q[2], q[6]));
      total = fadd(total, fadd(q[3], q[7]));
    }
    if (tid == 0) {
      for (size_t i = lim; i < n; i++) total = fadd(total, x[i]);
      out[0] = total;
    }
  }
}

}  // namespace

cudaError_t launch_loss(LossOp op, const float* p, const float* t, size_t n, float a, float b,
                        float* terms, float* sum_out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  In<2> in{{p, t}};
  cudaError_t e = cudaSuccess;
  switch (op) {
    case kLossMse: e = launch_map(TermMse{}, in, terms, n, s); break;
    case kLossL1: e = launch_map(TermL1{}, in, terms, n, s); break;
    case kLossSmoothL1: e = launch_map(TermSmoothL1{a, b}, in, terms, n, s); break;
    case kLossBce: e = launch_map(TermBce{a, b}, in, terms, n, s); break;
    case kLossCe: e = launch_map(TermCe{a}, in, terms, n, s); break;
  }
  if (e != cudaSuccess) return e;
  const size_t smem = (size_t)kOsStages * kOsTile * sizeof(float);
  if (op == kLossBce || op == kLossCe) {
    e = cudaFuncSetAttribute(ordered_sum_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    ordered_sum_kernel<1><<<1, kOsThreads, smem, s>>>(terms, n, -0.0f, sum_out);
  } else {
    e = cudaFuncSetAttribute(ordered_sum_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    ordered_sum_kernel<8><<<1, kOsThreads, smem, s>>>(terms, n, 0.0f, sum_out);
  }
  return cudaGetLastError();
}

}  // namespace rt
