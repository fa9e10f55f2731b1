// loss.cu — rusttorch-core's loss functions (src/ops/loss.rs) for f32.
//
// Each loss is the f32 sum of per-element terms, then (f64)sum / n.  The
// reference sums mse/l1/smooth_l1 terms with ndarray's sum() (unrolled_fold:
// eight sequential chains over elements i % 8, combined at the end) and
// bce/ce terms with Iterator::sum::<f32>() (one sequential chain from -0.0).
// Both orders are reproduced bit for bit.
//
// The term kernel computes the terms on every SM (HBM-bound), writing them
// chain-major with one f64 sum per 256-element block of each chain; the
// ordered sum (ordered_sum.cu) then reproduces the chains' f32 rounding
// exactly without running them one add at a time.
#include "rt_internal.h"
#include "rt_libm.cuh"
#include "rt_osum.cuh"

namespace rt {
namespace {

// The ordered-sum test hook's term: the first operand itself.
struct TermIdentity {
  RT_HD float operator()(float p, float) const { return p; }
};
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

int loss_chains(LossOp op) { return op == kLossBce || op == kLossCe ? 1 : 8; }

template <class Term>
cudaError_t launch_terms(const osum::Plan& plan, const float* p, const float* t, Term term,
                         cudaStream_t s) {
  const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(t)) & 15) == 0;
  const int grid = osum::term_grid(plan);
  if (plan.chains == 8)
    osum::osum_terms_kernel<Term, 8><<<grid, osum::kTermThreads, 0, s>>>(p, t, term, plan, vec);
  else
    osum::osum_terms_kernel<Term, 1><<<grid, osum::kTermThreads, 0, s>>>(p, t, term, plan, vec);
  return cudaGetLastError();
}

}  // namespace

size_t loss_scratch_bytes(LossOp op, size_t n) { return osum::scratch_bytes(n, loss_chains(op)); }

size_t ordered_sum_scratch_bytes(size_t n, int chains) { return osum::scratch_bytes(n, chains); }

cudaError_t launch_loss(LossOp op, const float* p, const float* t, size_t n, float a, float b,
                        void* scratch, float* sum_out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const osum::Plan plan = osum::make_plan(scratch, n, loss_chains(op));
  cudaError_t e = cudaSuccess;
  switch (op) {
    case kLossMse: e = launch_terms(plan, p, t, TermMse{}, s); break;
    case kLossL1: e = launch_terms(plan, p, t, TermL1{}, s); break;
    case kLossSmoothL1: e = launch_terms(plan, p, t, TermSmoothL1{a, b}, s); break;
    case kLossBce: e = launch_terms(plan, p, t, TermBce{a, b}, s); break;
    case kLossCe: e = launch_terms(plan, p, t, TermCe{a}, s); break;
  }
  if (e != cudaSuccess) return e;
  return osum::launch_ordered_sum(plan, -0.0f, sum_out, s);
}

// The ordered sum of x itself (a test hook for the algorithm): terms = x.
cudaError_t launch_ordered_sum_of(const float* x, size_t n, int chains, float init, void* scratch,
                                  float* sum_out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const osum::Plan plan = osum::make_plan(scratch, n, chains);
  cudaError_t e = launch_terms(plan, x, x, TermIdentity{}, s);
  if (e != cudaSuccess) return e;
  return osum::launch_ordered_sum(plan, init, sum_out, s);
}

}  // namespace rt
