// elementwise.cu — streaming kernels for the elementwise, scalar, activation
// and optimizer-update ops of rusttorch-core (ops/elementwise.rs, simd.rs,
// activation.rs, optimizer.rs).
//
// All of these are HBM-bound: per element they move 8 B (unary), 12 B
// (binary), 16 B (fma) or 28 B (Adam/AdamW) and do a few to a few dozen flops.
// Each thread moves 16-byte vectors (LDG.128 / STG.128) with U independent
// vectors per stream in flight, so an SM with 2048 resident threads keeps
// 2048 * U * 16 B * streams in flight — far above the ~40 KB per SM that
// Little's law asks for at HBM3e latency.  Loads and stores use the streaming
// cache hint (.cs): every byte is touched once.  Pointers that are not all
// 16-byte aligned take a scalar grid-stride kernel instead (same results).
#include "rt_internal.h"
#include "rt_map.cuh"
#include "rt_ops.cuh"

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

namespace rt {

int sm_count(int device) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0) device = 0;
  if ((size_t)device >= cache.size()) cache.resize(device + 1, 0);
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
      v = 148;
    cache[device] = v;
  }
  return cache[device];
}

// sqrt_2_over_pi = (2.0_f32 / PI).sqrt() (activation.rs:73): f32 division and
// square root, each correctly rounded.
float gelu_k() {
  volatile float two = 2.0f, pi = 3.14159265358979323846f;
  return sqrtf(two / pi);
}

namespace {
// -1: not yet read from RTC_MATH_MODE; 0: tolerance; 1: exact.
std::atomic<int> g_math_mode{-1};
}  // namespace

bool math_exact() {
  int m = g_math_mode.load(std::memory_order_relaxed);
  if (m < 0) {
    const char* env = std::getenv("RTC_MATH_MODE");
    const int want = (env && std::strcmp(env, "exact") == 0) ? 1 : 0;
    int expected = -1;
    g_math_mode.compare_exchange_strong(expected, want);
    m = g_math_mode.load(std::memory_order_relaxed);
  }
  return m == 1;
}

void set_math_exact(bool exact) { g_math_mode.store(exact ? 1 : 0); }

cudaError_t launch_unary(UnaryOp op, float param, const float* x, float* out, size_t n,
                         cudaStream_t s) {
  In<1> in{{x}};
  const bool exact = math_exact();
  switch (op) {
    case kRelu: return launch_map(OpRelu{}, in, out, n, s);
    case kLeakyRelu: return launch_map(OpLeakyRelu{param}, in, out, n, s);
    case kSigmoid:
      return exact ? launch_map(OpSigmoid{}, in, out, n, s)
                   : launch_map(OpSigmoidTol{}, in, out, n, s);
    case kTanh:
      return exact ? launch_map(OpTanh{}, in, out, n, s) : launch_map(OpTanhTol{}, in, out, n, s);
    case kGelu:
      return exact ? launch_map(OpGelu{gelu_k()}, in, out, n, s)
                   : launch_map_split(OpGeluTol{gelu_k()}, x, out, n, s);
    case kSwish:
      return exact ? launch_map(OpSwish{}, in, out, n, s) : launch_map(OpSwishTol{}, in, out, n, s);
    case kElu: return launch_map(OpElu{param}, in, out, n, s);
    case kSelu: {
      // activation.rs:236-251: f64 constants, cast to f32 at use.
      const float alpha = (float)1.6732632423543772, scale = (float)1.0507009873554805;
      return launch_map(OpSelu{alpha, scale}, in, out, n, s);
    }
    case kMish:
      return exact ? launch_map(OpMish{}, in, out, n, s) : launch_map(OpMishTol{}, in, out, n, s);
    case kSoftplus:
      return exact ? launch_map(OpSoftplus{}, in, out, n, s)
                   : launch_map(OpSoftplusTol{}, in, out, n, s);
    case kSoftsign: return launch_map(OpSoftsign{}, in, out, n, s);
    case kAddScalar: return launch_map(OpAddScalar{param}, in, out, n, s);
    case kMulScalar: return launch_map(OpMulScalar{param}, in, out, n, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_binary(BinaryOp op, float param, const float* a, const float* b, float* out,
                          size_t n, cudaStream_t s) {
  In<2> in{{a, b}};
  switch (op) {
    case kAdd: return launch_map(OpAdd{}, in, out, n, s);
    case kSub: return launch_map(OpSub{}, in, out, n, s);
    case kMul: return launch_map(OpMul{}, in, out, n, s);
    case kDiv: return launch_map(OpDiv{}, in, out, n, s);
    case kAddMulScalar: return launch_map(OpAddMulScalar{param}, in, out, n, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_fma(const float* a, const float* b, const float* c, float* out, size_t n,
                       cudaStream_t s) {
  In<3> in{{a, b, c}};
  return launch_map(OpFma{}, in, out, n, s);
}

// ----------------------------------------------------------------- optimizers

namespace {

// One Adam/AdamW element, in the order of optimizer.rs:293-309 and :413-421.
__device__ __forceinline__ void adam1(const AdamCoeffs& c, float p, float g, float m, float v,
                                      float& po, float& mo, float& vo) {
  const float nm = fadd(fmul(m, c.b1), fmul(g, c.one_minus_b1));
  const float nv = fadd(fmul(v, c.b2), fmul(fmul(g, g), c.one_minus_b2));
  const float mh = fdiv(nm, c.bc1);
  const float vh = fdiv(nv, c.bc2);
  const float den = fadd(fsqrt(vh), c.eps);
  float np = fsub(p, fmul(fdiv(mh, den), c.lr));
  if (c.decay) np = fsub(np, fmul(p, c.lr_wd));
  po = np;
  mo = nm;
  vo = nv;
}

template <int U>
__global__ void __launch_bounds__(kThreads)
adam_vec_kernel(const float* p, const float* g, const float* m, const float* v, float* po,
                float* mo, float* vo, size_t n, AdamCoeffs c) {
  const size_t n4 = n >> 2;
  const size_t tile = (size_t)kThreads * U;
  for (size_t base = (size_t)blockIdx.x * tile + threadIdx.x; base < n4;
       base += (size_t)gridDim.x * tile) {
    float4 P[U], G[U], M[U], V[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < n4) {
        P[u] = ld4(p + 4 * j);
        G[u] = ld4(g + 4 * j);
        M[u] = ld4(m + 4 * j);
        V[u] = ld4(v + 4 * j);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const size_t j = base + (size_t)u * kThreads;
      if (j < n4) {
        float4 a, b, d;
        adam1(c, P[u].x, G[u].x, M[u].x, V[u].x, a.x, b.x, d.x);
        adam1(c, P[u].y, G[u].y, M[u].y, V[u].y, a.y, b.y, d.y);
        adam1(c, P[u].z, G[u].z, M[u].z, V[u].z, a.z, b.z, d.z);
        adam1(c, P[u].w, G[u].w, M[u].w, V[u].w, a.w, b.w, d.w);
        st4(po + 4 * j, a);
        st4(mo + 4 * j, b);
        st4(vo + 4 * j, d);
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const size_t i = (n4 << 2) + threadIdx.x;
    float a, b, d;
    adam1(c, p[i], g[i], m[i], v[i], a, b, d);
    po[i] = a;
    mo[i] = b;
    vo[i] = d;
  }
}

__global__ void __launch_bounds__(kThreads)
adam_scalar_kernel(const float* p, const float* g, const float* m, const float* v, float* po,
                   float* mo, float* vo, size_t n, AdamCoeffs c) {
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    float a, b, d;
    adam1(c, p[i], g[i], m[i], v[i], a, b, d);
    po[i] = a;
    mo[i] = b;
    vo[i] = d;
  }
}

// nn/optim.rs:297-304: m' = b1*m + (1-b1)*g; v' = b2*v + ((1-b2)*g)*g;
// p' = p - (lr*(m'/bc1)) / (sqrt(v'/bc2) + eps)
__device__ __forceinline__ void nn_adam1(const NnAdamCoeffs& c, float p, float g, float m,
                                         float v, float& po, float& mo, float& vo) {
  const float nm = fadd(fmul(c.b1, m), fmul(c.one_minus_b1, g));
  const float nv = fadd(fmul(c.b2, v), fmul(fmul(c.one_minus_b2, g), g));
  const float mh = fdiv(nm, c.bc1);
  const float vh = fdiv(nv, c.bc2);
  po = fsub(p, fdiv(fmul(c.lr, mh), fadd(fsqrt(vh), c.eps)));
  mo = nm;
  vo = nv;
}

__global__ void __launch_bounds__(kThreads)
nn_adam_kernel(const float* p, const float* g, const float* m, const float* v, float* po,
               float* mo, float* vo, size_t n, NnAdamCoeffs c) {
  const size_t n4 = n >> 2;
  const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                     reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v) |
                     reinterpret_cast<uintptr_t>(po) | reinterpret_cast<uintptr_t>(mo) |
                     reinterpret_cast<uintptr_t>(vo)) & 15u) == 0;
  if (vec) {
    for (size_t j = (size_t)blockIdx.x * kThreads + threadIdx.x; j < n4;
         j += (size_t)gridDim.x * kThreads) {
      const float4 P = ld4(p + 4 * j), G = ld4(g + 4 * j), M = ld4(m + 4 * j), V = ld4(v + 4 * j);
      float4 a, b, d;
      nn_adam1(c, P.x, G.x, M.x, V.x, a.x, b.x, d.x);
      nn_adam1(c, P.y, G.y, M.y, V.y, a.y, b.y, d.y);
      nn_adam1(c, P.z, G.z, M.z, V.z, a.z, b.z, d.z);
      nn_adam1(c, P.w, G.w, M.w, V.w, a.w, b.w, d.w);
      st4(po + 4 * j, a);
      st4(mo + 4 * j, b);
      st4(vo + 4 * j, d);
    }
  }
  const size_t start = vec ? (n4 << 2) : 0;
  for (size_t i = start + (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    float a, b, d;
    nn_adam1(c, p[i], g[i], m[i], v[i], a, b, d);
    po[i] = a;
    mo[i] = b;
    vo[i] = d;
  }
}

// nn/optim.rs:182-190 (momentum > 0): v' = (momentum*v + g) + wd*p; p - lr*v'
struct NnSgdMomentum {
  float lr, mom, wd;
};
__global__ void __launch_bounds__(kThreads)
nn_sgd_momentum_kernel(const float* p, const float* g, const float* vel, float* po, float* vo,
                       size_t n, NnSgdMomentum c) {
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    const float nv = fadd(fadd(fmul(c.mom, vel[i]), g[i]), fmul(c.wd, p[i]));
    vo[i] = nv;
    po[i] = fsub(p[i], fmul(c.lr, nv));
  }
}

// nn/optim.rs:198-203 (no momentum): p - lr*(g + wd*p)
struct OpNnSgd {
  float lr, wd;
  RT_HD float operator()(float p, float g) const { return fsub(p, fmul(lr, fadd(g, fmul(wd, p)))); }
};

// optimizer.rs:150-153: v' = v*mom + g; p' = p - v'*lr
struct SgdMomentum {
  float lr, mom;
};
__global__ void __launch_bounds__(kThreads)
sgd_momentum_kernel(const float* p, const float* g, const float* vel, float* po, float* vo,
                    size_t n, SgdMomentum c) {
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    const float nv = fadd(fmul(vel[i], c.mom), g[i]);
    po[i] = fsub(p[i], fmul(nv, c.lr));
    vo[i] = nv;
  }
}

// optimizer.rs:72-74: p - g*lr
struct OpSgd {
  float lr;
  RT_HD float operator()(float p, float g) const { return fsub(p, fmul(g, lr)); }
};

}  // namespace

cudaError_t launch_adam(const float* p, const float* g, const float* m, const float* v,
                        float* p_out, float* m_out, float* v_out, size_t n, const AdamCoeffs& c,
                        cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const bool vec = aligned16(p) && aligned16(g) && aligned16(m) && aligned16(v) &&
                   aligned16(p_out) && aligned16(m_out) && aligned16(v_out);
  if (vec) {
    constexpr int U = 2;
    const unsigned grid = grid_for(std::max<size_t>(n >> 2, 1), (size_t)kThreads * U);
    adam_vec_kernel<U><<<grid, kThreads, 0, s>>>(p, g, m, v, p_out, m_out, v_out, n, c);
  } else {
    adam_scalar_kernel<<<grid_for(n, kThreads), kThreads, 0, s>>>(p, g, m, v, p_out, m_out,
                                                                    v_out, n, c);
  }
  return cudaGetLastError();
}

cudaError_t launch_nn_adam(const float* p, const float* g, const float* m, const float* v,
                           float* p_out, float* m_out, float* v_out, size_t n,
                           const NnAdamCoeffs& c, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  nn_adam_kernel<<<grid_for(std::max<size_t>(n >> 2, 1), kThreads), kThreads, 0, s>>>(
      p, g, m, v, p_out, m_out, v_out, n, c);
  return cudaGetLastError();
}

cudaError_t launch_nn_sgd(const float* p, const float* g, const float* vel, float* p_out,
                          float* vel_out, size_t n, float lr, float momentum, float wd,
                          cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (momentum > 0.0f) {
    nn_sgd_momentum_kernel<<<grid_for(n, kThreads), kThreads, 0, s>>>(
        p, g, vel, p_out, vel_out, n, NnSgdMomentum{lr, momentum, wd});
    return cudaGetLastError();
  }
  In<2> in{{p, g}};
  return launch_map(OpNnSgd{lr, wd}, in, p_out, n, s);
}

cudaError_t launch_sgd(const float* p, const float* g, float* p_out, size_t n, float lr,
                       cudaStream_t s) {
  In<2> in{{p, g}};
  return launch_map(OpSgd{lr}, in, p_out, n, s);
}

cudaError_t launch_sgd_momentum(const float* p, const float* g, const float* vel, float* p_out,
                                float* vel_out, size_t n, float lr, float momentum,
                                cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  sgd_momentum_kernel<<<grid_for(n, kThreads), kThreads, 0, s>>>(p, g, vel, p_out, vel_out, n,
                                                                  SgdMomentum{lr, momentum});
  return cudaGetLastError();
}

}  // namespace rt
