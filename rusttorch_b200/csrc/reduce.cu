// reduce.cu — global and dim reductions of rusttorch-core (ops/reduction.rs).
//
// Global sum/mean/max/min (reduction.rs:7-72).  One HBM pass computes the f64
// sum and the NaN-ignoring max/min of every block's contiguous share
// (4 B/element of traffic); a one-block kernel combines the per-block partials
// in block order, so the result is deterministic for a given device.  The
// reference folds max/min with partial_cmp (NaN compares Equal, Equal keeps
// the later element for max and the earlier for min); fmaxf/fminf give the
// same bits except when a NaN is present or the extreme is a zero, and the
// host repairs exactly those cases with one more scan (launch_index_scan).
//
// Dim reductions (reduction.rs:75-150, plus max along a dim), on a
// C-contiguous tensor viewed as [outer, len, inner].  ndarray's sum_axis
// reduces lane by lane only along the minimum-stride axis; for the default
// strides of a tensor built from a shape (IxDyn, all lengths > 0) that is the
// LAST axis, because the axes after it have stride 1 as well when they have
// length 1 and the reversed min_by_key keeps the last of equal strides.
//  * the last axis (inner == 1): ndarray reduces each lane with
//    numeric_util::unrolled_fold — eight strided partial sums combined as
//    0+(p0+p4), +(p1+p5), +(p2+p6), +(p3+p7), then the tail.  Eight threads
//    run the eight chains of one lane, each strictly sequential, so the result
//    is ndarray's bit for bit.  Max uses a warp per lane (order-independent
//    fmaxf) and re-folds a lane sequentially in the rare NaN/zero case.
//  * any other axis: ndarray accumulates `res = res + row` in row order, i.e.
//    each output is a sequential chain over len.  With inner > 1 one thread
//    owns one output column; a CTA owns a strip of W columns and streams the
//    rows through a multi-stage cp.async ring in shared memory, so HBM sees
//    fully coalesced 16-byte reads with ~150 KB in flight per SM while every
//    column is still summed in row order (bit-exact).  With inner == 1 (only
//    length-1 axes follow `dim`) the lanes are contiguous but still one
//    chain each: launch_lane_chain_sum.
#include "rt_internal.h"
#include "rt_fold.cuh"
#include "rt_ops.cuh"

#include <algorithm>
#include <cfloat>

namespace rt {

namespace {

constexpr int kStatsThreads = 512;

__device__ __forceinline__ double shfl_xor_d(double v, int m) {
  return __shfl_xor_sync(0xffffffffu, v, m);
}

struct Acc {
  double s;
  float mx, mn;
  __device__ void init() {
    s = 0.0;
    mx = -INFINITY;
    mn = INFINITY;
  }
  __device__ __forceinline__ void add(float v) {
    s = dadd(s, (double)v);
    mx = fmaxf(mx, v);
    mn = fminf(mn, v);
  }
  __device__ void merge(const Acc& o) {
    s = dadd(s, o.s);
    mx = fmaxf(mx, o.mx);
    mn = fminf(mn, o.mn);
  }
};

// Deterministic block reduction (fixed xor-butterfly and warp order).
template <int NT>
__device__ void block_reduce(Acc& a) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    Acc o;
    o.s = shfl_xor_d(a.s, m);
    o.mx = __shfl_xor_sync(0xffffffffu, a.mx, m);
    o.mn = __shfl_xor_sync(0xffffffffu, a.mn, m);
    a.merge(o);
  }
  constexpr int W = NT / 32;
  __shared__ double ss[W];
  __shared__ float smx[W], smn[W];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    ss[warp] = a.s;
    smx[warp] = a.mx;
    smn[warp] = a.mn;
  }
  __syncthreads();
  if (warp == 0) {
    if (lane < W) {
      a.s = ss[lane];
      a.mx = smx[lane];
      a.mn = smn[lane];
    } else {
      a.init();
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      Acc o;
      o.s = shfl_xor_d(a.s, m);
      o.mx = __shfl_xor_sync(0xffffffffu, a.mx, m);
      o.mn = __shfl_xor_sync(0xffffffffu, a.mn, m);
      a.merge(o);
    }
  }
}

// max/min of three floats in one instruction (sm_100a); NaN inputs are
// ignored as fmaxf/fminf ignore them, and the host repairs the NaN and zero
// cases exactly as for fmaxf/fminf.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// f64 value of x + y + z + w.  F32TREE: (x + y) + (z + w) in float32 and
// converted once — two roundings on each element's path, so the error is at
// most 2^-23 of |x| + |y| + |z| + |w| (the sum's tolerance is 1e-6 of
// sum|x|) — unless that overflows, when the tree is redone in float64 (an
// infinite or NaN input gives the same infinity or NaN either way).
// Otherwise every float is converted exactly and added in float64.
template <bool F32TREE>
__device__ __forceinline__ double sum4(const float4& v) {
  if (F32TREE) {
    const float t = fadd(fadd(v.x, v.y), fadd(v.z, v.w));
    if (fabsf(t) != INFINITY) return (double)t;
  }
  return dadd(dadd((double)v.x, (double)v.y), dadd((double)v.z, (double)v.w));
}

// Block b reduces the contiguous element range [b*chunk, (b+1)*chunk) with
// 16-byte loads (the unaligned head and the tail are read as scalars).  U
// loads per thread are in flight at once; each float4 is reduced as a tree
// (sum4, and three-input max/min) into one of two accumulators, so the
// dependent operations between one batch of loads and the next stay few: a
// warp spends most of its time with loads in flight, which is what a
// read-only stream needs to reach HBM bandwidth.
template <int NT, int U, bool F32TREE>
__global__ void __launch_bounds__(NT)
stats_kernel(const float* x, size_t n, size_t chunk, StatsPart* parts) {
  const size_t lo = (size_t)blockIdx.x * chunk;
  const size_t hi = min(n, lo + chunk);
  Acc a;
  a.init();
  double s1 = 0.0;
  if (lo < hi) {
    const float* p = x + lo;
    const size_t cnt = hi - lo;
    size_t head = ((16u - (reinterpret_cast<uintptr_t>(p) & 15u)) & 15u) >> 2;
    if (head > cnt) head = cnt;
    if (threadIdx.x < head) a.add(__ldcs(p + threadIdx.x));
    const float4* q = reinterpret_cast<const float4*>(p + head);
    const size_t n4 = (cnt - head) >> 2;
    size_t i = threadIdx.x;
    for (; i + (U - 1) * NT < n4; i += U * NT) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; u++) v[u] = __ldcs(q + i + u * NT);
#pragma unroll
      for (int u = 0; u < U; u++) {
        const double t = sum4<F32TREE>(v[u]);
        if (u & 1) s1 = dadd(s1, t);
        else a.s = dadd(a.s, t);
        a.mx = fmax3(fmax3(a.mx, v[u].x, v[u].y), v[u].z, v[u].w);
        a.mn = fmin3(fmin3(a.mn, v[u].x, v[u].y), v[u].z, v[u].w);
      }
    }
    for (; i < n4; i += NT) {
      const float4 v = __ldcs(q + i);
      a.add(v.x);
      a.add(v.y);
      a.add(v.z);
      a.add(v.w);
    }
    const size_t done = head + (n4 << 2);
    if (threadIdx.x < cnt - done) a.add(__ldcs(p + done + threadIdx.x));
  }
  a.s = dadd(a.s, s1);
  block_reduce<NT>(a);
  if (threadIdx.x == 0) parts[blockIdx.x] = StatsPart{a.s, a.mx, a.mn};
}

// The same statistics with the loads interleaved over the whole grid (block
// b, thread t reads float4 b*NT + t, then every gridDim*NT further, as one
// sweep of all SMs through the tensor) and software-pipelined: the next U
// loads are issued before the current U are reduced.  Block 0 also takes
// the unaligned head and the tail.
template <int NT, int U>
__global__ void __launch_bounds__(NT)
stats_gs_kernel(const float* x, size_t n, StatsPart* parts) {
  Acc a;
  a.init();
  double s1 = 0.0;
  size_t head = ((16u - (reinterpret_cast<uintptr_t>(x) & 15u)) & 15u) >> 2;
  if (head > n) head = n;
  const float4* q = reinterpret_cast<const float4*>(x + head);
  const size_t n4 = (n - head) >> 2;
  if (blockIdx.x == 0) {
    if (threadIdx.x < head) a.add(__ldcs(x + threadIdx.x));
    const size_t done = head + (n4 << 2);
    if (threadIdx.x < n - done) a.add(__ldcs(x + done + threadIdx.x));
  }
  const size_t stride = (size_t)gridDim.x * NT;
  size_t i = (size_t)blockIdx.x * NT + threadIdx.x;
  auto reduce = [&](const float4* v) {
#pragma unroll
    for (int u = 0; u < U; u++) {
      const double t = sum4<true>(v[u]);
      if (u & 1) s1 = dadd(s1, t);
      else a.s = dadd(a.s, t);
      a.mx = fmax3(fmax3(a.mx, v[u].x, v[u].y), v[u].z, v[u].w);
      a.mn = fmin3(fmin3(a.mn, v[u].x, v[u].y), v[u].z, v[u].w);
    }
  };
  if (i + (U - 1) * stride < n4) {
    float4 cur[U];
#pragma unroll
    for (int u = 0; u < U; u++) cur[u] = __ldcs(q + i + u * stride);
    for (; i + (2 * U - 1) * stride < n4; i += U * stride) {
      float4 nxt[U];
#pragma unroll
      for (int u = 0; u < U; u++) nxt[u] = __ldcs(q + i + (U + u) * stride);
      reduce(cur);
#pragma unroll
      for (int u = 0; u < U; u++) cur[u] = nxt[u];
    }
    reduce(cur);
    i += U * stride;
  }
  for (; i < n4; i += stride) {
    const float4 v = __ldcs(q + i);
    a.add(v.x);
    a.add(v.y);
    a.add(v.z);
    a.add(v.w);
  }
  a.s = dadd(a.s, s1);
  block_reduce<NT>(a);
  if (threadIdx.x == 0) parts[blockIdx.x] = StatsPart{a.s, a.mx, a.mn};
}

__global__ void __launch_bounds__(kStatsThreads)
stats_final_kernel(const StatsPart* parts, int nparts, StatsPart* out, double* sum_out) {
  Acc a;
  a.init();
  for (int i = threadIdx.x; i < nparts; i += kStatsThreads) {
    const StatsPart p = parts[i];
    Acc o;
    o.s = p.sum;
    o.mx = p.mx;
    o.mn = p.mn;
    a.merge(o);
  }
  block_reduce<kStatsThreads>(a);
  if (threadIdx.x == 0) {
    if (out) *out = StatsPart{a.s, a.mx, a.mn};
    if (sum_out) *sum_out = a.s;
  }
}

__global__ void index_scan_init(IndexScan* out) {
  out->last_nan = 0ull;
  out->first_zero = ~0ull;
  out->last_zero = 0ull;
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
  return __shfl_xor_sync(0xffffffffu, v, m);
}

__global__ void __launch_bounds__(kThreads)
index_scan_kernel(const float* x, size_t n, IndexScan* out) {
  unsigned long long ln = 0ull, fz = ~0ull, lz = 0ull;
  for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads) {
    const float v = x[i];
    const unsigned long long k = (unsigned long long)i + 1ull;
    if (v != v) ln = k;                 // indices only grow per thread
    if (v == 0.0f) {
      if (fz == ~0ull) fz = k;
      lz = k;
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    ln = max(ln, shfl_xor_u64(ln, m));
    fz = min(fz, shfl_xor_u64(fz, m));
    lz = max(lz, shfl_xor_u64(lz, m));
  }
  if ((threadIdx.x & 31) == 0) {
    if (ln) atomicMax(&out->last_nan, ln);
    if (fz != ~0ull) atomicMin(&out->first_zero, fz);
    if (lz) atomicMax(&out->last_zero, lz);
  }
}

// ------------------------------------------------------------ last-axis sum
// Eight threads per lane: thread j owns ndarray's partial sum p_j over
// elements j, j+8, j+16, ... of the lane, added strictly in order.  Loads are
// issued kBatch at a time ahead of the dependent adds.
constexpr int kLaneThreads = 64;      // 8 lanes per block
constexpr int kBatch = 64;

__global__ void __launch_bounds__(kLaneThreads)
lane_sum8_kernel(const float* x, size_t lanes, size_t len, float* out, int mean) {
  const size_t lane = (size_t)blockIdx.x * (kLaneThreads / 8) + (threadIdx.x >> 3);
  const int j = threadIdx.x & 7;
  const unsigned gmask = 0xffu << (threadIdx.x & 24);   // this lane's 8 threads
  float p = 0.0f;
  const bool active = lane < lanes;
  const float* base = x + (active ? lane : 0) * len + j;
  const size_t steps = active ? len / 8 : 0;
  size_t k = 0;
  for (; k + kBatch <= steps; k += kBatch) {
    float buf[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; b++) buf[b] = __ldcs(base + (k + b) * 8);
#pragma unroll
    for (int b = 0; b < kBatch; b++) p = fadd(p, buf[b]);
  }
  for (; k < steps; k++) p = fadd(p, __ldcs(base + k * 8));
  // Gather the eight partials on thread j == 0 of the lane.
  float q[8];
#pragma unroll
  for (int t = 0; t < 8; t++) q[t] = __shfl_sync(gmask, p, (threadIdx.x & 24) + t);
  if (active && j == 0) {
    float acc = 0.0f;
    acc = fadd(acc, fadd(q[0], q[4]));
    acc = fadd(acc, fadd(q[1], q[5]));
    acc = fadd(acc, fadd(q[2], q[6]));
    acc = fadd(acc, fadd(q[3], q[7]));
    const float* lp = x + lane * len;
    for (size_t t = steps * 8; t < len; t++) acc = fadd(acc, lp[t]);
    if (mean) acc = fdiv(acc, (float)len);
    out[lane] = acc;
  }
}

// ------------------------------------------------------------ last-axis max
// Warp per lane.  fmaxf is order-independent; it equals the reference fold
// unless the lane holds a NaN or its maximum is a zero (+0 and -0 compare
// Equal, and the fold keeps the last one).  Those lanes are re-folded
// sequentially by lane 0, which reproduces the reference exactly.
constexpr int kWarpLaneThreads = 256;

__global__ void __launch_bounds__(kWarpLaneThreads)
lane_max_kernel(const float* x, size_t lanes, size_t len, float* out) {
  const size_t lane = (size_t)blockIdx.x * (kWarpLaneThreads / 32) + (threadIdx.x >> 5);
  if (lane >= lanes) return;
  const int l = threadIdx.x & 31;
  const float* p = x + lane * len;
  float m = -INFINITY;
  bool nan = false;
  const bool vec = ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) && (len % 4 == 0);
  if (vec) {
    const float4* q = reinterpret_cast<const float4*>(p);
    const size_t n4 = len / 4;
    constexpr int U = 4;
    size_t i = l;
    for (; i + (U - 1) * 32 < n4; i += U * 32) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; u++) v[u] = __ldcs(q + i + u * 32);
#pragma unroll
      for (int u = 0; u < U; u++) {
        nan |= (v[u].x != v[u].x) | (v[u].y != v[u].y) | (v[u].z != v[u].z) | (v[u].w != v[u].w);
        m = fmaxf(fmaxf(m, v[u].x), fmaxf(v[u].y, fmaxf(v[u].z, v[u].w)));
      }
    }
    for (; i < n4; i += 32) {
      const float4 v = __ldcs(q + i);
      nan |= (v.x != v.x) | (v.y != v.y) | (v.z != v.z) | (v.w != v.w);
      m = fmaxf(fmaxf(m, v.x), fmaxf(v.y, fmaxf(v.z, v.w)));
    }
  } else {
    for (size_t i = l; i < len; i += 32) {
      const float v = p[i];
      nan |= (v != v);
      m = fmaxf(m, v);
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
  nan = __any_sync(0xffffffffu, nan);
  if (l == 0) {
    if (nan || m == 0.0f) {
      float acc = p[0];
      for (size_t i = 1; i < len; i++) acc = max_fold(acc, p[i]);
      m = acc;
    }
    out[lane] = m;
  }
}

// ------------------------------------------------- middle-axis, column strip
// CTA (o, s) reduces columns [c0, c0+W) of outer slice o over all `len` rows.
// Rows arrive R at a time through a kStages-deep cp.async ring in shared
// memory ([kStages][R][W] floats, R sized so the ring stays near kStripSmem).
constexpr int kStages = 6;
constexpr int kStripMaxW = 256;
constexpr size_t kStripSmem = 96 * 1024;   // two CTAs per SM

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Copy slots per thread and stage: a stage holds R*W <= 4096 floats = 1024
// 16-byte chunks, and the CTA has at least 128 threads.
constexpr int kStripSlots = 8;

template <int OP>
__global__ void strip_reduce_kernel(const float* x, size_t len, size_t inner, int W, int R,
                                    size_t strips, float* out) {
  extern __shared__ __align__(16) float smem[];
  const size_t o = blockIdx.x / strips;
  const size_t s = blockIdx.x % strips;
  const size_t c0 = s * (size_t)W;
  const int w_eff = (int)min((size_t)W, inner - c0);
  const int chunks_per_row = w_eff / 4;           // inner % 4 == 0 and c0 % 4 == 0
  const float* src = x + o * len * inner + c0;
  const size_t nstage = (len + R - 1) / R;
  const int tid = threadIdx.x, nt = blockDim.x;
  const size_t stage_floats = (size_t)R * W;

  // The chunks this thread copies are the same in every stage: precompute
  // their row, shared-memory offset and global offset once.
  int slot_row[kStripSlots];
  int slot_soff[kStripSlots];
  size_t slot_goff[kStripSlots];
#pragma unroll
  for (int q = 0; q < kStripSlots; q++) {
    const int t = tid + q * nt;
    const int r = chunks_per_row ? t / chunks_per_row : 0;
    const int c = chunks_per_row ? t % chunks_per_row : 0;
    slot_row[q] = (t < R * chunks_per_row) ? r : R;   // R = no chunk
    slot_soff[q] = r * W + 4 * c;
    slot_goff[q] = (size_t)r * inner + 4 * c;
  }

  auto issue = [&](size_t st) {
    if (st < nstage) {
      float* buf = smem + (st % kStages) * stage_floats;
      const size_t r0 = st * R;
      const int rows = (int)min((size_t)R, len - r0);
      const float* base = src + r0 * inner;
#pragma unroll
      for (int q = 0; q < kStripSlots; q++)
        if (slot_row[q] < rows) cp_async16(buf + slot_soff[q], base + slot_goff[q]);
    }
    cp_async_commit();   // always commit, so group counting stays in step
  };

  for (int st = 0; st < kStages - 1; st++) issue(st);

  // Sums are strictly sequential in row order.  Max keeps fmaxf's value
  // (order-independent) plus a NaN flag; a column holding a NaN, or whose
  // maximum is a zero, is re-folded sequentially at the end (rare).
  float acc = (OP == kDimMax) ? -INFINITY : 0.0f;
  bool nan = false;
  for (size_t st = 0; st < nstage; st++) {
    cp_async_wait<kStages - 2>();   // this thread's copies of stage st landed
    __syncthreads();                // everyone's did; stage st-1 is consumed
    issue(st + kStages - 1);        // refill the buffer stage st-1 used
    const float* buf = smem + (st % kStages) * stage_floats;
    const int rows = (int)min((size_t)R, len - st * R);
    if (tid < w_eff)
      fold_pipelined(buf + tid, W, rows, [&](float v) {
        if (OP == kDimMax) {
          nan |= v != v;
          acc = fmaxf(acc, v);
        } else {
          acc = fadd(acc, v);
        }
      });
  }
  cp_async_wait<0>();
  if (tid < w_eff) {
    if (OP == kDimMax && (nan || acc == 0.0f)) {
      const float* col = src + tid;
      float m = col[0];
      for (size_t l = 1; l < len; l++) m = max_fold(m, col[l * inner]);
      acc = m;
    }
    if (OP == kDimMean) acc = fdiv(acc, (float)len);
    out[o * inner + c0 + tid] = acc;
  }
}

// ------------------------------------------------ last-axis sum, staged
// The same eight sequential chains per lane as lane_sum8_kernel, but the
// lanes' bytes arrive through a cp.async ring: a CTA owns kLsRows lanes and
// streams their columns kLsCols at a time (rows padded by 8 floats so the
// 8 x kLsRows chain threads read shared memory without bank conflicts).
// Needs len % 4 == 0 and a 16-byte-aligned base.
constexpr int kLsRows = 4;
constexpr int kLsCols = 256;
constexpr int kLsPitch = kLsCols + 8;
constexpr int kLsThreads = 64;
constexpr int kLsSlots = kLsRows * (kLsCols / 4) / kLsThreads;   // 4 chunks per thread

// kLsStages-deep ring (3 to 6 stages; the launcher picks the deepest whose
// CTAs all fit on the GPU at once, since each CTA's lanes take equally long).
template <int kLsStages>
__global__ void __launch_bounds__(kLsThreads)
lane_sum8_staged_kernel(const float* x, size_t lanes, size_t len, float* out, int mean) {
  __shared__ __align__(16) float smem[kLsStages][kLsRows][kLsPitch];
  const size_t lane0 = (size_t)blockIdx.x * kLsRows;
  const int rows = (int)min((size_t)kLsRows, lanes - lane0);
  const size_t nstage = (len + kLsCols - 1) / kLsCols;
  const int tid = threadIdx.x;
  int slot_r[kLsSlots], slot_c[kLsSlots];
#pragma unroll
  for (int q = 0; q < kLsSlots; q++) {
    const int t = tid + q * kLsThreads;
    slot_r[q] = t / (kLsCols / 4);
    slot_c[q] = 4 * (t % (kLsCols / 4));
  }
  auto issue = [&](size_t st) {
    if (st < nstage) {
      const size_t col0 = st * kLsCols;
      const int cw = (int)min((size_t)kLsCols, len - col0);
#pragma unroll
      for (int q = 0; q < kLsSlots; q++)
        if (slot_r[q] < rows && slot_c[q] < cw)
          cp_async16(&smem[st % kLsStages][slot_r[q]][slot_c[q]],
                     x + (lane0 + slot_r[q]) * len + col0 + slot_c[q]);
    }
    cp_async_commit();
  };
  for (int st = 0; st < kLsStages - 1; st++) issue(st);

  const int r = tid >> 3, j = tid & 7;          // chain j of lane r (warp 0 only)
  const bool chain = tid < kLsRows * 8 && r < rows;
  const size_t steps = len / 8;                 // full groups of eight
  float p = 0.0f;
  for (size_t st = 0; st < nstage; st++) {
    cp_async_wait<kLsStages - 2>();
    __syncthreads();
    issue(st + kLsStages - 1);
    if (chain) {
      const size_t g0 = st * (kLsCols / 8);     // first group of this stage
      const int ng = (int)min((size_t)(kLsCols / 8), steps > g0 ? steps - g0 : 0);
      fold_pipelined(&smem[st % kLsStages][r][j], 8, ng, [&](float v) { p = fadd(p, v); });
    }
  }
  cp_async_wait<0>();
  if (tid < 32) {
    float q[8];
#pragma unroll
    for (int t = 0; t < 8; t++) q[t] = __shfl_sync(0xffffffffu, p, (tid & 24) + t);
    if (chain && j == 0) {
      float acc = 0.0f;
      acc = fadd(acc, fadd(q[0], q[4]));
      acc = fadd(acc, fadd(q[1], q[5]));
      acc = fadd(acc, fadd(q[2], q[6]));
      acc = fadd(acc, fadd(q[3], q[7]));
      const float* lp = x + (lane0 + r) * len;
      for (size_t t = steps * 8; t < len; t++) acc = fadd(acc, lp[t]);
      if (mean) acc = fdiv(acc, (float)len);
      out[lane0 + r] = acc;
    }
  }
}

// ------------------------------------------------ last-axis sum, one chain
// Each lane summed as ONE sequential f32 chain from 0.0, x[0] + x[1] + ...
// in order (autograd's reduce_to_shape row sums, autograd/ops.rs:650-656;
// ndarray's sum_axis over a non-last axis whose later axes all have length 1,
// reduction.rs:86, activation.rs:127).
// A CTA owns kLcRows lanes whose columns stream through a cp.async ring
// kLcCols at a time; thread r of the first warp runs lane r's chain out of
// shared memory.  Rows are padded to 68 floats so the chain threads' 16-byte
// reads hit distinct banks.  Needs len % 4 == 0 and a 16-byte-aligned base.
constexpr int kLcRows = 16;
constexpr int kLcCols = 64;
constexpr int kLcPitch = kLcCols + 4;
constexpr int kLcStages = 6;       // 26 KB: 8 CTAs (128 chains) per SM
constexpr int kLcThreads = 64;
constexpr int kLcSlots = kLcRows * (kLcCols / 4) / kLcThreads;   // 4 chunks per thread

__global__ void __launch_bounds__(kLcThreads)
lane_chain_sum_kernel(const float* x, size_t lanes, size_t len, float* out, bool mean) {
  __shared__ __align__(16) float smem[kLcStages][kLcRows][kLcPitch];
  const size_t lane0 = (size_t)blockIdx.x * kLcRows;
  const int rows = (int)min((size_t)kLcRows, lanes - lane0);
  const size_t nstage = (len + kLcCols - 1) / kLcCols;
  const int tid = threadIdx.x;
  int slot_r[kLcSlots], slot_c[kLcSlots];
#pragma unroll
  for (int q = 0; q < kLcSlots; q++) {
    const int t = tid + q * kLcThreads;
    slot_r[q] = t / (kLcCols / 4);
    slot_c[q] = 4 * (t % (kLcCols / 4));
  }
  auto issue = [&](size_t st) {
    if (st < nstage) {
      const size_t col0 = st * kLcCols;
      const int cw = (int)min((size_t)kLcCols, len - col0);
#pragma unroll
      for (int q = 0; q < kLcSlots; q++)
        if (slot_r[q] < rows && slot_c[q] < cw)
          cp_async16(&smem[st % kLcStages][slot_r[q]][slot_c[q]],
                     x + (lane0 + slot_r[q]) * len + col0 + slot_c[q]);
    }
    cp_async_commit();
  };
  for (int st = 0; st < kLcStages - 1; st++) issue(st);

  const bool chain = tid < rows;
  float acc = 0.0f;
  for (size_t st = 0; st < nstage; st++) {
    cp_async_wait<kLcStages - 2>();
    __syncthreads();
    issue(st + kLcStages - 1);
    if (chain) {
      const int n4 = (int)min((size_t)kLcCols, len - st * kLcCols) / 4;
      const float4* row = reinterpret_cast<const float4*>(&smem[st % kLcStages][tid][0]);
      // 16-byte reads, two groups of four ahead of the chain
      int c = 0;
      if (n4 >= 2) {
        float4 cur0 = row[0], cur1 = row[1];
        for (c = 2; c + 2 <= n4; c += 2) {
          const float4 nxt0 = row[c], nxt1 = row[c + 1];
          acc = fadd(fadd(fadd(fadd(acc, cur0.x), cur0.y), cur0.z), cur0.w);
          acc = fadd(fadd(fadd(fadd(acc, cur1.x), cur1.y), cur1.z), cur1.w);
          cur0 = nxt0;
          cur1 = nxt1;
        }
        acc = fadd(fadd(fadd(fadd(acc, cur0.x), cur0.y), cur0.z), cur0.w);
        acc = fadd(fadd(fadd(fadd(acc, cur1.x), cur1.y), cur1.z), cur1.w);
      }
      for (; c < n4; c++) {
        const float4 v = row[c];
        acc = fadd(fadd(fadd(fadd(acc, v.x), v.y), v.z), v.w);
      }
    }
  }
  cp_async_wait<0>();
  if (chain) out[lane0 + tid] = mean ? fdiv(acc, (float)len) : acc;
}

// out[i] /= (f32)len: the mean of lanes whose chains the ordered-sum kernels
// summed.
__global__ void div_by_len_kernel(float* out, size_t lanes, size_t len) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < lanes) out[i] = fdiv(out[i], (float)len);
}

// ------------------------------------------------ last-axis sum, 4 lanes per warp
// Four lanes (rows) per warp, each read front to back with 16-byte loads; the
// same eight ordered chains per row (ndarray's unrolled_fold), but all
// 32 threads run chains (thread 8r + j runs chain j of the warp's row r), so
// a chain step costs one warp instruction for 32 chains instead of 8.  Each
// tile step stages 128 floats of every row through a per-warp shared buffer
// (row pitch 136 floats: the four rows' chains read distinct banks), with the
// next kLqAhead tiles' 16-byte loads in flight in registers.  Only
// __syncwarp couples the threads.  Needs len % 4 == 0 and a 16-byte-aligned
// base.
// WARPS warps per CTA: small CTAs spread the warps evenly over the SMs (with
// 8-warp CTAs, cfg3's 256 CTAs put two on 108 SMs and one on the other 40,
// and the kernel waits for the busier SMs).
constexpr int kLqWarps = 2;
constexpr int kLqTile = 128;     // floats of each row per tile step
constexpr int kLqPitch = kLqTile + 8;
constexpr int kLqAhead = 4;

template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
lane_sum8_quad_kernel(const float* x, size_t lanes, size_t len, float* out, int mean) {
  __shared__ __align__(16) float tile_buf[WARPS][4 * kLqPitch];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t r0 = ((size_t)blockIdx.x * WARPS + warp) * 4;
  if (r0 >= lanes) return;                             // whole warp leaves together
  float* buf = tile_buf[warp];
  const size_t steps = len / 8;                        // chain steps per row
  const size_t ntiles = (8 * steps + kLqTile - 1) / kLqTile;
  const size_t n4 = len / 4;
  auto load = [&](size_t t, float4* v) {
    const size_t c = t * (kLqTile / 4) + lane;         // float4 index in each row
#pragma unroll
    for (int rr = 0; rr < 4; rr++) {
      const size_t row = r0 + rr;
      v[rr] = (c < n4 && row < lanes) ? __ldcs(reinterpret_cast<const float4*>(x + row * len) + c)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float4 pre[kLqAhead][4];
#pragma unroll
  for (int d = 0; d < kLqAhead; d++) load(d, pre[d]);
  const int rr = lane >> 3, j = lane & 7;
  const float* chain = buf + rr * kLqPitch + j;
  float p = 0.0f;
  for (size_t t0 = 0; t0 < ntiles; t0 += kLqAhead) {
#pragma unroll
    for (int d = 0; d < kLqAhead; d++) {
      const size_t t = t0 + d;
      if (t < ntiles) {
#pragma unroll
        for (int q = 0; q < 4; q++) reinterpret_cast<float4*>(buf + q * kLqPitch)[lane] = pre[d][q];
        load(t + kLqAhead, pre[d]);
        __syncwarp();
        const int n = (int)min((size_t)(kLqTile / 8), steps - t * (kLqTile / 8));
        fold_pipelined(chain, 8, n, [&](float v) { p = fadd(p, v); });
        __syncwarp();
      }
    }
  }
  float q[8];
#pragma unroll
  for (int k = 0; k < 8; k++) q[k] = __shfl_sync(0xffffffffu, p, (lane & ~7) + k);
  const size_t row = r0 + rr;
  if (j == 0 && row < lanes) {
    float acc = 0.0f;
    acc = fadd(acc, fadd(q[0], q[4]));
    acc = fadd(acc, fadd(q[1], q[5]));
    acc = fadd(acc, fadd(q[2], q[6]));
    acc = fadd(acc, fadd(q[3], q[7]));
    const float* xr = x + row * len;
    for (size_t t = steps * 8; t < len; t++) acc = fadd(acc, xr[t]);
    if (mean) acc = fdiv(acc, (float)len);
    out[row] = acc;
  }
}

// ------------------------------------------ last-axis sum, chains read directly
// The same eight chains per row as above, each run by one thread, but every
// chain reads its own floats straight from global memory: with CPT chains
// per thread (1, 2 or 4 adjacent chains, read together as a float, float2 or
// float4 at x[8k + CPT*j]), 8/CPT threads cover a row and read 32
// consecutive bytes of it per step, so no byte is fetched twice and nothing
// passes through shared memory; a warp holds 32*CPT/8 rows.  K loads per
// thread are in flight while the previous K are added (double-buffered
// registers), ~2 instructions per element instead of the staged kernel's
// ~13.  CPT > 1 needs rows aligned to 4*CPT bytes.
template <int CPT>
struct ChainVec;
template <>
struct ChainVec<1> {
  using T = float;
  __device__ static float get(const T& v, int) { return v; }
};
template <>
struct ChainVec<2> {
  using T = float2;
  __device__ static float get(const T& v, int c) { return c ? v.y : v.x; }
};
template <>
struct ChainVec<4> {
  using T = float4;
  __device__ static float get(const T& v, int c) {
    return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
  }
};

template <int WARPS, int K, int CPT>
__global__ void __launch_bounds__(WARPS * 32)
lane_sum8_direct_kernel(const float* x, size_t lanes, size_t len, float* out, int mean) {
  using V = typename ChainVec<CPT>::T;
  constexpr int TPR = 8 / CPT, RPW = 32 / TPR;      // threads per row, rows per warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t r0 = ((size_t)blockIdx.x * WARPS + warp) * RPW;
  if (r0 >= lanes) return;                             // whole warp leaves together
  const int rr = lane / TPR, j = lane % TPR;
  const size_t row = r0 + rr;
  const bool live = row < lanes;
  const float* xr = x + (live ? row : r0) * len;       // idle lanes reread row r0
  const V* p = reinterpret_cast<const V*>(xr + CPT * j);
  constexpr int kStep = 8 / CPT;                       // V elements per chain step
  const size_t steps = len / 8;                        // chain steps per row
  float acc[CPT];
#pragma unroll
  for (int c = 0; c < CPT; c++) acc[c] = 0.0f;
  auto add = [&](const V& v) {
#pragma unroll
    for (int c = 0; c < CPT; c++) acc[c] = fadd(acc[c], ChainVec<CPT>::get(v, c));
  };
  size_t k = 0;
  if (steps >= (size_t)K) {
    V cur[K];
#pragma unroll
    for (int u = 0; u < K; u++) cur[u] = __ldcs(p + kStep * u);
    p += kStep * K;
    for (k = K; k + K <= steps; k += K) {
      V nxt[K];
#pragma unroll
      for (int u = 0; u < K; u++) nxt[u] = __ldcs(p + kStep * u);
      p += kStep * K;
#pragma unroll
      for (int u = 0; u < K; u++) add(cur[u]);
#pragma unroll
      for (int u = 0; u < K; u++) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < K; u++) add(cur[u]);
  }
  for (; k < steps; k++, p += kStep) add(__ldcs(p));
  float q[8];
#pragma unroll
  for (int t = 0; t < TPR; t++)
#pragma unroll
    for (int c = 0; c < CPT; c++)
      q[t * CPT + c] = __shfl_sync(0xffffffffu, acc[c], (lane & ~(TPR - 1)) + t);
  if (j == 0 && live) {
    float r = 0.0f;
    r = fadd(r, fadd(q[0], q[4]));
    r = fadd(r, fadd(q[1], q[5]));
    r = fadd(r, fadd(q[2], q[6]));
    r = fadd(r, fadd(q[3], q[7]));
    for (size_t t = steps * 8; t < len; t++) r = fadd(r, xr[t]);
    if (mean) r = fdiv(r, (float)len);
    out[row] = r;
  }
}

// ---------------------------- last-axis sum, 128-byte row reads + transpose
// Four rows per warp, one thread per ndarray chain, as lane_sum8_direct, but
// the eight threads of a row read 128 contiguous bytes per load instruction
// (a float4 each: 32 floats = four chain steps of all eight chains) instead
// of 32.  Thread (q, g) of a row (sub-lane 2q + g) loads floats 4(2q+g) ..+3,
// i.e. step 4s + q of chains 4g..4g+3; a 4x4 transpose among the four
// threads of each g (two butterfly levels of two shuffles each) leaves
// thread (q, g) holding steps 4s..4s+3 of chain 4g + q, which it adds in
// order.  Needs len % 32 == 0 and 16-byte-aligned rows.
__device__ __forceinline__ void transpose4(float v[4], unsigned q) {
#pragma unroll
  for (int b = 1; b <= 2; b <<= 1) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
      if (c & b) continue;
      const bool hi = (q & (unsigned)b) != 0;
      const float send = hi ? v[c] : v[c ^ b];
      const float got = __shfl_xor_sync(0xffffffffu, send, 2 * b);
      if (hi) v[c] = got;
      else v[c ^ b] = got;
    }
  }
}

template <int WARPS, int K>
__global__ void __launch_bounds__(WARPS * 32)
lane_sum8_tr_kernel(const float* x, size_t lanes, size_t len, float* out, int mean) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t r0 = ((size_t)blockIdx.x * WARPS + warp) * 4;
  if (r0 >= lanes) return;                             // whole warp leaves together
  const int rr = lane >> 3, sub = lane & 7;
  const unsigned q = (unsigned)sub >> 1, g = (unsigned)sub & 1u;
  const size_t row = r0 + rr;
  const bool live = row < lanes;
  const float4* p = reinterpret_cast<const float4*>(x + (live ? row : r0) * len) + sub;
  const size_t segs = len / 32;                        // 32-float segments per row
  float acc = 0.0f;
  auto add = [&](float4 f) {
    float v[4] = {f.x, f.y, f.z, f.w};
    transpose4(v, q);
#pragma unroll
    for (int c = 0; c < 4; c++) acc = fadd(acc, v[c]);
  };
  size_t k = 0;
  if (segs >= (size_t)K) {
    float4 cur[K];
#pragma unroll
    for (int u = 0; u < K; u++) cur[u] = __ldcs(p + 8 * u);
    p += 8 * K;
    for (k = K; k + K <= segs; k += K) {
      float4 nxt[K];
#pragma unroll
      for (int u = 0; u < K; u++) nxt[u] = __ldcs(p + 8 * u);
      p += 8 * K;
#pragma unroll
      for (int u = 0; u < K; u++) add(cur[u]);
#pragma unroll
      for (int u = 0; u < K; u++) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < K; u++) add(cur[u]);
  }
  for (; k < segs; k++, p += 8) add(__ldcs(p));
  // thread (q, g) holds chain 4g + q; gather the row's eight chains
  const int base = lane & ~7;
  float pch[8];
#pragma unroll
  for (int c = 0; c < 8; c++) pch[c] = __shfl_sync(0xffffffffu, acc, base + 2 * (c & 3) + (c >> 2));
  if (sub == 0 && live) {
    float r = 0.0f;
    r = fadd(r, fadd(pch[0], pch[4]));
    r = fadd(r, fadd(pch[1], pch[5]));
    r = fadd(r, fadd(pch[2], pch[6]));
    r = fadd(r, fadd(pch[3], pch[7]));
    if (mean) r = fdiv(r, (float)len);
    out[row] = r;
  }
  (void)g;
}

template <int WARPS, int K>
void launch_lane_tr_w(const float* x, size_t lanes, size_t len, float* out, bool mean,
                      cudaStream_t s) {
  const size_t per_cta = (size_t)WARPS * 4;
  const size_t grid = (lanes + per_cta - 1) / per_cta;
  for (size_t g0 = 0; g0 < grid; g0 += 0x7fffffffull) {
    const size_t ng = std::min<size_t>(grid - g0, 0x7fffffffull);
    lane_sum8_tr_kernel<WARPS, K><<<(unsigned)ng, WARPS * 32, 0, s>>>(
        x + g0 * per_cta * len, lanes - g0 * per_cta, len, out + g0 * per_cta, mean);
  }
}

template <int WARPS, int K, int CPT = 1>
void launch_lane_direct_w(const float* x, size_t lanes, size_t len, float* out, bool mean,
                          cudaStream_t s) {
  const size_t per_cta = (size_t)WARPS * (32 * CPT / 8);      // rows
  const size_t grid = (lanes + per_cta - 1) / per_cta;
  for (size_t g0 = 0; g0 < grid; g0 += 0x7fffffffull) {
    const size_t ng = std::min<size_t>(grid - g0, 0x7fffffffull);
    lane_sum8_direct_kernel<WARPS, K, CPT><<<(unsigned)ng, WARPS * 32, 0, s>>>(
        x + g0 * per_cta * len, lanes - g0 * per_cta, len, out + g0 * per_cta, mean);
  }
}

template <int WARPS>
void launch_lane_quad_w(const float* x, size_t lanes, size_t len, float* out, bool mean,
                        cudaStream_t s) {
  const size_t per_cta = (size_t)WARPS * 4;      // rows
  const size_t grid = (lanes + per_cta - 1) / per_cta;
  for (size_t g0 = 0; g0 < grid; g0 += 0x7fffffffull) {
    const size_t ng = std::min<size_t>(grid - g0, 0x7fffffffull);
    lane_sum8_quad_kernel<WARPS><<<(unsigned)ng, WARPS * 32, 0, s>>>(
        x + g0 * per_cta * len, lanes - g0 * per_cta, len, out + g0 * per_cta, mean);
  }
}

cudaError_t launch_lane_quad(int warps, const float* x, size_t lanes, size_t len, float* out,
                             bool mean, cudaStream_t s) {
  switch (warps) {
    case 1: launch_lane_quad_w<1>(x, lanes, len, out, mean, s); break;
    case 2: launch_lane_quad_w<2>(x, lanes, len, out, mean, s); break;
    case 4: launch_lane_quad_w<4>(x, lanes, len, out, mean, s); break;
    case 8: launch_lane_quad_w<8>(x, lanes, len, out, mean, s); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Any layout: one thread per output, sequential over len (row order).
template <int OP>
__global__ void __launch_bounds__(kThreads)
lane_generic_kernel(const float* x, size_t outer, size_t len, size_t inner, float* out) {
  const size_t lanes = outer * inner;
  for (size_t t = (size_t)blockIdx.x * kThreads + threadIdx.x; t < lanes;
       t += (size_t)gridDim.x * kThreads) {
    const size_t o = t / inner, i = t % inner;
    const float* p = x + o * len * inner + i;
    float acc;
    size_t l = 0;
    if (OP == kDimMax) {
      acc = p[0];
      l = 1;
    } else {
      acc = 0.0f;
    }
    for (; l < len; l++) {
      const float v = p[l * inner];
      acc = (OP == kDimMax) ? max_fold(acc, v) : fadd(acc, v);
    }
    if (OP == kDimMean) acc = fdiv(acc, (float)len);
    out[t] = acc;
  }
}

int cur_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

template <int OP>
cudaError_t strip_launch(const float* x, size_t outer, size_t len, size_t inner, float* out,
                         cudaStream_t st) {
  const int sms = sm_count(cur_device());
  const size_t target = (size_t)sms * 2;
  const size_t per_outer = std::max<size_t>(1, (target + outer - 1) / outer);
  size_t W = (inner + per_outer - 1) / per_outer;
  W = (W + 3) & ~size_t(3);
  W = std::min<size_t>(std::max<size_t>(W, 32), kStripMaxW);
  W = std::min(W, (inner + 3) & ~size_t(3));
  const size_t strips = (inner + W - 1) / W;
  const int threads = (int)std::max<size_t>(128, (W + 31) & ~size_t(31));
  int R = (int)(kStripSmem / ((size_t)kStages * W * sizeof(float)));
  R = std::max(1, std::min(R, 64));
  // every chunk of a stage needs a copy slot
  while (R > 1 && (size_t)R * (W / 4) > (size_t)threads * kStripSlots) R--;
  const size_t smem = (size_t)kStages * R * W * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(strip_reduce_kernel<OP>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  strip_reduce_kernel<OP><<<(unsigned)(outer * strips), threads, smem, st>>>(
      x, len, inner, (int)W, R, strips, out);
  return cudaGetLastError();
}

// The global statistics run stats_gs_kernel<256, 4> with 8 blocks per SM
// (more than stay resident at once; the grid stride keeps every block's
// share equal): 0.99-1.00 of the measured copy bandwidth at cfg2, where the
// one-contiguous-range-per-block stats_kernel reached 0.86-0.89 in every
// shape (bench.py --probe).
constexpr int kStatsGsThreads = 256, kStatsGsU = 4, kStatsGsBlocksPerSm = 8;

template <int NT, int U, bool T>
int stats_resident(int device) {
  static int cached[64] = {0};
  if (device >= 0 && device < 64 && cached[device]) return cached[device];
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, stats_kernel<NT, U, T>, NT, 0) !=
          cudaSuccess || n < 1)
    n = 1;
  if (device >= 0 && device < 64) cached[device] = n;
  return n;
}

template <int NT, int U, bool T>
cudaError_t launch_stats_shape(const float* x, size_t n, StatsPart* parts, int nparts,
                               StatsPart* out, cudaStream_t s, double* sum_out,
                               bool combine = true) {
  const size_t chunk = (n + (size_t)nparts - 1) / (size_t)nparts;
  stats_kernel<NT, U, T><<<nparts, NT, 0, s>>>(x, n, chunk ? chunk : 1, parts);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !combine) return e;
  stats_final_kernel<<<1, kStatsThreads, 0, s>>>(parts, nparts, out, sum_out);
  return cudaGetLastError();
}

}  // namespace

int stats_max_parts(int device) { return sm_count(device) * kStatsGsBlocksPerSm; }

int stats_num_parts(int device, size_t n) {
  // At least ~16K elements per block so that small inputs use few blocks.
  const size_t want = (n + 16383) / 16384;
  return (int)std::max<size_t>(1, std::min<size_t>(want, (size_t)stats_max_parts(device)));
}

cudaError_t launch_stats(const float* x, size_t n, StatsPart* parts, int nparts, StatsPart* out,
                         cudaStream_t s, double* sum_out) {
  stats_gs_kernel<kStatsGsThreads, kStatsGsU><<<nparts, kStatsGsThreads, 0, s>>>(x, n, parts);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  stats_final_kernel<<<1, kStatsThreads, 0, s>>>(parts, nparts, out, sum_out);
  return cudaGetLastError();
}

cudaError_t launch_lane_sum_variant(int warps, const float* x, size_t lanes, size_t len,
                                    float* out, cudaStream_t s) {
  // warps >= 100: the 128-byte-read transpose kernel, warps = 100*K + warps per CTA
  if (warps >= 100) {
    const int K = warps / 100, w = warps % 100;
    if (len % 32 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) != 0) return cudaErrorInvalidValue;
    if (K == 8 && w == 2) launch_lane_tr_w<2, 8>(x, lanes, len, out, false, s);
    else if (K == 8 && w == 4) launch_lane_tr_w<4, 8>(x, lanes, len, out, false, s);
    else if (K == 8 && w == 8) launch_lane_tr_w<8, 8>(x, lanes, len, out, false, s);
    else if (K == 12 && w == 2) launch_lane_tr_w<2, 12>(x, lanes, len, out, false, s);
    else if (K == 12 && w == 4) launch_lane_tr_w<4, 12>(x, lanes, len, out, false, s);
    else if (K == 16 && w == 2) launch_lane_tr_w<2, 16>(x, lanes, len, out, false, s);
    else if (K == 16 && w == 1) launch_lane_tr_w<1, 16>(x, lanes, len, out, false, s);
    else if (K == 16 && w == 4) launch_lane_tr_w<4, 16>(x, lanes, len, out, false, s);
    else if (K == 16 && w == 8) launch_lane_tr_w<8, 16>(x, lanes, len, out, false, s);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
  }
  // warps < 0: the direct kernel with -warps = 1000*CPT + 10*K + warps per CTA
  if (warps < 0) {
    const int code = -warps, cpt = code / 1000, K = (code / 10) % 100, w = code % 10;
    if (len < 8 || (cpt > 1 && ((reinterpret_cast<uintptr_t>(x) | len * 4) % (4 * cpt)) != 0))
      return cudaErrorInvalidValue;
    if (cpt == 1 && K == 32 && w == 2) launch_lane_direct_w<2, 32, 1>(x, lanes, len, out, false, s);
    else if (cpt == 2 && K == 16 && w == 2) launch_lane_direct_w<2, 16, 2>(x, lanes, len, out, false, s);
    else if (cpt == 2 && K == 32 && w == 2) launch_lane_direct_w<2, 32, 2>(x, lanes, len, out, false, s);
    else if (cpt == 2 && K == 24 && w == 2) launch_lane_direct_w<2, 24, 2>(x, lanes, len, out, false, s);
    else if (cpt == 2 && K == 32 && w == 1) launch_lane_direct_w<1, 32, 2>(x, lanes, len, out, false, s);
    else if (cpt == 2 && K == 32 && w == 4) launch_lane_direct_w<4, 32, 2>(x, lanes, len, out, false, s);
    else if (cpt == 1 && K == 48 && w == 2) launch_lane_direct_w<2, 48, 1>(x, lanes, len, out, false, s);
    else if (cpt == 4 && K == 8 && w == 2) launch_lane_direct_w<2, 8, 4>(x, lanes, len, out, false, s);
    else if (cpt == 4 && K == 16 && w == 1) launch_lane_direct_w<1, 16, 4>(x, lanes, len, out, false, s);
    else if (cpt == 4 && K == 16 && w == 2) launch_lane_direct_w<2, 16, 4>(x, lanes, len, out, false, s);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
  }
  if (len % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) != 0) return cudaErrorInvalidValue;
  return launch_lane_quad(warps, x, lanes, len, out, false, s);
}

cudaError_t launch_stats_variant(int threads, int u, int blocks_per_sm, const float* x, size_t n,
                                 StatsPart* parts, int max_parts, cudaStream_t s,
                                 double* sum_out) {
  const int dev = cur_device();
  const size_t want = (n + 16383) / 16384;
  // u < 0: float32 trees per float4 (sum4<true>) with |u| loads in flight;
  // threads < 0: the partials only, without the combining kernel
  const bool combine = threads > 0;
  if (threads < 0) threads = -threads;
  const bool tree = u < 0;
  const int uu = tree ? -u : u;
#define RT_STATS_VARIANT(NT, UU, T)                                                       \
  if (threads == NT && uu == UU && tree == T) {                                           \
    const int per = blocks_per_sm > 0 ? blocks_per_sm : stats_resident<NT, UU, T>(dev);   \
    const int np = (int)std::max<size_t>(                                                 \
        1, std::min<size_t>(want, std::min<size_t>((size_t)per * sm_count(dev), max_parts))); \
    return launch_stats_shape<NT, UU, T>(x, n, parts, np, nullptr, s, sum_out, combine);  \
  }
  RT_STATS_VARIANT(256, 8, false)
  RT_STATS_VARIANT(512, 4, false)
  RT_STATS_VARIANT(512, 8, false)
  RT_STATS_VARIANT(256, 4, true)
  RT_STATS_VARIANT(256, 8, true)
  RT_STATS_VARIANT(512, 4, true)
  RT_STATS_VARIANT(512, 8, true)
  RT_STATS_VARIANT(1024, 4, true)
#undef RT_STATS_VARIANT
  return cudaErrorInvalidValue;
}

// The grid-stride, pipelined kernel: `threads` 256/512, `u` 2/4, blocks per
// SM as given (0: all that stay resident).
cudaError_t launch_stats_gs_variant(int threads, int u, int blocks_per_sm, const float* x,
                                    size_t n, StatsPart* parts, int max_parts, cudaStream_t s,
                                    double* sum_out) {
  const int dev = cur_device();
#define RT_STATS_GS(NT, UU)                                                                 \
  if (threads == NT && u == UU) {                                                           \
    int per = blocks_per_sm;                                                                \
    if (per <= 0 &&                                                                         \
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, stats_gs_kernel<NT, UU>, NT, 0) != \
            cudaSuccess)                                                                    \
      per = 1;                                                                              \
    const int np = std::max(1, std::min(per * sm_count(dev), max_parts));                   \
    stats_gs_kernel<NT, UU><<<np, NT, 0, s>>>(x, n, parts);                                 \
    cudaError_t e = cudaGetLastError();                                                     \
    if (e != cudaSuccess) return e;                                                         \
    stats_final_kernel<<<1, kStatsThreads, 0, s>>>(parts, np, nullptr, sum_out);            \
    return cudaGetLastError();                                                              \
  }
  RT_STATS_GS(256, 2)
  RT_STATS_GS(256, 4)
  RT_STATS_GS(512, 2)
  RT_STATS_GS(512, 4)
#undef RT_STATS_GS
  return cudaErrorInvalidValue;
}

cudaError_t launch_index_scan(const float* x, size_t n, IndexScan* out, cudaStream_t s) {
  index_scan_init<<<1, 1, 0, s>>>(out);
  const size_t want = (n + kThreads - 1) / kThreads;
  const unsigned grid =
      (unsigned)std::max<size_t>(1, std::min<size_t>(want, (size_t)sm_count(cur_device()) * 8));
  index_scan_kernel<<<grid, kThreads, 0, s>>>(x, n, out);
  return cudaGetLastError();
}

cudaError_t launch_reduce_dim(DimReduce op, const float* x, size_t outer, size_t len,
                              size_t inner, bool last_axis, float* out, cudaStream_t s) {
  const size_t lanes = outer * inner;
  if (lanes == 0) return cudaSuccess;
  if (inner == 1 && !last_axis && op != kDimMax)
    return launch_lane_chain_sum(x, lanes, len, out, s, op == kDimMean);
  if (inner == 1) {
    if (op == kDimMax) {
      const unsigned grid = (unsigned)((lanes + 7) / 8);
      lane_max_kernel<<<grid, kWarpLaneThreads, 0, s>>>(x, lanes, len, out);
    } else if (len >= 1024 && lanes >= (size_t)sm_count(cur_device()) * 28) {
      // enough lanes for ~7 warps per SM (fewer leave the warp kernel
      // under-occupied; the staged kernel below spreads 4 lanes per CTA):
      // the chains read straight from global memory.  Rows of whole
      // 128-byte segments on 16-byte boundaries: eight threads per row,
      // 16-byte loads and a 4x4 shuffle transpose, 16 loads in flight per
      // thread, 8 warps per CTA (0.85-0.86 of the measured bandwidth at
      // cfg3 for one launch, 0.89 for launches back to back).  Else two
      // adjacent chains per thread (float2 loads) when the rows are 8-byte
      // aligned (0.81-0.83), else one (0.80).  Four chains per thread reach
      // 0.59, the shared-memory-staged lane_sum8_quad_kernel 0.74-0.75 and
      // rows streamed through a cp.async.bulk ring 0.665 (bench.py --probe)
      if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && len % 32 == 0)
        launch_lane_tr_w<8, 16>(x, lanes, len, out, op == kDimMean, s);
      else if ((reinterpret_cast<uintptr_t>(x) & 7u) == 0 && len % 2 == 0)
        launch_lane_direct_w<2, 32, 2>(x, lanes, len, out, op == kDimMean, s);
      else
        launch_lane_direct_w<2, 32, 1>(x, lanes, len, out, op == kDimMean, s);
    } else if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && len % 4 == 0 && len >= 64) {
      const size_t grid = (lanes + kLsRows - 1) / kLsRows;
      // deepest ring whose CTAs are all resident in one wave (else 4)
      const size_t sms = (size_t)sm_count(cur_device());
      auto slots = [&](int stages) {
        const size_t smem = (size_t)stages * kLsRows * kLsPitch * sizeof(float) + 1024;
        return sms * std::min<size_t>((227u << 10) / smem, 2048 / kLsThreads);
      };
      int stages = 4;
      for (int c = 6; c >= 3; c--)
        if (grid <= slots(c)) {
          stages = c;
          break;
        }
      for (size_t g0 = 0; g0 < grid; g0 += 0x7fffffffull) {
        const size_t ng = std::min<size_t>(grid - g0, 0x7fffffffull);
        const float* xs = x + g0 * kLsRows * len;
        float* os = out + g0 * kLsRows;
        const size_t nl = lanes - g0 * kLsRows;
        switch (stages) {
          case 3: lane_sum8_staged_kernel<3><<<(unsigned)ng, kLsThreads, 0, s>>>(xs, nl, len, os, op == kDimMean); break;
          case 5: lane_sum8_staged_kernel<5><<<(unsigned)ng, kLsThreads, 0, s>>>(xs, nl, len, os, op == kDimMean); break;
          case 6: lane_sum8_staged_kernel<6><<<(unsigned)ng, kLsThreads, 0, s>>>(xs, nl, len, os, op == kDimMean); break;
          default: lane_sum8_staged_kernel<4><<<(unsigned)ng, kLsThreads, 0, s>>>(xs, nl, len, os, op == kDimMean); break;
        }
      }
    } else {
      const unsigned grid = (unsigned)((lanes + 7) / 8);
      lane_sum8_kernel<<<grid, kLaneThreads, 0, s>>>(x, lanes, len, out, op == kDimMean);
    }
    return cudaGetLastError();
  }
  {
    bool used = false;
    const cudaError_t e = launch_strip_tma(op, x, outer, len, inner, out, s, &used);
    if (e != cudaSuccess || used) return e;
  }
  const bool strip_ok = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && inner % 4 == 0 &&
                        inner >= 32 && len >= 1;
  if (strip_ok) {
    switch (op) {
      case kDimSum: return strip_launch<kDimSum>(x, outer, len, inner, out, s);
      case kDimMean: return strip_launch<kDimMean>(x, outer, len, inner, out, s);
      case kDimMax: return strip_launch<kDimMax>(x, outer, len, inner, out, s);
    }
  }
  const unsigned grid = (unsigned)std::max<size_t>(
      1, std::min<size_t>((lanes + kThreads - 1) / kThreads, (size_t)sm_count(cur_device()) * 8));
  switch (op) {
    case kDimSum: lane_generic_kernel<kDimSum><<<grid, kThreads, 0, s>>>(x, outer, len, inner, out); break;
    case kDimMean: lane_generic_kernel<kDimMean><<<grid, kThreads, 0, s>>>(x, outer, len, inner, out); break;
    case kDimMax: lane_generic_kernel<kDimMax><<<grid, kThreads, 0, s>>>(x, outer, len, inner, out); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_lane_chain_sum(const float* x, size_t lanes, size_t len, float* out,
                                  cudaStream_t s, bool mean) {
  if (lanes == 0) return cudaSuccess;
  if (len >= (size_t{1} << 18) && lanes <= (len >> 16)) {
    // Few long lanes: one thread per chain would take len dependent adds
    // (~2.6 ns each); the ordered-sum kernels reproduce the same chain with
    // every SM working on one lane at a time.
    const size_t bytes = ordered_sum_scratch_bytes(len, 1);
    void* scratch = nullptr;
    cudaError_t e = cudaMallocAsync(&scratch, bytes, s);
    if (e != cudaSuccess) return e;
    for (size_t l = 0; l < lanes && e == cudaSuccess; l++)
      e = launch_ordered_sum_of(x + l * len, len, 1, 0.0f, scratch, out + l, s);
    if (e == cudaSuccess && mean)
      div_by_len_kernel<<<(unsigned)((lanes + 255) / 256), 256, 0, s>>>(out, lanes, len);
    const cudaError_t ef = cudaFreeAsync(scratch, s);
    if (e == cudaSuccess) e = ef;
    return e == cudaSuccess ? cudaGetLastError() : e;
  }
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && len % 4 == 0) {
    const size_t grid = (lanes + kLcRows - 1) / kLcRows;
    for (size_t g0 = 0; g0 < grid; g0 += 0x7fffffffull) {
      const size_t ng = std::min<size_t>(grid - g0, 0x7fffffffull);
      lane_chain_sum_kernel<<<(unsigned)ng, kLcThreads, 0, s>>>(
          x + g0 * kLcRows * len, lanes - g0 * kLcRows, len, out + g0 * kLcRows, mean);
    }
    return cudaGetLastError();
  }
  // lane_generic_kernel is the same chain, one thread per lane
  const unsigned grid = (unsigned)std::max<size_t>(
      1, std::min<size_t>((lanes + kThreads - 1) / kThreads, (size_t)sm_count(cur_device()) * 8));
  if (mean)
    lane_generic_kernel<kDimMean><<<grid, kThreads, 0, s>>>(x, lanes, len, 1, out);
  else
    lane_generic_kernel<kDimSum><<<grid, kThreads, 0, s>>>(x, lanes, len, 1, out);
  return cudaGetLastError();
}

}  // namespace rt
