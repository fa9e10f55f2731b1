// ordered_sum.cu — the reference's sequential f32 sums of loss terms
// (ndarray's eight-chain unrolled_fold, or Iterator::sum's one chain),
// bit-exact and in parallel.  The algebra is in rt_osum.cuh.
//
// After a term kernel has written the terms (chain-major) and one f64 sum per
// 256-element block of each chain:
//   1. osum_chunk_kernel,  — per chain, an f64 prefix of the block sums (two
//      osum_code_kernel      wide passes: sums per 1024 blocks, then a scan
//                            inside each chunk); each block gets two
//                            candidate binade codes from its estimated start
//                            and end (rt_osum.cuh, Pair);
//   2. osum_summary_kernel — per block, the translation runs of its 256 terms
//                            under both codes (the moves from exact f32
//                            scaling and round-to-nearest-even, tau_pair_f),
//                            and per group of 32 blocks their composition
//                            under the first block's two codes;
//      osum_super_kernel   — and per 32 groups (1024 blocks) theirs;
//   3. osum_walk_kernel    — one warp per chain carries the running f32 sum
//                            across the super-groups, 32 at a time (the run whose
//                            code is the sum's binade, warp scan, ballot for
//                            the first that does not apply), then across the
//                            groups and blocks inside the one that does not,
//                            and folds a block whose runs do not
//                            apply with plain f32 adds in order (where the
//                            sum really crosses a power of two).  The first
//                            warp then combines the chains as unrolled_fold
//                            does and adds ndarray's remainder.
#include "rt_internal.h"
#include "rt_fold.cuh"
#include "rt_libm.cuh"
#include "rt_osum.cuh"

#include <algorithm>

namespace rt {
namespace osum {
namespace {

constexpr int kCodeThreads = kChunk;
constexpr int kSummWarps = 8;  // each warp of a group's CTA takes 4 of its blocks
constexpr int kMinBinade = -100;  // 2^(23 - e) must be a normal f32

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__device__ __forceinline__ int binade_code(int e, bool neg) {
  return neg ? -(e + kCodeBias) : e + kCodeBias;
}

// The two candidate codes of a block whose chain sum is estimated to run from
// start to end (f64): the binade(s) of the estimate, plus the neighbour when
// the estimate lies within 1/8 of a binade boundary (the f32 chain's drift
// from the exact prefix stays far below that in practice).  Binades below
// 2^-100 are left to the ordered fold.
__device__ __forceinline__ int2 classify(double start, double end) {
  if (start == 0.0 && end == 0.0) return make_int2(kCodeZero, kCodePoison);
  const uint64_t a = (uint64_t)__double_as_longlong(start);
  const uint64_t b = (uint64_t)__double_as_longlong(end);
  if (start == 0.0 || end == 0.0 || (a >> 63) != (b >> 63))
    return make_int2(kCodePoison, kCodePoison);
  const bool neg = (a >> 63) != 0;
  const int ea = (int)((a >> 52) & 0x7ff) - 1023, eb = (int)((b >> 52) & 0x7ff) - 1023;
  const int lo = min(ea, eb), hi = max(ea, eb);
  if (lo < kMinBinade || hi > 127) return make_int2(kCodePoison, kCodePoison);  // also NaN/inf
  if (hi == lo + 1) return make_int2(binade_code(ea, neg), binade_code(eb, neg));
  if (hi != lo) return make_int2(kCodePoison, kCodePoison);
  const double mid = fabs(0.5 * (start + end));
  const int other = mid < ldexp(1.125, ea) ? ea - 1 : (mid >= ldexp(1.75, ea) ? ea + 1 : 1000);
  const bool ok = other >= kMinBinade && other <= 127;
  return make_int2(binade_code(ea, neg), ok ? binade_code(other, neg) : kCodePoison);
}

// CTA-wide (1024 threads) inclusive f64 scan; returns this thread's
// inclusive value and *total = the CTA's sum.
__device__ __forceinline__ double cta_scan(double v, double* wsum, double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += y;
  }
  if (lane == 31) wsum[warp] = v;
  __syncthreads();
  if (warp == 0) {
    double w = wsum[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    wsum[lane] = w;
  }
  __syncthreads();
  *total = wsum[31];
  return v + (warp > 0 ? wsum[warp - 1] : 0.0);
}

// grid (chunks, chains): csum[c][k] = the sum of chunk k's 1024 block sums.
__global__ void __launch_bounds__(kCodeThreads) osum_chunk_kernel(Plan plan) {
  __shared__ double wsum[32];
  const int c = blockIdx.y;
  const size_t b = (size_t)blockIdx.x * kChunk + threadIdx.x;
  const double v = b < plan.blocks ? plan.bsum[c * plan.blocks + b] : 0.0;
  double total;
  cta_scan(v, wsum, &total);
  if (threadIdx.x == 0) plan.csum[c * plan.chunks + blockIdx.x] = total;
}

// grid (chunks, chains): each block's estimated start (the f64 sum of the
// block sums before it) and end, and the codes they give.
__global__ void __launch_bounds__(kCodeThreads) osum_code_kernel(Plan plan) {
  __shared__ double wsum[32];
  __shared__ double base_sh;
  const int c = blockIdx.y;
  const size_t k = blockIdx.x;
  if (threadIdx.x < 32) {
    double acc = 0.0;
    for (size_t j = threadIdx.x; j < k; j += 32) acc += plan.csum[c * plan.chunks + j];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (threadIdx.x == 0) base_sh = acc;
  }
  const size_t b = k * kChunk + threadIdx.x;
  const double v = b < plan.blocks ? plan.bsum[c * plan.blocks + b] : 0.0;
  double total;
  const double incl = cta_scan(v, wsum, &total);  // syncs, so base_sh is visible
  const double end = base_sh + incl;
  if (b < plan.blocks) plan.code[c * plan.blocks + b] = classify(end - v, end);
}

__device__ __forceinline__ Summ shfl_down_summ(const Summ& a, int off) {
  Summ r;
  r.code = __shfl_down_sync(0xffffffffu, a.code, off);
  r.t0 = __shfl_down_sync(0xffffffffu, a.t0, off);
  r.lo0 = __shfl_down_sync(0xffffffffu, a.lo0, off);
  r.hi0 = __shfl_down_sync(0xffffffffu, a.hi0, off);
  r.neg = __shfl_down_sync(0xffffffffu, a.neg, off);
  r.t1 = __shfl_down_sync(0xffffffffu, a.t1, off);
  r.lo1 = __shfl_down_sync(0xffffffffu, a.lo1, off);
  r.hi1 = __shfl_down_sync(0xffffffffu, a.hi1, off);
  return r;
}

__device__ __forceinline__ Summ shfl_up_summ(const Summ& a, int off) {
  Summ r;
  r.code = __shfl_up_sync(0xffffffffu, a.code, off);
  r.t0 = __shfl_up_sync(0xffffffffu, a.t0, off);
  r.lo0 = __shfl_up_sync(0xffffffffu, a.lo0, off);
  r.hi0 = __shfl_up_sync(0xffffffffu, a.hi0, off);
  r.neg = __shfl_up_sync(0xffffffffu, a.neg, off);
  r.t1 = __shfl_up_sync(0xffffffffu, a.t1, off);
  r.lo1 = __shfl_up_sync(0xffffffffu, a.lo1, off);
  r.hi1 = __shfl_up_sync(0xffffffffu, a.hi1, off);
  return r;
}

// Lane 0 gets lane 0's, then 1's, ..., then 31's run composed in lane order.
__device__ __forceinline__ Summ warp_compose(Summ a) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const Summ b = shfl_down_summ(a, off);
    if ((threadIdx.x & 31) + off < 32) a = summ_compose(a, b);
  }
  return a;
}

// Lane l gets lanes 0..l composed in order.
__device__ __forceinline__ Summ warp_scan(Summ a) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const Summ b = shfl_up_summ(a, off);
    if (lane >= off) a = summ_compose(b, a);
  }
  return a;
}

__device__ __forceinline__ Summ load_summ(const Summ* p) {
  const int4 a = __ldcg(reinterpret_cast<const int4*>(p));
  const int4 b = __ldcg(reinterpret_cast<const int4*>(p) + 1);
  return Summ{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
}

__device__ __forceinline__ void store_summ(Summ* p, const Summ& s) {
  reinterpret_cast<int4*>(p)[0] = make_int4(s.code, s.t0, s.lo0, s.hi0);
  reinterpret_cast<int4*>(p)[1] = make_int4(s.neg, s.t1, s.lo1, s.hi1);
}

// One-parity run (a block without ties): moves t, partial extremes lo/hi.
struct Run1 {
  int t, lo, hi;
};

__device__ __forceinline__ Run1 run1_compose(const Run1& a, const Run1& b) {
  return Run1{clamp_sat(a.t + b.t), min(a.lo, clamp_sat(a.t + b.lo)),
              max(a.hi, clamp_sat(a.t + b.hi))};
}

// Warp: the run of one block's terms (x: lane's 8 elements, elements past
// the block's end already replaced by 0 — they move by 0, so their partial
// sums repeat the last real one and change nothing) under a binade code.
__device__ __forceinline__ Summ block_run(const float (&x)[8], int cd) {
  const int lane = threadIdx.x & 31;
  const int e = (cd < 0 ? -cd : cd) - kCodeBias;
  const float scale = __uint_as_float((uint32_t)(23 - e + 127) << 23);  // 2^(23 - e)
  int m0[8], m1[8];
  bool tie = false;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    tau_pair_f(x[k], scale, m0[k], m1[k]);
    tie |= m0[k] != m1[k];
  }
  if (!__any_sync(0xffffffffu, tie)) {
    Run1 r{0, kLoId, kHiId};
#pragma unroll
    for (int k = 0; k < 8; k++) {  // |partial| <= 8 * 2^26: no overflow
      r.t += m0[k];
      r.lo = min(r.lo, r.t);
      r.hi = max(r.hi, r.t);
    }
    r = Run1{clamp_sat(r.t), clamp_sat(r.lo), clamp_sat(r.hi)};
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const Run1 o{__shfl_down_sync(0xffffffffu, r.t, off),
                   __shfl_down_sync(0xffffffffu, r.lo, off),
                   __shfl_down_sync(0xffffffffu, r.hi, off)};
      if (lane + off < 32) r = run1_compose(r, o);
    }
    return Summ{cd, r.t, r.lo, r.hi, 0, r.t, r.lo, r.hi};
  }
  Summ mine = summ_make(cd);
#pragma unroll
  for (int k = 0; k < 8; k++) summ_push(mine, m0[k], m1[k]);
  return warp_compose(mine);
}

__device__ __forceinline__ Summ pick(const Pair& p, int cd) {
  if (p.a.code == kCodeNone) return p.a;
  return p.a.code == cd ? p.a : (p.b.code == cd ? p.b : summ_make(kCodePoison));
}

// grid (groups, chains), 8 warps: each warp takes 4 of the group's blocks and
// computes their runs under both codes; warp 0 then composes the group under
// the first block's two codes.
__global__ void __launch_bounds__(32 * kSummWarps) osum_summary_kernel(Plan plan) {
  __shared__ Pair runs[kGroup];
  const int c = blockIdx.y;
  const size_t g = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = 0; i < kGroup / kSummWarps; i++) {
    const int wb = warp + kSummWarps * i;
    const size_t b = g * kGroup + wb;
    Pair pr{summ_make(kCodeNone), summ_make(kCodeNone)};
    if (b < plan.blocks) {
      const size_t first = b * kBlock;
      const int cnt = (int)min((size_t)kBlock, plan.len - first);
      const float* tb = plan.terms + c * plan.pitch + first;
      const int j0 = 8 * lane;
      // the chain pitch is a multiple of the block, so whole blocks are in bounds
      const float4 x0 = __ldcs(reinterpret_cast<const float4*>(tb + j0));
      const float4 x1 = __ldcs(reinterpret_cast<const float4*>(tb + j0 + 4));
      float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int k = 0; k < 8; k++) x[k] = j0 + k < cnt ? x[k] : 0.0f;
      const int2 cd = plan.code[c * plan.blocks + b];
      if (cd.x == kCodeZero) {
        bool allzero = true, allneg = true;
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const uint32_t u = __float_as_uint(x[k]);
          allzero &= (u & 0x7fffffffu) == 0;
          allneg &= j0 + k >= cnt || u == 0x80000000u;
        }
        pr.a = summ_make(__all_sync(0xffffffffu, allzero) ? kCodeZero : kCodePoison);
        pr.a.neg = __all_sync(0xffffffffu, allneg) ? 1 : 0;
        pr.b = summ_make(kCodePoison);
      } else {
        pr.a = cd.x != kCodePoison ? block_run(x, cd.x) : summ_make(kCodePoison);
        pr.b = cd.y != kCodePoison ? block_run(x, cd.y) : summ_make(kCodePoison);
      }
      if (lane == 0) {
        Pair* dst = plan.l0 + c * plan.blocks + b;
        store_summ(&dst->a, pr.a);
        store_summ(&dst->b, pr.b);
      }
    }
    if (lane == 0) runs[wb] = pr;
  }
  __syncthreads();
  if (warp == 0) {
    const Pair mine = runs[lane];
    const int c1 = runs[0].a.code, c2 = runs[0].b.code;
    const Summ g1 = warp_compose(pick(mine, c1));
    const Summ g2 = c2 != kCodePoison ? warp_compose(pick(mine, c2)) : summ_make(kCodePoison);
    if (lane == 0) {
      Pair* dst = plan.l1 + c * plan.groups + g;
      store_summ(&dst->a, g1);
      store_summ(&dst->b, g2);
    }
  }
}

// grid (supers, chains), one warp: the 32 group records of super-group q
// composed under the first group's two codes.
__global__ void __launch_bounds__(32) osum_super_kernel(Plan plan) {
  const int c = blockIdx.y, lane = threadIdx.x;
  const size_t q = blockIdx.x, g = q * kGroup + lane;
  const Pair* src = plan.l1 + c * plan.groups;
  Pair mine{summ_make(kCodeNone), summ_make(kCodeNone)};
  if (g < plan.groups) mine = Pair{load_summ(&src[g].a), load_summ(&src[g].b)};
  const int c1 = __shfl_sync(0xffffffffu, mine.a.code, 0);
  const int c2 = __shfl_sync(0xffffffffu, mine.b.code, 0);
  const Summ s1 = warp_compose(pick(mine, c1));
  const Summ s2 = c2 != kCodePoison ? warp_compose(pick(mine, c2)) : summ_make(kCodePoison);
  if (lane == 0) {
    Pair* dst = plan.l2 + c * plan.supers + q;
    store_summ(&dst->a, s1);
    store_summ(&dst->b, s2);
  }
}

// The code of the binade s lies in (kCodeZero for +-0; poison for
// subnormal, inf and NaN, which no run applies to).
__device__ __forceinline__ int code_of(float s) {
  const uint32_t u = __float_as_uint(s);
  const int ex = (int)((u >> 23) & 0xffu);
  if ((u & 0x7fffffffu) == 0) return kCodeZero;
  if (ex == 0 || ex == 0xff) return kCodePoison;
  return binade_code(ex - 127, (u >> 31) != 0);
}

// apply_prefix for runs that depend on parity (ties) or a zero sum: the
// full composition.
__device__ __forceinline__ int apply_prefix_general(const Summ& run, float& s) {
  const Summ x = warp_scan(run);
  float after;
  const bool ok = summ_apply(x, s, &after);
  const unsigned bal = __ballot_sync(0xffffffffu, ok);
  const int k = bal == 0xffffffffu ? 32 : __ffs(~bal) - 1;
  if (k > 0) s = __shfl_sync(0xffffffffu, after, k - 1);
  return k;
}

// One step over up to 32 runs (lane l: the run at position l, already picked
// for s's binade code cd; none for positions already behind, poison where the
// step must stop): applies the longest prefix that provably applies and
// returns the first lane that does not (32 if none).
__device__ __forceinline__ int apply_prefix(const Summ& run, int cd, float& s) {
  constexpr int kBig = 1 << 29;  // partial extremes are kept in [-kBig, kBig]
  const int lane = threadIdx.x & 31;
  if (cd == kCodePoison) return 0;  // s is subnormal or not finite: no run applies
  const bool none = run.code == kCodeNone;
  const bool stop = !none && run.code != cd;
  const bool flat = none || stop || (run.t0 == run.t1 && run.lo0 == run.lo1 && run.hi0 == run.hi1);
  constexpr int kMin = (1 << 23) + 1, kMax = (1 << 24) - 1;
  if (cd != kCodeZero && __all_sync(0xffffffffu, flat)) {
    // no run depends on parity: one inclusive scan of (moves, least partial,
    // greatest partial), composed as (ta + tb, min(la, ta + lb), max(ha, ta + hb))
    int t = none || stop ? 0 : run.t0;
    int lo = none ? kBig : (stop ? -kBig : run.lo0);
    int hi = none ? -kBig : (stop ? kBig : run.hi0);
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int ta = __shfl_up_sync(0xffffffffu, t, off);
      const int la = __shfl_up_sync(0xffffffffu, lo, off);
      const int ha = __shfl_up_sync(0xffffffffu, hi, off);
      if (lane >= off) {
        lo = min(la, min(max(ta + lo, -kBig), kBig));
        hi = max(ha, min(max(ta + hi, -kBig), kBig));
        t = clamp_sat(ta + t);
      }
    }
    const uint32_t sb = __float_as_uint(s);
    const bool neg = cd < 0;
    const int mag = (int)((sb & 0x7fffffu) | 0x800000u);
    const int S = neg ? -mag : mag;
    const bool ok = neg ? (S + hi <= -kMin && S + lo >= -kMax) : (S + lo >= kMin && S + hi <= kMax);
    const unsigned bal = __ballot_sync(0xffffffffu, ok);
    const int k = bal == 0xffffffffu ? 32 : __ffs(~bal) - 1;
    if (k > 0) {
      const int r = S + __shfl_sync(0xffffffffu, t, k - 1);
      const uint32_t rm = (uint32_t)(r < 0 ? -r : r);
      s = __uint_as_float((sb & 0xff800000u) | (rm - 0x800000u));
    }
    return k;
  }
  return apply_prefix_general(run, s);
}

__device__ __forceinline__ Pair load_pair(const Pair* p, bool valid) {
  if (!valid) return Pair{summ_make(kCodePoison), summ_make(kCodePoison)};
  return Pair{load_summ(&p->a), load_summ(&p->b)};
}

__device__ __forceinline__ Summ pick_run(const Pair& p, int cd) {
  return p.a.code == cd ? p.a : (p.b.code == cd ? p.b : summ_make(kCodePoison));
}

// With the running sum at +-inf only a NaN or the opposite infinity can change
// it, and a block holds one exactly when its f64 block sum is NaN or that
// opposite infinity (an f64 sum of f32 terms cannot overflow); the same holds
// for the 1024-block chunk sums.  The first block at or after b that can
// change s (nb if none), found from the chunk sums, then the block sums.
__device__ __forceinline__ size_t next_inf_breaker(const Plan& plan, int c, size_t b, bool pos) {
  const int lane = threadIdx.x & 31;
  const double other = pos ? -INFINITY : INFINITY;
  const double* bs = plan.bsum + c * plan.blocks;
  const double* cs = plan.csum + c * plan.chunks;
  const size_t nb = plan.blocks;
  while (b < nb) {
    if (b % kChunk == 0) {  // whole chunks
      const size_t k0 = b / kChunk;
      const double v = k0 + lane < plan.chunks ? __ldcg(cs + k0 + lane) : 0.0;
      const unsigned bad = __ballot_sync(0xffffffffu, v != v || v == other);
      if (!bad) {
        b = min(nb, (k0 + 32) * kChunk);
        continue;
      }
      b = (k0 + (__ffs(bad) - 1)) * kChunk;
    }
    const size_t cend = min(nb, (b / kChunk + 1) * kChunk);
    const double v = b + lane < cend ? __ldcg(bs + b + lane) : 0.0;
    const unsigned bad = __ballot_sync(0xffffffffu, v != v || v == other);
    if (bad) return b + (__ffs(bad) - 1);
    b = min(cend, b + 32);
  }
  return nb;
}

// One CTA (one warp) per chain, so that every chain's latency-bound walk has
// an SM to itself; the last chain to finish combines them.  Three levels: 32
// super-groups (1024 blocks each) per step, then 32 groups of the super-group
// that does not apply, then the blocks of the group that does not apply
// (their records loaded once), folding in order only a block none of whose
// runs applies.  A NaN sum ends the walk; an infinite one skips to the blocks
// that can still change it.
template <int CH>
__global__ void __launch_bounds__(32) osum_walk_kernel(Plan plan, float init, float* out) {
  constexpr size_t kSuper = (size_t)kGroup * kGroup;  // blocks per super-group
  __shared__ __align__(16) float buf[1][kBlock];
  const int c = blockIdx.x, lane = threadIdx.x;
  const size_t nb = plan.blocks, ng = plan.groups, nsg = plan.supers;
  const Pair* l0 = plan.l0 + c * nb;
  const Pair* l1 = plan.l1 + c * ng;
  const Pair* l2 = plan.l2 + c * nsg;
  float s = init;
  size_t b = 0;
  size_t next_q0 = 0;  // super-group records of the next 32, loaded ahead
  Pair next = load_pair(l2 + lane, lane < nsg);
  size_t rec1_super = ~(size_t)0;  // the super-group whose group records are in rec1
  Pair rec1;
  while (b < nb) {
    if (s != s) break;  // NaN + anything stays NaN
    if ((__float_as_uint(s) & 0x7fffffffu) == 0x7f800000u) {
      // +-inf: skip to the first block that can change it and fold that one
      b = next_inf_breaker(plan, c, b, s > 0.0f);
      if (b >= nb) break;
      const float4* tb = reinterpret_cast<const float4*>(plan.terms + c * plan.pitch + b * kBlock);
      reinterpret_cast<float4*>(buf[0])[2 * lane] = __ldcg(tb + 2 * lane);
      reinterpret_cast<float4*>(buf[0])[2 * lane + 1] = __ldcg(tb + 2 * lane + 1);
      __syncwarp();
      const int cnt = (int)min((size_t)kBlock, plan.len - b * kBlock);
      if (lane == 0) fold_pipelined(buf[0], 1, cnt, [&](float v) { s = fadd(s, v); });
      s = __shfl_sync(0xffffffffu, s, 0);
      __syncwarp();
      b++;
      continue;
    }
    if ((b % kSuper) == 0) {
      const size_t q0 = b / kSuper;
      const Pair rec = q0 == next_q0 ? next : load_pair(l2 + q0 + lane, q0 + lane < nsg);
      next_q0 = q0 + 32;
      next = load_pair(l2 + next_q0 + lane, next_q0 + lane < nsg);
      const int cd = code_of(s);
      const int k = apply_prefix(pick_run(rec, cd), cd, s);
      if (k > 0) {
        b = min(nb, (q0 + k) * kSuper);
        continue;
      }
    }
    if ((b % kGroup) == 0) {
      const size_t q = b / kSuper, gbase = q * kGroup;
      if (q != rec1_super) {
        rec1 = load_pair(l1 + gbase + lane, gbase + lane < ng);
        rec1_super = q;
      }
      const int off = (int)(b / kGroup - gbase);
      const int cd = code_of(s);
      const Summ run = lane < off ? summ_make(kCodeNone) : pick_run(rec1, cd);
      const int k = apply_prefix(run, cd, s);
      if (k > off) {
        b = min(nb, (gbase + k) * kGroup);
        continue;
      }
    }
    // the blocks of b's group
    const size_t base = b / kGroup * kGroup;
    const int end = (int)min((size_t)kGroup, nb - base);
    const Pair pr = load_pair(l0 + base + lane, lane < end);
    int pos = (int)(b - base);
    while (pos < end && s == s) {
      const int cd = code_of(s);
      const Summ run = lane < pos ? summ_make(kCodeNone) : pick_run(pr, cd);
      const int k = apply_prefix(run, cd, s);
      if (k > pos) {
        pos = k;
        continue;
      }
      // no run of block base + pos applies: fold it in order
      const size_t fb = base + pos;
      const int cnt = (int)min((size_t)kBlock, plan.len - fb * kBlock);
      const float4* tb = reinterpret_cast<const float4*>(plan.terms + c * plan.pitch + fb * kBlock);
      const float4 t0 = __ldcg(tb + 2 * lane), t1 = __ldcg(tb + 2 * lane + 1);
      reinterpret_cast<float4*>(buf[0])[2 * lane] = t0;
      reinterpret_cast<float4*>(buf[0])[2 * lane + 1] = t1;
      __syncwarp();
      if (lane == 0) fold_pipelined(buf[0], 1, cnt, [&](float v) { s = fadd(s, v); });
      s = __shfl_sync(0xffffffffu, s, 0);
      __syncwarp();
      pos++;
    }
    b = base + min(pos, end);
  }
  if (lane == 0) {
    plan.chain_out[c] = s;
    __threadfence();
    if (atomicAdd(plan.done, 1u) == CH - 1) {
      __threadfence();
      const volatile float* cs = plan.chain_out;
      float r = cs[0];
      if constexpr (CH == 8) {
        r = 0.0f;
        r = fadd(r, fadd(cs[0], cs[4]));
        r = fadd(r, fadd(cs[1], cs[5]));
        r = fadd(r, fadd(cs[2], cs[6]));
        r = fadd(r, fadd(cs[3], cs[7]));
        const size_t rest = plan.n - plan.len * CH;
        for (size_t i = 0; i < rest; i++) r = fadd(r, plan.terms[CH * plan.pitch + i]);
      }
      out[0] = r;
    }
  }
}

}  // namespace

Plan make_plan(void* scratch, size_t n, int chains) {
  Plan p;
  p.chains = chains;
  p.n = n;
  p.len = n / chains;
  p.blocks = (p.len + kBlock - 1) / kBlock;
  p.groups = (p.blocks + kGroup - 1) / kGroup;
  p.supers = (p.groups + kGroup - 1) / kGroup;
  p.pitch = p.blocks * kBlock;
  p.chunks = (p.blocks + kChunk - 1) / kChunk;
  char* at = static_cast<char*>(scratch);
  p.terms = reinterpret_cast<float*>(at);
  at += round_up((chains * p.pitch + 8) * sizeof(float), 256);
  p.bsum = reinterpret_cast<double*>(at);
  at += round_up(chains * p.blocks * sizeof(double), 256);
  p.csum = reinterpret_cast<double*>(at);
  at += round_up(chains * p.chunks * sizeof(double), 256);
  p.code = reinterpret_cast<int2*>(at);
  at += round_up(chains * p.blocks * sizeof(int2), 256);
  p.l0 = reinterpret_cast<Pair*>(at);
  at += round_up(chains * p.blocks * sizeof(Pair), 256);
  p.l1 = reinterpret_cast<Pair*>(at);
  at += round_up(chains * p.groups * sizeof(Pair), 256);
  p.l2 = reinterpret_cast<Pair*>(at);
  at += round_up(chains * p.supers * sizeof(Pair), 256);
  p.chain_out = reinterpret_cast<float*>(at);
  p.done = reinterpret_cast<unsigned*>(at + 64);
  return p;
}

size_t scratch_bytes(size_t n, int chains) {
  const Plan p = make_plan(nullptr, n, chains);
  return reinterpret_cast<size_t>(p.chain_out) + 256;
}

int term_grid(const Plan& plan) {
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t tiles = (plan.len * plan.chains + kTileIn - 1) / kTileIn;
  const size_t cap = (size_t)sm_count(dev) * 8;  // 8 CTAs of 256 threads per SM
  return (int)std::max<size_t>(1, std::min(tiles, cap));
}

cudaError_t launch_ordered_sum(const Plan& plan, float init, float* out, cudaStream_t s) {
  if (plan.blocks > 0) {
    const dim3 cgrid((unsigned)plan.chunks, (unsigned)plan.chains);
    osum_chunk_kernel<<<cgrid, kCodeThreads, 0, s>>>(plan);
    osum_code_kernel<<<cgrid, kCodeThreads, 0, s>>>(plan);
    const dim3 grid((unsigned)plan.groups, (unsigned)plan.chains);
    osum_summary_kernel<<<grid, 32 * kSummWarps, 0, s>>>(plan);
    osum_super_kernel<<<dim3((unsigned)plan.supers, (unsigned)plan.chains), 32, 0, s>>>(plan);
  }
  if (plan.chains == 8)
    osum_walk_kernel<8><<<8, 32, 0, s>>>(plan, 0.0f, out);
  else
    osum_walk_kernel<1><<<1, 32, 0, s>>>(plan, init, out);
  return cudaGetLastError();
}

}  // namespace osum
}  // namespace rt
