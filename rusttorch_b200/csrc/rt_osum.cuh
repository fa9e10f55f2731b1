// rt_osum.cuh — a sequential f32 sum (s = s + x[0] + x[1] + ..., every add
// rounded to nearest-even) computed in parallel, bit for bit.
//
// The reference sums loss terms with ndarray's sum (eight sequential f32
// chains) or Iterator::sum (one chain).  Reproducing that order by running
// the chain costs one dependent add per element.  This file restates the
// chain as something associative.
//
// The fact used: let s be an f32 of binade e (2^e <= |s| < 2^(e+1)) and u =
// 2^(e-23) that binade's ulp, so s = S*u for an integer S with 2^23 <= |S| <
// 2^24.  If the exact s + x also lies in binade e with the sign of s, then the
// f32 sum RN(s + x) is RN_u(s + x) = u * RN(S + x/u): the running sum moves by
// an integer tau = RN(S + x/u) - S that depends on x alone, except when x/u
// is an odd multiple of 1/2 (a tie), where it depends on the parity of S.  So
// inside one binade a run of adds is a translation of S, described for both
// parities of the start by (T: total move, lo/hi: the least and greatest
// partial move).  Two runs compose associatively (the end parity is the start
// parity plus T), and a run applies to a start S exactly when every partial
// sum stays strictly inside the binade: 2^23 < |S + partial| < 2^24, which
// also proves that each exact s + x was in the binade, so each rounding was
// the binade's own.  Runs that leave the binade (the sum crosses a power of
// two, hits zero, overflows, meets a NaN) fail that test and are re-run as a
// plain chain of f32 adds.
//
// Which binade a block of terms will see is guessed from an f64 prefix sum
// of block sums; a wrong guess costs only a sequential re-run of the block.
#pragma once

#include <cstdint>
#include <cmath>
#include <cstring>

namespace rt {
namespace osum {

constexpr int kBlock = 256;     // chain elements per block summary
constexpr int kGroup = 32;      // block summaries per group summary
constexpr int kTileIn = 2048;   // input elements per CTA tile of the term kernel
constexpr int kTermThreads = 256;

// Summary codes.  Binade codes are sign * (e + kCodeBias), e in [-126, 127].
constexpr int kCodePoison = 0;  // never applies: the walk folds the block in order
constexpr int kCodeZero = 1;    // every term is +-0 and the running sum is +-0
constexpr int kCodeNone = 2;    // empty (identity of composition)
constexpr int kCodeBias = 1000;

constexpr int kSat = 1 << 26;   // moves are clamped here; |move| >= 2^24 never applies
constexpr int kLoId = 1 << 30;  // lo of an empty run
constexpr int kHiId = -(1 << 30);

// 32 bytes: {code, t0, lo0, hi0} {neg, t1, lo1, hi1}.  t/lo/hi index = parity
// of S at the start.  neg (kCodeZero only): every term is -0.
struct Summ {
  int code, t0, lo0, hi0;
  int neg, t1, lo1, hi1;
};

__host__ __device__ __forceinline__ uint32_t bits_of(float x) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(x);
#else
  uint32_t u;
  memcpy(&u, &x, sizeof u);
  return u;
#endif
}

__host__ __device__ __forceinline__ float float_of(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float x;
  memcpy(&x, &u, sizeof x);
  return x;
#endif
}

__host__ __device__ __forceinline__ int clamp_sat(int v) { return min(max(v, -kSat), kSat); }

__host__ __device__ __forceinline__ Summ summ_make(int code) {
  return Summ{code, 0, kLoId, kHiId, 0, 0, kLoId, kHiId};
}

// The move of S for adding x on the grid u = 2^(e-23): m0 for even S, m1 for
// odd S (they differ only for a tie).  Exact integer arithmetic on x's bits,
// branch-free; NaN/inf and moves of 2^26 or more saturate (the run then never
// applies).
__host__ __device__ __forceinline__ void tau_pair(float x, int e, int& m0, int& m1) {
  const uint32_t bits = bits_of(x);
  const int ex = (int)((bits >> 23) & 0xffu);
  const uint32_t mant = (bits & 0x7fffffu) | (ex != 0 ? 0x800000u : 0u);
  const bool neg = (bits >> 31) != 0;
  // x/u = mant * 2^-r with r = (e - 23) - E and E = max(ex, 1) - 150
  const int r = (e - 23) - ((ex != 0 ? ex : 1) - 150);
  const bool big = ex == 0xff || r < -2;  // |x/u| >= 2^26 (or not finite)
  const int rs = min(max(r, 1), 31);
  const uint32_t a = r <= 0 ? mant << min(-r, 2) : mant >> rs;
  const uint32_t rem = r <= 0 ? 0u : mant & ((1u << rs) - 1u);
  const uint32_t half = r <= 0 ? 1u : 1u << (rs - 1);
  const int mag = (int)a + (rem > half ? 1 : 0);
  const int rounded = neg ? -mag : mag;
  // tie: the candidates are S + lo and S + lo + 1, and the even sum wins
  const int lo = neg ? -(int)a - 1 : (int)a;
  const int odd_lo = lo & 1;
  const bool tie = rem == half;
  const int sat = neg && ex != 0xff ? -kSat : kSat;
  m0 = big ? sat : (tie ? lo + odd_lo : rounded);
  m1 = big ? sat : (tie ? lo + (odd_lo ^ 1) : rounded);
}

// The same moves from f32 arithmetic, for a binade e in [-100, 127] given as
// scale = 2^(23 - e) (a normal f32).  q = x * scale = x/u is exact (or, when it
// underflows, far below 1/2); adding 1.5 * 2^23 rounds it to the nearest
// integer, ties to even, and since that constant is even the rounded q is the
// move for an even S.  For a tie the odd S takes the other neighbour.  Moves
// of 2^22 or more (and NaN/inf) saturate: a run needs |move| < 2^23 to apply,
// so this only sends terms as large as half the running sum to the ordered
// fold.  Equal to tau_pair for every x with |x/u| < 2^22.
__host__ __device__ __forceinline__ void tau_pair_f(float x, float scale, int& m0, int& m1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
#ifdef __CUDA_ARCH__
  const float q = __fmul_rn(x, scale);
  const float y = __fadd_rn(q, kMagic);
  const float r = __fsub_rn(y, kMagic);
  const float d = __fsub_rn(q, r);
#else
  const float q = x * scale;
  const float y = q + kMagic;
  const float r = y - kMagic;
  const float d = q - r;
#endif
  const bool ok = fabsf(q) < 4194304.0f;  // 2^22; false for NaN
  const int m = (int)(bits_of(y) - bits_of(kMagic));
  const int odd = fabsf(d) == 0.5f ? (d > 0.0f ? 1 : -1) : 0;
  const int sat = x < 0.0f ? -kSat : kSat;
  m0 = ok ? m : sat;
  m1 = ok ? m + odd : sat;
}

// Appends one element's move pair to a binade run (in order).
__host__ __device__ __forceinline__ void summ_push(Summ& a, int m0, int m1) {
  {
    const int mv = (a.t0 & 1) ? m1 : m0;
    a.t0 = clamp_sat(a.t0 + mv);
    a.lo0 = min(a.lo0, a.t0);
    a.hi0 = max(a.hi0, a.t0);
  }
  {
    const int mv = (a.t1 & 1) ? m0 : m1;  // parity of S + t1 with S odd
    a.t1 = clamp_sat(a.t1 + mv);
    a.lo1 = min(a.lo1, a.t1);
    a.hi1 = max(a.hi1, a.t1);
  }
}

// a then b.
__host__ __device__ __forceinline__ Summ summ_compose(const Summ& a, const Summ& b) {
  if (a.code == kCodeNone) return b;
  if (b.code == kCodeNone) return a;
  if (a.code == kCodePoison || b.code == kCodePoison || a.code != b.code)
    return summ_make(kCodePoison);
  Summ r = a;
  if (a.code == kCodeZero) {
    r.neg = a.neg & b.neg;
    return r;
  }
  // start parity 0: after a, S's parity is t0 & 1
  {
    const bool odd = (a.t0 & 1) != 0;
    const int bt = odd ? b.t1 : b.t0, bl = odd ? b.lo1 : b.lo0, bh = odd ? b.hi1 : b.hi0;
    r.t0 = clamp_sat(a.t0 + bt);
    r.lo0 = min(a.lo0, bl == kLoId ? kLoId : clamp_sat(a.t0 + bl));
    r.hi0 = max(a.hi0, bh == kHiId ? kHiId : clamp_sat(a.t0 + bh));
  }
  // start parity 1: after a, parity is (1 + t1) & 1
  {
    const bool odd = (a.t1 & 1) == 0;
    const int bt = odd ? b.t1 : b.t0, bl = odd ? b.lo1 : b.lo0, bh = odd ? b.hi1 : b.hi0;
    r.t1 = clamp_sat(a.t1 + bt);
    r.lo1 = min(a.lo1, bl == kLoId ? kLoId : clamp_sat(a.t1 + bl));
    r.hi1 = max(a.hi1, bh == kHiId ? kHiId : clamp_sat(a.t1 + bh));
  }
  return r;
}

// Applies a summary to the running sum s: true and *out = the chain's value
// after the run, or false if the run does not provably apply to s.
__host__ __device__ __forceinline__ bool summ_apply(const Summ& a, float s, float* out) {
  if (a.code == kCodeNone) {
    *out = s;
    return true;
  }
  if (a.code == kCodeZero) {
    // s + (+-0) = s for s != 0 (NaN stays NaN); -0 + -0 = -0; otherwise +0
    const uint32_t sb = bits_of(s);
    *out = (sb & 0x7fffffffu) != 0 ? s : ((sb >> 31) && a.neg ? -0.0f : 0.0f);
    return true;
  }
  if (a.code == kCodePoison) return false;
  const bool neg = a.code < 0;
  const int e = (neg ? -a.code : a.code) - kCodeBias;
  const uint32_t sb = bits_of(s);
  if ((int)((sb >> 23) & 0xffu) != e + 127 || ((sb >> 31) != 0) != neg) return false;
  const int mag = (int)((sb & 0x7fffffu) | 0x800000u);
  const int S = neg ? -mag : mag;
  const bool odd = (mag & 1) != 0;
  const int t = odd ? a.t1 : a.t0, lo = odd ? a.lo1 : a.lo0, hi = odd ? a.hi1 : a.hi0;
  constexpr int kMin = (1 << 23) + 1, kMax = (1 << 24) - 1;
  const bool ok = neg ? (hi == kHiId || S + hi <= -kMin) && (lo == kLoId || S + lo >= -kMax)
                      : (lo == kLoId || S + lo >= kMin) && (hi == kHiId || S + hi <= kMax);
  if (!ok) return false;
  const int r = S + t;
  const uint32_t rm = (uint32_t)(r < 0 ? -r : r);
  *out = float_of((sb & 0xff800000u) | (rm - 0x800000u));
  return true;
}

// Warp: sum of d[0..7] over the 32 lanes for each k, transposed so that lane l
// (l % 4 == 0) returns the total of slot 4*((l>>4)&1) + 2*((l>>3)&1) + ((l>>2)&1).
// Order of the f64 adds is unspecified (these sums only guess binades).
__device__ __forceinline__ double warp_sum8_transposed(const double (&d)[8], int lane) {
  double w[4], x[2];
  const bool b16 = (lane & 16) != 0, b8 = (lane & 8) != 0, b4 = (lane & 4) != 0;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const double send = b16 ? d[k] : d[k + 4];
    const double keep = b16 ? d[k + 4] : d[k];
    w[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const double send = b8 ? w[k] : w[k + 2];
    const double keep = b8 ? w[k + 2] : w[k];
    x[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  double y = (b4 ? x[1] : x[0]) + __shfl_xor_sync(0xffffffffu, b4 ? x[0] : x[1], 4);
  y += __shfl_xor_sync(0xffffffffu, y, 2);
  y += __shfl_xor_sync(0xffffffffu, y, 1);
  return y;
}

__device__ __forceinline__ int warp_sum8_slot(int lane) {
  return 4 * ((lane >> 4) & 1) + 2 * ((lane >> 3) & 1) + ((lane >> 2) & 1);
}

// Scratch of one ordered sum over n input elements with `chains` (1 or 8)
// chains: chain c's terms at terms[c * pitch + i], i < len; the n - chains *
// len trailing terms (ndarray's remainder, < 8) at terms[chains * pitch].
// Each block carries runs for two candidate binades: the one its estimated
// start lies in, and the neighbour on the nearer side (a block whose estimate
// crosses one power of two gets the binades on both sides).  The f32 chain
// drifts from the exact prefix that the estimate comes from (rounding of
// terms small against the running sum is biased), so the binade it is really
// in can be one off near a boundary; any drift below a factor of sqrt(2)
// still finds a candidate.
struct Pair {
  Summ a, b;
};

constexpr int kChunk = 1024;  // blocks per chunk of the binade-guess scan

struct Plan {
  int chains;
  size_t n, len, pitch, blocks, groups, supers, chunks;
  float* terms;
  double* bsum;   // [chains][blocks] f64 block sums (binade guesses)
  double* csum;   // [chains][chunks] their sums per 1024 blocks
  int2* code;     // [chains][blocks] the two candidate codes
  Pair* l0;       // [chains][blocks] the block's runs under its two codes
  Pair* l1;       // [chains][groups] the 32 blocks composed under the first
                  // block's two codes
  Pair* l2;       // [chains][supers] 32 groups (1024 blocks) composed likewise
  float* chain_out;   // [chains] each chain's sum
  unsigned* done;     // chains finished (zeroed by the term kernel)
};

// Term kernel: terms[] and block sums of term(p[i], t[i]) for i < n, laid out
// as the Plan says.  A CTA tile is 2048 inputs; thread j computes inputs
// 8j..8j+7 of the tile.  With 8 chains those are one element of each chain
// (chain = i % 8, position = i / 8), so the tile is block `tile` of all eight
// chains; with one chain, warp w's 256 inputs are block 8*tile + w.
template <class Term, int CH>
__global__ void __launch_bounds__(kTermThreads)
osum_terms_kernel(const float* __restrict__ p, const float* __restrict__ t, Term term, Plan plan,
                  bool vec) {
  static_assert(CH == 1 || CH == 8, "ndarray's eight chains or one");
  __shared__ double red[kTermThreads / 32][8];
  const size_t lim = plan.len * CH;
  const size_t ntiles = (lim + kTileIn - 1) / kTileIn;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (size_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const size_t base = tile * kTileIn + 8 * (size_t)tid;
    float v[8];
    if (vec && base + 8 <= lim) {
      const float4 a0 = __ldg(reinterpret_cast<const float4*>(p + base));
      const float4 a1 = __ldg(reinterpret_cast<const float4*>(p + base + 4));
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(t + base));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(t + base + 4));
      v[0] = term(a0.x, b0.x); v[1] = term(a0.y, b0.y);
      v[2] = term(a0.z, b0.z); v[3] = term(a0.w, b0.w);
      v[4] = term(a1.x, b1.x); v[5] = term(a1.y, b1.y);
      v[6] = term(a1.z, b1.z); v[7] = term(a1.w, b1.w);
    } else {
#pragma unroll
      for (int k = 0; k < 8; k++) v[k] = base + k < lim ? term(p[base + k], t[base + k]) : 0.0f;
    }
    if constexpr (CH == 8) {
      const size_t pos = tile * kBlock + tid;  // position in every chain
      if (pos < plan.len) {
#pragma unroll
        for (int k = 0; k < 8; k++) plan.terms[k * plan.pitch + pos] = v[k];
      }
      double d[8];
#pragma unroll
      for (int k = 0; k < 8; k++) d[k] = (double)v[k];
      const double r = warp_sum8_transposed(d, lane);
      if ((lane & 3) == 0) red[warp][warp_sum8_slot(lane)] = r;
      __syncthreads();
      if (tid < 8) {
        double acc = 0.0;
#pragma unroll
        for (int w = 0; w < kTermThreads / 32; w++) acc += red[w][tid];
        plan.bsum[tid * plan.blocks + tile] = acc;
      }
      __syncthreads();
    } else {
      if (vec && base + 8 <= lim) {
        *reinterpret_cast<float4*>(plan.terms + base) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(plan.terms + base + 4) = make_float4(v[4], v[5], v[6], v[7]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; k++)
          if (base + k < lim) plan.terms[base + k] = v[k];
      }
      double acc = 0.0;
#pragma unroll
      for (int k = 0; k < 8; k++) acc += (double)v[k];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      const size_t blk = tile * (kTileIn / kBlock) + warp;
      if (lane == 0 && blk < plan.blocks) plan.bsum[blk] = acc;
    }
  }
  if (blockIdx.x == 0 && tid == 0) *plan.done = 0u;
  // ndarray's remainder (n % 8 terms, summed after the chains)
  const size_t rest = plan.n - lim;
  if (blockIdx.x == 0 && (size_t)tid < rest)
    plan.terms[CH * plan.pitch + tid] = term(p[lim + tid], t[lim + tid]);
}

// Plan for n input elements with `chains` chains; scratch_bytes(n, chains)
// bytes of 256-byte-aligned device scratch.
size_t scratch_bytes(size_t n, int chains);
Plan make_plan(void* scratch, size_t n, int chains);
// After a term kernel filled plan.terms and plan.bsum: *out (device) = the
// ordered sum (ndarray's unrolled_fold for 8 chains, init + x0 + x1 + ...
// for one).
cudaError_t launch_ordered_sum(const Plan& plan, float init, float* out, cudaStream_t s);
// Grid of a term kernel for this plan.
int term_grid(const Plan& plan);

}  // namespace osum
}  // namespace rt
