// Host check of the losses' ordered-sum algebra (rusttorch_b200/csrc/rt_osum.cuh),
// built and run by tests/test_osum_algebra.py on the CPU (no GPU needed).
//
//   1. tau_pair_f (f32 rounding) equals tau_pair (integer restatement) for
//      every |x/ulp| < 2^22 and saturates beyond, on sampled floats of many
//      binades and on dense ties;
//   2. a run built with summ_push and applied with summ_apply gives exactly
//      the value of the sequential f32 adds whenever it applies, and
//      composing runs (in either grouping) gives the same run;
//   3. an emulation of the kernels' pipeline (f64 binade guesses, block runs
//      under two candidate codes, 32-block group runs, a walk that folds in
//      order where no run applies) reproduces ndarray's eight-chain sum and a
//      one-chain sum bit for bit on adversarial inputs.
// Prints one line per check and "ALL OK" when every check passed.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "rt_osum.cuh"

using namespace rt::osum;

static float add32(float a, float b) {
  volatile float r = a + b;
  return r;
}

static bool same(float a, float b) { return bits_of(a) == bits_of(b) || (a != a && b != b); }

static int failures = 0;
static void report(const char* what, long bad, long total) {
  std::printf("%-58s %s (%ld bad of %ld)\n", what, bad ? "FAIL" : "ok", bad, total);
  if (bad) failures++;
}

// ---- 1. moves ----------------------------------------------------------------
static void check_moves() {
  long bad = 0, total = 0;
  const int es[] = {-100, -40, -1, 0, 1, 7, 19, 23, 24, 60, 127};
  std::mt19937 rng(1);
  for (int e : es) {
    const float scale = std::ldexp(1.0f, 23 - e);
    for (int i = 0; i < 400000; i++) {
      const uint32_t u = rng();
      const float x = float_of(u);
      int a0, a1, f0, f1;
      tau_pair(x, e, a0, a1);
      tau_pair_f(x, scale, f0, f1);
      total++;
      const double q = std::fabs((double)x * std::ldexp(1.0, 23 - e));
      if (x == x && q < 4194304.0) {
        bad += a0 != f0 || a1 != f1;
      } else {
        bad += !((f0 == kSat || f0 == -kSat) && f1 == f0);
      }
    }
    for (int k = -3000; k < 3000; k++) {  // x/u an odd multiple of 1/2
      const float x = std::ldexp((float)k + 0.5f, e - 23);
      int a0, a1, f0, f1;
      tau_pair(x, e, a0, a1);
      tau_pair_f(x, scale, f0, f1);
      total++;
      bad += a0 != f0 || a1 != f1;
    }
  }
  report("tau_pair_f == tau_pair (sampled + ties)", bad, total);
}

// ---- 2. runs -----------------------------------------------------------------
static Summ run_of(const float* x, int n, int e, int code) {
  Summ r = summ_make(code);
  for (int i = 0; i < n; i++) {
    int m0, m1;
    tau_pair(x[i], e, m0, m1);
    summ_push(r, m0, m1);
  }
  return r;
}

static void check_runs() {
  std::mt19937 rng(2);
  std::uniform_real_distribution<float> U(0.0f, 1.0f);
  long bad = 0, total = 0, applied = 0;
  for (int trial = 0; trial < 20000; trial++) {
    // start in binade e, terms of several scales and signs, some ties
    const int e = (int)(rng() % 40) - 10;
    const float u = std::ldexp(1.0f, e - 23);
    float s = std::ldexp(1.0f + U(rng), e);
    if (rng() & 1) s = -s;
    const int code = s < 0 ? -(e + kCodeBias) : e + kCodeBias;
    const int n = 1 + (int)(rng() % 64);
    std::vector<float> x(n);
    for (int i = 0; i < n; i++) {
      const int kind = (int)(rng() % 4);
      if (kind == 0) x[i] = (float)((int)(rng() % 9) - 4) * 0.5f * u;    // ties and exact
      else if (kind == 1) x[i] = (U(rng) - 0.5f) * 1000.0f * u;
      else if (kind == 2) x[i] = (U(rng) - 0.3f) * std::ldexp(1.0f, e - 6);
      else x[i] = U(rng) * 1e-3f * u;
    }
    float want = s;
    for (int i = 0; i < n; i++) want = add32(want, x[i]);
    const Summ r = run_of(x.data(), n, e, code);
    float got;
    total++;
    if (summ_apply(r, s, &got)) {
      applied++;
      bad += !same(got, want);
    }
    // composition: (first part) then (rest) == whole, for a random split
    const int cut = (int)(rng() % (n + 1));
    const Summ a = run_of(x.data(), cut, e, code), b = run_of(x.data() + cut, n - cut, e, code);
    const Summ ab = summ_compose(a, b);
    float g2;
    const bool ok1 = summ_apply(r, s, &got), ok2 = summ_apply(ab, s, &g2);
    bad += ok1 != ok2 || (ok1 && !same(got, g2));
  }
  report("runs apply exactly and compose (20000 random runs)", bad, total);
  std::printf("  runs that applied: %ld of %ld\n", applied, total);
  if (applied < total / 4) {
    std::printf("  too few runs applied to be a test\n");
    failures++;
  }
}

// ---- 3. pipeline emulation ------------------------------------------------------
static int bcode(int e, bool neg) { return neg ? -(e + kCodeBias) : e + kCodeBias; }

static std::array<int, 2> classify(double start, double end) {
  if (start == 0.0 && end == 0.0) return {kCodeZero, kCodePoison};
  uint64_t a, b;
  std::memcpy(&a, &start, 8);
  std::memcpy(&b, &end, 8);
  if (start == 0.0 || end == 0.0 || (a >> 63) != (b >> 63)) return {kCodePoison, kCodePoison};
  const bool neg = a >> 63;
  const int ea = (int)((a >> 52) & 0x7ff) - 1023, eb = (int)((b >> 52) & 0x7ff) - 1023;
  const int lo = ea < eb ? ea : eb, hi = ea < eb ? eb : ea;
  if (lo < -100 || hi > 127) return {kCodePoison, kCodePoison};
  if (hi == lo + 1) return {bcode(ea, neg), bcode(eb, neg)};
  if (hi != lo) return {kCodePoison, kCodePoison};
  const double mid = std::fabs(0.5 * (start + end));
  const int other = mid < std::ldexp(1.125, ea) ? ea - 1 : (mid >= std::ldexp(1.75, ea) ? ea + 1 : 1000);
  const bool ok = other >= -100 && other <= 127;
  return {bcode(ea, neg), ok ? bcode(other, neg) : kCodePoison};
}

static int code_of(float s) {
  const uint32_t u = bits_of(s);
  const int ex = (int)((u >> 23) & 0xff);
  if ((u & 0x7fffffffu) == 0) return kCodeZero;
  if (ex == 0 || ex == 0xff) return kCodePoison;
  return bcode(ex - 127, u >> 31);
}

static Summ block_run(const float* x, int cnt, int code) {
  const int e = (code < 0 ? -code : code) - kCodeBias;
  const float scale = std::ldexp(1.0f, 23 - e);
  Summ r = summ_make(code);
  for (int j = 0; j < kBlock; j++) {  // past the end: moves of 0
    int m0, m1;
    tau_pair_f(j < cnt ? x[j] : 0.0f, scale, m0, m1);
    summ_push(r, m0, m1);
  }
  return r;
}

static Summ pick(const Summ& a, const Summ& b, int cd) {
  return a.code == cd ? a : (b.code == cd ? b : summ_make(kCodePoison));
}

// One chain's ordered sum from init, the way the kernels compute it.
static float chain_sum(const std::vector<float>& x, float init) {
  const size_t len = x.size(), nb = (len + kBlock - 1) / kBlock, ng = (nb + kGroup - 1) / kGroup;
  std::vector<std::array<int, 2>> code(nb);
  double est = 0.0;
  for (size_t b = 0; b < nb; b++) {
    double bs = 0.0;
    for (size_t i = b * kBlock; i < std::min(len, (b + 1) * kBlock); i++) bs += x[i];
    code[b] = classify(est, est + bs);
    est += bs;
  }
  std::vector<Summ> A(nb), B(nb), GA(ng), GB(ng);
  for (size_t b = 0; b < nb; b++) {
    const int cnt = (int)std::min((size_t)kBlock, len - b * kBlock);
    const float* tb = x.data() + b * kBlock;
    if (code[b][0] == kCodeZero) {
      bool allzero = true, allneg = true;
      for (int j = 0; j < cnt; j++) {
        allzero &= (bits_of(tb[j]) & 0x7fffffffu) == 0;
        allneg &= bits_of(tb[j]) == 0x80000000u;
      }
      A[b] = summ_make(allzero ? kCodeZero : kCodePoison);
      A[b].neg = allneg;
      B[b] = summ_make(kCodePoison);
    } else {
      A[b] = code[b][0] != kCodePoison ? block_run(tb, cnt, code[b][0]) : summ_make(kCodePoison);
      B[b] = code[b][1] != kCodePoison ? block_run(tb, cnt, code[b][1]) : summ_make(kCodePoison);
    }
  }
  for (size_t g = 0; g < ng; g++) {
    const int c1 = A[g * kGroup].code, c2 = B[g * kGroup].code;
    Summ ga = summ_make(kCodeNone), gb = summ_make(kCodeNone);
    for (size_t b = g * kGroup; b < std::min(nb, (g + 1) * kGroup); b++) {
      ga = summ_compose(ga, pick(A[b], B[b], c1));
      gb = summ_compose(gb, pick(A[b], B[b], c2));
    }
    GA[g] = ga;
    GB[g] = c2 != kCodePoison ? gb : summ_make(kCodePoison);
  }
  float s = init;
  size_t b = 0;
  while (b < nb) {
    if (s != s) break;
    if (b % kGroup == 0) {  // whole groups while they apply
      float t;
      if (summ_apply(pick(GA[b / kGroup], GB[b / kGroup], code_of(s)), s, &t)) {
        s = t;
        b = std::min(nb, b + kGroup);
        continue;
      }
    }
    float t;
    if (summ_apply(pick(A[b], B[b], code_of(s)), s, &t)) {
      s = t;
    } else {
      for (size_t i = b * kBlock; i < std::min(len, (b + 1) * kBlock); i++) s = add32(s, x[i]);
    }
    b++;
  }
  return s;
}

static float eight_chain_sum(const std::vector<float>& t) {
  const size_t n = t.size(), len = n / 8;
  float p[8];
  for (int c = 0; c < 8; c++) {
    std::vector<float> ch(len);
    for (size_t i = 0; i < len; i++) ch[i] = t[8 * i + c];
    p[c] = chain_sum(ch, 0.0f);
  }
  float acc = 0.0f;
  for (int j = 0; j < 4; j++) acc = add32(acc, add32(p[j], p[j + 4]));
  for (size_t i = len * 8; i < n; i++) acc = add32(acc, t[i]);
  return acc;
}

static float eight_chain_ref(const std::vector<float>& t) {
  const size_t n = t.size(), lim = n / 8 * 8;
  float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t i = 0; i < lim; i++) p[i % 8] = add32(p[i % 8], t[i]);
  float acc = 0.0f;
  for (int j = 0; j < 4; j++) acc = add32(acc, add32(p[j], p[j + 4]));
  for (size_t i = lim; i < n; i++) acc = add32(acc, t[i]);
  return acc;
}

static void check_pipeline() {
  std::mt19937_64 rng(3);
  std::uniform_real_distribution<float> U(0.0f, 1.0f);
  std::normal_distribution<float> N(0.0f, 1.0f);
  struct Case {
    const char* name;
    size_t n;
    int kind;
  };
  const Case cases[] = {{"uniform", 300001, 0},       {"squares of normal", 262147, 1},
                        {"ties on a grid", 262144, 2}, {"mixed signs", 131072, 3},
                        {"zeros then values", 200000, 4}, {"all -0", 70000, 5},
                        {"NaN inside", 100000, 6},     {"overflow to inf", 90000, 7},
                        {"small n", 13, 0},            {"n = 1", 1, 0}};
  long bad = 0, total = 0;
  for (const Case& cs : cases) {
    std::vector<float> x(cs.n);
    for (size_t i = 0; i < cs.n; i++) {
      switch (cs.kind) {
        case 0: x[i] = U(rng); break;
        case 1: { const float d = N(rng); x[i] = d * d; break; }
        case 2: x[i] = i == 0 ? 1.0f : (float)(rng() % 4) * 0x1p-24f; break;
        case 3: x[i] = N(rng); break;
        case 4: x[i] = i < 70000 ? 0.0f : U(rng); break;
        case 5: x[i] = -0.0f; break;
        case 6: x[i] = i == 77777 ? NAN : U(rng); break;
        default: x[i] = 3.0e33f * U(rng); break;
      }
    }
    const bool ok8 = same(eight_chain_sum(x), eight_chain_ref(x));
    float ref1 = -0.0f;
    for (float v : x) ref1 = add32(ref1, v);
    const bool ok1 = same(chain_sum(x, -0.0f), ref1);
    total += 2;
    bad += !ok8 + !ok1;
    if (!ok8 || !ok1) std::printf("  mismatch: %s (eight chains %s, one chain %s)\n", cs.name,
                                  ok8 ? "ok" : "differs", ok1 ? "ok" : "differs");
  }
  report("pipeline emulation == sequential folds (10 inputs x 2 orders)", bad, total);
}

int main() {
  check_moves();
  check_runs();
  check_pipeline();
  std::printf(failures ? "FAILED %d\n" : "ALL OK\n", failures);
  return failures ? 1 : 0;
}
