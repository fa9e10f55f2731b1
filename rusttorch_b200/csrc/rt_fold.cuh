// rt_fold.cuh — sequential folds out of shared memory with the loads one
// batch ahead of the chain.
//
// A sequential chain (acc = acc + v, in order) is bound by the add's latency
// only if the next values are already in registers.  fold_pipelined loads
// values k+8..k+15 before adding values k..k+7, so shared-memory latency is
// overlapped with the eight dependent adds.
#pragma once

namespace rt {

// step(v) for v = p[0], p[s], p[2s], ..., p[(n-1)s], in that order.
template <class Step>
__device__ __forceinline__ void fold_pipelined(const float* p, int s, int n, Step&& step) {
  int k = 0;
  if (n >= 8) {
    float cur[8];
#pragma unroll
    for (int u = 0; u < 8; u++) cur[u] = p[u * s];
    for (k = 8; k + 8 <= n; k += 8) {
      float nxt[8];
#pragma unroll
      for (int u = 0; u < 8; u++) nxt[u] = p[(k + u) * s];
#pragma unroll
      for (int u = 0; u < 8; u++) step(cur[u]);
#pragma unroll
      for (int u = 0; u < 8; u++) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < 8; u++) step(cur[u]);
  }
  for (; k < n; k++) step(p[k * s]);
}

// The same with the stride S known at compile time: every load of a batch
// is an immediate offset from one pointer, which steps once per batch.
template <int S, class Step>
__device__ __forceinline__ void fold_pipelined_fixed(const float* p, int n, Step&& step) {
  int k = 0;
  if (n >= 8) {
    float cur[8];
#pragma unroll
    for (int u = 0; u < 8; u++) cur[u] = p[u * S];
    const float* q = p + 8 * S;
    for (k = 8; k + 8 <= n; k += 8, q += 8 * S) {
      float nxt[8];
#pragma unroll
      for (int u = 0; u < 8; u++) nxt[u] = q[u * S];
#pragma unroll
      for (int u = 0; u < 8; u++) step(cur[u]);
#pragma unroll
      for (int u = 0; u < 8; u++) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < 8; u++) step(cur[u]);
  }
  for (; k < n; k++) step(p[k * S]);
}

}  // namespace rt
