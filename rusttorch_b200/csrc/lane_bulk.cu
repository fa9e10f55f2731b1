// lane_bulk.cu — sum (or mean) along the last axis, rows streamed through a
// cp.async.bulk ring (ops/reduction.rs:75-150, sum_dim / mean_dim).
//
// ndarray reduces each row ("lane") with unrolled_fold: eight strictly
// sequential chains p_j over elements j, j+8, j+16, ..., combined as
// 0 + (p0+p4) + (p1+p5) + (p2+p6) + (p3+p7), then the remaining len % 8
// elements in order.  Here every chain is one thread (a warp = four rows x
// eight chains), and the rows reach shared memory by bulk copies: one thread
// per CTA keeps kStages stages of kChunk floats of each of the CTA's rows in
// flight, so the loads cost the SMs almost no instructions and HBM sees
// long contiguous reads.  A chain thread then adds its floats of the stage
// (kChunk / 8 of them) in order out of shared memory; the row pitch is
// kChunk + 8 floats, so the 32 threads of a warp (rows r..r+3, chains 0..7)
// read 32 different banks.  After a stage is consumed the CTA syncs and the
// copy thread refills it with the chunk kStages further on.
//
// Every wait on a stage is bounded (rt_tma.cuh, 2 s): a CTA that gives up
// raises the library's wait-timeout flag (rtc_synchronize reports it), waits
// (bounded again) for its copies in flight, and returns.  No multicast: each
// copy fills the issuing CTA's own shared memory.
#include "rt_internal.h"
#include "rt_ops.cuh"
#include "rt_tma.cuh"

#include <algorithm>

namespace rt {
namespace {

constexpr int kLbWarps = 4;
constexpr int kLbRows = kLbWarps * 4;             // rows per CTA
constexpr int kLbChunk = 128;                     // floats of each row per stage
constexpr int kLbPitch = kLbChunk + 8;            // floats
constexpr int kLbStages = 4;
constexpr size_t kLbStageFloats = (size_t)kLbRows * kLbPitch;
constexpr size_t kLbSmem = kLbStages * kLbStageFloats * sizeof(float);

__global__ void __launch_bounds__(kLbWarps * 32)
lane_sum8_bulk_kernel(const float* x, size_t lanes, size_t len, float* out, int mean, int* err) {
  extern __shared__ __align__(128) float ring[];
  __shared__ __align__(8) uint64_t full[kLbStages];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t r0 = (size_t)blockIdx.x * kLbRows;
  const int nrows = (int)std::min<size_t>(kLbRows, lanes - r0);
  const size_t steps = len / 8;                    // chain steps per row
  const size_t body = steps * 8;                   // floats the chains cover
  const size_t nchunks = (body + kLbChunk - 1) / kLbChunk;
  if (tid == 0) {
    for (int s = 0; s < kLbStages; s++) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  auto issue = [&](size_t c, int s) {              // chunk c of every row into stage s
    const size_t f0 = c * kLbChunk;
    const unsigned bytes = (unsigned)(std::min<size_t>(kLbChunk, body - f0) * sizeof(float));
    mbar_arrive_expect_tx(&full[s], bytes * (unsigned)nrows);
    float* dst = ring + (size_t)s * kLbStageFloats;
    for (int r = 0; r < nrows; r++)
      bulk_load(dst + (size_t)r * kLbPitch, x + (r0 + r) * len + f0, bytes, &full[s]);
  };
  if (tid == 0)
    for (int s = 0; s < kLbStages && (size_t)s < nchunks; s++) issue(s, s);

  const int rr = lane >> 3, j = lane & 7;
  const int row = warp * 4 + rr;                   // this thread's row in the CTA
  float acc = 0.0f;
  size_t c = 0;
  bool gave_up = false;
  for (; c < nchunks; c++) {
    const int s = (int)(c % kLbStages);
    const unsigned parity = (unsigned)((c / kLbStages) & 1);
    gave_up = __syncthreads_or(!mbar_wait(&full[s], parity));
    if (gave_up) break;
    const float* src = ring + (size_t)s * kLbStageFloats + (size_t)row * kLbPitch + j;
    const int n = (int)(std::min<size_t>(kLbChunk, body - c * kLbChunk) / 8);
    if (n == kLbChunk / 8) {
      float v[kLbChunk / 8];
#pragma unroll
      for (int k = 0; k < kLbChunk / 8; k++) v[k] = src[8 * k];
#pragma unroll
      for (int k = 0; k < kLbChunk / 8; k++) acc = fadd(acc, v[k]);
    } else {
      for (int k = 0; k < n; k++) acc = fadd(acc, src[8 * k]);
    }
    __syncthreads();                               // every thread is done with stage s
    if (tid == 0 && c + kLbStages < nchunks) {
      fence_proxy_async_smem();
      issue(c + kLbStages, s);
    }
  }
  if (gave_up) {
    if (tid == 0) {
      atomicExch(err, 1);
      for (size_t d = c; d < nchunks && d < c + kLbStages; d++)
        mbar_wait(&full[d % kLbStages], (unsigned)((d / kLbStages) & 1));
    }
    return;
  }
  float q[8];
#pragma unroll
  for (int t = 0; t < 8; t++) q[t] = __shfl_sync(0xffffffffu, acc, (lane & ~7) + t);
  if (j == 0 && row < nrows) {
    float r = 0.0f;
    r = fadd(r, fadd(q[0], q[4]));
    r = fadd(r, fadd(q[1], q[5]));
    r = fadd(r, fadd(q[2], q[6]));
    r = fadd(r, fadd(q[3], q[7]));
    const float* xr = x + (r0 + row) * len;
    for (size_t t = body; t < len; t++) r = fadd(r, xr[t]);
    if (mean) r = fdiv(r, (float)len);
    out[r0 + row] = r;
  }
}

}  // namespace

cudaError_t launch_lane_sum_bulk(const float* x, size_t lanes, size_t len, float* out, bool mean,
                                 cudaStream_t s, bool* used) {
  *used = false;
  // 16-byte-aligned row starts for the bulk copies; rows long enough to be
  // worth a ring; enough rows to give every SM a few CTAs.
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0 || len % 4 != 0 || len < 1024 || lanes == 0)
    return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  int* err = wait_timeout_flag(dev);
  if (!err) return cudaSuccess;
  static bool attr_set[64] = {false};
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(
        lane_sum8_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kLbSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const size_t grid = (lanes + kLbRows - 1) / kLbRows;
  for (size_t g0 = 0; g0 < grid; g0 += 0x7fffffffull) {
    const size_t ng = std::min<size_t>(grid - g0, 0x7fffffffull);
    lane_sum8_bulk_kernel<<<(unsigned)ng, kLbWarps * 32, kLbSmem, s>>>(
        x + g0 * kLbRows * len, lanes - g0 * kLbRows, len, out + g0 * kLbRows, mean, err);
  }
  *used = true;
  return cudaGetLastError();
}

}  // namespace rt
