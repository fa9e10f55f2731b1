// strip_tma.cu — reductions along a non-last axis with TMA-staged tiles.
//
// x is C-contiguous [outer, len, inner]; out[o, c] folds x[o, 0..len, c] in
// row order (ndarray's sum_axis / fold_axis: res = res + row), strictly
// sequentially per column, so the result is bit-identical to the reference.
//
// CTA (o, s) owns columns [c0, c0 + W).  One producer thread streams
// [R rows x W columns] tiles of its strip into an S-deep shared-memory ring
// with TMA (cp.async.bulk.tensor, completion counted on a "full" mbarrier per
// slot); each consumer thread runs one column's chain out of shared memory
// and each consumer warp releases a slot through its "empty" mbarrier.  The
// producer runs ahead of the chains by up to S tiles with no CTA-wide
// barrier, so HBM latency is hidden by bytes in flight while the chains —
// the only sequential part — run back to back.
#include "rt_internal.h"
#include "rt_fold.cuh"
#include "rt_ops.cuh"
#include "rt_tma.cuh"

#include <algorithm>

namespace rt {
namespace {

constexpr int kMaxStages = 8;
constexpr int kStageAlign = 128;            // bytes; TMA destinations are 16-byte aligned

// WT > 0: the strip width W known at compile time, so a column's chain walks
// the tile with immediate offsets (one pointer step per eight rows) instead
// of a multiply-add per element; WT = 0: W at run time.
template <int OP, int WT>
__global__ void __launch_bounds__(288)
strip_tma_kernel(const __grid_constant__ CUtensorMap tm, const float* x, size_t len,
                 size_t inner, int W_rt, int R, int S, size_t strips, float* out, int* err) {
  const int W = WT > 0 ? WT : W_rt;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  const size_t o = blockIdx.x / strips;
  const size_t s = blockIdx.x % strips;
  const size_t c0 = s * (size_t)W;
  const int w_eff = (int)min((size_t)W, inner - c0);
  const size_t nstage = (len + R - 1) / R;
  const int consumer_warps = (W + 31) / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t stage_floats =
      (((size_t)R * W * sizeof(float) + kStageAlign - 1) / kStageAlign) * kStageAlign / 4;
  float* ring = reinterpret_cast<float*>(smem_raw);
  const unsigned tile_bytes = (unsigned)((size_t)R * W * sizeof(float));

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], consumer_warps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == consumer_warps) {
    // ---- producer
    if (lane == 0) {
      size_t issued = 0;
      bool ok = true;
      int slot = 0;
      unsigned round = 0;              // parity of st / S
      for (size_t st = 0; st < nstage; st++) {
        // slot's previous tile (round - 1) must have been consumed
        if (st >= (size_t)S && !mbar_wait(&empty[slot], round ^ 1u)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[slot], tile_bytes);
        tma_load_3d(ring + slot * stage_floats, &tm, &full[slot], (int)c0, (int)(st * R), (int)o);
        issued = st + 1;
        if (++slot == S) {
          slot = 0;
          round ^= 1u;
        }
      }
      // Wait (bounded) until every tile this thread issued has landed, so no
      // copy is still writing when the CTA exits.
      for (int k = 0; k < S && (size_t)k < issued; k++) {
        const size_t last = k + ((issued - 1 - k) / S) * S;
        if (!mbar_wait(&full[k], (unsigned)(last / S) & 1u)) ok = false;
      }
      if (!ok) atomicExch(err, 1);
    }
    return;
  }

  // ---- consumers: thread tid folds column c0 + tid
  const int tid = threadIdx.x;
  float acc = (OP == kDimMax) ? -INFINITY : 0.0f;
  bool nan = false;
  int slot = 0;
  unsigned round = 0;
  for (size_t st = 0; st < nstage; st++) {
    if (!mbar_wait(&full[slot], round)) {
      atomicExch(err, 1);
      return;
    }
    const int rows = (int)min((size_t)R, len - st * R);
    auto step = [&](float v) {
      if (OP == kDimMax) {
        nan |= v != v;
        acc = fmaxf(acc, v);
      } else {
        acc = fadd(acc, v);
      }
    };
    if (tid < w_eff) {
      if constexpr (WT > 0)
        fold_pipelined_fixed<WT>(ring + slot * stage_floats + tid, rows, step);
      else
        fold_pipelined(ring + slot * stage_floats + tid, W, rows, step);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (++slot == S) {
      slot = 0;
      round ^= 1u;
    }
  }
  if (tid < w_eff) {
    // fmaxf's maximum equals the reference fold except with a NaN present
    // or a zero maximum (sign of zero); re-fold those columns in order.
    if (OP == kDimMax && (nan || acc == 0.0f)) {
      const float* col = x + o * len * inner + c0 + tid;
      float m = col[0];
      for (size_t l = 1; l < len; l++) m = max_fold(m, col[l * inner]);
      acc = m;
    }
    if (OP == kDimMean) acc = fdiv(acc, (float)len);
    out[o * inner + c0 + tid] = acc;
  }
}

int cur_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

}  // namespace

cudaError_t launch_strip_tma(DimReduce op, const float* x, size_t outer, size_t len,
                             size_t inner, float* out, cudaStream_t st, bool* used) {
  *used = false;
  // TMA: 16-byte-aligned base and row stride, coordinates fit in int32.
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || inner % 4 || inner < 4 || len == 0 ||
      len >= (1ull << 31) || inner >= (1ull << 31) || outer >= (1ull << 31))
    return cudaSuccess;
  const int sms = sm_count(cur_device());
  // Every CTA folds its strip over all `len` rows, so a second, partial wave
  // of CTAs would nearly double the time: pick the narrowest strip (at
  // least 32 columns, when there are enough columns) whose CTAs all fit on
  // the GPU at once.  A stage is about 10 KB (R rows x W columns); S = 4.
  const int S = 4;
  const size_t cols = outer * inner;
  auto rows_for = [&](size_t w) {
    return std::min<size_t>(len, std::min<size_t>(256, std::max<size_t>(32, 10240 / (4 * w))));
  };
  auto smem_for = [&](size_t w) {
    return (size_t)S * (((rows_for(w) * w * sizeof(float)) + kStageAlign - 1) / kStageAlign) *
           kStageAlign;
  };
  auto resident = [&](size_t w) {
    const size_t by_smem = (size_t)(227u << 10) / (smem_for(w) + 1024);
    const size_t by_threads = 2048 / (((w + 31) / 32 + 1) * 32);
    return (size_t)sms * std::min<size_t>({by_smem, by_threads, 32});
  };
  size_t W = (cols + 2 * (size_t)sms - 1) / (2 * (size_t)sms);   // about 2 CTAs per SM
  W = std::min<size_t>(32, std::max<size_t>(4, (W + 3) & ~size_t(3)));
  while (W < 256 && outer * ((inner + W - 1) / W) > resident(W)) W += 16;
  W = std::min(W, inner);
  const size_t ctas = outer * ((inner + W - 1) / W);
  size_t R = rows_for(W);
  size_t stage = smem_for(W) / S;
  // With at most two CTAs per SM (few, narrow strips: e.g. 4096 columns
  // folded over many rows) each CTA can take tiles of 256 rows and a deeper
  // ring at no cost in residency, keeping two CTAs' rings within an SM.
  int stages = S;
  // The compiled-in widths pay off where the chains are long and few CTAs
  // share an SM ([1, C] gradient of cfg4: 0.48 -> 0.62); with many CTAs per
  // SM (cfg3's dim-0 sums) the run-time-width kernel measured 0.966 against
  // 0.943.
  const bool few = ctas <= 2 * (size_t)sms;
  if (few) {
    const size_t half = (size_t)(227u << 10) / 2 - 1024;   // one of two CTAs per SM
    R = std::min<size_t>({len, 256, std::max<size_t>(8, half / 2 / (W * sizeof(float)))});
    stage = ((R * W * sizeof(float) + kStageAlign - 1) / kStageAlign) * kStageAlign;
    stages = (int)std::min<size_t>(kMaxStages, std::max<size_t>(2, half / stage));
  }
  return launch_strip_tma_shape(op, x, outer, len, inner, out, st, used, W, R, stages, few);
}

// The launch for a given strip width W (columns per CTA), tile height R and
// ring depth; *used = false (nothing launched) when the shape cannot be
// encoded or does not fit in shared memory.  W is a multiple of 4, so every
// strip's first column c0 = s*W — the tiles' innermost TMA coordinate —
// starts on a 16-byte boundary.
cudaError_t launch_strip_tma_shape(DimReduce op, const float* x, size_t outer, size_t len,
                                   size_t inner, float* out, cudaStream_t st, bool* used,
                                   size_t W, size_t R, int stages, bool fixed_width) {
  *used = false;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || inner % 4 || inner < 4 || len == 0 ||
      len >= (1ull << 31) || inner >= (1ull << 31) || outer >= (1ull << 31) || W < 4 ||
      W % 4 || W > 256 || W > inner || R < 1 || R > 256 || R > len || stages < 2 ||
      stages > kMaxStages)
    return cudaSuccess;
  const int dev = cur_device();
  int* err = wait_timeout_flag(dev);
  if (!err) return cudaSuccess;
  const size_t strips = (inner + W - 1) / W;
  const size_t ctas = outer * strips;
  if (ctas >= (1ull << 31)) return cudaSuccess;
  const size_t stage = ((R * W * sizeof(float) + kStageAlign - 1) / kStageAlign) * kStageAlign;
  const size_t smem = stage * stages;
  if (smem > (227u << 10)) return cudaSuccess;

  CUtensorMap tm;
  const uint64_t dims[3] = {inner, len, outer};
  const uint64_t strides[2] = {inner * sizeof(float), len * inner * sizeof(float)};
  const uint32_t box[3] = {(uint32_t)W, (uint32_t)R, 1};
  if (!encode_tensor_map_f32(&tm, x, 3, dims, strides, box)) return cudaSuccess;

  const int threads = ((int)((W + 31) / 32) + 1) * 32;
  auto go = [&](auto kernel) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    kernel<<<(unsigned)ctas, threads, smem, st>>>(tm, x, len, inner, (int)W, (int)R, stages,
                                                  strips, out, err);
    return cudaGetLastError();
  };
  cudaError_t e = cudaErrorInvalidValue;
  const int wt = fixed_width ? (int)W : 0;
  switch (op) {
#define RT_STRIP_TMA(OPV)                                               \
  case OPV:                                                             \
    e = wt == 16   ? go(strip_tma_kernel<OPV, 16>)                      \
        : wt == 32 ? go(strip_tma_kernel<OPV, 32>)                      \
                   : go(strip_tma_kernel<OPV, 0>);                      \
    break;
    RT_STRIP_TMA(kDimSum)
    RT_STRIP_TMA(kDimMean)
    RT_STRIP_TMA(kDimMax)
#undef RT_STRIP_TMA
  }
  if (e == cudaSuccess) *used = true;
  return e;
}

}  // namespace rt
