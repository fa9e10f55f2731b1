// staging.cu — ops on tensors in host memory (rtc_tensor.device ==
// RTC_HOST_MEMORY), streamed through the calling thread's current GPU.
//
// The work is cut into chunks; chunk c uses slot c % kSlots, each slot with
// its own device buffers and stream, so the H2D copy of one chunk, the kernel
// of the previous one and the D2H copy of the one before that run at the same
// time (two copy engines, PCIe being full duplex).  Each chunk's copies and
// kernel are ordered on its slot's stream, which also makes buffer reuse
// safe.  Host memory should be page-locked (rtc_host_alloc) for full PCIe
// bandwidth; pageable memory works at the driver's staging speed.
#include "rt_abi_util.h"
#include "rt_staging.h"

#include <algorithm>
#include <cmath>
#include <vector>

namespace rt {

namespace {

constexpr int kSlots = 3;

struct Streams {
  cudaStream_t s[kSlots] = {};
  cudaError_t err = cudaSuccess;
  Streams() {
    for (int i = 0; i < kSlots && err == cudaSuccess; i++)
      err = cudaStreamCreateWithFlags(&s[i], cudaStreamNonBlocking);
  }
  ~Streams() {
    for (auto st : s)
      if (st) cudaStreamDestroy(st);
  }
  cudaError_t sync() {
    cudaError_t e = cudaSuccess;
    for (auto st : s) {
      cudaError_t e2 = cudaStreamSynchronize(st);
      if (e == cudaSuccess) e = e2;
    }
    return e;
  }
};

struct DeviceBlock {
  void* p = nullptr;
  cudaStream_t s = nullptr;
  ~DeviceBlock() {
    if (p) {
      cudaStreamSynchronize(s);
      cudaFreeAsync(p, s);
    }
  }
};

}  // namespace

size_t staged_chunk_units(const std::vector<size_t>& in_unit, const std::vector<size_t>& out_unit,
                          const std::vector<int>& out_alias) {
  size_t unit_bytes = 0;
  for (size_t b : in_unit) unit_bytes += b;
  for (size_t m = 0; m < out_unit.size(); m++)
    if (out_alias[m] < 0) unit_bytes += out_unit[m];
  return std::max<size_t>(1, kStagedSlotBytes / std::max<size_t>(unit_bytes, 1));
}

cudaError_t staged_map(const std::vector<const void*>& hin, const std::vector<size_t>& in_unit,
                       const std::vector<void*>& hout, const std::vector<size_t>& out_unit,
                       const std::vector<int>& out_alias, size_t units, size_t chunk_units,
                       const StagedLaunch& launch) {
  if (units == 0) return cudaSuccess;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  keep_pool_memory(device);
  const size_t chunk = std::min(std::max<size_t>(chunk_units, 1), units);
  const size_t nchunks = (units + chunk - 1) / chunk;
  const int slots = (int)std::min<size_t>(kSlots, nchunks);

  Streams st;
  if (st.err != cudaSuccess) return st.err;
  // One device block per slot: [inputs..., non-aliased outputs...], each
  // region 256-byte aligned.
  std::vector<size_t> in_off(hin.size()), out_off(hout.size());
  size_t slot_bytes = 0;
  for (size_t k = 0; k < hin.size(); k++) {
    in_off[k] = slot_bytes;
    slot_bytes += (chunk * in_unit[k] + 255) & ~size_t(255);
  }
  for (size_t m = 0; m < hout.size(); m++) {
    if (out_alias[m] >= 0) continue;
    out_off[m] = slot_bytes;
    slot_bytes += (chunk * out_unit[m] + 255) & ~size_t(255);
  }
  DeviceBlock block;
  block.s = st.s[0];
  e = cudaMallocAsync(&block.p, slot_bytes * slots, st.s[0]);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(st.s[0]);
  if (e != cudaSuccess) return e;

  std::vector<const void*> din(hin.size());
  std::vector<void*> dout(hout.size());
  for (size_t c = 0; c < nchunks; c++) {
    const int slot = (int)(c % slots);
    cudaStream_t s = st.s[slot];
    char* base = static_cast<char*>(block.p) + slot * slot_bytes;
    const size_t u0 = c * chunk;
    const size_t cu = std::min(chunk, units - u0);
    for (size_t k = 0; k < hin.size(); k++) {
      din[k] = base + in_off[k];
      e = cudaMemcpyAsync(base + in_off[k], static_cast<const char*>(hin[k]) + u0 * in_unit[k],
                          cu * in_unit[k], cudaMemcpyHostToDevice, s);
      if (e != cudaSuccess) return e;
    }
    for (size_t m = 0; m < hout.size(); m++)
      dout[m] = out_alias[m] >= 0 ? const_cast<void*>(din[out_alias[m]]) : base + out_off[m];
    e = launch(din.data(), dout.data(), u0, cu, s);
    if (e != cudaSuccess) return e;
    for (size_t m = 0; m < hout.size(); m++) {
      if (!hout[m]) continue;
      e = cudaMemcpyAsync(static_cast<char*>(hout[m]) + u0 * out_unit[m], dout[m],
                          cu * out_unit[m], cudaMemcpyDeviceToHost, s);
      if (e != cudaSuccess) return e;
    }
  }
  return st.sync();
}

cudaError_t staged_global_stats(const float* host, size_t n,
                                std::vector<rtc_shard_summary>* out) {
  out->clear();
  if (n == 0) return cudaSuccess;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  keep_pool_memory(device);
  const size_t chunk = std::min(n, kStagedSlotBytes / sizeof(float));
  const size_t nchunks = (n + chunk - 1) / chunk;
  const int maxp = stats_num_parts(device, chunk);
  // Per chunk: one StatsPart result slot; per stream slot: block partials.
  StatsPart* results = nullptr;
  e = cudaMallocAsync(reinterpret_cast<void**>(&results), nchunks * sizeof(StatsPart),
                      thread_stream());
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(thread_stream());
  std::vector<StatsPart> host_parts(nchunks);
  const size_t parts_bytes = ((size_t)maxp * sizeof(StatsPart) + 255) & ~size_t(255);
  if (e == cudaSuccess) {
    e = staged_map({host}, {sizeof(float)}, {}, {}, {}, n, chunk,
                   [&](const void* const* din, void* const*, size_t u0, size_t cu,
                       cudaStream_t s) -> cudaError_t {
                     // Block partials live in a small per-chunk scratch from the pool.
                     StatsPart* parts = nullptr;
                     cudaError_t e2 = cudaMallocAsync(reinterpret_cast<void**>(&parts),
                                                      parts_bytes, s);
                     if (e2 != cudaSuccess) return e2;
                     const int np = stats_num_parts(device, cu);
                     e2 = launch_stats(static_cast<const float*>(din[0]), cu, parts, np,
                                       results + u0 / chunk, s);
                     cudaFreeAsync(parts, s);
                     return e2;
                   });
  }
  if (e == cudaSuccess)
    e = cudaMemcpy(host_parts.data(), results, nchunks * sizeof(StatsPart),
                   cudaMemcpyDeviceToHost);
  cudaFreeAsync(results, thread_stream());
  if (e != cudaSuccess) return e;

  // Chunks whose fast statistics may differ from the reference's fold (a NaN,
  // or a zero extreme) are copied once more and summarised exactly.
  float* redo = nullptr;
  for (size_t c = 0; c < nchunks; c++) {
    const size_t u0 = c * chunk, cu = std::min(chunk, n - u0);
    const StatsPart& h = host_parts[c];
    rtc_shard_summary s{};
    s.count = cu;
    s.sum = h.sum;
    if (!std::isnan(h.sum) && h.mx != 0.0f && h.mn != 0.0f) {
      s.max = h.mx;
      s.max_kind = 1;
      s.min_nonnan = h.mn;
      s.first_nan = 0;
    } else {
      cudaStream_t ts = thread_stream();
      if (!redo) {
        e = cudaMallocAsync(reinterpret_cast<void**>(&redo), chunk * sizeof(float), ts);
        if (e != cudaSuccess) return e;
      }
      e = cudaMemcpyAsync(redo, host + u0, cu * sizeof(float), cudaMemcpyHostToDevice, ts);
      GlobalStats g;
      if (e == cudaSuccess)
        e = exact_global_stats(redo, cu, device, kStatSum | kStatMax | kStatMin, ts, &g);
      if (e != cudaSuccess) {
        cudaFreeAsync(redo, ts);
        return e;
      }
      s.sum = g.sum;
      s.max = g.max;
      s.max_kind = g.max_const ? 2 : 1;
      s.min_nonnan = g.min_nonnan;
      s.first_nan = g.first_nan ? 1 : 0;
    }
    out->push_back(s);
  }
  if (redo) {
    cudaFreeAsync(redo, thread_stream());
    e = cudaStreamSynchronize(thread_stream());
  }
  return e;
}

// Composition of the shards' fold functions (reduction.rs:36-40, :58-62):
// for max, a shard holding a NaN restarts the fold (the value after it no
// longer depends on earlier shards), and Equal keeps the later element; for
// min, NaN is skipped unless it is the very first element, and Equal keeps
// the earlier element.
rtc_shard_summary compose_summaries(const rtc_shard_summary* parts, size_t n) {
  rtc_shard_summary t{};
  t.min_nonnan = INFINITY;
  for (size_t i = 0; i < n; i++) {
    const rtc_shard_summary& p = parts[i];
    t.sum += p.sum;
    if (p.count == 0) continue;
    if (t.count == 0) {
      t.first_nan = p.first_nan;
      t.max_kind = p.max_kind;
      t.max = p.max;
    } else if (p.max_kind == 2) {
      t.max_kind = 2;
      t.max = p.max;
    } else {
      t.max = t.max > p.max ? t.max : p.max;
    }
    t.min_nonnan = t.min_nonnan > p.min_nonnan ? p.min_nonnan : t.min_nonnan;
    t.count += p.count;
  }
  return t;
}

bool combine_summaries(const rtc_shard_summary* parts, size_t n, double out[4]) {
  const rtc_shard_summary t = compose_summaries(parts, n);
  out[0] = t.sum;
  if (t.count == 0) {
    out[1] = out[2] = out[3] = NAN;
    return false;
  }
  out[1] = t.sum / (double)t.count;
  out[2] = (double)t.max;
  out[3] = t.first_nan ? (double)NAN : (double)t.min_nonnan;
  return true;
}

}  // namespace rt
