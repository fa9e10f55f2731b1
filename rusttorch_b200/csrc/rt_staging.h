// rt_staging.h — streaming host-memory tensors through the GPU (staging.cu).
#pragma once

#include "../../include/rusttorch_cuda.h"
#include "rt_internal.h"

#include <functional>
#include <vector>

namespace rt {

// Runs one chunk on the device: din/dout are the chunk's device buffers,
// [u0, u0 + cu) the chunk's units.
using StagedLaunch = std::function<cudaError_t(const void* const* din, void* const* dout,
                                               size_t u0, size_t cu, cudaStream_t s)>;

// Default chunk: about kStagedSlotBytes of device memory per pipeline slot.
constexpr size_t kStagedSlotBytes = size_t(64) << 20;
size_t staged_chunk_units(const std::vector<size_t>& in_unit, const std::vector<size_t>& out_unit,
                          const std::vector<int>& out_alias);

// `units` units; input k has in_unit[k] bytes per unit at hin[k], output m
// out_unit[m] bytes per unit at hout[m] (host pointers; hout[m] may be NULL
// to skip the copy back).  out_alias[m] >= 0 makes output m reuse input
// out_alias[m]'s device buffer (in-place kernels).  Synchronous.
cudaError_t staged_map(const std::vector<const void*>& hin, const std::vector<size_t>& in_unit,
                       const std::vector<void*>& hout, const std::vector<size_t>& out_unit,
                       const std::vector<int>& out_alias, size_t units, size_t chunk_units,
                       const StagedLaunch& launch);

// Exact summaries of consecutive chunks of a host float array (in order).
cudaError_t staged_global_stats(const float* host, size_t n,
                                std::vector<rtc_shard_summary>* out);

// The summary of the concatenation of n shards, in order.
rtc_shard_summary compose_summaries(const rtc_shard_summary* parts, size_t n);
// Folds shard summaries in order (see rtc_shard_combine).  Returns false if
// the total is empty (out[0] = sum is still written).
bool combine_summaries(const rtc_shard_summary* parts, size_t n, double out[4]);

}  // namespace rt
