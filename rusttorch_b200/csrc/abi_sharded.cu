// abi_sharded.cu — one process driving a tensor split over several GPUs.
//
// The reference has no multi-device path; these entry points are the
// single-process form of the sharding bench.py does with one process per
// GPU.  A logical tensor is given as n shards (one rtc_tensor each, each on
// its own device); every op here is one whose shards need no exchange:
//  - elementwise (add -> mul_scalar) and AdamW: shard i of every operand
//    holds the same elements, any split;
//  - softmax and the dim reductions: the split axis is not the reduced one
//    (row blocks for the last axis, column blocks for dim 0 of a matrix:
//    each column block is its own contiguous [R, C_i] tensor).
// Each call checks every shard first (so an argument error launches
// nothing), waits for the work already queued on the shards' devices (the
// shards may come from other streams), queues every shard on a stream of its
// device owned by the library — all devices work at once, launched from the
// calling thread — and returns when every shard is done.  Per-shard work is
// the single-device entry point's, so results are those of rtc_add_mul_scalar,
// rtc_softmax, rtc_sum_dim, rtc_adamw_update on each shard.
#include "../../include/rusttorch_cuda.h"
#include "rt_abi_util.h"
#include "rt_internal.h"

#include <algorithm>
#include <functional>
#include <mutex>
#include <string>
#include <vector>

using namespace rt;

namespace {

std::mutex g_stream_mu;
std::vector<cudaStream_t> g_streams;   // one per device, created on first use

// The library's stream on `device` (the device must be current).
cudaError_t device_stream(int device, cudaStream_t* out) {
  std::lock_guard<std::mutex> lock(g_stream_mu);
  if ((size_t)device >= g_streams.size()) g_streams.resize(device + 1, nullptr);
  if (!g_streams[device]) {
    cudaError_t e = cudaStreamCreateWithFlags(&g_streams[device], cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      g_streams[device] = nullptr;
      return e;
    }
  }
  *out = g_streams[device];
  return cudaSuccess;
}

// Every tensor of one shard on one GPU, f32, C-contiguous descriptors.
rtc_result check_shard(const rtc_tensor* const* ts, size_t k, const char* what) {
  for (size_t j = 0; j < k; j++) {
    TRY(check_desc(ts[j], what));
    if (ts[j]->device < 0)
      return unsupported(std::string(what) + ": sharded ops take device tensors");
    if (ts[j]->device != ts[0]->device)
      return invalid_argument("shards", "every tensor of a shard must be on one device");
    TRY(require_f32(ts[j], what));
  }
  return ok();
}

// Runs launch(i) for every shard i on shard i's device with the library's
// stream as the calling thread's stream, after waiting for the devices' queued
// work; then waits for every device's stream.  Returns the first error.
rtc_result run_sharded(size_t n, const std::function<int(size_t)>& device_of,
                       const std::function<rtc_result(size_t)>& launch) {
  std::vector<int> devices;
  for (size_t i = 0; i < n; i++) {
    const int d = device_of(i);
    if (std::find(devices.begin(), devices.end(), d) == devices.end()) devices.push_back(d);
  }
  for (int d : devices) {
    DeviceScope scope(d);
    if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return backend_error("cudaDeviceSynchronize", e);
  }
  const cudaStream_t caller = thread_stream();
  rtc_result first = ok();
  for (size_t i = 0; i < n && first.success; i++) {
    DeviceScope scope(device_of(i));
    if (!scope.ok()) {
      first = backend_error("cudaSetDevice", scope.error());
      break;
    }
    cudaStream_t s = nullptr;
    cudaError_t e = device_stream(device_of(i), &s);
    if (e != cudaSuccess) {
      first = backend_error("cudaStreamCreate", e);
      break;
    }
    set_thread_stream(s);
    first = launch(i);
  }
  set_thread_stream(caller);
  for (int d : devices) {
    DeviceScope scope(d);
    cudaStream_t s = nullptr;
    if (!scope.ok() || device_stream(d, &s) != cudaSuccess) continue;
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess && first.success) first = backend_error("cudaStreamSynchronize", e);
  }
  return first;
}

rtc_result check_list(const void* p, size_t n, const char* name) {
  if (n > 0 && !p) return invalid_argument(name, "must not be null");
  return ok();
}

// Shapes of corresponding shards must match (a, b and out of one op).
rtc_result same_shapes(const rtc_tensor* a, const rtc_tensor* b, const char* context) {
  if (!same_shape(a, b)) return shape_mismatch(context, a, b);
  return ok();
}

}  // namespace

namespace rt {
void release_sharded_streams() {
  std::lock_guard<std::mutex> lock(g_stream_mu);
  for (size_t d = 0; d < g_streams.size(); d++) {
    if (!g_streams[d]) continue;
    DeviceScope scope((int)d);
    cudaStreamDestroy(g_streams[d]);
    g_streams[d] = nullptr;
  }
}
}  // namespace rt

// ------------------------------------------------------------ entry points

extern "C" rtc_result rtc_sharded_add_mul_scalar(const rtc_tensor* a, const rtc_tensor* b,
                                                 float scalar, const rtc_tensor* out,
                                                 size_t n_shards) {
  RTC_OP_RANGE();
  TRY(check_list(a, n_shards, "a"));
  TRY(check_list(b, n_shards, "b"));
  TRY(check_list(out, n_shards, "out"));
  for (size_t i = 0; i < n_shards; i++) {
    const rtc_tensor* t[3] = {&a[i], &b[i], &out[i]};
    TRY(check_shard(t, 3, "shard"));
    TRY(same_shapes(&a[i], &b[i], "add"));
    TRY(same_shapes(&a[i], &out[i], "add_mul_scalar output"));
  }
  return run_sharded(
      n_shards, [&](size_t i) { return a[i].device; },
      [&](size_t i) { return rtc_add_mul_scalar(&a[i], &b[i], scalar, &out[i]); });
}

extern "C" rtc_result rtc_sharded_softmax(const rtc_tensor* x, size_t dim, const rtc_tensor* out,
                                          size_t n_shards) {
  RTC_OP_RANGE();
  TRY(check_list(x, n_shards, "x"));
  TRY(check_list(out, n_shards, "out"));
  for (size_t i = 0; i < n_shards; i++) {
    const rtc_tensor* t[2] = {&x[i], &out[i]};
    TRY(check_shard(t, 2, "shard"));
    if (dim >= x[i].ndim) return invalid_dimension("softmax", dim, x[i].ndim == 0 ? 0 : x[i].ndim - 1);
    TRY(same_shapes(&x[i], &out[i], "softmax output"));
  }
  if (dim == 0 && n_shards > 1)
    return invalid_argument("dim", "the shards split axis 0 (row blocks): softmax along it "
                                   "would need an exchange between shards");
  return run_sharded(
      n_shards, [&](size_t i) { return x[i].device; },
      [&](size_t i) { return rtc_softmax(&x[i], dim, &out[i]); });
}

namespace {

rtc_result sharded_dim(rtc_result (*fn)(const rtc_tensor*, size_t, const rtc_tensor*),
                       const char* context, const rtc_tensor* x, size_t dim,
                       const rtc_tensor* out, size_t n_shards) {
  TRY(check_list(x, n_shards, "x"));
  TRY(check_list(out, n_shards, "out"));
  for (size_t i = 0; i < n_shards; i++) {
    const rtc_tensor* t[2] = {&x[i], &out[i]};
    TRY(check_shard(t, 2, "shard"));
    if (dim >= x[i].ndim) return invalid_dimension(context, dim, x[i].ndim == 0 ? 0 : x[i].ndim - 1);
    if (shape_vec(&out[i]) != reduced_shape(&x[i], dim))
      return shape_mismatch_vec(context, reduced_shape(&x[i], dim), shape_vec(&out[i]));
  }
  return run_sharded(
      n_shards, [&](size_t i) { return x[i].device; },
      [&](size_t i) { return fn(&x[i], dim, &out[i]); });
}

}  // namespace

extern "C" rtc_result rtc_sharded_sum_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out,
                                          size_t n_shards) {
  RTC_OP_RANGE();
  return sharded_dim(rtc_sum_dim, "sum_dim", x, dim, out, n_shards);
}

extern "C" rtc_result rtc_sharded_mean_dim(const rtc_tensor* x, size_t dim,
                                           const rtc_tensor* out, size_t n_shards) {
  RTC_OP_RANGE();
  return sharded_dim(rtc_mean_dim, "mean_dim", x, dim, out, n_shards);
}

extern "C" rtc_result rtc_sharded_max_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out,
                                          size_t n_shards) {
  RTC_OP_RANGE();
  return sharded_dim(rtc_max_dim, "max_dim", x, dim, out, n_shards);
}

extern "C" rtc_result rtc_sharded_adamw_update(const rtc_tensor* params, const rtc_tensor* grads,
                                               const rtc_tensor* m, const rtc_tensor* v,
                                               double learning_rate, double beta1, double beta2,
                                               double epsilon, double weight_decay,
                                               uint64_t timestep, size_t n_shards) {
  RTC_OP_RANGE();
  TRY(check_list(params, n_shards, "params"));
  TRY(check_list(grads, n_shards, "grads"));
  TRY(check_list(m, n_shards, "m"));
  TRY(check_list(v, n_shards, "v"));
  for (size_t i = 0; i < n_shards; i++) {
    const rtc_tensor* t[4] = {&params[i], &grads[i], &m[i], &v[i]};
    TRY(check_shard(t, 4, "shard"));
    TRY(same_shapes(&params[i], &grads[i], "adamw_update"));
    TRY(same_shapes(&params[i], &m[i], "adamw_update"));
    TRY(same_shapes(&params[i], &v[i], "adamw_update"));
  }
  // The hyperparameters are the same for every shard: shard 0's call rejects
  // bad ones before anything is launched.
  return run_sharded(
      n_shards, [&](size_t i) { return params[i].device; },
      [&](size_t i) {
        return rtc_adamw_update(&params[i], &grads[i], &m[i], &v[i], learning_rate, beta1, beta2,
                                epsilon, weight_decay, timestep, &params[i], &m[i], &v[i]);
      });
}
