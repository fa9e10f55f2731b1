// rt_abi_util.h — helpers of the C-ABI layer: results and error text,
// descriptor checks, device/stream scope, and the exact global statistics.
#pragma once

#include "../../include/rusttorch_cuda.h"
#include "rt_internal.h"

#include <nvtx3/nvToolsExt.h>

#include <string>
#include <vector>

namespace rt {

// ---- results (error text follows rusttorch-core/src/error.rs:69-160) -------
rtc_result ok();
rtc_result fail(int code, const std::string& msg);
rtc_result shape_mismatch(const std::string& context, const rtc_tensor* expected,
                          const rtc_tensor* actual);
rtc_result shape_mismatch_vec(const std::string& context, const std::vector<size_t>& expected,
                              const std::vector<size_t>& actual);
rtc_result dtype_mismatch(const std::string& context, const std::string& expected,
                          const std::string& actual);
rtc_result empty_tensor(const std::string& operation);
rtc_result invalid_dimension(const std::string& context, size_t dim, size_t max_dim);
rtc_result invalid_argument(const std::string& parameter, const std::string& reason);
rtc_result unsupported(const std::string& msg);
rtc_result backend_error(const std::string& what, cudaError_t e);
// Converts a launcher's status into a result.
rtc_result launched(cudaError_t e, const char* what);

#define TRY(expr)                      \
  do {                                 \
    rtc_result _r = (expr);            \
    if (!_r.success) return _r;        \
  } while (0)

// Rust's `{:?}` of a shape ("[2, 3]").
std::string fmt_shape_pub(const std::vector<size_t>& s);
// Rust's `{}` for f64 (shortest round-trip digits, positional notation).
std::string rust_f64(double v);
// Rust's `{:?}` (DType::Float32 ...) and `{}` (float32 ...) for a dtype code.
std::string dtype_debug(int dtype);
std::string dtype_display(int dtype);

// ---- tracing ----------------------------------------------------------------
// An NVTX range named after the C-ABI entry point around each op call, when
// the environment variable RTC_NVTX is 1 at the first call (otherwise one
// load and branch).  Profilers that record NVTX (ncu --nvtx, nsys) then show
// which op every kernel belongs to.  NVTX is header-only: nothing is linked.
bool nvtx_enabled();
struct OpRange {
  bool on;
  explicit OpRange(const char* name) : on(nvtx_enabled()) {
    if (on) nvtxRangePushA(name);
  }
  ~OpRange() {
    if (on) nvtxRangePop();
  }
  OpRange(const OpRange&) = delete;
  OpRange& operator=(const OpRange&) = delete;
};
#define RTC_OP_RANGE() ::rt::OpRange rtc_op_range_(__func__)

// ---- descriptors ------------------------------------------------------------
rtc_result check_desc(const rtc_tensor* t, const char* name);   // structural sanity
bool is_float(int dtype);
bool same_shape(const rtc_tensor* a, const rtc_tensor* b);
std::vector<size_t> shape_vec(const rtc_tensor* t);
std::vector<size_t> reduced_shape(const rtc_tensor* t, size_t dim);
// out must have x's shape and dtype.
rtc_result check_output(const rtc_tensor* x, const rtc_tensor* out, const char* context);
rtc_result require_f32(const rtc_tensor* t, const char* context);
rtc_result same_device(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* c);
void split_dims(const rtc_tensor* t, size_t dim, size_t* outer, size_t* len, size_t* inner);

inline const float* cf(const rtc_tensor* t) { return static_cast<const float*>(t->data); }
inline float* f(const rtc_tensor* t) { return static_cast<float*>(t->data); }

// ---- device / stream --------------------------------------------------------
class DeviceScope {
 public:
  explicit DeviceScope(int device);
  ~DeviceScope();
  bool ok() const { return err_ == cudaSuccess; }
  cudaError_t error() const { return err_; }

 private:
  int prev_ = -1;
  bool changed_ = false;
  cudaError_t err_ = cudaSuccess;
};

cudaStream_t thread_stream();
void set_thread_stream(cudaStream_t s);
// Keeps freed stream-ordered allocations cached in the device's default pool
// (scratch of the reductions is allocated per call with cudaMallocAsync).
void keep_pool_memory(int device);
void release_library_state();
// Destroys the per-device streams of the sharded entry points (abi_sharded.cu).
void release_sharded_streams();

// ---- exact global statistics ------------------------------------------------
// Sum (f64) and the reference's max/min fold results of x[0..n), n > 0.
struct GlobalStats {
  double sum = 0.0;
  float max = 0.0f;
  float min = 0.0f;
  // Order-aware summary used to combine shards (see comm.cu):
  //   max_const: the shard contains a NaN, so the fold's result after this
  //   shard no longer depends on what came before (it is `max`).
  //   first_nan: x[0] is NaN (the min fold then stays NaN).
  bool max_const = false;
  bool first_nan = false;
  // The min fold over the non-NaN elements only (+inf if there are none);
  // equals `min` unless first_nan.
  float min_nonnan = 0.0f;
};
enum { kStatSum = 1, kStatMax = 2, kStatMin = 4 };
// Synchronises `s`.  `x` is a device pointer on the current device.
cudaError_t exact_global_stats(const float* x, size_t n, int device, int want, cudaStream_t s,
                               GlobalStats* out);

}  // namespace rt
