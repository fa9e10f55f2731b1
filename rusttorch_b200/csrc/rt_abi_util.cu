// rt_abi_util.cu — see rt_abi_util.h.
#include "rt_abi_util.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace rt {

// ------------------------------------------------------------------- results

rtc_result ok() {
  rtc_result r;
  r.success = true;
  r.error_msg = nullptr;
  r.code = RTC_OK;
  return r;
}

rtc_result fail(int code, const std::string& msg) {
  rtc_result r;
  r.success = false;
  r.code = code;
  r.error_msg = static_cast<char*>(std::malloc(msg.size() + 1));
  if (r.error_msg) std::memcpy(r.error_msg, msg.c_str(), msg.size() + 1);
  return r;
}

static std::string fmt_shape(const std::vector<size_t>& s) {
  std::string out = "[";
  for (size_t i = 0; i < s.size(); i++) {
    if (i) out += ", ";
    out += std::to_string(s[i]);
  }
  return out + "]";
}

std::string fmt_shape_pub(const std::vector<size_t>& s) { return fmt_shape(s); }

rtc_result shape_mismatch_vec(const std::string& context, const std::vector<size_t>& expected,
                              const std::vector<size_t>& actual) {
  return fail(RTC_SHAPE_MISMATCH, "Shape mismatch in " + context + ": expected " +
                                      fmt_shape(expected) + ", got " + fmt_shape(actual));
}

rtc_result shape_mismatch(const std::string& context, const rtc_tensor* expected,
                          const rtc_tensor* actual) {
  return shape_mismatch_vec(context, shape_vec(expected), shape_vec(actual));
}

rtc_result dtype_mismatch(const std::string& context, const std::string& expected,
                          const std::string& actual) {
  return fail(RTC_DTYPE_MISMATCH,
              "Data type mismatch in " + context + ": expected " + expected + ", got " + actual);
}

rtc_result empty_tensor(const std::string& operation) {
  return fail(RTC_EMPTY_TENSOR, "Cannot perform " + operation + " on empty tensor");
}

rtc_result invalid_dimension(const std::string& context, size_t dim, size_t max_dim) {
  return fail(RTC_INVALID_DIMENSION, "Invalid dimension in " + context + ": " +
                                         std::to_string(dim) + " (max: " +
                                         std::to_string(max_dim) + ")");
}

rtc_result invalid_argument(const std::string& parameter, const std::string& reason) {
  return fail(RTC_INVALID_ARGUMENT, "Invalid argument '" + parameter + "': " + reason);
}

rtc_result unsupported(const std::string& msg) { return fail(RTC_UNSUPPORTED, msg); }

rtc_result backend_error(const std::string& what, cudaError_t e) {
  return fail(RTC_BACKEND_ERROR, "CUDA error in " + what + ": " + cudaGetErrorName(e) + " (" +
                                     cudaGetErrorString(e) + ")");
}

rtc_result launched(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return backend_error(what, e);
  return ok();
}

std::string rust_f64(double v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v < 0 ? "-inf" : "inf";
  if (v == 0.0) return std::signbit(v) ? "-0" : "0";
  // Shortest digit string that round-trips (what Rust's Display prints).
  char buf[64];
  int prec = 1;
  for (; prec <= 17; prec++) {
    std::snprintf(buf, sizeof buf, "%.*e", prec - 1, v);
    if (std::strtod(buf, nullptr) == v) break;
  }
  std::string s(buf);
  const bool neg = s[0] == '-';
  if (neg) s.erase(0, 1);
  const size_t epos = s.find('e');
  const int exp10 = std::atoi(s.c_str() + epos + 1);
  std::string digits;
  for (size_t i = 0; i < epos; i++)
    if (s[i] != '.') digits += s[i];
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  std::string out;
  const int nd = (int)digits.size();
  if (exp10 >= nd - 1) {
    out = digits + std::string((size_t)(exp10 - (nd - 1)), '0');
  } else if (exp10 >= 0) {
    out = digits.substr(0, (size_t)exp10 + 1) + "." + digits.substr((size_t)exp10 + 1);
  } else {
    out = "0." + std::string((size_t)(-exp10 - 1), '0') + digits;
  }
  return neg ? "-" + out : out;
}

std::string dtype_debug(int dtype) {
  switch (dtype) {
    case RTC_F32: return "Float32";
    case RTC_F64: return "Float64";
    case RTC_I32: return "Int32";
    case RTC_I64: return "Int64";
  }
  return "Unknown(" + std::to_string(dtype) + ")";
}

std::string dtype_display(int dtype) {
  switch (dtype) {
    case RTC_F32: return "float32";
    case RTC_F64: return "float64";
    case RTC_I32: return "int32";
    case RTC_I64: return "int64";
  }
  return "unknown(" + std::to_string(dtype) + ")";
}

// --------------------------------------------------------------- descriptors

rtc_result check_desc(const rtc_tensor* t, const char* name) {
  if (!t) return invalid_argument(name, "tensor descriptor must not be null");
  if (t->dtype < RTC_F32 || t->dtype > RTC_I64)
    return invalid_argument("dtype", "Unknown dtype code: " + std::to_string(t->dtype));
  if (t->ndim > 0 && !t->shape) return invalid_argument(name, "shape must not be null");
  size_t prod = 1;
  for (size_t i = 0; i < t->ndim; i++) {
    if (t->shape[i] != 0 && prod > SIZE_MAX / t->shape[i])
      return fail(RTC_SIZE_OVERFLOW, "Tensor size overflow: dimensions " +
                                         fmt_shape(shape_vec(t)) + " would exceed maximum size");
    prod *= t->shape[i];
  }
  if (prod != t->numel)
    return invalid_argument("shape", "Shape and data length mismatch: shape " +
                                         fmt_shape(shape_vec(t)) + " holds " +
                                         std::to_string(prod) + " elements, numel is " +
                                         std::to_string(t->numel));
  if (t->strides) {
    size_t expect = 1;
    for (size_t i = t->ndim; i-- > 0;) {
      if (t->shape[i] != 1 && t->strides[i] != expect)
        return unsupported(std::string(name) +
                           ": non-contiguous tensors are not supported by the CUDA path");
      expect *= t->shape[i];
    }
  }
  if (t->numel > 0 && !t->data) return invalid_argument(name, "data must not be null");
  return ok();
}

bool is_float(int dtype) { return dtype == RTC_F32 || dtype == RTC_F64; }

std::vector<size_t> shape_vec(const rtc_tensor* t) {
  std::vector<size_t> v;
  for (size_t i = 0; i < t->ndim; i++) v.push_back(t->shape[i]);
  return v;
}

std::vector<size_t> reduced_shape(const rtc_tensor* t, size_t dim) {
  std::vector<size_t> v;
  for (size_t i = 0; i < t->ndim; i++)
    if (i != dim) v.push_back(t->shape[i]);
  return v;
}

bool same_shape(const rtc_tensor* a, const rtc_tensor* b) {
  if (a->ndim != b->ndim) return false;
  for (size_t i = 0; i < a->ndim; i++)
    if (a->shape[i] != b->shape[i]) return false;
  return true;
}

rtc_result check_output(const rtc_tensor* x, const rtc_tensor* out, const char* context) {
  if (!same_shape(x, out)) return shape_mismatch(std::string(context) + " (output)", x, out);
  if (out->dtype != x->dtype)
    return dtype_mismatch(std::string(context) + " (output)", dtype_debug(x->dtype),
                          dtype_debug(out->dtype));
  return ok();
}

rtc_result require_f32(const rtc_tensor* t, const char* context) {
  if (t->dtype != RTC_F32)
    return unsupported(std::string(context) + ": " + dtype_display(t->dtype) +
                       " tensors are not supported by the CUDA path (float32 only)");
  return ok();
}

rtc_result same_device(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* c) {
  const bool ha = a->device == RTC_HOST_MEMORY, hb = b->device == RTC_HOST_MEMORY,
             hc = c->device == RTC_HOST_MEMORY;
  if (ha != hb || ha != hc)
    return invalid_argument("device", "host-memory and device tensors cannot be mixed in one call");
  if (a->device != b->device || a->device != c->device)
    return invalid_argument("device", "all tensors of one call must be on the same device");
  if (a->device < RTC_HOST_MEMORY) return invalid_argument("device", "invalid device ordinal");
  return ok();
}

void split_dims(const rtc_tensor* t, size_t dim, size_t* outer, size_t* len, size_t* inner) {
  size_t o = 1, in = 1;
  for (size_t d = 0; d < dim; d++) o *= t->shape[d];
  for (size_t d = dim + 1; d < t->ndim; d++) in *= t->shape[d];
  *outer = o;
  *len = t->shape[dim];
  *inner = in;
}

// ------------------------------------------------------------ device/stream

DeviceScope::DeviceScope(int device) {
  err_ = cudaGetDevice(&prev_);
  if (err_ != cudaSuccess) return;
  if (prev_ != device) {
    err_ = cudaSetDevice(device);
    changed_ = err_ == cudaSuccess;
  }
}

DeviceScope::~DeviceScope() {
  if (changed_) cudaSetDevice(prev_);
}

static thread_local cudaStream_t t_stream = cudaStreamPerThread;

cudaStream_t thread_stream() { return t_stream; }
void set_thread_stream(cudaStream_t s) { t_stream = s ? s : cudaStreamPerThread; }

static std::mutex g_pool_mu;
static std::vector<bool> g_pool_set;

void keep_pool_memory(int device) {
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (device < 0) return;
  if ((size_t)device >= g_pool_set.size()) g_pool_set.resize(device + 1, false);
  if (g_pool_set[device]) return;
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  }
  g_pool_set[device] = true;
}

bool nvtx_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("RTC_NVTX");
    return v && std::strcmp(v, "1") == 0;
  }();
  return on;
}

void release_library_state() {
  release_sharded_streams();
  std::lock_guard<std::mutex> lock(g_pool_mu);
  for (size_t d = 0; d < g_pool_set.size(); d++) {
    if (!g_pool_set[d]) continue;
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, (int)d) == cudaSuccess) cudaMemPoolTrimTo(pool, 0);
  }
}

// ------------------------------------------------------ exact global stats

// A small page-locked buffer per host thread for the scalars these paths
// return: a device-to-host copy into pinned memory is one DMA, where pageable
// memory goes through the driver's staging buffer.  Allocated on first use
// and kept for the thread's life (256 bytes).
static void* pinned_scratch() {
  static thread_local void* p = nullptr;
  if (!p && cudaHostAlloc(&p, 256, cudaHostAllocPortable) != cudaSuccess) p = nullptr;
  return p;
}

// Copies `bytes` (<= 256) from the device to *dst through the pinned buffer
// (or directly when it is unavailable) and waits for them.
static cudaError_t fetch(void* dst, const void* src, size_t bytes, cudaStream_t s) {
  void* pin = pinned_scratch();
  cudaError_t e = cudaMemcpyAsync(pin ? pin : dst, src, bytes, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && pin) std::memcpy(dst, pin, bytes);
  return e;
}

static cudaError_t read_elem(const float* x, size_t i, cudaStream_t s, float* v) {
  return fetch(v, x + i, sizeof(float), s);
}

#define CK(call)                         \
  do {                                   \
    cudaError_t _e = (call);             \
    if (_e != cudaSuccess) {             \
      cudaFreeAsync(scratch, s);         \
      return _e;                         \
    }                                    \
  } while (0)

cudaError_t exact_global_stats(const float* x, size_t n, int device, int want, cudaStream_t s,
                               GlobalStats* out) {
  keep_pool_memory(device);
  const int nparts = stats_num_parts(device, n);
  const size_t parts_bytes = ((size_t)nparts * sizeof(StatsPart) + 255) & ~size_t(255);
  const size_t bytes = parts_bytes + 256 + sizeof(IndexScan);
  char* scratch = nullptr;
  cudaError_t e0 = cudaMallocAsync(reinterpret_cast<void**>(&scratch), bytes, s);
  if (e0 != cudaSuccess) return e0;
  StatsPart* parts = reinterpret_cast<StatsPart*>(scratch);
  StatsPart* res = reinterpret_cast<StatsPart*>(scratch + parts_bytes);
  IndexScan* scan = reinterpret_cast<IndexScan*>(scratch + parts_bytes + 256);

  CK(launch_stats(x, n, parts, nparts, res, s));
  StatsPart h;
  CK(fetch(&h, res, sizeof h, s));
  out->sum = h.sum;
  out->max = h.mx;
  out->min = h.mn;
  out->max_const = false;
  out->first_nan = false;
  out->min_nonnan = h.mn;

  const bool sum_nan = std::isnan(h.sum);
  const bool fix_max = (want & kStatMax) && (sum_nan || h.mx == 0.0f);
  const bool fix_min = (want & kStatMin) && (sum_nan || h.mn == 0.0f);
  if (fix_max || fix_min) {
    IndexScan hs;
    CK(launch_index_scan(x, n, scan, s));
    CK(fetch(&hs, scan, sizeof hs, s));
    if (fix_max) {
      // The fold restarts after the last NaN; if x[n-1] is NaN it ends there.
      if (hs.last_nan == n) {
        CK(read_elem(x, n - 1, s, &out->max));
        out->max_const = true;
      } else {
        float m = h.mx;
        if (hs.last_nan > 0) {
          const size_t start = hs.last_nan;
          const int np2 = stats_num_parts(device, n - start);
          CK(launch_stats(x + start, n - start, parts, np2, res, s));
          StatsPart h2;
          CK(fetch(&h2, res, sizeof h2, s));
          m = h2.mx;
          out->max_const = true;
        }
        // A zero maximum keeps the sign of the last zero.
        if (m == 0.0f) CK(read_elem(x, hs.last_zero - 1, s, &m));
        out->max = m;
      }
    }
    if (fix_min) {
      // fminf skips NaN as the fold does; a zero minimum keeps the first zero.
      float m = h.mn;
      if (m == 0.0f) CK(read_elem(x, hs.first_zero - 1, s, &m));
      out->min_nonnan = m;
      float x0;
      CK(read_elem(x, 0, s, &x0));
      if (std::isnan(x0)) {
        out->min = x0;          // the fold never leaves a NaN first element
        out->first_nan = true;
      } else {
        out->min = m;
      }
    }
  }
  return cudaFreeAsync(scratch, s);
}

}  // namespace rt
