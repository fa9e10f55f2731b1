/*
 * rusttorch_cuda.h — C ABI of the B200 (sm_100a) implementation of
 * rusttorch-core's data-parallel tensor hot path.
 *
 * The library (librusttorch_cuda.so) is the device-side counterpart of
 * rusttorch-core's `ffi` feature (rusttorch-core/src/ffi/{mod,tensor,ops}.rs):
 * the same descriptor and result conventions, one entry point per hot-path op,
 * with tensors living in GPU memory instead of being copied in and out of
 * Rust-owned host arrays.  A `Tensor` device-storage variant in rusttorch-core
 * dispatches its ops here; the ops API and the PyO3 bindings do not change.
 *
 * Conventions
 *  - Every fallible call returns rtc_result by value.  On failure `error_msg`
 *    is a NUL-terminated message owned by the caller until passed to
 *    rtc_free_error_message(), formatted like rusttorch's TensorError Display
 *    (rusttorch-core/src/error.rs:69-160), and `code` names the variant.
 *  - Inputs are validated on the host before anything is launched, in the
 *    reference's order (dtype before shape for binary ops, shapes before
 *    hyperparameters for the optimizers).  The library never aborts.
 *  - Tensors are C-contiguous (`strides` NULL or row-major).  `data` is a
 *    device pointer on `device`; outputs are preallocated by the caller and
 *    may alias inputs of the same shape (in-place use).
 *  - Kernels run on the calling thread's stream (rtc_set_stream; default: the
 *    per-thread default stream) and calls return once the work is queued,
 *    except the scalar reductions (rtc_sum/mean/max/min, rtc_sharded_*),
 *    which return their value and so wait for it.
 *  - Host memory: a tensor whose `device` is RTC_HOST_MEMORY lives in host
 *    memory.  When every tensor of a call does, the op streams the data
 *    through the calling thread's current GPU (rtc_set_device) in chunks,
 *    with host-to-device copies, kernels and device-to-host copies of
 *    consecutive chunks overlapped on three streams, and returns when the
 *    results are in host memory.  Page-locked memory (rtc_host_alloc) runs at
 *    full PCIe bandwidth.  Mixing host and device tensors in one call is an
 *    error.
 *  - dtype: every op implements float32 (RTC_F32).  Other dtypes return
 *    RTC_UNSUPPORTED after the reference's own dtype checks have run.
 */
#ifndef RUSTTORCH_CUDA_H
#define RUSTTORCH_CUDA_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RTC_VERSION_STRING "0.1.0"

/* rtc_tensor.device value for a tensor in host memory (see Conventions). */
#define RTC_HOST_MEMORY (-1)

/* dtype codes of CTensorDescriptor.dtype (rusttorch-core/src/ffi/tensor.rs:25) */
enum { RTC_F32 = 0, RTC_F64 = 1, RTC_I32 = 2, RTC_I64 = 3 };

/* rtc_result.code: the TensorError variant (rusttorch-core/src/error.rs:10-67) */
typedef enum {
  RTC_OK = 0,
  RTC_SHAPE_MISMATCH = 1,    /* TensorError::ShapeMismatch     error.rs:12-16 */
  RTC_DTYPE_MISMATCH = 2,    /* TensorError::DTypeMismatch     error.rs:19-23 */
  RTC_EMPTY_TENSOR = 3,      /* TensorError::EmptyTensor       error.rs:26 */
  RTC_INVALID_DIMENSION = 4, /* TensorError::InvalidDimension  error.rs:29-33 */
  RTC_INVALID_ARGUMENT = 5,  /* TensorError::InvalidArgument   error.rs:46 */
  RTC_SIZE_OVERFLOW = 6,     /* TensorError::SizeOverflow      error.rs:43 */
  RTC_UNSUPPORTED = 7,       /* dtype/layout this library does not implement */
  RTC_BACKEND_ERROR = 8,     /* CUDA or NCCL failure (TensorError::Other, error.rs:66) */
  RTC_BROADCAST_ERROR = 9    /* TensorError::BroadcastError    error.rs:36-40 */
} rtc_status;

/* CTensorDescriptor (rusttorch-core/src/ffi/tensor.rs:13-26) plus the device
 * that holds `data`. */
typedef struct {
  void* data;            /* device pointer (or NULL when numel == 0) */
  const size_t* shape;   /* ndim extents */
  const size_t* strides; /* element strides; NULL means C-contiguous */
  size_t ndim;
  size_t numel;          /* must equal the product of shape */
  int dtype;             /* RTC_F32 ... RTC_I64 */
  int device;            /* CUDA device ordinal */
} rtc_tensor;

/* CResult (rusttorch-core/src/ffi/tensor.rs:38-64) plus the variant code.
 * The first two members have CResult's layout. */
typedef struct {
  bool success;
  char* error_msg; /* NULL on success */
  int code;        /* rtc_status */
} rtc_result;

/* ---------------------------------------------------------------- lifecycle */
/* rusttorch_version, ffi/mod.rs:45-48.  Static string, do not free. */
const char* rtc_version(void);
/* rusttorch_init, ffi/mod.rs:25-32: initialises the CUDA context of every
 * visible device.  Optional; every entry point initialises lazily. */
rtc_result rtc_init(void);
/* rusttorch_cleanup, ffi/mod.rs:38-41: releases library-held device state. */
void rtc_cleanup(void);
/* rusttorch_free_error_message, ffi/tensor.rs:68-73 */
void rtc_free_error_message(char* msg);

/* Stream (a cudaStream_t) for the calling thread's subsequent calls; NULL
 * selects the per-thread default stream. */
rtc_result rtc_set_stream(void* stream);
void* rtc_get_stream(void);
/* Waits for the calling thread's stream on its current GPU (rtc_set_device),
 * then reports RTC_BACKEND_ERROR if a kernel on that GPU gave up one of its
 * bounded waits since the last call (its results are then incomplete). */
rtc_result rtc_synchronize(void);
/* Failure-path self-test (no reference counterpart): queues a one-thread
 * kernel on the current GPU whose bounded mbarrier wait runs out after 50 ms,
 * as a TMA consumer's would if its tile never landed.  The next
 * rtc_synchronize returns RTC_BACKEND_ERROR for it; the context stays usable
 * and the call after that returns RTC_OK.  Nothing faults or hangs. */
rtc_result rtc_selftest_bounded_wait(void);
/* Test hook for the losses' ordered sum: *out_value = the f32 sum of x (f32,
 * on a device) in ndarray's unrolled_fold order (chains = 8: eight chains over
 * i % 8 from 0.0, combined as (p0+p4), (p1+p5), (p2+p6), (p3+p7) onto 0.0,
 * then the remainder in order) or as one chain from init (chains = 1, the
 * order of Iterator::sum with init = -0.0), bit for bit. */
rtc_result rtc_selftest_ordered_sum(const rtc_tensor* x, int chains, float init,
                                    float* out_value);
/* Math mode of the transcendental activations (sigmoid, tanh, gelu, swish,
 * mish, softplus) and softmax; no reference counterpart.
 *  RTC_MATH_TOLERANCE (default): within 1e-6 relative error or 4 ulp of the
 *    reference's result on every float input, from single-precision
 *    exp/tanh/log (at most 5.8e-7 relative over all 2^32 inputs); where the
 *    reference's own formula cancels (gelu's 1 + tanh for inputs below
 *    -1.58, softplus and mish's 1 + exp) the exact glibc steps are kept.
 *  RTC_MATH_EXACT: glibc's expf/tanhf reproduced bit for bit (softplus and
 *    mish still use a correctly rounded log: within 1 and 6 ulp).
 * Process-wide; the environment variable RTC_MATH_MODE=exact|tolerance sets
 * the initial mode.  Kernels already queued keep the mode they were queued
 * with.  ELU, SELU, the backward ops and the losses are the same in both. */
enum { RTC_MATH_TOLERANCE = 0, RTC_MATH_EXACT = 1 };
rtc_result rtc_set_math_mode(int mode);
int rtc_get_math_mode(void);
/* Test hook (no reference counterpart): out[i] = the tolerance mode's
 * primitive `which` of x[i] on the current GPU (0 exp, 1 log for positive
 * normal x, 2 tanh, 3 the correctly rounded reciprocal for x in [1, 2^64]);
 * device pointers, returns once queued. */
rtc_result rtc_selftest_fastmath(int which, const float* x, float* out, size_t n);
int rtc_device_count(void);
/* The calling thread's current GPU (host-memory ops and the flat *_f32 API
 * run there). */
rtc_result rtc_set_device(int device);
int rtc_get_device(void);

/* Memory helpers for callers without the CUDA runtime (no reference
 * counterpart: the reference owns host memory through ndarray). */
rtc_result rtc_malloc(int device, size_t bytes, void** out);
rtc_result rtc_free(int device, void* ptr);
rtc_result rtc_memcpy_h2d(int device, void* dst, const void* src, size_t bytes);
rtc_result rtc_memcpy_d2h(int device, void* dst, const void* src, size_t bytes);
rtc_result rtc_host_alloc(size_t bytes, void** out); /* page-locked host memory */
rtc_result rtc_host_free(void* ptr);

/* Seeded synthetic data on the device: element i depends only on
 * (seed, offset + i).  uniform in [lo, hi); normal(mean, std). */
rtc_result rtc_fill_uniform(const rtc_tensor* out, uint64_t seed, uint64_t offset, float lo,
                            float hi);
rtc_result rtc_fill_normal(const rtc_tensor* out, uint64_t seed, uint64_t offset, float mean,
                           float std);

/* -------------------------------------------------- elementwise (f32, bit-exact) */
/* rusttorch_add, ffi/ops.rs:21-40 -> ops::add, ops/elementwise.rs:14-94 */
rtc_result rtc_add(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
/* rusttorch_mul, ffi/ops.rs:44-63 -> ops::mul, ops/elementwise.rs:97-127 */
rtc_result rtc_mul(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
/* rusttorch_sub, ffi/ops.rs:67-86 -> ops::sub, ops/elementwise.rs:130-160 */
rtc_result rtc_sub(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
/* rusttorch_div, ffi/ops.rs:90-109 -> ops::div, ops/elementwise.rs:163-197 */
rtc_result rtc_div(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
/* ops::add_scalar, ops/elementwise.rs:200-210 (no reference FFI export) */
rtc_result rtc_add_scalar(const rtc_tensor* x, float scalar, const rtc_tensor* out);
/* ops::mul_scalar, ops/elementwise.rs:213-223 (no reference FFI export) */
rtc_result rtc_mul_scalar(const rtc_tensor* x, float scalar, const rtc_tensor* out);
/* ops::mul_scalar(&ops::add(a, b)?, s) in one pass (elementwise.rs:14 then :213) */
rtc_result rtc_add_mul_scalar(const rtc_tensor* a, const rtc_tensor* b, float scalar,
                              const rtc_tensor* out);
/* ops::fused_multiply_add, ops/simd.rs:275-370: a*b + c, two roundings */
rtc_result rtc_fused_multiply_add(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* c,
                                  const rtc_tensor* out);
/* ops::add_simd / mul_simd / relu_simd / mul_scalar_simd (ops/simd.rs:14, :95,
 * :176, :225): same values as the plain ops, their own error contexts. */
rtc_result rtc_add_simd(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
rtc_result rtc_mul_simd(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
rtc_result rtc_relu_simd(const rtc_tensor* x, const rtc_tensor* out);
rtc_result rtc_mul_scalar_simd(const rtc_tensor* x, float scalar, const rtc_tensor* out);

/* ------------------------------------------------------------- activations */
/* rusttorch_relu, ffi/ops.rs:117-132 -> ops::relu, ops/activation.rs:8-18 */
rtc_result rtc_relu(const rtc_tensor* x, const rtc_tensor* out);
/* rusttorch_leaky_relu, ffi/ops.rs:199-215 -> ops::leaky_relu, activation.rs:170-191 */
rtc_result rtc_leaky_relu(const rtc_tensor* x, const rtc_tensor* out, float alpha);
/* rusttorch_sigmoid, ffi/ops.rs:136-153 -> ops::sigmoid, activation.rs:21-37 */
rtc_result rtc_sigmoid(const rtc_tensor* x, const rtc_tensor* out);
/* rusttorch_tanh, ffi/ops.rs:157-174 -> ops::tanh, activation.rs:40-56 */
rtc_result rtc_tanh(const rtc_tensor* x, const rtc_tensor* out);
/* rusttorch_gelu, ffi/ops.rs:178-195 -> ops::gelu, activation.rs:61-88 */
rtc_result rtc_gelu(const rtc_tensor* x, const rtc_tensor* out);
/* ops::swish (SiLU), activation.rs:263-279 */
rtc_result rtc_swish(const rtc_tensor* x, const rtc_tensor* out);
/* ops::elu, activation.rs:195-222 (alpha <= 0 -> RTC_INVALID_ARGUMENT) */
rtc_result rtc_elu(const rtc_tensor* x, const rtc_tensor* out, float alpha);
/* ops::selu, activation.rs:228-259 */
rtc_result rtc_selu(const rtc_tensor* x, const rtc_tensor* out);
/* ops::mish, activation.rs:284-314 */
rtc_result rtc_mish(const rtc_tensor* x, const rtc_tensor* out);
/* ops::softplus, activation.rs:319-346 */
rtc_result rtc_softplus(const rtc_tensor* x, const rtc_tensor* out);
/* ops::softsign, activation.rs:351-367 */
rtc_result rtc_softsign(const rtc_tensor* x, const rtc_tensor* out);
/* ops::softmax(t, dim), activation.rs:92-167 */
rtc_result rtc_softmax(const rtc_tensor* x, size_t dim, const rtc_tensor* out);

/* -------------------------------------------------------------- reductions */
/* rusttorch_sum, ffi/ops.rs:223-238 -> ops::sum, ops/reduction.rs:7-14 */
rtc_result rtc_sum(const rtc_tensor* x, double* out_value);
/* rusttorch_mean, ffi/ops.rs:241-256 -> ops::mean, reduction.rs:17-26 */
rtc_result rtc_mean(const rtc_tensor* x, double* out_value);
/* rusttorch_max, ffi/ops.rs:259-274 -> ops::max, reduction.rs:29-49 */
rtc_result rtc_max(const rtc_tensor* x, double* out_value);
/* rusttorch_min, ffi/ops.rs:277-292 -> ops::min, reduction.rs:52-72 */
rtc_result rtc_min(const rtc_tensor* x, double* out_value);
/* ops::sum without waiting: queues the sum of the device tensor x on the
 * calling thread's stream; the f64 result lands in *device_out (device
 * memory on x's device).  Same value as rtc_sum. */
rtc_result rtc_sum_device(const rtc_tensor* x, double* device_out);
/* rtc_sum_device for callers that must not allocate GPU memory (no
 * counterpart in the reference).  rtc_sum_device draws its scratch (one
 * partial sum per thread block) from the stream-ordered pool; callers whose
 * GPU memory is already reserved by another allocator, or whose policy or
 * latency budget rules out allocation, can call this instead: the scratch is
 * a fixed array inside the library (room for 2048 partials, 32 KB per GPU,
 * held by every GPU that loads the library until exit).  The first call on a
 * device looks up that array's device address, so make it before any stream
 * capture; the address is kept, so do not use the library on a device after
 * resetting it.  Calls share the array: calls that overlap on the GPU race.
 * Fails with RTC_INVALID_ARGUMENT if x would need more partials than the
 * array holds (only on GPUs with more than 256 SMs). */
rtc_result rtc_sum_device_noalloc(const rtc_tensor* x, double* device_out);
/* sum, mean, max and min from one pass over x (no reference counterpart; each
 * value equals the corresponding single op).  out[4] = {sum, mean, max, min}. */
rtc_result rtc_stats(const rtc_tensor* x, double out[4]);
/* ops::sum_dim, reduction.rs:75-108: out has shape without `dim`. */
rtc_result rtc_sum_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out);
/* ops::mean_dim, reduction.rs:111-150 */
rtc_result rtc_mean_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out);
/* max along `dim` (no reference counterpart: the reference's global max fold,
 * reduction.rs:29-49, applied to every lane). */
rtc_result rtc_max_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out);

/* ------------------------------------------------------- optimizer updates */
/* ops::adam_update, ops/optimizer.rs:207-354.  Writes p', m', v' into the
 * *_out tensors (which may be p, m, v themselves). */
rtc_result rtc_adam_update(const rtc_tensor* params, const rtc_tensor* grads, const rtc_tensor* m,
                           const rtc_tensor* v, double learning_rate, double beta1, double beta2,
                           double epsilon, uint64_t timestep, const rtc_tensor* params_out,
                           const rtc_tensor* m_out, const rtc_tensor* v_out);
/* ops::adamw_update, ops/optimizer.rs:379-440 */
rtc_result rtc_adamw_update(const rtc_tensor* params, const rtc_tensor* grads,
                            const rtc_tensor* m, const rtc_tensor* v, double learning_rate,
                            double beta1, double beta2, double epsilon, double weight_decay,
                            uint64_t timestep, const rtc_tensor* params_out,
                            const rtc_tensor* m_out, const rtc_tensor* v_out);
/* ops::sgd_update, ops/optimizer.rs:42-86 */
rtc_result rtc_sgd_update(const rtc_tensor* params, const rtc_tensor* grads,
                          double learning_rate, const rtc_tensor* params_out);
/* ops::sgd_momentum_update, ops/optimizer.rs:108-177 */
rtc_result rtc_sgd_momentum_update(const rtc_tensor* params, const rtc_tensor* grads,
                                   const rtc_tensor* velocity, double learning_rate,
                                   double momentum, const rtc_tensor* params_out,
                                   const rtc_tensor* velocity_out);

/* --------------------------------------------- sharded global reductions */
/* A tensor split into contiguous shards, one per GPU or process, reduces to
 * the reference's sum/mean/max/min of the whole (reduction.rs:7-72) in two
 * steps: every shard is summarised on its own GPU, the summaries (a few bytes
 * each) are exchanged by any collective (NCCL all-gather in bench.py), and
 * rtc_shard_combine folds them in shard order.  The summary keeps what the
 * reference's order-dependent max/min folds need across shard boundaries. */
typedef struct {
  double sum;          /* f64 sum of the shard */
  uint64_t count;      /* elements in the shard */
  float max;           /* the shard's max fold (see max_kind) */
  float min_nonnan;    /* min fold over the shard's non-NaN elements (+inf if none) */
  int32_t max_kind;    /* 0: empty shard; 1: max fold of the shard alone;
                          2: the shard holds a NaN, so the fold's value after
                             it is `max` whatever came before */
  int32_t first_nan;   /* the shard's first element is NaN */
} rtc_shard_summary;

/* Summarise one shard (a device tensor, or host memory streamed through the
 * current GPU).  Waits for the result. */
rtc_result rtc_shard_summary_local(const rtc_tensor* shard, rtc_shard_summary* out);
/* Fold n summaries in shard order (host only, no GPU needed).
 * out[4] = {sum, mean, max, min} of the concatenated tensor; an empty total
 * writes out[0] = 0 and returns RTC_EMPTY_TENSOR. */
rtc_result rtc_shard_combine(const rtc_shard_summary* parts, size_t n, double out[4]);
/* One process driving several GPUs: summarise every shard on its own device
 * (concurrently, one host thread per device) and fold the summaries in shard
 * order; out[4] = {sum, mean, max, min} of the concatenated tensor.  Waits
 * for the work already queued on the shards' devices first.  No reference
 * counterpart (the reference has no multi-device path); it is the
 * single-process form of rtc_shard_summary_local + rtc_shard_combine. */
rtc_result rtc_sharded_stats(const rtc_tensor* shards, size_t n_shards, double out[4]);

/* More single-process sharded ops (no reference counterpart: the reference
 * has no multi-device path; each is the sharded form of the reference export
 * named).  A logical tensor is given as n_shards descriptors, shard i of
 * every operand on one device (any device per shard), all f32.  Each call
 * checks every shard before anything is launched (an argument error changes
 * nothing), waits for the work already queued on the shards' devices, runs
 * the shards at once (one library stream per device, launched from the
 * calling thread) and returns when all are done.  No shard exchanges data
 * with another: the results are those of the single-GPU op on each shard. */
/* ops::add then ops::mul_scalar (ffi/ops.rs:21-40 rusttorch_add), any split. */
rtc_result rtc_sharded_add_mul_scalar(const rtc_tensor* a, const rtc_tensor* b, float scalar,
                                      const rtc_tensor* out, size_t n_shards);
/* ops::softmax (activation.rs:92-167) of row blocks: the shards split axis 0,
 * so dim must be >= 1 when there is more than one shard. */
rtc_result rtc_sharded_softmax(const rtc_tensor* x, size_t dim, const rtc_tensor* out,
                               size_t n_shards);
/* ops::sum_dim / mean_dim (reduction.rs:75-150) and max along dim, each shard
 * reduced on its own GPU: the shards split an axis other than dim (row blocks
 * for the last axis; column blocks — each its own contiguous [R, C_i]
 * tensor — for dim 0 of a matrix).  out[i] has shard i's reduced shape. */
rtc_result rtc_sharded_sum_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out,
                               size_t n_shards);
rtc_result rtc_sharded_mean_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out,
                                size_t n_shards);
rtc_result rtc_sharded_max_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out,
                               size_t n_shards);
/* ops::adamw_update (optimizer.rs:379-440) on every shard, in place
 * (params, m and v are overwritten with p', m', v'); any split. */
rtc_result rtc_sharded_adamw_update(const rtc_tensor* params, const rtc_tensor* grads,
                                    const rtc_tensor* m, const rtc_tensor* v,
                                    double learning_rate, double beta1, double beta2,
                                    double epsilon, double weight_decay, uint64_t timestep,
                                    size_t n_shards);

/* One process per GPU: the global sum's exchange over peer memory (no
 * reference counterpart; the reference has no multi-device path).  Each rank
 * allocates a slot array of rtc_peer_slot_bytes(world) bytes with rtc_malloc
 * (a whole allocation: IPC maps allocations, not offsets into them), zeroes
 * it, passes its handle (rtc_ipc_handle) to the other ranks by any host
 * channel, and opens theirs (rtc_ipc_open).  Then
 * rtc_peer_allreduce_sum_f64(device, local, slots, world, rank, g, out), with
 * slots[p] = rank p's slot array as mapped on this rank (its own for p =
 * rank) and g = 1, 2, 3, ... on successive calls (the same g on every rank),
 * writes into *out (device) the sum of every rank's *local, added in rank
 * order from 0.0 — the same bits on every rank.  Queued on the calling
 * thread's stream, one kernel; it waits at most 2 s for the other ranks, then
 * writes NaN and raises the flag rtc_synchronize reports.  rtc_ipc_close
 * unmaps a peer's array (before the peer frees it). */
#define RTC_IPC_HANDLE_BYTES 64
#define RTC_PEER_MAX_RANKS 8
rtc_result rtc_ipc_handle(int device, const void* dev_ptr, void* handle_out);
rtc_result rtc_ipc_open(int device, const void* handle, void** dev_ptr_out);
rtc_result rtc_ipc_close(int device, void* dev_ptr);
size_t rtc_peer_slot_bytes(int world);
rtc_result rtc_peer_allreduce_sum_f64(int device, const double* local, void* const* slots,
                                      int world, int rank, unsigned long long generation,
                                      double* out);

/* -------------------------------------------------------- broadcasting */
/* ops::add_broadcast / sub_broadcast / mul_broadcast / div_broadcast
 * (ops/broadcast.rs:177-198): NumPy broadcasting of a and b (dtype checked
 * first, context "broadcast_tensors"; incompatible shapes give
 * RTC_BROADCAST_ERROR), then the plain op.  `out` has the broadcast shape.
 * The operands are read in place through zero strides; nothing is
 * materialised.  Device tensors only. */
rtc_result rtc_add_broadcast(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
rtc_result rtc_sub_broadcast(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
rtc_result rtc_mul_broadcast(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);
rtc_result rtc_div_broadcast(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out);

/* ------------------------------------------------------- nn optimizers */
/* nn::Adam::step (nn/optim.rs:262-313) for one parameter: f32
 * hyperparameters, bias corrections 1 - powf(beta, t) in f32, and the
 * module's own operation order (it differs from ops::adam_update).  `t` is
 * the step count after this step's increment (:264); pass zero tensors for
 * m and v on the first step.  The reference indexes g, m and v by p's length
 * and panics on a shorter one; here that is RTC_SHAPE_MISMATCH. */
rtc_result rtc_nn_adam_step(const rtc_tensor* params, const rtc_tensor* grads,
                            const rtc_tensor* m, const rtc_tensor* v, float lr, float beta1,
                            float beta2, float eps, uint64_t t, const rtc_tensor* params_out,
                            const rtc_tensor* m_out, const rtc_tensor* v_out);
/* nn::SGD::step (nn/optim.rs:148-208) for one parameter.  With momentum > 0
 * it updates `velocity` (zeros on the first step) into velocity_out;
 * otherwise velocity and velocity_out may be NULL.  Element counts of params
 * and grads must match ("SGD step", :160-166). */
rtc_result rtc_nn_sgd_step(const rtc_tensor* params, const rtc_tensor* grads,
                           const rtc_tensor* velocity, float lr, float momentum,
                           float weight_decay, const rtc_tensor* params_out,
                           const rtc_tensor* velocity_out);

/* ---- loss functions (rusttorch-core src/ops/loss.rs) --------------------
 * No C entry point in the reference (Rust functions returning Result<f64>).
 * *out_value = the reference's f64 result: the f32 sum of the per-element
 * terms, in the reference's order, as f64, divided by the element count.
 * mse/l1/smooth_l1 sum like ndarray's sum() (eight sequential chains) and
 * are bit-identical; bce/ce sum one chain from -0.0 like Iterator::sum and
 * use a correctly rounded logf (glibc's logf differs from it in the last
 * bit for about 0.02% of inputs).  The chains are serial: their time is
 * about n/8 (or n) dependent f32 adds on one SM.  Device f32 tensors;
 * synchronous. */

/* mse_loss (loss.rs:41-85): mean((p - t)^2). */
rtc_result rtc_mse_loss(const rtc_tensor* predictions, const rtc_tensor* targets,
                        double* out_value);
/* l1_loss (loss.rs:102-144): mean(|p - t|). */
rtc_result rtc_l1_loss(const rtc_tensor* predictions, const rtc_tensor* targets,
                       double* out_value);
/* smooth_l1_loss (loss.rs:165-229); beta <= 0 is RTC_INVALID_ARGUMENT. */
rtc_result rtc_smooth_l1_loss(const rtc_tensor* predictions, const rtc_tensor* targets,
                              double beta, double* out_value);
/* binary_cross_entropy_loss (loss.rs:249-315); epsilon must be in (0, 1). */
rtc_result rtc_binary_cross_entropy_loss(const rtc_tensor* predictions,
                                         const rtc_tensor* targets, double epsilon,
                                         double* out_value);
/* cross_entropy_loss (loss.rs:332-391); epsilon must be in (0, 1). */
rtc_result rtc_cross_entropy_loss(const rtc_tensor* predictions, const rtc_tensor* targets,
                                  double epsilon, double* out_value);

/* ---- autograd backward (rusttorch-core src/autograd/ops.rs) -------------
 * No C entry point in the reference: its GradFn::backward methods compose
 * ops::* calls on the CPU.  Each function below returns the same tensors
 * from one fused kernel.  A NULL gradient output is the reference's `None`
 * (that input does not require grad).  Errors are those of the first
 * ops::* call that would fail in the reference.  MulScalarBackward
 * (ops.rs:583-593) is rtc_mul_scalar(grad_output, scalar). */

/* ReluBackward (ops.rs:375-390): grad_output * (input > 0 ? 1 : 0). */
rtc_result rtc_relu_backward(const rtc_tensor* grad_output, const rtc_tensor* input,
                             const rtc_tensor* grad_input);
/* SigmoidBackward (ops.rs:419-431): grad_output * (y * (1 - y)), y the
 * saved sigmoid output. */
rtc_result rtc_sigmoid_backward(const rtc_tensor* grad_output, const rtc_tensor* output,
                                const rtc_tensor* grad_input);
/* TanhBackward (ops.rs:460-472): grad_output * (1 - y*y), y the saved tanh
 * output. */
rtc_result rtc_tanh_backward(const rtc_tensor* grad_output, const rtc_tensor* output,
                             const rtc_tensor* grad_input);
/* GeluBackward (ops.rs:3102-3125), from the saved input, with glibc tanhf. */
rtc_result rtc_gelu_backward(const rtc_tensor* grad_output, const rtc_tensor* input,
                             const rtc_tensor* grad_input);
/* autograd's GELU forward (ops.rs:3131-3141), which rounds its cubic term as
 * ((0.044715*x)*x)*x, unlike ops::gelu (rtc_gelu). */
rtc_result rtc_autograd_gelu(const rtc_tensor* input, const rtc_tensor* output);
/* AddBackward (ops.rs:133-149): both gradients are grad_output. */
rtc_result rtc_add_backward(const rtc_tensor* grad_output, const rtc_tensor* grad_a,
                            const rtc_tensor* grad_b);
/* SubBackward (ops.rs:175-192): grad_a = grad_output, grad_b = -grad_output. */
rtc_result rtc_sub_backward(const rtc_tensor* grad_output, const rtc_tensor* grad_a,
                            const rtc_tensor* grad_b);
/* MulBackward (ops.rs:219-236): grad_a = grad_output * b,
 * grad_b = grad_output * a; one pass when both are wanted. */
rtc_result rtc_mul_backward(const rtc_tensor* grad_output, const rtc_tensor* a,
                            const rtc_tensor* b, const rtc_tensor* grad_a,
                            const rtc_tensor* grad_b);
/* DivBackward (ops.rs:267-290): grad_a = grad_output / b,
 * grad_b = grad_output * ((-a) / (b*b)). */
rtc_result rtc_div_backward(const rtc_tensor* grad_output, const rtc_tensor* a,
                            const rtc_tensor* b, const rtc_tensor* grad_a,
                            const rtc_tensor* grad_b);
/* SumBackward (ops.rs:501-511): grad_input filled with the one element of
 * grad_output (item(): any other element count is RTC_INVALID_ARGUMENT).
 * Device tensors only; the value is read on the device. */
rtc_result rtc_sum_backward(const rtc_tensor* grad_output, const rtc_tensor* grad_input);
/* MeanBackward (ops.rs:542-552): filled with (f32)((f64)g / n), n =
 * grad_input's element count.  Device tensors only. */
rtc_result rtc_mean_backward(const rtc_tensor* grad_output, const rtc_tensor* grad_input);
/* BroadcastAddBackward (ops.rs:615-693): grad_output folded back onto each
 * operand's original shape (given by grad_a / grad_b) by reduce_to_shape
 * (:627-681), in its order: 2-D [1,C] column sums and [R,1] row sums, a copy
 * for equal element counts, else result[i % m] += grad[i].  Device only. */
rtc_result rtc_broadcast_add_backward(const rtc_tensor* grad_output, const rtc_tensor* grad_a,
                                      const rtc_tensor* grad_b);

/* ------------------------------------------------------------ diagnostics */
/* Bandwidth probes (no reference counterpart): the read ceiling the
 * reductions are measured against and the sizing of the small fused map.
 * mode 0/1: read `bytes` of src with 16-byte loads, p1 (4, 8, 16) loads in
 * flight per thread, p0 threads per block, p2 blocks per SM (0: grid-stride,
 * 1: one contiguous range per block); 2/3: read src through a cp.async.bulk
 * ring into shared memory, p1 slots of p0 bytes per CTA, p2 CTAs per SM (3:
 * every thread also folds each slot); 4: copy src to dst as mode 0; 5/6: the
 * add->mul_scalar map over a = src, b = src + bytes/2 into dst with U = p1
 * (1, 2, 4, 8) and p2 blocks per SM (5: grid-stride, p2 = 0 one resident
 * wave, p2 < 0 one block per tile; 6: one balanced range per block); 7: the
 * global sum/max/min kernel over bytes/4 floats of src with p0 threads, |p1|
 * loads in flight per thread (p1 < 0: each float4 summed as a float32 tree)
 * and p2 blocks per SM (0: all that stay resident); 8: the last-axis sum of
 * src viewed as [bytes/4/p0, p0] into dst: p1 (1, 2, 4, 8) warps per CTA of the
 * shared-memory-staged kernel, -(1000*C + 10*K + w) the direct-chain kernel
 * (C chains per thread, K loads ahead, w warps per CTA), 100*K + w (>= 100)
 * the 128-byte-read transpose kernel.
 * Device pointers on the current GPU, 16-byte aligned; returns once queued. */
rtc_result rtc_probe_stream(int mode, const void* src, void* dst, size_t bytes, int p0, int p1,
                            int p2);

/* ------------------------------------- flat float32 API (device pointers) */
/* rusttorch_relu_f32 / add_f32 / mul_f32, ffi/ops.rs:348-389: contiguous f32
 * buffers of `size` elements on the current device. */
rtc_result rtc_relu_f32(const float* input, float* output, size_t size);
rtc_result rtc_add_f32(const float* a, const float* b, float* output, size_t size);
rtc_result rtc_mul_f32(const float* a, const float* b, float* output, size_t size);

#ifdef __cplusplus
}
#endif

#endif /* RUSTTORCH_CUDA_H */
