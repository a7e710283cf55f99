/*
 * pvb2.h -- C-ABI of the B200 kernel library (libpvb2.so) behind the `ocl`
 * (PrivateUse1) PyTorch backend.
 *
 * Everything here is plain C: raw device pointers, sizes and strides, an
 * opaque stream handle, an int status.  No torch types cross this boundary,
 * so the library can be bound from ctypes, cffi or any C++ host.
 *
 * Each entry point names the reference interface it replaces.  In the
 * reference (pytorch_ocl 0.2.0) those are ATen kernels registered with
 * TORCH_LIBRARY_IMPL(aten, PrivateUse1) that forward to dlprimitives'
 * OpenCL kernels; the host layer of this project (csrc/host/*.cpp) keeps the
 * same ATen registrations and forwards to the functions below instead.
 *
 * Conventions
 *   - Every function returns PVB2_OK (0) or an error code; it never aborts.
 *     pvb2_last_error() returns a thread-local message for the last failure.
 *   - Launchers validate shapes, dtypes and alignment before launching.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy
 *     default stream.
 *   - Strides are in elements, like torch.
 *   - No launcher allocates device memory.  Scratch space ("workspace") is
 *     passed in by the caller; *_workspace_size() reports how much is needed.
 */
#ifndef PVB2_H
#define PVB2_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PVB2_API __attribute__((visibility("default")))
#else
#define PVB2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ */
/* status, dtypes, tensor descriptor                                    */
/* ------------------------------------------------------------------ */
enum {
  PVB2_OK = 0,
  PVB2_ERR_INVALID = 1,     /* bad argument (shape, dtype, alignment)    */
  PVB2_ERR_UNSUPPORTED = 2, /* valid request this library does not do    */
  PVB2_ERR_CUDA = 3,        /* CUDA runtime error                        */
  PVB2_ERR_OOM = 4,         /* cudaMalloc / cudaHostAlloc failed         */
  PVB2_ERR_NCCL = 5,        /* NCCL error                                */
  PVB2_ERR_TIMEOUT = 6      /* a bounded wait ran out                    */
};

/* dtype codes follow the reference's dtype map (src/utils.cpp:5-32). */
enum {
  PVB2_F32 = 0, PVB2_F64 = 1, PVB2_F16 = 2, PVB2_BF16 = 3,
  PVB2_I64 = 4, PVB2_I32 = 5, PVB2_I16 = 6, PVB2_I8 = 7,
  PVB2_U8 = 8, PVB2_BOOL = 9
};

#define PVB2_MAX_DIMS 8

/* A strided view of device memory.  Replaces the reference's
 * torch::Tensor -> dlprim::Tensor bridge `todp()` (src/utils.cpp:44-59),
 * which required contiguous tensors; here strides are carried through. */
typedef struct pvb2_tensor {
  void* data;                       /* points at element [0,...,0]      */
  int64_t sizes[PVB2_MAX_DIMS];
  int64_t strides[PVB2_MAX_DIMS];   /* in elements                      */
  int32_t ndim;
  int32_t dtype;                    /* PVB2_* dtype code                */
} pvb2_tensor;

typedef void* pvb2_stream;          /* cudaStream_t */
typedef void* pvb2_event;           /* cudaEvent_t  */
typedef void* pvb2_graph;           /* a captured, instantiated CUDA graph */

/* ------------------------------------------------------------------ */
/* runtime: devices, memory, streams, events                           */
/* Replaces CLContextManager (src/CLTensor.h:87-282) and the OpenCL     */
/* buffer/queue calls made by CLCache (src/CLTensor.cpp:9-92).          */
/* ------------------------------------------------------------------ */
PVB2_API const char* pvb2_last_error(void);
PVB2_API int pvb2_version(void);
PVB2_API int pvb2_device_count(int* count);                         /* CLTensor.h:230-258 */
PVB2_API int pvb2_set_device(int device);
PVB2_API int pvb2_get_device(int* device);
PVB2_API int pvb2_device_name(int device, char* buf, int buflen);
PVB2_API int pvb2_device_synchronize(void);                         /* python_iface.cpp:34-47 */
PVB2_API int pvb2_mem_get_info(size_t* free_bytes, size_t* total_bytes);
PVB2_API int pvb2_malloc(void** ptr, size_t bytes);                 /* CLCache::allocate backing store, CLTensor.cpp:81-92 */
PVB2_API int pvb2_free(void* ptr);
PVB2_API int pvb2_host_alloc(void** ptr, size_t bytes);             /* pinned host memory */
PVB2_API int pvb2_host_free(void* ptr);
PVB2_API int pvb2_pointer_info(const void* ptr, int* is_device, int* is_pinned_host, int* device);
PVB2_API int pvb2_stream_create(pvb2_stream* stream, int priority); /* the reference's single in-order queue, CLTensor.h:260-276 */
PVB2_API int pvb2_stream_destroy(pvb2_stream stream);
PVB2_API int pvb2_stream_synchronize(pvb2_stream stream);           /* queue.finish(), registeration.cpp:71-74 */
PVB2_API int pvb2_stream_query(pvb2_stream stream, int* done);      /* registeration.cpp:68-70 (was always false) */
PVB2_API int pvb2_stream_wait_event(pvb2_stream stream, pvb2_event event);
PVB2_API int pvb2_event_create(pvb2_event* event, int timing);
PVB2_API int pvb2_event_destroy(pvb2_event event);
PVB2_API int pvb2_event_record(pvb2_event event, pvb2_stream stream);
PVB2_API int pvb2_event_synchronize(pvb2_event event);
PVB2_API int pvb2_event_query(pvb2_event event, int* done);
PVB2_API int pvb2_event_elapsed_ms(pvb2_event start, pvb2_event end, float* ms);
/* kind: 0 host->device, 1 device->host, 2 device->device, 3 inferred */
PVB2_API int pvb2_memcpy_async(void* dst, const void* src, size_t bytes, int kind, pvb2_stream stream);
PVB2_API int pvb2_memset_async(void* dst, int value, size_t bytes, pvb2_stream stream);
/* number of kernels this library has launched in this process (all devices) */
PVB2_API int64_t pvb2_launch_count(void);
/* CUDA graphs: the work this library issues to `stream` between
 * pvb2_graph_capture_begin and pvb2_graph_capture_end (relaxed capture mode;
 * the stream must be one of pvb2_stream_create's) becomes one graph that
 * pvb2_graph_launch replays on a stream with a single launch, the pointers
 * and arguments of the capture baked in.  Nothing may synchronise with the
 * stream while it is captured (a read back to the host, a stream or device
 * synchronisation), and memory the captured work uses must stay allocated,
 * unchanged in address, for as long as the graph is replayed.  Each replay
 * adds the number of kernels captured to pvb2_launch_count.  The reference
 * has no counterpart: it issued every kernel from the host, one by one
 * (dlprimitives through its OpenCL queue). */
PVB2_API int pvb2_graph_capture_begin(pvb2_stream stream);
PVB2_API int pvb2_graph_capture_end(pvb2_stream stream, pvb2_graph* graph);
PVB2_API int pvb2_graph_launch(pvb2_graph graph, pvb2_stream stream);
PVB2_API int pvb2_graph_kernel_count(pvb2_graph graph, int64_t* kernels);
PVB2_API int pvb2_graph_destroy(pvb2_graph graph);
PVB2_API int pvb2_stream_is_capturing(pvb2_stream stream, int* capturing);

/* ------------------------------------------------------------------ */
/* tensor plumbing (src/tensor_ops.cpp)                                 */
/* ------------------------------------------------------------------ */
/* fill_.Scalar / zero_, tensor_ops.cpp:204-225 */
PVB2_API int pvb2_fill(const pvb2_tensor* out, double value, pvb2_stream stream);
/* strided copy with dtype conversion: copy_strided in _copy_from,
 * tensor_ops.cpp:118-186 (same sizes required; any strides, any dtypes) */
PVB2_API int pvb2_copy(const pvb2_tensor* dst, const pvb2_tensor* src, pvb2_stream stream);
/* arange.start_out, pointwise_ops.cpp (arange_out): out[i] = start + i*step */
PVB2_API int pvb2_arange(const pvb2_tensor* out, double start, double step, pvb2_stream stream);
/* masked_select / nonzero, tensor_ops.cpp:303-356 (the reference copied to
 * the host; here the compaction runs on the device).  `mask` (bool/u8) and
 * `src` have equal sizes (broadcast by the caller); elements are taken in
 * row-major order of those sizes.
 *   1. pvb2_select_count: per-block counts and their prefix into workspace,
 *      total count into *d_total (device int64).
 *   2. pvb2_select_gather: out[k] = k-th selected element of src, or, with
 *      src == NULL, the k-th selected element's coordinates as
 *      out[k*ndim + d] (int64), which is nonzero(). */
PVB2_API size_t pvb2_select_workspace_size(int64_t n);
PVB2_API int pvb2_select_count(const pvb2_tensor* mask, void* workspace, size_t workspace_bytes,
                               int64_t* d_total, pvb2_stream stream);
PVB2_API int pvb2_select_gather(const pvb2_tensor* src, const pvb2_tensor* mask, void* out,
                                const void* workspace, pvb2_stream stream);
/* index.Tensor_out (advanced indexing): out[i] = src[i + sum_k idx_k[i] *
 * index_strides[k]] where src (already restrided: indexed dims have stride
 * 0) and the int64 index tensors are broadcast to out's sizes; negative
 * indices wrap by index_sizes[k].  At most 4 index tensors. */
PVB2_API int pvb2_index_gather(const pvb2_tensor* out, const pvb2_tensor* src, int n_index,
                               const pvb2_tensor* indices, const int64_t* index_sizes,
                               const int64_t* index_strides, pvb2_stream stream);
/* cat.out along `dim`, pointwise_ops.cpp:689-705 (SliceCopy) */
PVB2_API int pvb2_cat(const pvb2_tensor* out, const pvb2_tensor* inputs, int n_inputs, int dim, pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* pointwise (src/pointwise_ops.cpp)                                    */
/* All operands are already broadcast to out's sizes (stride 0 on       */
/* broadcast dims).  `compute_dtype` is the promoted dtype that the     */
/* arithmetic runs in (PVB2_F32 / PVB2_F64 / PVB2_I64 / PVB2_I32 /      */
/* PVB2_BOOL); operands are converted on load and out on store.         */
/* ------------------------------------------------------------------ */
enum {
  /* unary: out = f(x; p0, p1) */
  PVB2_UN_COPY = 0, PVB2_UN_RELU = 1, PVB2_UN_HARDTANH = 2, PVB2_UN_GELU_ERF = 3,
  PVB2_UN_GELU_TANH = 4, PVB2_UN_NEG = 5, PVB2_UN_EXP = 6, PVB2_UN_LOG = 7,
  PVB2_UN_SQRT = 8, PVB2_UN_ABS = 9, PVB2_UN_SIGMOID = 10, PVB2_UN_TANH = 11,
  PVB2_UN_RECIPROCAL = 12, PVB2_UN_SILU = 13, PVB2_UN_AFFINE = 14, /* x*p0+p1 */
  PVB2_UN_POW = 15, PVB2_UN_CLAMP = 16, PVB2_UN_LEAKY_RELU = 17, PVB2_UN_SGN = 18,
  PVB2_UN_HARDSIGMOID = 19, PVB2_UN_HARDSWISH = 20, PVB2_UN_CEIL = 21,
  PVB2_UN_ROUND = 22, PVB2_UN_ATAN = 23, PVB2_UN_RSQRT = 24, PVB2_UN_LOG_SIGMOID = 25,
  PVB2_UN_BITWISE_NOT = 26, PVB2_UN_CLAMP_MIN = 27, PVB2_UN_FLOOR = 28, PVB2_UN_TRUNC = 29,
  PVB2_UN_LOGICAL_NOT = 30, PVB2_UN_ISNAN = 31, PVB2_UN_ISINF = 32, PVB2_UN_ISPOSINF = 33,
  PVB2_UN_ISNEGINF = 34, PVB2_UN_ISFINITE = 35, PVB2_UN_LOGIT = 36 /* p0 = eps, <0 for none */
};
enum {
  /* binary: out = f(a, b; p0, p1) */
  PVB2_BIN_ADD = 0,        /* a + p0*b                            add_out, pointwise_ops.cpp:133-172 */
  PVB2_BIN_SUB = 1,        /* a - p0*b                            sub_out, :206-210 */
  PVB2_BIN_MUL = 2,        /*                                      mul_out, :407-411 */
  PVB2_BIN_DIV = 3,        /*                                      div_out, :318-344 */
  PVB2_BIN_MAXIMUM = 4, PVB2_BIN_MINIMUM = 5,
  PVB2_BIN_EQ = 6, PVB2_BIN_NE = 7, PVB2_BIN_LT = 8, PVB2_BIN_LE = 9, PVB2_BIN_GT = 10, PVB2_BIN_GE = 11,
  PVB2_BIN_THRESHOLD_BWD = 12, /* b <= p0 ? 0 : a   (a=grad, b=self) threshold_backward, :437-455 */
  PVB2_BIN_HARDTANH_BWD = 13,  /* (b > p0 && b < p1) ? a : 0          hardtanh_backward, :590-603 */
  PVB2_BIN_GELU_ERF_BWD = 14,  /* a * gelu'(b)                         gelu_backward, :1360-1393 */
  PVB2_BIN_GELU_TANH_BWD = 15,
  PVB2_BIN_SIGMOID_BWD = 16,   /* a * b*(1-b)   (b = sigmoid output) */
  PVB2_BIN_TANH_BWD = 17,      /* a * (1-b*b)   (b = tanh output)    */
  PVB2_BIN_SILU_BWD = 18,
  PVB2_BIN_LEAKY_RELU_BWD = 19,
  PVB2_BIN_HARDSIGMOID_BWD = 20, PVB2_BIN_HARDSWISH_BWD = 21,
  PVB2_BIN_BITWISE_AND = 22, PVB2_BIN_BITWISE_OR = 23, PVB2_BIN_BITWISE_XOR = 24,
  PVB2_BIN_LERP = 25,          /* a + p0*(b-a) */
  PVB2_BIN_POW = 26, PVB2_BIN_ATAN2 = 27, PVB2_BIN_LOG_SIGMOID_BWD = 28,
  PVB2_BIN_DIV_TRUNC = 29, PVB2_BIN_DIV_FLOOR = 30, PVB2_BIN_REMAINDER = 31,
  PVB2_BIN_MSE_BWD = 32        /* p0 * (a - b) */
};
enum {
  /* ternary: out = f(a, b, c; p0) */
  PVB2_TER_ADDCMUL = 0,  /* a + p0*b*c   addcmul_out, pointwise_ops.cpp:214-234 */
  PVB2_TER_ADDCDIV = 1,  /* a + p0*b/c   addcdiv_out, :414-434 */
  PVB2_TER_WHERE = 2     /* a(bool) ? b : c */
};
PVB2_API int pvb2_unary(int op, const pvb2_tensor* out, const pvb2_tensor* x, double p0, double p1,
               int compute_dtype, pvb2_stream stream);
PVB2_API int pvb2_binary(int op, const pvb2_tensor* out, const pvb2_tensor* a, const pvb2_tensor* b,
                double p0, double p1, int compute_dtype, pvb2_stream stream);
/* binary op with one operand a host scalar: scalar_first=0 computes
 * f(t, scalar), scalar_first=1 computes f(scalar, t).  Used for the wrapped
 * CPU numbers of add(x, 2), mul_(0.9), rsub, ... (isCPUScalar fast path of
 * the reference, pointwise_ops.cpp:33-52). */
PVB2_API int pvb2_binary_scalar(int op, const pvb2_tensor* out, const pvb2_tensor* t, double scalar,
                                int scalar_first, double p0, double p1, int compute_dtype, pvb2_stream stream);
PVB2_API int pvb2_ternary(int op, const pvb2_tensor* out, const pvb2_tensor* a, const pvb2_tensor* b,
                 const pvb2_tensor* c, double p0, int compute_dtype, pvb2_stream stream);

/* reductions: sum/mean/prod/amax/amin/argmax, red_op_out pointwise_ops.cpp:501-555.
 * `in` has the full shape; `out` has the same ndim with every reduced dim of
 * size 1.  `scale` multiplies the result (1/count for mean). */
enum { PVB2_RED_SUM = 0, PVB2_RED_PROD = 1, PVB2_RED_MAX = 2, PVB2_RED_MIN = 3,
       PVB2_RED_ARGMAX = 4, PVB2_RED_ARGMIN = 5, PVB2_RED_SUMSQ = 6 };
PVB2_API int pvb2_reduce(int op, const pvb2_tensor* out, const pvb2_tensor* in, double scale,
                int compute_dtype, pvb2_stream stream);
/* Same, with scratch for splitting long reduced ranges over many blocks
 * (partials combined in a fixed order, so results depend only on the
 * shape).  workspace may be NULL (no split); otherwise it must hold
 * pvb2_reduce_workspace_size() bytes, which is 0 when no split applies. */
PVB2_API size_t pvb2_reduce_workspace_size(int op, const pvb2_tensor* out, const pvb2_tensor* in,
                                           int compute_dtype);
PVB2_API int pvb2_reduce_ws(int op, const pvb2_tensor* out, const pvb2_tensor* in, double scale,
                            int compute_dtype, void* workspace, size_t workspace_bytes, pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* normalisation (src/norm_ops.cpp)                                     */
/* x, y: [N, C, inner] described by a 4-D NCHW tensor (any of NCHW or   */
/* channels-last strides).  mean/invstd: [C] fp32.                      */
/* ------------------------------------------------------------------ */
/* native_batch_norm (train), norm_ops.cpp:19-84: batch stats, running-stat
 * update with unbiased variance, normalise.  Returns save_mean and
 * save_invstd (torch's convention; the reference returned var).
 * gamma/beta/running_* may be NULL.  workspace >= pvb2_batch_norm_workspace_size. */
PVB2_API size_t pvb2_batch_norm_workspace_size(const pvb2_tensor* x);
PVB2_API int pvb2_batch_norm_fwd_train(const pvb2_tensor* x, const float* gamma, const float* beta,
                              float* running_mean, float* running_var, double momentum, double eps,
                              const pvb2_tensor* y, float* save_mean, float* save_invstd,
                              void* workspace, size_t workspace_bytes, pvb2_stream stream);
/* Training backward below a ReLU: grad_above is the gradient of the ReLU's
 * output relu_out; the gradient of the batch-norm output,
 *     dy = relu_out <= 0 ? 0 : grad_above     (threshold_backward),
 * is formed in the first pass, stored to dy, and the backward proceeds as
 * pvb2_batch_norm_bwd (train) would on it.  One pass fewer than
 * threshold_backward followed by pvb2_batch_norm_bwd (norm_ops.cpp:87-164,
 * pointwise_ops.cpp:437-455).  Needs pvb2_batch_norm_fwd_split_ok(x). */
PVB2_API int pvb2_batch_norm_bwd_relu(const pvb2_tensor* grad_above, const pvb2_tensor* relu_out,
                                      const pvb2_tensor* x, const float* gamma, const float* mean,
                                      const float* invstd, const pvb2_tensor* dy, const pvb2_tensor* dx,
                                      float* dgamma, float* dbeta, void* workspace, size_t workspace_bytes,
                                      pvb2_stream stream);
/* The same below ReLU (act = 1, exactly pvb2_batch_norm_bwd_relu) or ReLU6
 * (act = 2): with act_out the ReLU6 output,
 *     dy = (act_out <= 0 || act_out >= 6) ? 0 : grad_above
 * as hardtanh_backward(grad_above, act_out, 0, 6) computes it
 * (pointwise_ops.cpp:559-603).  MobileNet-v2's conv -> batch norm -> ReLU6. */
PVB2_API int pvb2_batch_norm_bwd_act(int act, const pvb2_tensor* grad_above, const pvb2_tensor* act_out,
                                     const pvb2_tensor* x, const float* gamma, const float* mean,
                                     const float* invstd, const pvb2_tensor* dy, const pvb2_tensor* dx,
                                     float* dgamma, float* dbeta, void* workspace, size_t workspace_bytes,
                                     pvb2_stream stream);
/* The activation's mask formed from x instead of read from its output.
 * pvb2_batch_norm_fwd_apply_ab is pvb2_batch_norm_fwd_apply that also writes
 * each channel's (a, b) of the normalising pass, y = fmaf(x, a, b), to
 * ab_out (2*C floats: a at [c], b at [C + c]).  When that pass applied the
 * activation act with no residual, its output is act(fmaf(x, a, b)) bit for
 * bit, and pvb2_batch_norm_bwd_act_ab forms the same gradient as
 * pvb2_batch_norm_bwd_act from x and ab without reading that output:
 * grad_above is the gradient above the activation, dy (may be NULL) receives
 * the gradient below it, dx the input gradient.  The reference ran
 * threshold_backward (pointwise_ops.cpp) before its batch-norm backward
 * (norm_ops.cpp:87-164), each as its own pass. */
PVB2_API int pvb2_batch_norm_fwd_apply_ab(const pvb2_tensor* x, const float* gamma, const float* beta,
                                          float* running_mean, float* running_var, double momentum, double eps,
                                          const pvb2_tensor* y, float* save_mean, float* save_invstd,
                                          const pvb2_tensor* residual, int act, const pvb2_tensor* sum_out,
                                          const void* workspace, size_t workspace_bytes, float* ab_out,
                                          pvb2_stream stream);
PVB2_API int pvb2_batch_norm_bwd_act_ab(int act, const pvb2_tensor* grad_above, const pvb2_tensor* x,
                                        const float* ab, const float* gamma, const float* mean,
                                        const float* invstd, const pvb2_tensor* dy, const pvb2_tensor* dx,
                                        float* dgamma, float* dbeta, void* workspace, size_t workspace_bytes,
                                        pvb2_stream stream);
/* Training forward in two calls, so that a host can fuse what follows the
 * normalisation into the second pass: pvb2_batch_norm_fwd_stats writes the
 * per-CTA partial sums of x into the workspace; pvb2_batch_norm_fwd_apply
 * folds them (mean, invstd, running statistics, save_mean / save_invstd as
 * pvb2_batch_norm_fwd_train) and writes
 *     y = act(gamma * (x - mean) * invstd + beta + residual)
 * with residual optional (NULL, or contiguous and shaped like x) and act the
 * identity (act = 0), ReLU (act = 1) or ReLU6 = hardtanh(0, 6) (act = 2),
 * NaN kept by both; other values are rejected.  With sum_out given (it may
 * be the residual tensor itself), y receives the plain normalised values and
 * sum_out the epilogue result (a host keeps a copy of the values before an
 * in-place activation this way, or adds the output into another tensor).  With residual
 * NULL and act 0 the pair computes exactly what pvb2_batch_norm_fwd_train
 * does.
 * Both need pvb2_batch_norm_fwd_split_ok(x) (contiguous fp32 NCHW within the
 * streaming kernels' size limits) and the workspace of
 * pvb2_batch_norm_workspace_size, untouched between the two calls.  The
 * reference's torch front end ran batch norm, the residual add and the ReLU
 * (or ReLU6) as three ops (norm_ops.cpp:19-84, pointwise_ops.cpp:55-113,
 * :559-603). */
PVB2_API int pvb2_batch_norm_fwd_split_ok(const pvb2_tensor* x);
PVB2_API int pvb2_batch_norm_fwd_stats(const pvb2_tensor* x, void* workspace, size_t workspace_bytes,
                                       pvb2_stream stream);
/* The same, also adding 1 to *counter (device memory, or NULL) in the same
 * launch: the batch-norm module's num_batches_tracked += 1 (torch's
 * BatchNorm2d.forward in training), which otherwise costs a launch of its
 * own per layer. */
PVB2_API int pvb2_batch_norm_fwd_stats_count(const pvb2_tensor* x, void* workspace, size_t workspace_bytes,
                                             int64_t* counter, pvb2_stream stream);
PVB2_API int pvb2_batch_norm_fwd_apply(const pvb2_tensor* x, const float* gamma, const float* beta,
                                       float* running_mean, float* running_var, double momentum, double eps,
                                       const pvb2_tensor* y, float* save_mean, float* save_invstd,
                                       const pvb2_tensor* residual, int act, const pvb2_tensor* sum_out,
                                       const void* workspace, size_t workspace_bytes, pvb2_stream stream);
/* Batch-norm training forward that allocates nothing and takes no workspace.
 * No counterpart in the reference: it exists for callers that cannot
 * allocate device memory at the point of the call -- code running while a
 * CUDA stream is being captured into a graph (cudaMalloc is not allowed
 * there), or hosts whose memory is fully owned by another allocator and that
 * hand out only their tensors' pointers.  Results equal
 * pvb2_batch_norm_fwd_train's.  Its scratch (per-CTA partial sums) is a
 * fixed 1 MiB array inside this library, resident on every GPU that loads
 * it until the process exits.  The partials take C x splits x 8 bytes, and
 * splits grows with N*H*W (about N*H*W / 16384 per channel for large
 * inputs, at most N on the path for inputs of 2^30 or more elements per
 * channel), so inputs needing more than PVB2_BN_NOALLOC_SCRATCH_BYTES are
 * rejected with PVB2_ERR_INVALID: roughly, inputs of more than about 2^31
 * elements whatever their channel count, or more than about 130k channels.
 * A call is accepted whenever pvb2_batch_norm_workspace_size(x) is at most
 * PVB2_BN_NOALLOC_SCRATCH_BYTES.  The first call on each device looks
 * up that device's copy of the array (make it before any stream capture).
 * All calls share the one array: calls that may overlap on the GPU (other
 * streams, other host threads) race and must be serialised by the caller. */
#define PVB2_BN_NOALLOC_SCRATCH_BYTES (1u << 20)
PVB2_API int pvb2_batch_norm_fwd_train_noalloc(const pvb2_tensor* x, const float* gamma, const float* beta,
                              float* running_mean, float* running_var, double momentum, double eps,
                              const pvb2_tensor* y, float* save_mean, float* save_invstd,
                              pvb2_stream stream);
/* native_batch_norm (eval): uses running stats */
PVB2_API int pvb2_batch_norm_fwd_eval(const pvb2_tensor* x, const float* gamma, const float* beta,
                             const float* running_mean, const float* running_var, double eps,
                             const pvb2_tensor* y, pvb2_stream stream);
/* native_batch_norm_backward (training statistics), norm_ops.cpp:87-164.
 * mean/invstd are save_mean/save_invstd of the forward; `train` must be 1.
 * dx/dgamma/dbeta may be NULL. */
PVB2_API int pvb2_batch_norm_bwd(const pvb2_tensor* dy, const pvb2_tensor* x, const float* gamma,
                        const float* mean, const float* invstd, int train,
                        const pvb2_tensor* dx, float* dgamma, float* dbeta,
                        void* workspace, size_t workspace_bytes, pvb2_stream stream);
/* native_batch_norm_backward with running statistics (eval mode):
 * dx = dy * gamma / sqrt(running_var + eps) */
PVB2_API int pvb2_batch_norm_bwd_eval(const pvb2_tensor* dy, const float* gamma, const float* running_var,
                             double eps, const pvb2_tensor* dx, pvb2_stream stream);
/* native_layer_norm / _backward, norm_ops.cpp:167-351.  x: [M, N] rows
 * (contiguous), gamma/beta: [N] or NULL.  mean/rstd: [M]. */
PVB2_API int pvb2_layer_norm_fwd(const float* x, const float* gamma, const float* beta, int64_t M, int64_t N,
                        double eps, float* y, float* mean, float* rstd, pvb2_stream stream);
PVB2_API size_t pvb2_layer_norm_bwd_workspace_size(int64_t M, int64_t N);
PVB2_API int pvb2_layer_norm_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                        const float* gamma, int64_t M, int64_t N, float* dx, float* dgamma, float* dbeta,
                        void* workspace, size_t workspace_bytes, pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* pooling (src/vision_ops.cpp)                                         */
/* ------------------------------------------------------------------ */
typedef struct pvb2_pool2d_desc {
  int32_t kh, kw, sh, sw, ph, pw, dh, dw;
  int32_t ceil_mode;
  int32_t count_include_pad;   /* avg pool */
  int32_t divisor_override;    /* avg pool, 0 = none */
} pvb2_pool2d_desc;
/* max_pool2d_cls forward, vision_ops.cpp:353-410.  x,y NCHW (contiguous or
 * channels-last); indices int64 with y's layout (flat h*W+w, torch's
 * convention, bit-exact with CPU) or NULL. */
PVB2_API int pvb2_max_pool2d_fwd(const pvb2_pool2d_desc* d, const pvb2_tensor* x, const pvb2_tensor* y,
                        int64_t* indices, pvb2_stream stream);
/* max_pool2d_cls backward, vision_ops.cpp:411-438 (indices-based here) */
PVB2_API int pvb2_max_pool2d_bwd(const pvb2_pool2d_desc* d, const pvb2_tensor* dy, const int64_t* indices,
                        const pvb2_tensor* dx, pvb2_stream stream);
/* avg_pool2d.out / avg_pool2d_backward, vision_ops.cpp:448-511 */
PVB2_API int pvb2_avg_pool2d_fwd(const pvb2_pool2d_desc* d, const pvb2_tensor* x, const pvb2_tensor* y, pvb2_stream stream);
PVB2_API int pvb2_avg_pool2d_bwd(const pvb2_pool2d_desc* d, const pvb2_tensor* dy, const pvb2_tensor* dx, pvb2_stream stream);
/* _adaptive_avg_pool2d / _backward, vision_ops.cpp:188-241 (general
 * adaptive windows; the reference supported global pooling only) */
PVB2_API int pvb2_adaptive_avg_pool2d_fwd(const pvb2_tensor* x, const pvb2_tensor* y, pvb2_stream stream);
PVB2_API int pvb2_adaptive_avg_pool2d_bwd(const pvb2_tensor* dy, const pvb2_tensor* dx, pvb2_stream stream);

/* upsample_nearest2d, _upsample_nearest_exact2d, upsample_bilinear2d and their
 * backward passes (no reference kernel: the reference ran them on its CPU
 * fallback, tensor_ops.cpp:423-429, for the nets its README lists).
 * mode: PVB2_UPSAMPLE_*.  scale_h / scale_w: the input/output coordinate
 * ratio as torch computes it in fp32 (1/scale_factor when the caller gave
 * one, else in/out; (in-1)/(out-1) for align_corners bilinear).  x, y (dy, dx)
 * NCHW contiguous fp32.  Backward passes gather (deterministic). */
enum { PVB2_UPSAMPLE_NEAREST = 0, PVB2_UPSAMPLE_NEAREST_EXACT = 1, PVB2_UPSAMPLE_BILINEAR = 2 };
PVB2_API int pvb2_upsample2d_fwd(int mode, int align_corners, float scale_h, float scale_w, const pvb2_tensor* x,
                                 const pvb2_tensor* y, pvb2_stream stream);
PVB2_API int pvb2_upsample2d_bwd(int mode, int align_corners, float scale_h, float scale_w, const pvb2_tensor* dy,
                                 const pvb2_tensor* dx, pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* softmax and losses (src/loss_ops.cpp)                                */
/* x viewed as (outer, dim, inner), contiguous.                         */
/* ------------------------------------------------------------------ */
/* _log_softmax.out / _softmax.out, loss_ops.cpp:137-175 */
PVB2_API int pvb2_softmax_fwd(int log_softmax, const float* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                     pvb2_stream stream);
/* _log_softmax_backward_data.out / _softmax_backward_data.out, loss_ops.cpp:177-213 */
PVB2_API int pvb2_softmax_bwd(int log_softmax, const float* dy, const float* y, float* dx, int64_t outer, int64_t dim,
                     int64_t inner, pvb2_stream stream);
/* nll_loss_forward.output, loss_ops.cpp:23-44.  x [N, C] (or [C] with N=1),
 * target int64 [N].  reduction 0 none / 1 mean / 2 sum.  weight may be NULL.
 * out: [N] for none, [] otherwise; total_weight: [] */
PVB2_API int pvb2_nll_loss_fwd(const float* x, const int64_t* target, const float* weight, int64_t N, int64_t C,
                      int reduction, int64_t ignore_index, float* out, float* total_weight,
                      pvb2_stream stream);
/* nll_loss_backward.grad_input, loss_ops.cpp:46-65 */
PVB2_API int pvb2_nll_loss_bwd(const float* grad_out, const int64_t* target, const float* weight,
                      const float* total_weight, int64_t N, int64_t C, int reduction,
                      int64_t ignore_index, float* grad_in, pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* GEMM (src/vision_ops.cpp:513-673 mm/bmm/addmm, :243-351 linear)      */
/* C[b] = alpha * A[b] @ B[b] + beta * C[b] (+ bias broadcast)          */
/* A: [batch, M, K], B: [batch, K, N], C: [batch, M, N]; any strides.   */
/* bias: NULL, or [N] (bias_dim=1) / [M] (bias_dim=0), added after      */
/* alpha/beta.                                                          */
/* math: 0 = TF32 tensor cores where the shapes allow, 1 = exact fp32   */
/*       (SIMT).  2 (3xTF32) is reserved: GEMM and convolution entry    */
/*       points reject it with PVB2_ERR_UNSUPPORTED.                    */
/* ------------------------------------------------------------------ */
enum { PVB2_MATH_TF32 = 0, PVB2_MATH_FP32 = 1, PVB2_MATH_3XTF32 = 2 };
PVB2_API int pvb2_gemm(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C,
              const float* bias, int bias_dim, double alpha, double beta, int math,
              pvb2_stream stream);
/* Same, with scratch for splitting K over more CTAs when the output has too
 * few 128 x BN tiles to occupy every SM (a linear layer's weight gradient:
 * small output, K = tokens); the split partials are summed in a fixed order.
 * workspace may be NULL (no split); otherwise it holds
 * pvb2_gemm_workspace_size() bytes, 0 when no split applies. */
PVB2_API size_t pvb2_gemm_workspace_size(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C,
                                         int math);
/* Which engine pvb2_gemm runs these operands on (host logic, no GPU
 * needed): 1 the TF32 tensor cores, 0 exact fp32 on the CUDA cores, -1 an
 * invalid request.  The operands' data pointers and strides count (TMA
 * wants 16-byte aligned bases and row pitches). */
PVB2_API int pvb2_gemm_path(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, int math);
PVB2_API int pvb2_gemm_ws(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C,
                          const float* bias, int bias_dim, double alpha, double beta, int math,
                          void* workspace, size_t workspace_bytes, pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* fused scaled-dot-product attention (the reference's ViT attention ran */
/* as bmm + softmax: mm_bmm_out, vision_ops.cpp:541-626, and            */
/* _softmax_out / _softmax_backward_data_out, loss_ops.cpp:137-213).    */
/* Serves _scaled_dot_product_fused_attention_overrideable(_backward).   */
/* q [B,H,Lq,D], k and v [B,H,Lk,D], any strides over (b, h, l) that     */
/* keep 16-byte rows, unit stride along d; D in {32, 64, 128}.  No mask  */
/* or dropout; causal = query i sees keys j <= i.  fp32 throughout.      */
/* lse: [B,H,Lq] logsumexp of the scaled scores, written by the forward */
/* and read by the backward.                                            */
/* ------------------------------------------------------------------ */
typedef struct pvb2_sdpa_desc {
  int32_t B, H, Lq, Lk, D;
  float scale;                 /* usually 1/sqrt(D)                      */
  int32_t causal;
  int32_t math;                /* PVB2_MATH_TF32: tensor cores (D 32, 64); */
                               /* PVB2_MATH_FP32: exact fp32 CUDA cores     */
} pvb2_sdpa_desc;
PVB2_API int pvb2_sdpa_fwd(const pvb2_sdpa_desc* d, const pvb2_tensor* q, const pvb2_tensor* k, const pvb2_tensor* v,
                           const pvb2_tensor* out, float* lse, pvb2_stream stream);
/* Backward workspace: D_i = rowsum(dO * O) and, unless they would pass
 * 2 GiB, one dQ slice per 64-key block (summed in a fixed order).  A
 * workspace of only the D_i part (B*H*Lq floats, rounded up to 256 bytes) is
 * accepted too: dQ is then recomputed per query block. */
PVB2_API size_t pvb2_sdpa_bwd_workspace_size(const pvb2_sdpa_desc* d);
PVB2_API int pvb2_sdpa_bwd(const pvb2_sdpa_desc* d, const pvb2_tensor* q, const pvb2_tensor* k, const pvb2_tensor* v,
                           const pvb2_tensor* out, const pvb2_tensor* dout, const float* lse, const pvb2_tensor* dq,
                           const pvb2_tensor* dk, const pvb2_tensor* dv, void* workspace, size_t workspace_bytes,
                           pvb2_stream stream);

/* Tensor-core watchdogs (no counterpart in the reference, whose OpenCL   */
/* kernels had no internal waits).  Every mbarrier wait in the tcgen05    */
/* GEMM / convolution kernels gives up after about 2 s and sets a device  */
/* flag instead of spinning forever; these read it (synchronising the    */
/* current device) into *timed_out, and clear it when reset != 0.         */
PVB2_API int pvb2_tc_status(int* timed_out, int reset);
PVB2_API int pvb2_conv_tc_status(int* timed_out, int reset);

/* ------------------------------------------------------------------ */
/* convolution (src/vision_ops.cpp:30-186)                              */
/* ------------------------------------------------------------------ */
typedef struct pvb2_conv2d_desc {
  int32_t N, C, H, W;          /* input                                 */
  int32_t K, R, S;             /* output channels, kernel h, kernel w    */
  int32_t P, Q;                /* output h, w                            */
  int32_t stride_h, stride_w, pad_h, pad_w, dil_h, dil_w;
  int32_t groups;
  int32_t math;                /* PVB2_MATH_*                            */
} pvb2_conv2d_desc;
/* which: 0 fwd, 1 bwd data, 2 bwd filter */
PVB2_API size_t pvb2_conv2d_workspace_size(const pvb2_conv2d_desc* d, int which);
/* Keeping the staged input between forward and weight gradient: the
 * tensor-core paths read x as a channels-last copy or as im2col columns,
 * made in the forward and again in the weight gradient.
 * pvb2_conv2d_staged_input_bytes gives that copy's size (0 when the path
 * stages nothing); pvb2_conv2d_fwd_staged leaves it in the caller's `staged`
 * buffer (*staged_written = 1 when it did), and
 * pvb2_conv2d_bwd_filter_staged reads it from there instead of staging x
 * again.  The caller keeps the buffer between the calls and passes it only
 * while x is unchanged.  The reference staged nothing (its kernels read
 * NCHW directly, vision_ops.cpp:61-186). */
/* Input gradient accumulated into another gradient in one pass:
 * dx = conv2d_bwd_data(dy, w) + addend, the sum formed in the dgrad's
 * epilogue (a residual block's first convolution, whose input gradient the
 * autograd engine adds to the identity branch's; the reference ran the
 * dgrad, vision_ops.cpp:116-186, then its add, pointwise_ops.cpp:133-172).
 * Offered for 1x1 stride-1 convolutions on the TF32 path with 16-byte
 * aligned operands: pvb2_conv2d_bwd_data_acc_ok says whether the pointers
 * and descriptor qualify (1) or not (0), and pvb2_conv2d_bwd_data_acc
 * returns PVB2_ERR_UNSUPPORTED when they do not.  addend may be dx itself
 * (an in-place accumulation); otherwise it must not overlap dx, dy or w.
 * Each element is dgrad + addend rounded once, as the separate add gives. */
PVB2_API int pvb2_conv2d_bwd_data_acc_ok(const pvb2_conv2d_desc* d, const void* dy, const float* w,
                                         const void* dx, const void* addend);
PVB2_API int pvb2_conv2d_bwd_data_acc(const pvb2_conv2d_desc* d, const pvb2_tensor* dy, const float* w,
                                      const pvb2_tensor* dx, const pvb2_tensor* addend, pvb2_stream stream);
PVB2_API size_t pvb2_conv2d_staged_input_bytes(const pvb2_conv2d_desc* d);
/* Which engine a convolution pass runs on (host logic, no GPU needed):
 * which = 0 forward, 1 input gradient, 2 weight gradient.  Returns 1 for the
 * TF32 tensor cores, 0 for exact fp32 on the CUDA cores (math = 1, grouped
 * and depthwise convolutions, shapes too small or not expressible as TMA
 * boxes), -1 for an invalid descriptor.  Assumes 16-byte aligned tensors
 * and the workspace of pvb2_conv2d_workspace_size.  No counterpart in the
 * reference (whose dlprim kernels had one precision); it tells a caller,
 * and the TF32-emulating oracle, where operands are cut to TF32. */
PVB2_API int pvb2_conv2d_path(const pvb2_conv2d_desc* d, int which);
PVB2_API int pvb2_conv2d_fwd_staged(const pvb2_conv2d_desc* d, const pvb2_tensor* x, const float* w,
                                    const float* b, const pvb2_tensor* y, void* workspace, size_t workspace_bytes,
                                    float* staged, size_t staged_bytes, int* staged_written, pvb2_stream stream);
PVB2_API int pvb2_conv2d_bwd_filter_staged(const pvb2_conv2d_desc* d, const pvb2_tensor* x,
                                           const pvb2_tensor* dy, float* dw, float* db, void* workspace,
                                           size_t workspace_bytes, const float* staged, size_t staged_bytes,
                                           pvb2_stream stream);
/* Keeping the staged output gradient between input and weight gradient:
 * both passes of the tap-box path (3x3 and larger filters, and 1x1 layers
 * whose planes are not a multiple of 4 pixels) read dy as a channels-last
 * copy with K padded to 4.  pvb2_conv2d_staged_grad_bytes gives its size
 * (0 when either pass reads dy another way); pvb2_conv2d_bwd_data_staged
 * leaves the copy in the caller's `staged_dy` buffer (*staged_written = 1
 * when it did), and pvb2_conv2d_bwd_filter_staged_grad reads it from there
 * (staged_dy non-null) beside the forward's staged x, instead of staging dy
 * a second time.  The caller passes it only while dy is unchanged.  The
 * reference's convolution_backward (vision_ops.cpp:116-186) ran its data and
 * filter passes on NCHW tensors and staged nothing. */
PVB2_API size_t pvb2_conv2d_staged_grad_bytes(const pvb2_conv2d_desc* d);
PVB2_API int pvb2_conv2d_bwd_data_staged(const pvb2_conv2d_desc* d, const pvb2_tensor* dy, const float* w,
                                         const pvb2_tensor* dx, void* workspace, size_t workspace_bytes,
                                         float* staged_dy, size_t staged_dy_bytes, int* staged_written,
                                         pvb2_stream stream);
PVB2_API int pvb2_conv2d_bwd_filter_staged_grad(const pvb2_conv2d_desc* d, const pvb2_tensor* x,
                                                const pvb2_tensor* dy, float* dw, float* db, void* workspace,
                                                size_t workspace_bytes, const float* staged, size_t staged_bytes,
                                                const float* staged_dy, size_t staged_dy_bytes,
                                                pvb2_stream stream);
/* convolution_overrideable, vision_ops.cpp:61-113: y = conv(x, w) + b
 * x [N,C,H,W], w [K,C/g,R,S] contiguous, y [N,K,P,Q]; x/y NCHW-contiguous
 * or channels-last.  b may be NULL. */
PVB2_API int pvb2_conv2d_fwd(const pvb2_conv2d_desc* d, const pvb2_tensor* x, const float* w, const float* b,
                    const pvb2_tensor* y, void* workspace, size_t workspace_bytes, pvb2_stream stream);
/* convolution_backward_overrideable, data branch, vision_ops.cpp:116-163 */
PVB2_API int pvb2_conv2d_bwd_data(const pvb2_conv2d_desc* d, const pvb2_tensor* dy, const float* w,
                         const pvb2_tensor* dx, void* workspace, size_t workspace_bytes, pvb2_stream stream);
/* convolution_backward_overrideable, filter and bias branches,
 * vision_ops.cpp:145-180.  dw [K,C/g,R,S]; db [K] or NULL. */
PVB2_API int pvb2_conv2d_bwd_filter(const pvb2_conv2d_desc* d, const pvb2_tensor* x, const pvb2_tensor* dy,
                           float* dw, float* db, void* workspace, size_t workspace_bytes,
                           pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* optimizer: SGD with momentum over many tensors in one launch.        */
/* Replaces the per-tensor mul_/add_ loop that torch.optim.SGD's        */
/* foreach path falls into on the reference (add_out / mul_out,         */
/* pointwise_ops.cpp:115-172,407-411).                                  */
/* For every i:  g = grads[i] * grad_scale + weight_decay * params[i]   */
/*   momentum != 0: buf = first_step ? g : momentum*buf + (1-dampening)*g */
/*                  g = nesterov ? g + momentum*buf : buf               */
/*   params[i] -= lr * g                                                */
/* ------------------------------------------------------------------ */
PVB2_API int pvb2_sgd_multi(int n, float* const* params, const float* const* grads, float* const* momentum_bufs,
                   const int64_t* numels, double lr, double momentum, double dampening,
                   double weight_decay, int nesterov, int first_step, double grad_scale,
                   pvb2_stream stream);
/* _foreach_* helpers: out[i] = a[i] (op) (b ? b[i] : scalar) with alpha,
 * for op in {ADD, SUB, MUL, DIV}; out may alias a.  fp32 only. */
PVB2_API int pvb2_foreach_binary(int op, int n, float* const* out, const float* const* a, const float* const* b,
                        const int64_t* numels, double scalar, double alpha, pvb2_stream stream);
/* gather many tensors into one flat buffer (or scatter back): used by the
 * data-parallel gradient buckets.  direction 0: flat <- tensors, 1: tensors <- flat */
PVB2_API int pvb2_flatten_multi(int n, float* const* tensors, const int64_t* numels, float* flat, int direction,
                       double scale, pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* random (src/random_ops.cpp): Philox-4x32-10 counter-based generator  */
/* (Salmon et al., SC'11).  Element i of the output uses counter        */
/* (offset + i/4) and key `seed`, lane i%4.                             */
/* ------------------------------------------------------------------ */
/* uniform_ :37-45 -> [lo, hi) ; normal_ :47-56 -> mean, std ; bernoulli_ :58-67 -> p */
enum { PVB2_RNG_UNIFORM = 0, PVB2_RNG_NORMAL = 1, PVB2_RNG_BERNOULLI = 2 };
PVB2_API int pvb2_philox_fill(int dist, const pvb2_tensor* out, uint64_t seed, uint64_t offset,
                     double p0, double p1, pvb2_stream stream);
/* native_dropout, random_ops.cpp:69-89: mask = u >= p, y = x*mask/(1-p) */
PVB2_API int pvb2_dropout_fwd(const float* x, float* y, uint8_t* mask, int64_t n, double p, uint64_t seed,
                     uint64_t offset, pvb2_stream stream);
/* native_dropout_backward, random_ops.cpp:91-105 */
PVB2_API int pvb2_dropout_bwd(const float* dy, const uint8_t* mask, float* dx, int64_t n, double scale,
                     pvb2_stream stream);

/* ------------------------------------------------------------------ */
/* data-parallel gradient exchange (no counterpart in the reference,    */
/* which has no multi-device code): NCCL over NVLink / NVSwitch.        */
/* ------------------------------------------------------------------ */
#define PVB2_NCCL_ID_BYTES 128
PVB2_API int pvb2_nccl_get_unique_id(uint8_t id[PVB2_NCCL_ID_BYTES]);
PVB2_API int pvb2_nccl_comm_init(void** comm, int nranks, const uint8_t id[PVB2_NCCL_ID_BYTES], int rank);
/* op: 0 sum, 1 avg.  dtype: PVB2_F32 / PVB2_F64 / PVB2_I64 */
PVB2_API int pvb2_nccl_allreduce(void* comm, const void* send, void* recv, size_t count, int dtype, int op,
                        pvb2_stream stream);
PVB2_API int pvb2_nccl_broadcast(void* comm, void* buf, size_t count, int dtype, int root, pvb2_stream stream);
PVB2_API int pvb2_nccl_comm_destroy(void* comm);
PVB2_API int pvb2_nccl_comm_abort(void* comm);

#ifdef __cplusplus
}
#endif
#endif /* PVB2_H */
