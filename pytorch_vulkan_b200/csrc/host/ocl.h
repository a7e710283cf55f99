// Shared declarations of the `ocl` (PrivateUse1) host extension: device and
// stream registry, tensor descriptors for the C-ABI, allocation helpers,
// op tracing.  Every op in ops_*.cpp goes through these.
#pragma once
#include <ATen/ATen.h>
#include <c10/core/Allocator.h>
#include <c10/core/DeviceGuard.h>
#include <torch/library.h>
#include <atomic>
#include <string>
#include <vector>
#include "pvb2.h"

namespace ocl {

constexpr c10::DeviceType kOcl = c10::DeviceType::PrivateUse1;

// ------------------------------------------------------------------ errors
#define OCL_CHECK(expr)                                                                               \
  do {                                                                                                \
    int _s = (expr);                                                                                  \
    TORCH_CHECK(_s == PVB2_OK, "ocl backend: ", #expr, " failed (status ", _s, "): ", pvb2_last_error()); \
  } while (0)

// ---------------------------------------------------------- device/stream
int device_count();
int current_device();
void set_device(int device);
void ensure_device(int device);          // make `device` current for this thread if it is not
pvb2_stream stream_for(int device);      // the current stream of `device` for this thread
pvb2_stream current_stream();            // stream_for(current_device())
void after_op(int device);               // sync-after-op debug mode (OPENCL_NO_MEM_CACHE)

// sets the current device to the tensor's for the scope of an op
struct DeviceScope {
  int prev;
  bool changed;
  explicit DeviceScope(const at::Tensor& t);
  // flush = false: only makes `device` current, leaving deferred work
  // pending (allocations, which neither launch work nor read memory: every
  // pending launch holds references to the tensors it touches)
  explicit DeviceScope(int device, bool flush = true);
  ~DeviceScope();
};

// --------------------------------------------------------------- tracing
// Replaces ExecGuard / the GUARD macro (src/guard.cpp, src/CLTensor.h:24-37):
// OPENCL_DEBUG_MODE (or B200_DEBUG_MODE) = 1 reports the failing op, = 2
// prints an indented trace; while torch.ocl.profile is active each op is
// bracketed by CUDA events for the CSV log.
struct ExecGuard {
  const char* name;
  int device;
  int slot;
  ExecGuard(const char* name, int device);
  ~ExecGuard();
};
extern std::atomic<int> g_trace_mode;
extern std::atomic<bool> g_profiling;
#define OCL_OP(name_str, device_index) ::ocl::ExecGuard _ocl_guard((name_str), (device_index))

// ------------------------------------------------------ tensor <-> C-ABI
int dtype_code(c10::ScalarType t);
pvb2_tensor desc(const at::Tensor& t);
// descriptor of `t` broadcast (expanded) to `sizes`
pvb2_tensor desc_expanded(const at::Tensor& t, c10::IntArrayRef sizes);

// --------------------------------------------------------------- memory
c10::Allocator* allocator();
at::Tensor empty(c10::IntArrayRef sizes, c10::ScalarType dtype, int device,
                 c10::MemoryFormat mf = c10::MemoryFormat::Contiguous);
at::Tensor empty_like_dev(const at::Tensor& t);          // contiguous, same dtype/device
at::Tensor empty_strided_dev(c10::IntArrayRef sizes, c10::IntArrayRef strides, c10::ScalarType dtype, int device);
// scratch buffer from the caching allocator, released at scope exit
struct Workspace {
  c10::DataPtr ptr;
  size_t bytes = 0;
  Workspace(size_t bytes, int device);
  void* get() const { return ptr.get(); }
};
void allocator_record_stream(const c10::DataPtr& ptr, pvb2_stream stream);

// ------------------------------------------------------ deferred epilogue
// A training batch norm may leave its normalising pass pending so that an
// in-place residual add and ReLU of its output join it (deferred.cpp).
// flush_deferred() launches whatever is pending; every op entry, stream and
// event call and synchronisation calls it first.
void flush_deferred();
bool defer_bn_apply(const at::Tensor& x, const at::Tensor& y, const std::optional<at::Tensor>& weight,
                    const std::optional<at::Tensor>& bias, const std::optional<at::Tensor>& running_mean,
                    const std::optional<at::Tensor>& running_var, const at::Tensor& save_mean,
                    const at::Tensor& save_invstd, double momentum, double eps, Workspace&& ws, pvb2_stream stream,
                    int64_t* counter);
// `self += other * alpha` of an int64 scalar by 1 (a batch norm's
// num_batches_tracked) left pending (true) for the statistics kernel of the
// training batch norm that follows; any other op launches it first
bool defer_counter_increment(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha);
// the pending increment's tensor when it lives on `device` (cleared), else
// an undefined tensor
at::Tensor take_pending_counter(int device);
// true when `self += other * alpha` was folded into the pending pass
bool fuse_deferred_add(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha);
// true when `dst.copy_(src)` of the pending pass's output into a contiguous
// tensor was folded into that pass (dst then takes the plain normalised values)
bool fuse_deferred_copy(const at::Tensor& dst, const at::Tensor& src);
// true when `relu_(self)` (act 1) or `hardtanh_(self, 0, 6)` (act 2) was
// folded into the pending pass (and launched it)
bool fuse_deferred_act(const at::Tensor& self, int act);
// threshold_backward(grad, self, 0) (act 1) or hardtanh_backward(grad, self,
// 0, 6) (act 2) into `out`, left pending (true) so that a following
// batch-norm backward can form it in its first pass
bool defer_threshold_bwd(const at::Tensor& grad, const at::Tensor& self, const at::Tensor& out, int act);
// when the pending activation gradient wrote grad_out: hand over its inputs
// and kind (the batch-norm backward then stores grad_out itself) and clear it
bool take_deferred_threshold(const at::Tensor& grad_out, at::Tensor* grad_above, at::Tensor* relu_out, int* act);
// the forward's (a, b) when act_out = act(fmaf(x, a, b)) came from a
// normalising pass of x (the record is consumed), else an undefined tensor
at::Tensor take_act_record(const at::Tensor& act_out, const at::Tensor& x, int act);
// `out` = the activation gradient of (grad, act_out), formed by a batch-norm
// backward but not stored: written at the next flush if still held
void defer_unwritten_act_grad(const at::Tensor& out, const at::Tensor& grad, const at::Tensor& act_out, int act);
// input gradient of a convolution whose dgrad can also form a sum
// (pvb2_conv2d_bwd_data_acc_ok), left pending so that a following add of it
// joins the dgrad's epilogue
bool conv_dgrad_deferrable(const pvb2_conv2d_desc& d, const at::Tensor& gy, const at::Tensor& w, const at::Tensor& gx);
void defer_conv_dgrad(const pvb2_conv2d_desc& d, const at::Tensor& gy, const at::Tensor& w, const at::Tensor& gx);
// true when `out = self + other * alpha` was formed by the pending dgrad
bool fuse_deferred_dgrad_add(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha,
                             const at::Tensor& out);

// ------------------------------------------ staged convolution inputs
// Channels-last / im2col copies of convolution inputs kept from a training
// forward for the weight gradient (ops_nn.cpp); released by empty_cache.
void clear_staged_inputs();
size_t staged_input_bytes();  // bytes the kept copies hold now

// ------------------------------------------------------------- settings
int math_mode();                 // PVB2_MATH_* for convolution / GEMM
void set_math_mode(int mode);

// -------------------------------------------------------------- helpers
inline bool is_ocl(const at::Tensor& t) { return t.defined() && t.device().type() == kOcl; }
// a 0-dim CPU tensor (e.g. a wrapped Python number) used as an operand
inline bool is_cpu_scalar(const at::Tensor& t) {
  return t.defined() && t.device().is_cpu() && t.dim() == 0;
}
// the element type the arithmetic runs in
int compute_code(c10::ScalarType t);
// copy src (any device) into dst (ocl), handling dtype and strides on device
void copy_into(const at::Tensor& dst, const at::Tensor& src, bool non_blocking);
// dst = src laid out contiguously (returns src itself if already so)
at::Tensor contiguous(const at::Tensor& t);
// out may be non-contiguous or of another dtype: run `fn` on a contiguous
// temp of `dtype` and copy back if needed
at::Tensor& write_back(at::Tensor& out, const at::Tensor& tmp);

}  // namespace ocl
