// Deferred batch-norm epilogue (forward) and ReLU gradient (backward).
//
// ResNet-style blocks run `y = bn(x); y += identity; y = relu(y)` as three
// ops, each a full pass over the activation (the reference did the same:
// norm_ops.cpp:19-84, pointwise_ops.cpp:55-113).  Here a training batch norm
// launches its statistics pass at once and leaves the normalising pass
// pending; an in-place add of a residual into its output and an in-place
// ReLU of its output join that pass (pvb2_batch_norm_fwd_apply with a
// residual and relu = 1) instead of re-reading the tensor.  Anything else
// that touches the device first launches what is pending: every op entry
// (DeviceScope, ExecGuard), stream and event calls, synchronisation.  The
// pending state holds references to every tensor the pass reads or writes,
// so none of them can be freed or reused before it runs.
//
// Backward, the mirror image: threshold_backward (the ReLU gradient) is left
// pending, and when the next op is the backward of the batch norm that fed
// that ReLU, its first pass forms the gradient from the ReLU output on the
// fly (pvb2_batch_norm_bwd_relu), still storing it to the op's output tensor.
// B200_DEFER_BN=0 turns both deferrals off.
#include <cstdlib>
#include <mutex>
#include <optional>

#include "ocl.h"

namespace ocl {

namespace {

struct PendingBn {
  // out: where the epilogue result goes when it is not y itself (an in-place
  // add into another tensor of the pending output, `out += y`)
  at::Tensor x, y, weight, bias, running_mean, running_var, save_mean, save_invstd, residual, out;
  double momentum = 0.0, eps = 0.0;
  c10::DataPtr ws;
  size_t ws_bytes = 0;
  pvb2_stream stream = nullptr;
  int device = 0;
  bool relu = false;
};

struct PendingThr {  // grad_input = self <= 0 ? 0 : grad
  at::Tensor grad, self, out;
  pvb2_stream stream = nullptr;
  int device = 0;
};

std::mutex g_mutex;
std::optional<PendingBn> g_pending;
std::optional<PendingThr> g_thr;
std::atomic<bool> g_any{false};
thread_local bool t_flushing = false;

bool defer_enabled() {
  static const bool on = [] {
    const char* v = getenv("B200_DEFER_BN");
    return !(v && v[0] == '0');
  }();
  return on;
}

float* fptr(const at::Tensor& t) { return t.defined() ? t.data_ptr<float>() : nullptr; }

void launch(PendingBn& p, const char* name) {
  DeviceScope scope(p.device);
  OCL_OP(name, p.device);
  const pvb2_tensor xd = desc(p.x), yd = desc(p.y);
  pvb2_tensor rd, od;
  if (p.residual.defined()) rd = desc(p.residual);
  if (p.out.defined()) od = desc(p.out);
  OCL_CHECK(pvb2_batch_norm_fwd_apply(&xd, fptr(p.weight), fptr(p.bias), fptr(p.running_mean), fptr(p.running_var),
                                      p.momentum, p.eps, &yd, fptr(p.save_mean), fptr(p.save_invstd),
                                      p.residual.defined() ? &rd : nullptr, p.relu ? 1 : 0,
                                      p.out.defined() ? &od : nullptr, p.ws.get(), p.ws_bytes, p.stream));
}

void launch_thr(PendingThr& t) {
  DeviceScope scope(t.device);
  OCL_OP("threshold_backward", t.device);
  const pvb2_tensor od = desc(t.out), gd = desc(t.grad), sd = desc(t.self);
  OCL_CHECK(pvb2_binary(PVB2_BIN_THRESHOLD_BWD, &od, &gd, &sd, 0.0, 0.0, PVB2_F32, t.stream));
}

std::pair<std::optional<PendingBn>, std::optional<PendingThr>> take() {
  std::lock_guard<std::mutex> g(g_mutex);
  std::pair<std::optional<PendingBn>, std::optional<PendingThr>> p{std::move(g_pending), std::move(g_thr)};
  g_pending.reset();
  g_thr.reset();
  g_any.store(false, std::memory_order_release);
  return p;
}

}  // namespace

void flush_deferred() {
  if (!g_any.load(std::memory_order_acquire) || t_flushing) return;
  t_flushing = true;
  try {
    auto p = take();
    if (p.first) launch(*p.first, p.first->residual.defined() ? "native_batch_norm+add_" : "native_batch_norm");
    if (p.second) launch_thr(*p.second);
  } catch (...) {
    t_flushing = false;
    throw;
  }
  t_flushing = false;
}

bool defer_bn_apply(const at::Tensor& x, const at::Tensor& y, const std::optional<at::Tensor>& weight,
                    const std::optional<at::Tensor>& bias, const std::optional<at::Tensor>& running_mean,
                    const std::optional<at::Tensor>& running_var, const at::Tensor& save_mean,
                    const at::Tensor& save_invstd, double momentum, double eps, Workspace&& ws, pvb2_stream stream) {
  if (!defer_enabled()) return false;
  const pvb2_tensor xd = desc(x);
  if (!pvb2_batch_norm_fwd_split_ok(&xd)) return false;
  PendingBn p;
  p.x = x;
  p.y = y;
  auto opt = [](const std::optional<at::Tensor>& t) { return t.has_value() && t->defined() ? *t : at::Tensor(); };
  p.weight = opt(weight);
  p.bias = opt(bias);
  p.running_mean = opt(running_mean);
  p.running_var = opt(running_var);
  p.save_mean = save_mean;
  p.save_invstd = save_invstd;
  p.momentum = momentum;
  p.eps = eps;
  p.ws = std::move(ws.ptr);
  p.ws_bytes = ws.bytes;
  p.stream = stream;
  p.device = (int)x.device().index();
  OCL_CHECK(pvb2_batch_norm_fwd_stats(&xd, p.ws.get(), p.ws_bytes, stream));
  for (;;) {
    flush_deferred();  // one pending pass at a time (another thread may have left one)
    std::lock_guard<std::mutex> g(g_mutex);
    if (g_pending.has_value() || g_thr.has_value()) continue;
    g_pending = std::move(p);
    g_any.store(true, std::memory_order_release);
    return true;
  }
}

static bool same_tensor(const at::Tensor& a, const at::Tensor& b) {
  return a.defined() && b.defined() && a.data_ptr() == b.data_ptr() && a.sizes().equals(b.sizes()) &&
         a.strides().equals(b.strides()) && a.scalar_type() == b.scalar_type();
}

bool fuse_deferred_add(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
  if (!g_any.load(std::memory_order_acquire)) return false;
  std::lock_guard<std::mutex> g(g_mutex);
  if (!g_pending || g_pending->relu || g_pending->residual.defined()) return false;
  PendingBn& p = *g_pending;
  if (alpha.isComplex() || alpha.toDouble() != 1.0) return false;
  // `y += other` (ResNet's out += identity) or `self += y` (the same add when
  // the identity branch is the pending batch norm: a downsampling
  // projection); the sum is the same either way, y + other == other + y
  const bool y_is_self = same_tensor(self, p.y);
  const at::Tensor& r = y_is_self ? other : self;
  if (!y_is_self && !same_tensor(other, p.y)) return false;
  if (!is_ocl(r) || r.device() != p.y.device() || r.scalar_type() != at::kFloat || !r.is_contiguous() ||
      !r.sizes().equals(p.y.sizes()))
    return false;
  if (r.is_alias_of(p.y) || r.is_alias_of(p.x)) return false;
  p.residual = r;
  if (!y_is_self) p.out = self;  // y stays the plain normalised values
  return true;
}

bool fuse_deferred_relu(const at::Tensor& self) {
  if (!g_any.load(std::memory_order_acquire)) return false;
  std::optional<PendingBn> p;
  {
    std::lock_guard<std::mutex> g(g_mutex);
    if (!g_pending || !same_tensor(self, g_pending->out.defined() ? g_pending->out : g_pending->y)) return false;
    p = std::move(g_pending);
    g_pending.reset();
    g_any.store(false, std::memory_order_release);
  }
  p->relu = true;
  launch(*p, p->residual.defined() ? "native_batch_norm+add_+relu_" : "native_batch_norm+relu_");
  return true;
}

bool defer_threshold_bwd(const at::Tensor& grad, const at::Tensor& self, const at::Tensor& out) {
  if (!defer_enabled()) return false;
  for (const at::Tensor* t : {&grad, &self, &out})
    if (!is_ocl(*t) || t->scalar_type() != at::kFloat || !t->is_contiguous() || !t->sizes().equals(out.sizes()))
      return false;
  if (grad.device() != out.device() || self.device() != out.device()) return false;
  if (out.is_alias_of(self) || out.is_alias_of(grad) || out.numel() == 0) return false;
  PendingThr t;
  t.grad = grad;
  t.self = self;
  t.out = out;
  t.device = (int)out.device().index();
  t.stream = stream_for(t.device);
  for (;;) {
    flush_deferred();
    std::lock_guard<std::mutex> g(g_mutex);
    if (g_pending.has_value() || g_thr.has_value()) continue;
    g_thr = std::move(t);
    g_any.store(true, std::memory_order_release);
    return true;
  }
}

bool take_deferred_threshold(const at::Tensor& grad_out, at::Tensor* grad_above, at::Tensor* relu_out) {
  if (!g_any.load(std::memory_order_acquire)) return false;
  std::lock_guard<std::mutex> g(g_mutex);
  if (!g_thr || !same_tensor(grad_out, g_thr->out)) return false;
  *grad_above = g_thr->grad;
  *relu_out = g_thr->self;
  g_thr.reset();
  g_any.store(false, std::memory_order_release);
  return true;
}

}  // namespace ocl
