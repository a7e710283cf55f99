// Deferred batch-norm epilogue (forward) and ReLU gradient (backward).
//
// ResNet-style blocks run `y = bn(x); y += identity; y = relu(y)` as three
// ops, each a full pass over the activation (the reference did the same:
// norm_ops.cpp:19-84, pointwise_ops.cpp:55-113).  Here a training batch norm
// launches its statistics pass at once and leaves the normalising pass
// pending; an in-place add of a residual into its output and an in-place
// ReLU of its output join that pass (pvb2_batch_norm_fwd_apply with a
// residual and act = 1), as does MobileNet's in-place ReLU6 (act = 2),
// instead of re-reading the tensor.  The autograd kernel of an in-place
// hardtanh_ first clones its input (the backward reads the values before the
// activation): a copy of the pending output into a fresh contiguous tensor
// joins the pass too, which then writes the plain values to the copy and the
// activated ones to y.  Anything else
// that touches the device first launches what is pending: every op entry
// (DeviceScope, ExecGuard), stream and event calls, synchronisation.  The
// pending state holds references to every tensor the pass reads or writes,
// so none of them can be freed or reused before it runs.
//
// Backward, the mirror image: threshold_backward (the ReLU gradient) or
// hardtanh_backward(.., 0, 6) (ReLU6's) is left pending, and when the next op
// is the backward of the batch norm that fed that activation, its first pass
// forms the gradient from the activation's output on the fly
// (pvb2_batch_norm_bwd_act), still storing it to the op's output tensor.
//
// When the activation joined a pass with no residual, its output is
// act(fmaf(x, a, b)) with that pass's per-channel (a, b): the pass writes
// them to a small tensor and a record remembers which output they belong to
// (holding its storage and x's only weakly).  The batch-norm backward that
// takes the activation gradient then forms the mask from x
// (pvb2_batch_norm_bwd_act_ab) instead of reading the activation's output,
// and does not store the gradient below the activation either: that tensor
// is left as an unwritten record, written by the next flush only if
// something still holds its storage (the engine drops it after the batch
// norm's backward, the usual case).
//
// Input gradients of 1x1 stride-1 convolutions (a residual block's first
// convolution) are left pending as well: when the next op adds that gradient
// to another (the autograd engine summing the identity branch's gradient
// with it), the dgrad's epilogue forms the sum (pvb2_conv2d_bwd_data_acc)
// and the gradient itself is not written.  A record of it stays behind,
// holding its storage only weakly: the next flush writes the gradient after
// all if its storage is still alive (someone kept it), and otherwise (the
// engine dropped it after the add, the usual case) just forgets it.
// A training batch norm's module first adds 1 to its num_batches_tracked
// (an int64 scalar): that add is left pending too, and the batch norm that
// follows hands it to its statistics kernel (pvb2_batch_norm_fwd_stats_count)
// instead of a launch of its own; any other op launches it as the add it is.
// B200_DEFER_BN=0 turns all four deferrals off.
#include <cstdlib>
#include <deque>
#include <mutex>
#include <optional>
#include <vector>

#include "ocl.h"

namespace ocl {

namespace {

struct PendingBn {
  // out: where the epilogue result goes when it is not y itself (an in-place
  // add into another tensor of the pending output, `out += y`)
  // copy: a tensor that takes the plain normalised values, y then taking the
  // epilogue result (a clone of y made before an in-place activation)
  at::Tensor x, y, weight, bias, running_mean, running_var, save_mean, save_invstd, residual, out, copy;
  double momentum = 0.0, eps = 0.0;
  c10::DataPtr ws;
  size_t ws_bytes = 0;
  pvb2_stream stream = nullptr;
  int device = 0;
  int act = 0;  // 0 none, 1 ReLU, 2 ReLU6
};

struct PendingThr {  // act 1: out = self <= 0 ? 0 : grad; act 2: (self <= 0 || self >= 6) ? 0 : grad
  at::Tensor grad, self, out;
  int act = 1;
  pvb2_stream stream = nullptr;
  int device = 0;
  // after a batch-norm backward that formed the gradient without storing
  // it: out is not held, only its storage weakly, with its descriptor;
  // written at the next flush if that storage is still alive
  std::optional<c10::weak_intrusive_ptr<c10::StorageImpl>> unwritten;
  pvb2_tensor out_desc;
};

// an activation output y = act(fmaf(x, a, b)) of a normalising pass, with
// the pass's (a, b) (ab: a at [c], b at [C + c])
struct ActRecord {
  ActRecord(c10::weak_intrusive_ptr<c10::StorageImpl> y, c10::weak_intrusive_ptr<c10::StorageImpl> x)
      : y_storage(std::move(y)), x_storage(std::move(x)) {}
  c10::weak_intrusive_ptr<c10::StorageImpl> y_storage, x_storage;
  const void* y_data = nullptr;
  const void* x_data = nullptr;
  std::vector<int64_t> sizes;
  at::Tensor ab;
  int act = 0;
};
constexpr size_t kMaxActRecords = 1024;
std::mutex g_rec_mutex;
std::deque<ActRecord> g_act_records;

struct PendingDgrad {  // gx = conv2d_bwd_data(gy, w)
  pvb2_conv2d_desc d;
  at::Tensor gy, w, gx;
  pvb2_stream stream = nullptr;
  int device = 0;
  // after a fused add: gx is not held, only its storage weakly, with its
  // descriptor; written at the next flush if that storage is still alive
  std::optional<c10::weak_intrusive_ptr<c10::StorageImpl>> unwritten;
  pvb2_tensor gx_desc;
};

std::mutex g_mutex;
std::optional<PendingBn> g_pending;
std::optional<PendingThr> g_thr;
std::optional<PendingDgrad> g_dgrad;
std::optional<at::Tensor> g_counter;  // a pending `+= 1` of this int64 scalar
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

// the op name of a pending pass, by what joined it
const char* apply_name(const PendingBn& p) {
  static const char* const names[2][2][3] = {
      {{"native_batch_norm.apply", "native_batch_norm.apply+relu_", "native_batch_norm.apply+hardtanh_"},
       {"native_batch_norm.apply+add_", "native_batch_norm.apply+add_+relu_",
        "native_batch_norm.apply+add_+hardtanh_"}},
      {{"native_batch_norm.apply+copy_", "native_batch_norm.apply+copy_+relu_",
        "native_batch_norm.apply+copy_+hardtanh_"},
       {"native_batch_norm.apply+copy_+add_", "native_batch_norm.apply+copy_+add_+relu_",
        "native_batch_norm.apply+copy_+add_+hardtanh_"}}};
  return names[p.copy.defined()][p.residual.defined()][p.act];
}

void launch(PendingBn& p) {
  DeviceScope scope(p.device);
  OCL_OP(apply_name(p), p.device);
  // the kernel's y takes the plain values, its sum_out the epilogue result
  const at::Tensor& plain = p.copy.defined() ? p.copy : p.y;
  const at::Tensor& epi = p.copy.defined() ? p.y : p.out;
  const pvb2_tensor xd = desc(p.x), yd = desc(plain);
  pvb2_tensor rd, od;
  if (p.residual.defined()) rd = desc(p.residual);
  if (epi.defined()) od = desc(epi);
  // y = act(fmaf(x, a, b)) exactly: keep (a, b) for the backward
  const bool record = p.act != 0 && !p.residual.defined() && !p.copy.defined() && !p.out.defined();
  at::Tensor ab = record ? empty({2 * p.x.size(1)}, at::kFloat, p.device) : at::Tensor();
  OCL_CHECK(pvb2_batch_norm_fwd_apply_ab(&xd, fptr(p.weight), fptr(p.bias), fptr(p.running_mean),
                                         fptr(p.running_var), p.momentum, p.eps, &yd, fptr(p.save_mean),
                                         fptr(p.save_invstd), p.residual.defined() ? &rd : nullptr, p.act,
                                         epi.defined() ? &od : nullptr, p.ws.get(), p.ws_bytes, fptr(ab),
                                         p.stream));
  if (!record) return;
  ActRecord r(p.y.storage().getWeakStorageImpl(), p.x.storage().getWeakStorageImpl());
  r.y_data = p.y.data_ptr();
  r.x_data = p.x.data_ptr();
  r.sizes = p.y.sizes().vec();
  r.ab = std::move(ab);
  r.act = p.act;
  std::lock_guard<std::mutex> g(g_rec_mutex);
  // forget records whose tensors are gone (a forward without a backward)
  for (auto it = g_act_records.begin(); it != g_act_records.end();)
    it = it->y_storage.expired() || it->x_storage.expired() ? g_act_records.erase(it) : it + 1;
  if (g_act_records.size() >= kMaxActRecords) g_act_records.pop_front();
  g_act_records.push_back(std::move(r));
}

void launch_thr(PendingThr& t) {
  if (t.unwritten) {
    const c10::intrusive_ptr<c10::StorageImpl> st = t.unwritten->lock();
    if (!st || st->data() != t.out_desc.data) return;  // nobody kept it
  }
  DeviceScope scope(t.device);
  OCL_OP(t.act == 2 ? "hardtanh_backward" : "threshold_backward", t.device);
  const pvb2_tensor od = t.unwritten ? t.out_desc : desc(t.out), gd = desc(t.grad), sd = desc(t.self);
  if (t.act == 2)
    OCL_CHECK(pvb2_binary(PVB2_BIN_HARDTANH_BWD, &od, &gd, &sd, 0.0, 6.0, PVB2_F32, t.stream));
  else
    OCL_CHECK(pvb2_binary(PVB2_BIN_THRESHOLD_BWD, &od, &gd, &sd, 0.0, 0.0, PVB2_F32, t.stream));
}

// dx: where the gradient goes (gx, or the sum's output when addend is set)
void launch_dgrad(PendingDgrad& p, const at::Tensor& dx, const at::Tensor& addend) {
  DeviceScope scope(p.device);
  OCL_OP(addend.defined() ? "convolution_backward+add" : "convolution_backward", p.device);
  const pvb2_tensor gyd = desc(p.gy), dxd = desc(dx);
  if (addend.defined()) {
    const pvb2_tensor ad = desc(addend);
    OCL_CHECK(pvb2_conv2d_bwd_data_acc(&p.d, &gyd, p.w.data_ptr<float>(), &dxd, &ad, p.stream));
    return;
  }
  Workspace ws(pvb2_conv2d_workspace_size(&p.d, 1), p.device);
  OCL_CHECK(pvb2_conv2d_bwd_data(&p.d, &gyd, p.w.data_ptr<float>(), &dxd, ws.get(), ws.bytes, p.stream));
}

struct Taken {
  std::optional<PendingBn> bn;
  std::optional<PendingThr> thr;
  std::optional<PendingDgrad> dgrad;
  std::optional<at::Tensor> counter;
};

Taken take() {
  std::lock_guard<std::mutex> g(g_mutex);
  Taken t{std::move(g_pending), std::move(g_thr), std::move(g_dgrad), std::move(g_counter)};
  g_pending.reset();
  g_thr.reset();
  g_dgrad.reset();
  g_counter.reset();
  g_any.store(false, std::memory_order_release);
  return t;
}

bool anything_pending() {
  return g_pending.has_value() || g_thr.has_value() || g_dgrad.has_value() || g_counter.has_value();
}

}  // namespace

void flush_deferred() {
  if (!g_any.load(std::memory_order_acquire) || t_flushing) return;
  t_flushing = true;
  try {
    auto p = take();
    if (p.counter) p.counter->add_(1);  // the add itself (t_flushing: not deferred again)
    if (p.bn) launch(*p.bn);
    if (p.thr) launch_thr(*p.thr);
    if (p.dgrad && !p.dgrad->unwritten) launch_dgrad(*p.dgrad, p.dgrad->gx, at::Tensor());
    if (p.dgrad && p.dgrad->unwritten) {
      const c10::intrusive_ptr<c10::StorageImpl> st = p.dgrad->unwritten->lock();
      if (st && st->data() == p.dgrad->gx_desc.data) {  // kept by someone: write it now
        PendingDgrad& q = *p.dgrad;
        DeviceScope scope(q.device);
        OCL_OP("convolution_backward", q.device);
        const pvb2_tensor gyd = desc(q.gy);
        Workspace ws(pvb2_conv2d_workspace_size(&q.d, 1), q.device);
        OCL_CHECK(pvb2_conv2d_bwd_data(&q.d, &gyd, q.w.data_ptr<float>(), &q.gx_desc, ws.get(), ws.bytes, q.stream));
      }
    }
  } catch (...) {
    t_flushing = false;
    throw;
  }
  t_flushing = false;
}

bool defer_bn_apply(const at::Tensor& x, const at::Tensor& y, const std::optional<at::Tensor>& weight,
                    const std::optional<at::Tensor>& bias, const std::optional<at::Tensor>& running_mean,
                    const std::optional<at::Tensor>& running_var, const at::Tensor& save_mean,
                    const at::Tensor& save_invstd, double momentum, double eps, Workspace&& ws, pvb2_stream stream,
                    int64_t* counter) {
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
  OCL_CHECK(pvb2_batch_norm_fwd_stats_count(&xd, p.ws.get(), p.ws_bytes, counter, stream));
  for (;;) {
    flush_deferred();  // one pending pass at a time (another thread may have left one)
    std::lock_guard<std::mutex> g(g_mutex);
    if (anything_pending()) continue;
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
  if (!g_pending || g_pending->act || g_pending->residual.defined() || g_pending->copy.defined()) return false;
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

bool fuse_deferred_copy(const at::Tensor& dst, const at::Tensor& src) {
  if (!g_any.load(std::memory_order_acquire)) return false;
  std::lock_guard<std::mutex> g(g_mutex);
  if (!g_pending || g_pending->act || g_pending->residual.defined() || g_pending->copy.defined()) return false;
  PendingBn& p = *g_pending;
  if (!same_tensor(src, p.y)) return false;
  if (!is_ocl(dst) || dst.device() != p.y.device() || dst.scalar_type() != at::kFloat || !dst.is_contiguous() ||
      !dst.sizes().equals(p.y.sizes()))
    return false;
  for (const at::Tensor* t : {&p.x, &p.y, &p.weight, &p.bias, &p.running_mean, &p.running_var, &p.save_mean,
                              &p.save_invstd})
    if (t->defined() && dst.is_alias_of(*t)) return false;
  p.copy = dst;
  return true;
}

bool fuse_deferred_act(const at::Tensor& self, int act) {
  if (!g_any.load(std::memory_order_acquire)) return false;
  std::optional<PendingBn> p;
  {
    std::lock_guard<std::mutex> g(g_mutex);
    if (!g_pending || !same_tensor(self, g_pending->out.defined() ? g_pending->out : g_pending->y)) return false;
    p = std::move(g_pending);
    g_pending.reset();
    g_any.store(false, std::memory_order_release);
  }
  p->act = act;
  launch(*p);
  return true;
}

bool defer_threshold_bwd(const at::Tensor& grad, const at::Tensor& self, const at::Tensor& out, int act) {
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
  t.act = act;
  t.device = (int)out.device().index();
  t.stream = stream_for(t.device);
  for (;;) {
    flush_deferred();
    std::lock_guard<std::mutex> g(g_mutex);
    if (anything_pending()) continue;
    g_thr = std::move(t);
    g_any.store(true, std::memory_order_release);
    return true;
  }
}

bool take_deferred_threshold(const at::Tensor& grad_out, at::Tensor* grad_above, at::Tensor* relu_out, int* act) {
  if (!g_any.load(std::memory_order_acquire)) return false;
  std::lock_guard<std::mutex> g(g_mutex);
  if (!g_thr || !same_tensor(grad_out, g_thr->out)) return false;
  *grad_above = g_thr->grad;
  *relu_out = g_thr->self;
  *act = g_thr->act;
  g_thr.reset();
  g_any.store(false, std::memory_order_release);
  return true;
}

bool conv_dgrad_deferrable(const pvb2_conv2d_desc& d, const at::Tensor& gy, const at::Tensor& w, const at::Tensor& gx) {
  return defer_enabled() && gx.numel() > 0 &&
         pvb2_conv2d_bwd_data_acc_ok(&d, gy.data_ptr(), w.data_ptr<float>(), gx.data_ptr(), gx.data_ptr()) == 1;
}

void defer_conv_dgrad(const pvb2_conv2d_desc& d, const at::Tensor& gy, const at::Tensor& w, const at::Tensor& gx) {
  PendingDgrad p;
  p.d = d;
  p.gy = gy;
  p.w = w;
  p.gx = gx;
  p.device = (int)gx.device().index();
  p.stream = stream_for(p.device);
  for (;;) {
    flush_deferred();
    std::lock_guard<std::mutex> g(g_mutex);
    if (anything_pending()) continue;
    g_dgrad = std::move(p);
    g_any.store(true, std::memory_order_release);
    return;
  }
}

bool fuse_deferred_dgrad_add(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha,
                             const at::Tensor& out) {
  if (!g_any.load(std::memory_order_acquire)) return false;
  std::optional<PendingDgrad> p;
  at::Tensor addend;
  {
    std::lock_guard<std::mutex> g(g_mutex);
    if (!g_dgrad || alpha.isComplex() || alpha.toDouble() != 1.0) return false;
    const PendingDgrad& q = *g_dgrad;
    const bool gx_self = same_tensor(self, q.gx), gx_other = same_tensor(other, q.gx);
    if (gx_self == gx_other) return false;  // neither operand, or gx + gx
    addend = gx_self ? other : self;
    for (const at::Tensor* t : {static_cast<const at::Tensor*>(&addend), &out})
      if (!is_ocl(*t) || t->device() != q.gx.device() || t->scalar_type() != at::kFloat || !t->is_contiguous() ||
          !t->sizes().equals(q.gx.sizes()))
        return false;
    // the sum goes to `out`: gx itself (an in-place add into it) or apart from it
    if (!same_tensor(out, q.gx) && out.is_alias_of(q.gx)) return false;
    // the addend is read where the sum is stored: the same tensor or apart
    if (!same_tensor(addend, out) && addend.is_alias_of(out)) return false;
    if (out.is_alias_of(q.gy) || out.is_alias_of(q.w)) return false;
    if (pvb2_conv2d_bwd_data_acc_ok(&q.d, q.gy.data_ptr(), q.w.data_ptr<float>(), out.data_ptr(),
                                    addend.data_ptr()) != 1)
      return false;
    p = std::move(g_dgrad);
    g_dgrad.reset();
    g_any.store(false, std::memory_order_release);
  }
  launch_dgrad(*p, out, addend);
  if (same_tensor(out, p->gx)) return true;
  // gx was not written: leave the record that writes it if it is still
  // alive at the next flush (installed after the launch, whose own device
  // entry flushes)
  p->gx_desc = desc(p->gx);
  p->unwritten = p->gx.storage().getWeakStorageImpl();
  p->gx = at::Tensor();
  for (;;) {
    flush_deferred();  // one pending record at a time (another thread may have left one)
    std::lock_guard<std::mutex> g(g_mutex);
    if (anything_pending()) continue;
    g_dgrad = std::move(p);
    g_any.store(true, std::memory_order_release);
    return true;
  }
}

at::Tensor take_act_record(const at::Tensor& act_out, const at::Tensor& x, int act) {
  if (!act_out.defined() || !x.defined()) return at::Tensor();
  std::lock_guard<std::mutex> g(g_rec_mutex);
  for (auto it = g_act_records.begin(); it != g_act_records.end(); ++it) {
    if (it->y_data != act_out.data_ptr()) continue;
    const c10::intrusive_ptr<c10::StorageImpl> ys = it->y_storage.lock(), xs = it->x_storage.lock();
    const bool match = ys && xs && ys.get() == act_out.storage().unsafeGetStorageImpl() &&
                       xs.get() == x.storage().unsafeGetStorageImpl() && it->x_data == x.data_ptr() &&
                       it->act == act && act_out.sizes().equals(it->sizes) && x.sizes().equals(it->sizes) &&
                       act_out.is_contiguous() && x.is_contiguous();
    if (!match) continue;
    at::Tensor ab = std::move(it->ab);
    g_act_records.erase(it);
    return ab;
  }
  return at::Tensor();
}

void defer_unwritten_act_grad(const at::Tensor& out, const at::Tensor& grad, const at::Tensor& act_out, int act) {
  PendingThr t;
  t.grad = grad;
  t.self = act_out;
  t.act = act;
  t.device = (int)out.device().index();
  t.stream = stream_for(t.device);
  t.out_desc = desc(out);
  t.unwritten = out.storage().getWeakStorageImpl();
  for (;;) {
    flush_deferred();  // one pending record at a time
    std::lock_guard<std::mutex> g(g_mutex);
    if (anything_pending()) continue;
    g_thr = std::move(t);
    g_any.store(true, std::memory_order_release);
    return;
  }
}

// `self += 1` of an int64 scalar (a batch norm's num_batches_tracked) left
// pending for the statistics launch of the batch norm that follows
bool defer_counter_increment(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
  if (!defer_enabled() || t_flushing) return false;
  if (!is_ocl(self) || self.scalar_type() != at::kLong || self.numel() != 1 || !self.is_contiguous()) return false;
  if (!other.device().is_cpu() || other.numel() != 1 || other.is_floating_point() || other.is_complex() ||
      other.scalar_type() == at::kBool)
    return false;
  if (alpha.isComplex() || alpha.isFloatingPoint() || alpha.toLong() != 1 || other.item().toLong() != 1) return false;
  for (;;) {
    flush_deferred();
    std::lock_guard<std::mutex> g(g_mutex);
    if (anything_pending()) continue;
    g_counter = self;
    g_any.store(true, std::memory_order_release);
    return true;
  }
}

at::Tensor take_pending_counter(int device) {
  if (!g_any.load(std::memory_order_acquire)) return at::Tensor();
  std::lock_guard<std::mutex> g(g_mutex);
  if (!g_counter || g_counter->device().index() != device) return at::Tensor();
  at::Tensor t = std::move(*g_counter);
  g_counter.reset();
  g_any.store(anything_pending(), std::memory_order_release);
  return t;
}

}  // namespace ocl
