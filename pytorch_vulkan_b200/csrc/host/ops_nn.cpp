// Neural-network ops of the `ocl` device: convolution, GEMM family, batch /
// layer norm, pooling, (log)softmax, NLL loss, dropout and random fills.
//
// Mirrors the registrations of src/vision_ops.cpp:833-858,
// src/norm_ops.cpp:354-359, src/loss_ops.cpp:268-280 and
// src/random_ops.cpp:109-115.  Max-pool is registered as the indices-based
// torch op pair (max_pool2d_with_indices[_backward]) instead of the
// reference's autograd override (vision_ops.cpp:353-445), so the indices are
// the CPU's, bit for bit.
#include <deque>
#include <mutex>
#include <utility>

#include <ATen/core/grad_mode.h>

#include "ocl.h"

namespace ocl {

std::pair<uint64_t, uint64_t> philox_reserve(const std::optional<at::Generator>& gen, int device, int64_t n);

// ============================================================ convolution
static pvb2_conv2d_desc conv_desc(const at::Tensor& x, const at::Tensor& w, at::IntArrayRef stride,
                                  at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups) {
  TORCH_CHECK(x.dim() == 4 && w.dim() == 4, "ocl conv: only 2-D convolution (4-D tensors) is supported");
  TORCH_CHECK(stride.size() == 2 && padding.size() == 2 && dilation.size() == 2,
              "ocl conv: expecting stride/padding/dilation of size 2");
  pvb2_conv2d_desc d;
  d.N = (int32_t)x.size(0);
  d.C = (int32_t)x.size(1);
  d.H = (int32_t)x.size(2);
  d.W = (int32_t)x.size(3);
  d.K = (int32_t)w.size(0);
  d.R = (int32_t)w.size(2);
  d.S = (int32_t)w.size(3);
  d.stride_h = (int32_t)stride[0];
  d.stride_w = (int32_t)stride[1];
  d.pad_h = (int32_t)padding[0];
  d.pad_w = (int32_t)padding[1];
  d.dil_h = (int32_t)dilation[0];
  d.dil_w = (int32_t)dilation[1];
  d.groups = (int32_t)groups;
  d.P = (d.H + 2 * d.pad_h - d.dil_h * (d.R - 1) - 1) / d.stride_h + 1;
  d.Q = (d.W + 2 * d.pad_w - d.dil_w * (d.S - 1) - 1) / d.stride_w + 1;
  d.math = math_mode();
  TORCH_CHECK(w.size(1) * groups == x.size(1), "ocl conv: weight/input channel mismatch");
  return d;
}

// transposed conv y = conv_transpose(x, w): the data-gradient of the forward
// conv that maps y-shaped inputs to x-shaped outputs
static pvb2_conv2d_desc tconv_desc(const at::Tensor& x, const at::Tensor& w, at::IntArrayRef stride,
                                   at::IntArrayRef padding, at::IntArrayRef dilation, at::IntArrayRef output_padding,
                                   int64_t groups) {
  pvb2_conv2d_desc d;
  d.N = (int32_t)x.size(0);
  d.K = (int32_t)x.size(1);  // forward conv's output channels = transposed input channels
  d.P = (int32_t)x.size(2);
  d.Q = (int32_t)x.size(3);
  d.C = (int32_t)(w.size(1) * groups);
  d.R = (int32_t)w.size(2);
  d.S = (int32_t)w.size(3);
  d.stride_h = (int32_t)stride[0];
  d.stride_w = (int32_t)stride[1];
  d.pad_h = (int32_t)padding[0];
  d.pad_w = (int32_t)padding[1];
  d.dil_h = (int32_t)dilation[0];
  d.dil_w = (int32_t)dilation[1];
  d.groups = (int32_t)groups;
  d.H = (d.P - 1) * d.stride_h - 2 * d.pad_h + d.dil_h * (d.R - 1) + (int32_t)output_padding[0] + 1;
  d.W = (d.Q - 1) * d.stride_w - 2 * d.pad_w + d.dil_w * (d.S - 1) + (int32_t)output_padding[1] + 1;
  d.math = math_mode();
  return d;
}

// ------------------------------------------- staged input kept for wgrad
// The tensor-core convolution reads its input as a channels-last copy (or
// im2col columns) that it makes on the device, and the weight gradient reads
// the same copy.  A training forward (grad mode on, weight requiring grad)
// leaves it in a buffer kept here, keyed by the input's storage, offset,
// sizes, strides, version counter and the convolution's geometry; the
// backward that finds a match reads it instead of staging its input again
// and drops the entry.  Entries also go when their input's storage is freed
// or the input is modified (its version counter moves), oldest first past a
// byte cap (B200_CONV_STAGE_CACHE_MB, default 4096;
// 0 turns the cache off), and on empty_cache.  The autograd engine runs a
// backward on the stream its forward used, so the buffer is written and read
// in that stream's order, like any workspace.
namespace {
struct StagedInput {
  StagedInput(c10::weak_intrusive_ptr<c10::StorageImpl> s, c10::VariableVersion v)
      : storage(std::move(s)), vc(std::move(v)) {}
  c10::weak_intrusive_ptr<c10::StorageImpl> storage;
  c10::VariableVersion vc;  // the input's version counter (shared, not the tensor)
  int64_t offset = 0, version = 0;
  std::vector<int64_t> sizes, strides;
  pvb2_conv2d_desc d;
  int device = 0;
  c10::DataPtr buf;
  size_t bytes = 0;
};

std::mutex g_stage_mutex;
// never destroyed: entries may outlive the allocator at process exit
std::deque<StagedInput>& staged_inputs() {
  static auto* q = new std::deque<StagedInput>();
  return *q;
}
size_t g_staged_bytes = 0;

size_t stage_cap() {
  static const size_t cap = [] {
    const char* v = getenv("B200_CONV_STAGE_CACHE_MB");
    const long long mb = v ? atoll(v) : 4096;
    return mb > 0 ? (size_t)mb << 20 : (size_t)0;
  }();
  return cap;
}

bool same_desc(const pvb2_conv2d_desc& a, const pvb2_conv2d_desc& b) {
  return a.N == b.N && a.C == b.C && a.H == b.H && a.W == b.W && a.K == b.K && a.R == b.R && a.S == b.S &&
         a.P == b.P && a.Q == b.Q && a.stride_h == b.stride_h && a.stride_w == b.stride_w && a.pad_h == b.pad_h &&
         a.pad_w == b.pad_w && a.dil_h == b.dil_h && a.dil_w == b.dil_w && a.groups == b.groups && a.math == b.math;
}

bool staged_matches(const StagedInput& e, const at::Tensor& x, const pvb2_conv2d_desc& d) {
  if (e.storage.expired()) return false;
  return e.storage.lock().get() == x.storage().unsafeGetStorageImpl() && e.offset == x.storage_offset() &&
         e.version == x._version() && x.sizes().equals(e.sizes) && x.strides().equals(e.strides) &&
         e.device == (int)x.device().index() && same_desc(e.d, d);
}

// drop entries whose input is gone or has changed since (they can never
// match again), then the oldest until `need` more fits
void staged_make_room(size_t need) {
  auto& q = staged_inputs();
  for (auto it = q.begin(); it != q.end();) {
    if (it->storage.expired() || (int64_t)it->vc.current_version() != it->version) {
      g_staged_bytes -= it->bytes;
      it = q.erase(it);
    } else {
      ++it;
    }
  }
  while (!q.empty() && g_staged_bytes + need > stage_cap()) {
    g_staged_bytes -= q.front().bytes;
    q.pop_front();
  }
}

// the backward's lookup: hands over the buffer (the entry is dropped)
c10::DataPtr take_staged_input(const at::Tensor& x, const pvb2_conv2d_desc& d, size_t* bytes) {
  if (!x.unsafeGetTensorImpl()->version_counter().enabled()) return c10::DataPtr();  // never cached
  std::lock_guard<std::mutex> g(g_stage_mutex);
  auto& q = staged_inputs();
  for (auto it = q.begin(); it != q.end(); ++it) {
    if (!staged_matches(*it, x, d)) continue;
    c10::DataPtr p = std::move(it->buf);
    *bytes = it->bytes;
    g_staged_bytes -= it->bytes;
    q.erase(it);
    return p;
  }
  return c10::DataPtr();
}
}  // namespace

size_t staged_input_bytes() {
  std::lock_guard<std::mutex> g(g_stage_mutex);
  return g_staged_bytes;
}

void clear_staged_inputs() {
  std::lock_guard<std::mutex> g(g_stage_mutex);
  staged_inputs().clear();
  g_staged_bytes = 0;
}

// convolution_overrideable, vision_ops.cpp:61-113
static at::Tensor convolution(const at::Tensor& input, const at::Tensor& weight, const std::optional<at::Tensor>& bias,
                              at::IntArrayRef stride, at::IntArrayRef padding, at::IntArrayRef dilation,
                              bool transposed, at::IntArrayRef output_padding, int64_t groups) {
  const int dev = input.device().index();
  DeviceScope scope(dev);
  OCL_OP("convolution", dev);
  at::Tensor x = contiguous(input), w = contiguous(weight);
  const float* b = nullptr;
  at::Tensor bc;
  if (bias.has_value() && bias->defined()) {
    bc = contiguous(*bias);
    b = bc.data_ptr<float>();
  }
  TORCH_CHECK(x.scalar_type() == at::kFloat, "ocl conv: float32 only");
  pvb2_stream st = stream_for(dev);
  if (!transposed) {
    pvb2_conv2d_desc d = conv_desc(x, w, stride, padding, dilation, groups);
    at::Tensor y = empty({d.N, d.K, d.P, d.Q}, at::kFloat, dev);
    if (y.numel() == 0) return y;
    Workspace ws(pvb2_conv2d_workspace_size(&d, 0), dev);
    pvb2_tensor xd = desc(x), yd = desc(y);
    const size_t sb = at::GradMode::is_enabled() && weight.requires_grad() && stage_cap() > 0 &&
                              x.unsafeGetTensorImpl()->version_counter().enabled()
                          ? pvb2_conv2d_staged_input_bytes(&d)
                          : 0;
    if (sb == 0 || sb > stage_cap()) {
      OCL_CHECK(pvb2_conv2d_fwd(&d, &xd, w.data_ptr<float>(), b, &yd, ws.get(), ws.bytes, st));
      return y;
    }
    {
      std::lock_guard<std::mutex> g(g_stage_mutex);
      staged_make_room(sb);
    }
    Workspace staged(sb, dev);
    int written = 0;
    OCL_CHECK(pvb2_conv2d_fwd_staged(&d, &xd, w.data_ptr<float>(), b, &yd, ws.get(), ws.bytes,
                                     (float*)staged.get(), sb, &written, st));
    if (written) {
      StagedInput e(x.storage().getWeakStorageImpl(), x.unsafeGetTensorImpl()->version_counter());
      e.offset = x.storage_offset();
      e.version = x._version();
      e.sizes = x.sizes().vec();
      e.strides = x.strides().vec();
      e.d = d;
      e.device = dev;
      e.buf = std::move(staged.ptr);
      e.bytes = sb;
      std::lock_guard<std::mutex> g(g_stage_mutex);
      g_staged_bytes += sb;
      staged_inputs().push_back(std::move(e));
    }
    return y;
  }
  pvb2_conv2d_desc d = tconv_desc(x, w, stride, padding, dilation, output_padding, groups);
  at::Tensor y = empty({d.N, d.C, d.H, d.W}, at::kFloat, dev);
  if (y.numel() == 0) return y;
  Workspace ws(pvb2_conv2d_workspace_size(&d, 1), dev);
  pvb2_tensor xd = desc(x), yd = desc(y);
  OCL_CHECK(pvb2_conv2d_bwd_data(&d, &xd, w.data_ptr<float>(), &yd, ws.get(), ws.bytes, st));
  if (b) {
    pvb2_tensor bd = desc(bc.view({1, d.C, 1, 1}).expand(y.sizes()));
    OCL_CHECK(pvb2_binary(PVB2_BIN_ADD, &yd, &yd, &bd, 1.0, 0.0, PVB2_F32, st));
  }
  return y;
}

// convolution_backward_overrideable, vision_ops.cpp:116-186
static std::tuple<at::Tensor, at::Tensor, at::Tensor> convolution_backward(
    const at::Tensor& grad_output, const at::Tensor& input, const at::Tensor& weight, at::IntArrayRef stride,
    at::IntArrayRef padding, at::IntArrayRef dilation, bool transposed, at::IntArrayRef output_padding, int64_t groups,
    std::array<bool, 3> output_mask) {
  const int dev = input.device().index();
  DeviceScope scope(dev);
  OCL_OP("convolution_backward", dev);
  at::Tensor x = contiguous(input), w = contiguous(weight), gy = contiguous(grad_output);
  pvb2_stream st = stream_for(dev);
  at::Tensor gx, gw, gb;
  if (!transposed) {
    pvb2_conv2d_desc d = conv_desc(x, w, stride, padding, dilation, groups);
    pvb2_tensor xd = desc(x), gyd = desc(gy);
    bool dgrad_later = false;  // left pending after the weight gradient (deferred.cpp)
    if (output_mask[0]) {
      gx = empty(x.sizes(), at::kFloat, dev);
      dgrad_later = conv_dgrad_deferrable(d, gy, w, gx);
    }
    // the input gradient's channels-last copy of dy, kept for the weight gradient
    const size_t gsb = output_mask[0] && !dgrad_later && output_mask[1] ? pvb2_conv2d_staged_grad_bytes(&d) : 0;
    Workspace staged_gy(gsb, dev);
    int gy_staged = 0;
    if (output_mask[0] && !dgrad_later) {
      Workspace ws(pvb2_conv2d_workspace_size(&d, 1), dev);
      pvb2_tensor gxd = desc(gx);
      OCL_CHECK(pvb2_conv2d_bwd_data_staged(&d, &gyd, w.data_ptr<float>(), &gxd, ws.get(), ws.bytes,
                                            (float*)staged_gy.get(), gsb, &gy_staged, st));
    }
    if (output_mask[1] || output_mask[2]) {
      if (output_mask[1]) gw = empty(w.sizes(), at::kFloat, dev);
      if (output_mask[2]) gb = empty({d.K}, at::kFloat, dev);
      Workspace ws(output_mask[1] ? pvb2_conv2d_workspace_size(&d, 2) : 0, dev);
      size_t sb = 0;
      c10::DataPtr staged = output_mask[1] ? take_staged_input(x, d, &sb) : c10::DataPtr();
      OCL_CHECK(pvb2_conv2d_bwd_filter_staged_grad(
          &d, &xd, &gyd, output_mask[1] ? gw.data_ptr<float>() : nullptr,
          output_mask[2] ? gb.data_ptr<float>() : nullptr, ws.get(), ws.bytes, (const float*)staged.get(), sb,
          gy_staged ? (const float*)staged_gy.get() : nullptr, gsb, st));
    }
    if (dgrad_later) defer_conv_dgrad(d, gy, w, gx);
    return {gx, gw, gb};
  }
  // transposed: forward was y = dgrad(x); so dx = conv_fwd(dy), dw = wgrad(input=dy, grad=x)
  pvb2_conv2d_desc d = tconv_desc(x, w, stride, padding, dilation, output_padding, groups);
  pvb2_tensor xd = desc(x), gyd = desc(gy);
  if (output_mask[0]) {
    gx = empty(x.sizes(), at::kFloat, dev);
    Workspace ws(pvb2_conv2d_workspace_size(&d, 0), dev);
    pvb2_tensor gxd = desc(gx);
    OCL_CHECK(pvb2_conv2d_fwd(&d, &gyd, w.data_ptr<float>(), nullptr, &gxd, ws.get(), ws.bytes, st));
  }
  if (output_mask[1]) {
    gw = empty(w.sizes(), at::kFloat, dev);
    Workspace ws(pvb2_conv2d_workspace_size(&d, 2), dev);
    OCL_CHECK(pvb2_conv2d_bwd_filter(&d, &gyd, &xd, gw.data_ptr<float>(), nullptr, ws.get(), ws.bytes, st));
  }
  if (output_mask[2]) gb = gy.sum({0, 2, 3});
  return {gx, gw, gb};
}

// ================================================================== GEMM
// 2-D / 3-D operand as a 3-D [batch, rows, cols] descriptor
static pvb2_tensor as3d(const at::Tensor& t) {
  pvb2_tensor d = desc(t);
  if (t.dim() == 2) {
    d.ndim = 3;
    d.sizes[2] = d.sizes[1];
    d.sizes[1] = d.sizes[0];
    d.sizes[0] = 1;
    d.strides[2] = d.strides[1];
    d.strides[1] = d.strides[0];
    d.strides[0] = 0;
  }
  return d;
}

static void gemm(const at::Tensor& a, const at::Tensor& b, const at::Tensor& c, const float* bias, int bias_dim,
                 double alpha, double beta) {
  const int dev = c.device().index();
  pvb2_tensor A = as3d(a), B = as3d(b), C = as3d(c);
  const int math = math_mode();
  const size_t wsb = pvb2_gemm_workspace_size(&A, &B, &C, math);
  if (wsb == 0) {
    OCL_CHECK(pvb2_gemm(&A, &B, &C, bias, bias_dim, alpha, beta, math, stream_for(dev)));
  } else {
    Workspace ws(wsb, dev);
    OCL_CHECK(pvb2_gemm_ws(&A, &B, &C, bias, bias_dim, alpha, beta, math, ws.get(), ws.bytes, stream_for(dev)));
  }
}

// mm.out, vision_ops.cpp:513-560
static at::Tensor& mm_out(const at::Tensor& self, const at::Tensor& mat2, at::Tensor& out) {
  const int dev = out.device().index();
  DeviceScope scope(dev);
  OCL_OP("mm", dev);
  TORCH_CHECK(self.dim() == 2 && mat2.dim() == 2 && self.size(1) == mat2.size(0), "mm: shape mismatch");
  if (!out.sizes().equals({self.size(0), mat2.size(1)})) out.resize_({self.size(0), mat2.size(1)});
  if (out.numel() == 0) return out;
  if (self.size(1) == 0) return out.zero_();
  gemm(self, mat2, out, nullptr, 0, 1.0, 0.0);
  return out;
}

// bmm.out, vision_ops.cpp:562-626
static at::Tensor& bmm_out(const at::Tensor& self, const at::Tensor& mat2, at::Tensor& out) {
  const int dev = out.device().index();
  DeviceScope scope(dev);
  OCL_OP("bmm", dev);
  TORCH_CHECK(self.dim() == 3 && mat2.dim() == 3 && self.size(0) == mat2.size(0) && self.size(2) == mat2.size(1),
              "bmm: shape mismatch");
  if (!out.sizes().equals({self.size(0), self.size(1), mat2.size(2)}))
    out.resize_({self.size(0), self.size(1), mat2.size(2)});
  if (out.numel() == 0) return out;
  if (self.size(2) == 0) return out.zero_();
  gemm(self, mat2, out, nullptr, 0, 1.0, 0.0);
  return out;
}

// addmm.out, vision_ops.cpp:628-673:  out = beta*self + alpha*(mat1 @ mat2)
static at::Tensor& addmm_out(const at::Tensor& self, const at::Tensor& mat1, const at::Tensor& mat2,
                             const at::Scalar& beta, const at::Scalar& alpha, at::Tensor& out) {
  const int dev = out.device().index();
  DeviceScope scope(dev);
  OCL_OP("addmm", dev);
  TORCH_CHECK(mat1.dim() == 2 && mat2.dim() == 2 && mat1.size(1) == mat2.size(0), "addmm: shape mismatch");
  const int64_t M = mat1.size(0), N = mat2.size(1);
  if (!out.sizes().equals({M, N})) out.resize_({M, N});
  if (out.numel() == 0) return out;
  const double b = beta.toDouble(), a = alpha.toDouble();
  // linear's case: a bias row added once
  const bool bias_row = b == 1.0 && !out.is_same(self) && self.dim() <= 2 && self.numel() == N &&
                        (self.dim() == 1 || self.size(0) == 1) && self.scalar_type() == at::kFloat;
  if (bias_row && mat1.size(1) > 0) {
    at::Tensor bc = contiguous(self.reshape({N}));
    gemm(mat1, mat2, out, bc.data_ptr<float>(), 1, a, 0.0);
    return out;
  }
  if (!out.is_same(self)) {
    if (b == 0.0) out.zero_();
    else out.copy_(self.expand({M, N}));
  }
  if (mat1.size(1) == 0) {
    if (b != 1.0) out.mul_(b);
    return out;
  }
  gemm(mat1, mat2, out, nullptr, 0, a, b);
  return out;
}

// baddbmm.out: out = beta*self + alpha*(batch1 @ batch2)
static at::Tensor& baddbmm_out(const at::Tensor& self, const at::Tensor& b1, const at::Tensor& b2,
                               const at::Scalar& beta, const at::Scalar& alpha, at::Tensor& out) {
  const int dev = out.device().index();
  DeviceScope scope(dev);
  OCL_OP("baddbmm", dev);
  const int64_t B = b1.size(0), M = b1.size(1), N = b2.size(2);
  if (!out.sizes().equals({B, M, N})) out.resize_({B, M, N});
  if (out.numel() == 0) return out;
  const double bb = beta.toDouble();
  if (!out.is_same(self)) {
    if (bb == 0.0) out.zero_();
    else out.copy_(self.expand({B, M, N}));
  }
  gemm(b1, b2, out, nullptr, 0, alpha.toDouble(), bb);
  return out;
}

// =========================================================== batch norm
// native_batch_norm, norm_ops.cpp:19-84 (returns save_mean/save_invstd)
static std::tuple<at::Tensor, at::Tensor, at::Tensor> native_batch_norm(
    const at::Tensor& input, const std::optional<at::Tensor>& weight, const std::optional<at::Tensor>& bias,
    const std::optional<at::Tensor>& running_mean, const std::optional<at::Tensor>& running_var, bool training,
    double momentum, double eps) {
  const int dev = input.device().index();
  TORCH_CHECK(input.scalar_type() == at::kFloat, "ocl batch_norm: float32 only");
  for (const auto* t : {&weight, &bias, &running_mean, &running_var})
    if (t->has_value() && (*t)->defined()) TORCH_CHECK((*t)->is_contiguous(), "ocl batch_norm: parameters must be contiguous");
  // the module's `num_batches_tracked += 1` just before, when it was left
  // pending: taken before the op entry flushes it, applied by the
  // statistics kernel below (or launched as the add it is)
  at::Tensor counter = training ? take_pending_counter(dev) : at::Tensor();
  auto count_apart = [&] {
    if (counter.defined()) std::exchange(counter, at::Tensor()).add_(1);
  };
  try {
    DeviceScope scope(dev);
    OCL_OP("native_batch_norm", dev);
    at::Tensor x = contiguous(input);
    const int64_t C = x.size(1);
    auto ptr = [](const std::optional<at::Tensor>& t) -> float* {
      return t.has_value() && t->defined() ? t->data_ptr<float>() : nullptr;
    };
    at::Tensor y = empty(x.sizes(), at::kFloat, dev);
    pvb2_tensor xd = desc(x), yd = desc(y);
    pvb2_stream st = stream_for(dev);
    if (training) {
      at::Tensor mean = empty({C}, at::kFloat, dev), invstd = empty({C}, at::kFloat, dev);
      Workspace ws(pvb2_batch_norm_workspace_size(&xd), dev);
      // statistics now, the normalising pass when the next op needs it (or
      // fused with an in-place residual add / ReLU of y)
      if (defer_bn_apply(x, y, weight, bias, running_mean, running_var, mean, invstd, momentum, eps, std::move(ws), st,
                         counter.defined() ? counter.data_ptr<int64_t>() : nullptr))
        return {y, mean, invstd};
      count_apart();
      OCL_CHECK(pvb2_batch_norm_fwd_train(&xd, ptr(weight), ptr(bias), ptr(running_mean), ptr(running_var),
                                          momentum, eps, &yd, mean.data_ptr<float>(), invstd.data_ptr<float>(),
                                          ws.get(), ws.bytes, st));
      return {y, mean, invstd};
    }
  } catch (...) {
    count_apart();
    throw;
  }
  DeviceScope scope(dev);
  OCL_OP("native_batch_norm", dev);
  at::Tensor x = contiguous(input);
  auto ptr = [](const std::optional<at::Tensor>& t) -> float* {
    return t.has_value() && t->defined() ? t->data_ptr<float>() : nullptr;
  };
  at::Tensor y = empty(x.sizes(), at::kFloat, dev);
  pvb2_tensor xd = desc(x), yd = desc(y);
  pvb2_stream st = stream_for(dev);
  TORCH_CHECK(ptr(running_mean) && ptr(running_var), "ocl batch_norm: running stats required in eval mode");
  OCL_CHECK(pvb2_batch_norm_fwd_eval(&xd, ptr(weight), ptr(bias), ptr(running_mean), ptr(running_var), eps, &yd, st));
  return {y, empty({0}, at::kFloat, dev), empty({0}, at::kFloat, dev)};
}

// native_batch_norm_backward, norm_ops.cpp:87-164
static std::tuple<at::Tensor, at::Tensor, at::Tensor> native_batch_norm_backward(
    const at::Tensor& grad_out, const at::Tensor& input, const std::optional<at::Tensor>& weight,
    const std::optional<at::Tensor>& running_mean, const std::optional<at::Tensor>& running_var,
    const std::optional<at::Tensor>& save_mean, const std::optional<at::Tensor>& save_invstd, bool train, double eps,
    std::array<bool, 3> output_mask) {
  const int dev = input.device().index();
  // grad_out still pending as a ReLU's or ReLU6's gradient: form it in the
  // first pass
  at::Tensor relu_grad, relu_out;
  bool below_relu = false;
  int act = 0;
  if (train && input.is_contiguous() && input.scalar_type() == at::kFloat && save_mean.has_value() &&
      save_invstd.has_value()) {
    const pvb2_tensor xd0 = desc(input);
    below_relu = pvb2_batch_norm_fwd_split_ok(&xd0) && take_deferred_threshold(grad_out, &relu_grad, &relu_out, &act);
  }
  // the forward's (a, b) when the activation's output came from this input's
  // normalising pass: the mask is then formed from x ("@x" in the op name)
  const at::Tensor ab = below_relu ? take_act_record(relu_out, input, act) : at::Tensor();
  static const char* const names[2][3] = {
      {"native_batch_norm_backward", "threshold_backward+native_batch_norm_backward",
       "hardtanh_backward+native_batch_norm_backward"},
      {"native_batch_norm_backward", "threshold_backward@x+native_batch_norm_backward",
       "hardtanh_backward@x+native_batch_norm_backward"}};
  DeviceScope scope(dev);
  OCL_OP(names[ab.defined()][below_relu ? act : 0], dev);
  at::Tensor x = contiguous(input), gy = below_relu ? grad_out : contiguous(grad_out);
  const int64_t C = x.size(1);
  const float* g = weight.has_value() && weight->defined() ? weight->data_ptr<float>() : nullptr;
  at::Tensor gx, gw, gb;
  if (output_mask[0]) gx = empty(x.sizes(), at::kFloat, dev);
  if (output_mask[1]) gw = empty({C}, at::kFloat, dev);
  if (output_mask[2]) gb = empty({C}, at::kFloat, dev);
  pvb2_stream st = stream_for(dev);
  pvb2_tensor xd = desc(x), gyd = desc(gy);
  if (train) {
    TORCH_CHECK(save_mean.has_value() && save_invstd.has_value(), "ocl batch_norm_backward: saved stats required");
    pvb2_tensor gxd;
    if (output_mask[0]) gxd = desc(gx);
    Workspace ws(pvb2_batch_norm_workspace_size(&xd), dev);
    if (below_relu) {
      const pvb2_tensor rgd = desc(relu_grad), rod = desc(relu_out);
      // the activation's mask from x with the forward's (a, b); its gradient
      // (grad_out) is stored only if someone still holds it at the next flush
      if (ab.defined()) {
        OCL_CHECK(pvb2_batch_norm_bwd_act_ab(act, &rgd, &xd, ab.data_ptr<float>(), g, save_mean->data_ptr<float>(),
                                             save_invstd->data_ptr<float>(), nullptr,
                                             output_mask[0] ? &gxd : nullptr,
                                             output_mask[1] ? gw.data_ptr<float>() : nullptr,
                                             output_mask[2] ? gb.data_ptr<float>() : nullptr, ws.get(), ws.bytes, st));
        defer_unwritten_act_grad(gy, relu_grad, relu_out, act);
        return {gx, gw, gb};
      }
      OCL_CHECK(pvb2_batch_norm_bwd_act(act, &rgd, &rod, &xd, g, save_mean->data_ptr<float>(),
                                        save_invstd->data_ptr<float>(), &gyd, output_mask[0] ? &gxd : nullptr,
                                        output_mask[1] ? gw.data_ptr<float>() : nullptr,
                                        output_mask[2] ? gb.data_ptr<float>() : nullptr, ws.get(), ws.bytes, st));
      return {gx, gw, gb};
    }
    OCL_CHECK(pvb2_batch_norm_bwd(&gyd, &xd, g, save_mean->data_ptr<float>(), save_invstd->data_ptr<float>(), 1,
                                  output_mask[0] ? &gxd : nullptr, output_mask[1] ? gw.data_ptr<float>() : nullptr,
                                  output_mask[2] ? gb.data_ptr<float>() : nullptr, ws.get(), ws.bytes, st));
    return {gx, gw, gb};
  }
  // running statistics (eval-mode backward)
  TORCH_CHECK(running_mean.has_value() && running_var.has_value(), "ocl batch_norm_backward: running stats required");
  if (output_mask[0]) {
    pvb2_tensor gxd = desc(gx);
    OCL_CHECK(pvb2_batch_norm_bwd_eval(&gyd, g, running_var->data_ptr<float>(), eps, &gxd, st));
  }
  std::vector<int64_t> red{0};
  for (int64_t d = 2; d < x.dim(); ++d) red.push_back(d);
  std::vector<int64_t> bshape(x.dim(), 1);
  bshape[1] = C;
  if (output_mask[2]) gb.copy_(gy.sum(red));
  if (output_mask[1]) {
    at::Tensor invstd = (*running_var + eps).rsqrt();
    gw.copy_((gy * (x - running_mean->view(bshape)) * invstd.view(bshape)).sum(red));
  }
  return {gx, gw, gb};
}

// =========================================================== layer norm
// native_layer_norm, norm_ops.cpp:167-235
static std::tuple<at::Tensor, at::Tensor, at::Tensor> native_layer_norm(const at::Tensor& input,
                                                                         at::IntArrayRef normalized_shape,
                                                                         const std::optional<at::Tensor>& weight,
                                                                         const std::optional<at::Tensor>& bias,
                                                                         double eps) {
  const int dev = input.device().index();
  DeviceScope scope(dev);
  OCL_OP("native_layer_norm", dev);
  at::Tensor x = contiguous(input);
  const int64_t axis = x.dim() - (int64_t)normalized_shape.size();
  int64_t M = 1, N = 1;
  for (int64_t d = 0; d < x.dim(); ++d) (d < axis ? M : N) *= x.size(d);
  std::vector<int64_t> stat_shape;
  for (int64_t d = 0; d < x.dim(); ++d) stat_shape.push_back(d < axis ? x.size(d) : 1);
  at::Tensor y = empty(x.sizes(), at::kFloat, dev);
  at::Tensor mean = empty(stat_shape, at::kFloat, dev), rstd = empty(stat_shape, at::kFloat, dev);
  at::Tensor w, b;
  if (weight.has_value() && weight->defined()) w = contiguous(*weight);
  if (bias.has_value() && bias->defined()) b = contiguous(*bias);
  OCL_CHECK(pvb2_layer_norm_fwd(x.data_ptr<float>(), w.defined() ? w.data_ptr<float>() : nullptr,
                                b.defined() ? b.data_ptr<float>() : nullptr, M, N, eps, y.data_ptr<float>(),
                                mean.data_ptr<float>(), rstd.data_ptr<float>(), stream_for(dev)));
  return {y, mean, rstd};
}

// native_layer_norm_backward, norm_ops.cpp:237-351
static std::tuple<at::Tensor, at::Tensor, at::Tensor> native_layer_norm_backward(
    const at::Tensor& grad_out, const at::Tensor& input, at::IntArrayRef normalized_shape, const at::Tensor& mean,
    const at::Tensor& rstd, const std::optional<at::Tensor>& weight, const std::optional<at::Tensor>& bias,
    std::array<bool, 3> output_mask) {
  const int dev = input.device().index();
  DeviceScope scope(dev);
  OCL_OP("native_layer_norm_backward", dev);
  at::Tensor x = contiguous(input), gy = contiguous(grad_out);
  const int64_t axis = x.dim() - (int64_t)normalized_shape.size();
  int64_t M = 1, N = 1;
  for (int64_t d = 0; d < x.dim(); ++d) (d < axis ? M : N) *= x.size(d);
  at::Tensor w;
  if (weight.has_value() && weight->defined()) w = contiguous(*weight);
  at::Tensor gx, gw, gb;
  if (output_mask[0]) gx = empty(x.sizes(), at::kFloat, dev);
  if (output_mask[1] && w.defined()) gw = empty(w.sizes(), at::kFloat, dev);
  if (output_mask[2] && bias.has_value() && bias->defined()) gb = empty(bias->sizes(), at::kFloat, dev);
  Workspace ws(pvb2_layer_norm_bwd_workspace_size(M, N), dev);
  OCL_CHECK(pvb2_layer_norm_bwd(gy.data_ptr<float>(), x.data_ptr<float>(), contiguous(mean).data_ptr<float>(),
                                contiguous(rstd).data_ptr<float>(), w.defined() ? w.data_ptr<float>() : nullptr, M, N,
                                gx.defined() ? gx.data_ptr<float>() : nullptr,
                                gw.defined() ? gw.data_ptr<float>() : nullptr,
                                gb.defined() ? gb.data_ptr<float>() : nullptr, ws.get(), ws.bytes, stream_for(dev)));
  return {gx, gw, gb};
}

// ============================================================== pooling
static pvb2_pool2d_desc pool_desc(at::IntArrayRef k, at::IntArrayRef s, at::IntArrayRef p, at::IntArrayRef d,
                                  bool ceil_mode) {
  pvb2_pool2d_desc pd;
  memset(&pd, 0, sizeof(pd));
  pd.kh = (int32_t)k[0];
  pd.kw = (int32_t)(k.size() > 1 ? k[1] : k[0]);
  pd.sh = s.empty() ? pd.kh : (int32_t)s[0];
  pd.sw = s.empty() ? pd.kw : (int32_t)(s.size() > 1 ? s[1] : s[0]);
  pd.ph = (int32_t)p[0];
  pd.pw = (int32_t)(p.size() > 1 ? p[1] : p[0]);
  pd.dh = d.empty() ? 1 : (int32_t)d[0];
  pd.dw = d.empty() ? 1 : (int32_t)(d.size() > 1 ? d[1] : d[0]);
  pd.ceil_mode = ceil_mode ? 1 : 0;
  return pd;
}

static at::Tensor as4d(const at::Tensor& t) { return t.dim() == 3 ? t.unsqueeze(0) : t; }

// max_pool2d_with_indices.out (forward of max_pool2d_cls, vision_ops.cpp:353-410)
static std::tuple<at::Tensor&, at::Tensor&> max_pool2d_with_indices_out(const at::Tensor& self, at::IntArrayRef k,
                                                                         at::IntArrayRef s, at::IntArrayRef p,
                                                                         at::IntArrayRef d, bool ceil_mode,
                                                                         at::Tensor& out, at::Tensor& indices) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("max_pool2d_with_indices", dev);
  if (out.numel() == 0) return {out, indices};
  pvb2_pool2d_desc pd = pool_desc(k, s, p, d, ceil_mode);
  at::Tensor x = as4d(contiguous(self));
  at::Tensor o = out.is_contiguous() ? out : empty(out.sizes(), at::kFloat, dev);
  at::Tensor ind = indices.is_contiguous() ? indices : empty(indices.sizes(), at::kLong, dev);
  pvb2_tensor xd = desc(x), od = desc(as4d(o));
  OCL_CHECK(pvb2_max_pool2d_fwd(&pd, &xd, &od, ind.data_ptr<int64_t>(), stream_for(dev)));
  write_back(out, o);
  write_back(indices, ind);
  return {out, indices};
}

// max_pool2d_with_indices_backward.grad_input (max_pool2d_cls backward, vision_ops.cpp:411-438)
static at::Tensor& max_pool2d_with_indices_backward_out(const at::Tensor& grad_output, const at::Tensor& self,
                                                        at::IntArrayRef k, at::IntArrayRef s, at::IntArrayRef p,
                                                        at::IntArrayRef d, bool ceil_mode, const at::Tensor& indices,
                                                        at::Tensor& grad_input) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("max_pool2d_with_indices_backward", dev);
  if (grad_input.numel() == 0) return grad_input;
  pvb2_pool2d_desc pd = pool_desc(k, s, p, d, ceil_mode);
  at::Tensor gy = as4d(contiguous(grad_output)), ind = contiguous(indices);
  at::Tensor gi = grad_input.is_contiguous() ? grad_input : empty(grad_input.sizes(), at::kFloat, dev);
  pvb2_tensor gyd = desc(gy), gid = desc(as4d(gi));
  OCL_CHECK(pvb2_max_pool2d_bwd(&pd, &gyd, ind.data_ptr<int64_t>(), &gid, stream_for(dev)));
  write_back(grad_input, gi);
  return grad_input;
}

// avg_pool2d.out / avg_pool2d_backward.grad_input, vision_ops.cpp:448-511
static at::Tensor& avg_pool2d_out(const at::Tensor& self, at::IntArrayRef k, at::IntArrayRef s, at::IntArrayRef p,
                                  bool ceil_mode, bool count_include_pad, std::optional<int64_t> divisor_override,
                                  at::Tensor& out) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("avg_pool2d", dev);
  if (out.numel() == 0) return out;
  pvb2_pool2d_desc pd = pool_desc(k, s, p, {}, ceil_mode);
  pd.count_include_pad = count_include_pad ? 1 : 0;
  pd.divisor_override = divisor_override.has_value() ? (int32_t)*divisor_override : 0;
  at::Tensor x = as4d(contiguous(self));
  at::Tensor o = out.is_contiguous() ? out : empty(out.sizes(), at::kFloat, dev);
  pvb2_tensor xd = desc(x), od = desc(as4d(o));
  OCL_CHECK(pvb2_avg_pool2d_fwd(&pd, &xd, &od, stream_for(dev)));
  write_back(out, o);
  return out;
}

static at::Tensor& avg_pool2d_backward_out(const at::Tensor& grad_output, const at::Tensor& self, at::IntArrayRef k,
                                           at::IntArrayRef s, at::IntArrayRef p, bool ceil_mode,
                                           bool count_include_pad, std::optional<int64_t> divisor_override,
                                           at::Tensor& grad_input) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("avg_pool2d_backward", dev);
  if (grad_input.numel() == 0) return grad_input;
  pvb2_pool2d_desc pd = pool_desc(k, s, p, {}, ceil_mode);
  pd.count_include_pad = count_include_pad ? 1 : 0;
  pd.divisor_override = divisor_override.has_value() ? (int32_t)*divisor_override : 0;
  at::Tensor gy = as4d(contiguous(grad_output));
  at::Tensor gi = grad_input.is_contiguous() ? grad_input : empty(grad_input.sizes(), at::kFloat, dev);
  pvb2_tensor gyd = desc(gy), gid = desc(as4d(gi));
  OCL_CHECK(pvb2_avg_pool2d_bwd(&pd, &gyd, &gid, stream_for(dev)));
  write_back(grad_input, gi);
  return grad_input;
}

// _adaptive_avg_pool2d / _backward, vision_ops.cpp:188-241
static at::Tensor adaptive_avg_pool2d(const at::Tensor& self, at::IntArrayRef output_size) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("_adaptive_avg_pool2d", dev);
  at::Tensor x = as4d(contiguous(self));
  std::vector<int64_t> osz(self.sizes().begin(), self.sizes().end());
  osz[osz.size() - 2] = output_size[0];
  osz[osz.size() - 1] = output_size[1];
  at::Tensor y = empty(osz, at::kFloat, dev);
  if (y.numel() == 0) return y;
  pvb2_tensor xd = desc(x), yd = desc(as4d(y));
  OCL_CHECK(pvb2_adaptive_avg_pool2d_fwd(&xd, &yd, stream_for(dev)));
  return y;
}

static at::Tensor adaptive_avg_pool2d_backward(const at::Tensor& grad_output, const at::Tensor& self) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("_adaptive_avg_pool2d_backward", dev);
  at::Tensor gy = as4d(contiguous(grad_output));
  at::Tensor gx = empty(self.sizes(), at::kFloat, dev);
  if (gx.numel() == 0) return gx;
  pvb2_tensor gyd = desc(gy), gxd = desc(as4d(gx));
  OCL_CHECK(pvb2_adaptive_avg_pool2d_bwd(&gyd, &gxd, stream_for(dev)));
  return gx;
}

// ======================================================= softmax / loss
static void split_dim(const at::Tensor& t, int64_t dim, int64_t& outer, int64_t& D, int64_t& inner) {
  const int64_t d = c10::maybe_wrap_dim(dim, std::max<int64_t>(t.dim(), 1));
  outer = 1;
  inner = 1;
  D = t.dim() ? t.size(d) : 1;
  for (int64_t i = 0; i < d; ++i) outer *= t.size(i);
  for (int64_t i = d + 1; i < t.dim(); ++i) inner *= t.size(i);
}

// _log_softmax.out / _softmax.out, loss_ops.cpp:137-175
static at::Tensor& softmax_out_impl(bool log, const at::Tensor& self, int64_t dim, at::Tensor& out) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP(log ? "_log_softmax" : "_softmax", dev);
  if (out.numel() == 0) return out;
  TORCH_CHECK(self.scalar_type() == at::kFloat, "ocl softmax: float32 only");
  at::Tensor x = contiguous(self);
  at::Tensor o = out.is_contiguous() ? out : empty(out.sizes(), at::kFloat, dev);
  int64_t outer, D, inner;
  split_dim(x, dim, outer, D, inner);
  OCL_CHECK(pvb2_softmax_fwd(log ? 1 : 0, x.data_ptr<float>(), o.data_ptr<float>(), outer, D, inner, stream_for(dev)));
  write_back(out, o);
  return out;
}
static at::Tensor& log_softmax_out(const at::Tensor& self, int64_t dim, bool half_to_float, at::Tensor& out) {
  return softmax_out_impl(true, self, dim, out);
}
static at::Tensor& softmax_out(const at::Tensor& self, int64_t dim, bool half_to_float, at::Tensor& out) {
  return softmax_out_impl(false, self, dim, out);
}

// _log_softmax_backward_data.out / _softmax_backward_data.out, loss_ops.cpp:177-213
static at::Tensor& softmax_bwd_impl(bool log, const at::Tensor& grad_output, const at::Tensor& output, int64_t dim,
                                    at::Tensor& out) {
  const int dev = output.device().index();
  DeviceScope scope(dev);
  OCL_OP(log ? "_log_softmax_backward" : "_softmax_backward", dev);
  if (out.numel() == 0) return out;
  at::Tensor gy = contiguous(grad_output), y = contiguous(output);
  at::Tensor o = out.is_contiguous() ? out : empty(out.sizes(), at::kFloat, dev);
  int64_t outer, D, inner;
  split_dim(y, dim, outer, D, inner);
  OCL_CHECK(pvb2_softmax_bwd(log ? 1 : 0, gy.data_ptr<float>(), y.data_ptr<float>(), o.data_ptr<float>(), outer, D,
                             inner, stream_for(dev)));
  write_back(out, o);
  return out;
}
static at::Tensor& log_softmax_backward_out(const at::Tensor& grad_output, const at::Tensor& output, int64_t dim,
                                            at::ScalarType input_dtype, at::Tensor& out) {
  return softmax_bwd_impl(true, grad_output, output, dim, out);
}
static at::Tensor& softmax_backward_out(const at::Tensor& grad_output, const at::Tensor& output, int64_t dim,
                                        at::ScalarType input_dtype, at::Tensor& out) {
  return softmax_bwd_impl(false, grad_output, output, dim, out);
}

// nll_loss_forward.output, loss_ops.cpp:23-44
static std::tuple<at::Tensor&, at::Tensor&> nll_loss_forward_out(const at::Tensor& self, const at::Tensor& target,
                                                                 const std::optional<at::Tensor>& weight,
                                                                 int64_t reduction, int64_t ignore_index,
                                                                 at::Tensor& output, at::Tensor& total_weight) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("nll_loss_forward", dev);
  at::Tensor x = contiguous(self), t = contiguous(target);
  const int64_t N = x.dim() == 1 ? 1 : x.size(0), C = x.size(-1);
  at::Tensor w;
  if (weight.has_value() && weight->defined()) w = contiguous(*weight);
  at::Tensor o = output.is_contiguous() ? output : empty(output.sizes(), at::kFloat, dev);
  OCL_CHECK(pvb2_nll_loss_fwd(x.data_ptr<float>(), t.data_ptr<int64_t>(), w.defined() ? w.data_ptr<float>() : nullptr,
                              N, C, (int)reduction, ignore_index, o.data_ptr<float>(),
                              total_weight.data_ptr<float>(), stream_for(dev)));
  write_back(output, o);
  return {output, total_weight};
}

// nll_loss_backward.grad_input, loss_ops.cpp:46-65
static at::Tensor& nll_loss_backward_out(const at::Tensor& grad_output, const at::Tensor& self,
                                         const at::Tensor& target, const std::optional<at::Tensor>& weight,
                                         int64_t reduction, int64_t ignore_index, const at::Tensor& total_weight,
                                         at::Tensor& grad_input) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("nll_loss_backward", dev);
  at::Tensor t = contiguous(target), go = contiguous(grad_output);
  const int64_t N = self.dim() == 1 ? 1 : self.size(0), C = self.size(-1);
  at::Tensor w;
  if (weight.has_value() && weight->defined()) w = contiguous(*weight);
  at::Tensor gi = grad_input.is_contiguous() ? grad_input : empty(grad_input.sizes(), at::kFloat, dev);
  OCL_CHECK(pvb2_nll_loss_bwd(go.data_ptr<float>(), t.data_ptr<int64_t>(), w.defined() ? w.data_ptr<float>() : nullptr,
                              total_weight.data_ptr<float>(), N, C, (int)reduction, ignore_index,
                              gi.data_ptr<float>(), stream_for(dev)));
  write_back(grad_input, gi);
  return grad_input;
}

// ================================================================ random
// bernoulli_/normal_/uniform_, random_ops.cpp:37-67
static at::Tensor& philox_fill(at::Tensor& self, int dist, double p0, double p1,
                               const std::optional<at::Generator>& gen, const char* name) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP(name, dev);
  if (self.numel() == 0) return self;
  auto so = philox_reserve(gen, dev, self.numel());
  pvb2_tensor d = desc(self);
  OCL_CHECK(pvb2_philox_fill(dist, &d, so.first, so.second, p0, p1, stream_for(dev)));
  return self;
}
static at::Tensor& uniform_(at::Tensor& self, double from, double to, std::optional<at::Generator> gen) {
  return philox_fill(self, PVB2_RNG_UNIFORM, from, to, gen, "uniform_");
}
static at::Tensor& normal_(at::Tensor& self, double mean, double std, std::optional<at::Generator> gen) {
  return philox_fill(self, PVB2_RNG_NORMAL, mean, std, gen, "normal_");
}
static at::Tensor& bernoulli_(at::Tensor& self, double p, std::optional<at::Generator> gen) {
  return philox_fill(self, PVB2_RNG_BERNOULLI, p, 0, gen, "bernoulli_");
}

// native_dropout / native_dropout_backward, random_ops.cpp:69-105
static std::tuple<at::Tensor, at::Tensor> native_dropout(const at::Tensor& input, double p, std::optional<bool> train) {
  const int dev = input.device().index();
  DeviceScope scope(dev);
  OCL_OP("native_dropout", dev);
  at::Tensor x = contiguous(input);
  at::Tensor y = empty(x.sizes(), x.scalar_type(), dev);
  at::Tensor mask = empty(x.sizes(), at::kBool, dev);
  if (!train.value_or(true) || p == 0.0) {
    y.copy_(x);
    mask.fill_(true);
    return {y, mask};
  }
  TORCH_CHECK(x.scalar_type() == at::kFloat, "ocl dropout: float32 only");
  auto so = philox_reserve(std::nullopt, dev, x.numel());
  OCL_CHECK(pvb2_dropout_fwd(x.data_ptr<float>(), y.data_ptr<float>(), (uint8_t*)mask.data_ptr(), x.numel(), p,
                             so.first, so.second, stream_for(dev)));
  return {y, mask};
}

static at::Tensor native_dropout_backward(const at::Tensor& grad_output, const at::Tensor& mask, double scale) {
  const int dev = grad_output.device().index();
  DeviceScope scope(dev);
  OCL_OP("native_dropout_backward", dev);
  at::Tensor gy = contiguous(grad_output), m = contiguous(mask);
  at::Tensor gx = empty(gy.sizes(), gy.scalar_type(), dev);
  OCL_CHECK(pvb2_dropout_bwd(gy.data_ptr<float>(), (const uint8_t*)m.data_ptr(), gx.data_ptr<float>(), gy.numel(),
                             scale, stream_for(dev)));
  return gx;
}

// ------------------------------------------------------------ upsample
// upsample_nearest2d / _upsample_nearest_exact2d / upsample_bilinear2d and
// their backward passes; the reference had no device kernel for them (its
// CPU fallback ran them, tensor_ops.cpp:423-429).  Scales follow torch's fp32
// rules (area_pixel_compute_scale / compute_scales_value).
static float up_scale(int64_t in, int64_t out, bool align, std::optional<double> scale, bool linear) {
  if (linear && align) return out > 1 ? (float)(in - 1) / (float)(out - 1) : 0.f;
  return (scale.has_value() && *scale > 0.) ? (float)(1.0 / *scale) : (float)in / (float)out;
}

static at::Tensor& upsample_fwd(const char* name, int mode, const at::Tensor& self, at::IntArrayRef output_size,
                                bool align, std::optional<double> sh, std::optional<double> sw, at::Tensor& out) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP(name, dev);
  TORCH_CHECK(self.dim() == 4 && output_size.size() == 2, name, ": 4-D input and 2 output sizes expected");
  TORCH_CHECK(self.scalar_type() == at::kFloat, name, ": only float32 is supported");
  const std::vector<int64_t> osz = {self.size(0), self.size(1), output_size[0], output_size[1]};
  if (out.sizes() != c10::IntArrayRef(osz)) out.resize_(osz);
  if (out.numel() == 0) return out;
  const bool lin = mode == PVB2_UPSAMPLE_BILINEAR;
  const float fh = up_scale(self.size(2), output_size[0], align, sh, lin);
  const float fw = up_scale(self.size(3), output_size[1], align, sw, lin);
  at::Tensor x = contiguous(self);
  at::Tensor o = out.is_contiguous() ? out : empty(osz, at::kFloat, dev);
  pvb2_tensor xd = desc(x), od = desc(o);
  OCL_CHECK(pvb2_upsample2d_fwd(mode, align ? 1 : 0, fh, fw, &xd, &od, stream_for(dev)));
  write_back(out, o);
  return out;
}

static at::Tensor& upsample_bwd(const char* name, int mode, const at::Tensor& grad_output, at::IntArrayRef output_size,
                                at::IntArrayRef input_size, bool align, std::optional<double> sh,
                                std::optional<double> sw, at::Tensor& grad_input) {
  const int dev = grad_output.device().index();
  DeviceScope scope(dev);
  OCL_OP(name, dev);
  TORCH_CHECK(input_size.size() == 4 && output_size.size() == 2, name, ": 4 input and 2 output sizes expected");
  if (grad_input.sizes() != input_size) grad_input.resize_(input_size);
  if (grad_input.numel() == 0) return grad_input;
  const bool lin = mode == PVB2_UPSAMPLE_BILINEAR;
  const float fh = up_scale(input_size[2], output_size[0], align, sh, lin);
  const float fw = up_scale(input_size[3], output_size[1], align, sw, lin);
  at::Tensor gy = contiguous(grad_output);
  at::Tensor gi = grad_input.is_contiguous() ? grad_input : empty(input_size, at::kFloat, dev);
  pvb2_tensor gyd = desc(gy), gid = desc(gi);
  OCL_CHECK(pvb2_upsample2d_bwd(mode, align ? 1 : 0, fh, fw, &gyd, &gid, stream_for(dev)));
  write_back(grad_input, gi);
  return grad_input;
}

static at::Tensor& upsample_nearest2d_out(const at::Tensor& self, at::IntArrayRef osz, std::optional<double> sh,
                                          std::optional<double> sw, at::Tensor& out) {
  return upsample_fwd("upsample_nearest2d", PVB2_UPSAMPLE_NEAREST, self, osz, false, sh, sw, out);
}
static at::Tensor& upsample_nearest2d_backward_out(const at::Tensor& gy, at::IntArrayRef osz, at::IntArrayRef isz,
                                                   std::optional<double> sh, std::optional<double> sw,
                                                   at::Tensor& gi) {
  return upsample_bwd("upsample_nearest2d_backward", PVB2_UPSAMPLE_NEAREST, gy, osz, isz, false, sh, sw, gi);
}
static at::Tensor& upsample_nearest_exact2d_out(const at::Tensor& self, at::IntArrayRef osz, std::optional<double> sh,
                                                std::optional<double> sw, at::Tensor& out) {
  return upsample_fwd("_upsample_nearest_exact2d", PVB2_UPSAMPLE_NEAREST_EXACT, self, osz, false, sh, sw, out);
}
static at::Tensor& upsample_nearest_exact2d_backward_out(const at::Tensor& gy, at::IntArrayRef osz,
                                                         at::IntArrayRef isz, std::optional<double> sh,
                                                         std::optional<double> sw, at::Tensor& gi) {
  return upsample_bwd("_upsample_nearest_exact2d_backward", PVB2_UPSAMPLE_NEAREST_EXACT, gy, osz, isz, false, sh, sw,
                      gi);
}
static at::Tensor& upsample_bilinear2d_out(const at::Tensor& self, at::IntArrayRef osz, bool align,
                                           std::optional<double> sh, std::optional<double> sw, at::Tensor& out) {
  return upsample_fwd("upsample_bilinear2d", PVB2_UPSAMPLE_BILINEAR, self, osz, align, sh, sw, out);
}
static at::Tensor& upsample_bilinear2d_backward_out(const at::Tensor& gy, at::IntArrayRef osz, at::IntArrayRef isz,
                                                    bool align, std::optional<double> sh, std::optional<double> sw,
                                                    at::Tensor& gi) {
  return upsample_bwd("upsample_bilinear2d_backward", PVB2_UPSAMPLE_BILINEAR, gy, osz, isz, align, sh, sw, gi);
}

// ------------------------------------------------------------ MSE / BCE
// mse_loss and binary_cross_entropy (no reference kernel; its CPU fallback
// ran them) composed from this backend's own pointwise and reduction kernels.
// Reduction codes: 0 none, 1 mean, 2 sum.  BCE clamps each log term at -100
// like the CPU kernel.
static at::Tensor reduce_loss(const at::Tensor& l, int64_t reduction) {
  if (reduction == 1) return at::mean(l);
  if (reduction == 2) return at::sum(l);
  return l;
}

static at::Tensor& put(at::Tensor& out, const at::Tensor& v) {
  if (out.sizes() != v.sizes()) out.resize_(v.sizes());
  out.copy_(v);
  return out;
}

static at::Tensor& mse_loss_out(const at::Tensor& self, const at::Tensor& target, int64_t reduction, at::Tensor& out) {
  OCL_OP("mse_loss", self.device().index());
  const at::Tensor d = at::sub(self, target);
  return put(out, reduce_loss(at::mul(d, d), reduction));
}

static at::Tensor mse_loss_backward_fn(const at::Tensor& gy, const at::Tensor& self, const at::Tensor& target,
                                       int64_t reduction) {
  OCL_OP("mse_loss_backward", self.device().index());
  const double norm = reduction == 1 ? 2.0 / (double)std::max<int64_t>(self.numel(), 1) : 2.0;
  return at::mul(at::mul(at::sub(self, target), norm), gy);
}

static at::Tensor& mse_loss_backward_out(const at::Tensor& gy, const at::Tensor& self, const at::Tensor& target,
                                         int64_t reduction, at::Tensor& grad_input) {
  return put(grad_input, mse_loss_backward_fn(gy, self, target, reduction));
}

static at::Tensor binary_cross_entropy_fn(const at::Tensor& self, const at::Tensor& target,
                                          const std::optional<at::Tensor>& weight, int64_t reduction) {
  OCL_OP("binary_cross_entropy", self.device().index());
  const at::Tensor lx = at::clamp_min(at::log(self), -100.0);
  const at::Tensor l1x = at::clamp_min(at::log(at::rsub(self, 1.0)), -100.0);
  // -(t*log x + (1-t)*log(1-x)) = (t - 1)*log(1-x) - t*log x
  at::Tensor l = at::sub(at::mul(at::sub(target, 1.0), l1x), at::mul(target, lx));
  if (weight.has_value() && weight->defined()) l = at::mul(l, *weight);
  return reduce_loss(l, reduction);
}

static at::Tensor& binary_cross_entropy_out(const at::Tensor& self, const at::Tensor& target,
                                            const std::optional<at::Tensor>& weight, int64_t reduction,
                                            at::Tensor& out) {
  return put(out, binary_cross_entropy_fn(self, target, weight, reduction));
}

static at::Tensor binary_cross_entropy_backward_fn(const at::Tensor& gy, const at::Tensor& self,
                                                   const at::Tensor& target, const std::optional<at::Tensor>& weight,
                                                   int64_t reduction) {
  OCL_OP("binary_cross_entropy_backward", self.device().index());
  // (x - t) / max((1 - x) * x, eps) * gy, eps = 1e-12
  const at::Tensor den = at::clamp_min(at::mul(at::rsub(self, 1.0), self), 1e-12);
  at::Tensor g = at::mul(at::div(at::sub(self, target), den), gy);
  if (weight.has_value() && weight->defined()) g = at::mul(g, *weight);
  if (reduction == 1) g = at::div(g, (double)std::max<int64_t>(self.numel(), 1));
  return g;
}

static at::Tensor& binary_cross_entropy_backward_out(const at::Tensor& gy, const at::Tensor& self,
                                                     const at::Tensor& target, const std::optional<at::Tensor>& weight,
                                                     int64_t reduction, at::Tensor& grad_input) {
  return put(grad_input, binary_cross_entropy_backward_fn(gy, self, target, weight, reduction));
}

}  // namespace ocl

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  using namespace ocl;
  m.impl("convolution_overrideable", &convolution);
  m.impl("convolution_backward_overrideable", &convolution_backward);
  m.impl("mm.out", &mm_out);
  m.impl("bmm.out", &bmm_out);
  m.impl("addmm.out", &addmm_out);
  m.impl("baddbmm.out", &baddbmm_out);
  m.impl("native_batch_norm", &native_batch_norm);
  m.impl("native_batch_norm_backward", &native_batch_norm_backward);
  m.impl("native_layer_norm", &native_layer_norm);
  m.impl("native_layer_norm_backward", &native_layer_norm_backward);
  m.impl("max_pool2d_with_indices.out", &max_pool2d_with_indices_out);
  m.impl("max_pool2d_with_indices_backward.grad_input", &max_pool2d_with_indices_backward_out);
  m.impl("avg_pool2d.out", &avg_pool2d_out);
  m.impl("avg_pool2d_backward.grad_input", &avg_pool2d_backward_out);
  m.impl("_adaptive_avg_pool2d", &adaptive_avg_pool2d);
  m.impl("_adaptive_avg_pool2d_backward", &adaptive_avg_pool2d_backward);
  m.impl("_log_softmax.out", &log_softmax_out);
  m.impl("_softmax.out", &softmax_out);
  m.impl("_log_softmax_backward_data.out", &log_softmax_backward_out);
  m.impl("_softmax_backward_data.out", &softmax_backward_out);
  m.impl("nll_loss_forward.output", &nll_loss_forward_out);
  m.impl("nll_loss_backward.grad_input", &nll_loss_backward_out);
  m.impl("uniform_", &uniform_);
  m.impl("normal_", &normal_);
  m.impl("bernoulli_.float", &bernoulli_);
  m.impl("native_dropout", &native_dropout);
  m.impl("native_dropout_backward", &native_dropout_backward);
  m.impl("upsample_nearest2d.out", &upsample_nearest2d_out);
  m.impl("upsample_nearest2d_backward.grad_input", &upsample_nearest2d_backward_out);
  m.impl("_upsample_nearest_exact2d.out", &upsample_nearest_exact2d_out);
  m.impl("_upsample_nearest_exact2d_backward.grad_input", &upsample_nearest_exact2d_backward_out);
  m.impl("upsample_bilinear2d.out", &upsample_bilinear2d_out);
  m.impl("upsample_bilinear2d_backward.grad_input", &upsample_bilinear2d_backward_out);
  m.impl("mse_loss.out", &mse_loss_out);
  m.impl("mse_loss_backward", &mse_loss_backward_fn);
  m.impl("mse_loss_backward.grad_input", &mse_loss_backward_out);
  m.impl("binary_cross_entropy", &binary_cross_entropy_fn);
  m.impl("binary_cross_entropy.out", &binary_cross_entropy_out);
  m.impl("binary_cross_entropy_backward", &binary_cross_entropy_backward_fn);
  m.impl("binary_cross_entropy_backward.grad_input", &binary_cross_entropy_backward_out);
}
