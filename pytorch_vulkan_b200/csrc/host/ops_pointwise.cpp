// Pointwise, reduction, cat/where and multi-tensor (_foreach_*, _fused_sgd_)
// ops of the `ocl` device.
//
// Mirrors the registrations of src/pointwise_ops.cpp:1556-1648 (structured
// `.out` kernels; torch's generated wrappers provide the functional and
// in-place variants) and adds the multi-tensor kernels that the reference
// lacked (its optimizer step ran one launch per tensor).
#include "ocl.h"

namespace ocl {

std::pair<uint64_t, uint64_t> philox_reserve(const std::optional<at::Generator>& gen, int device, int64_t n);

static double sc(const at::Scalar& s) { return s.isBoolean() ? (s.toBool() ? 1.0 : 0.0) : s.toDouble(); }

static void check_dev(const at::Tensor& t, int dev, const char* op) {
  TORCH_CHECK(is_cpu_scalar(t) || (is_ocl(t) && t.device().index() == dev), "ocl: ", op,
              ": expected all tensors on ocl:", dev, ", got ", t.device());
}

// ------------------------------------------------------------------ unary
static at::Tensor& unary_out(int op, const at::Tensor& x, at::Tensor& out, double p0 = 0, double p1 = 0,
                             const char* name = "unary") {
  const int dev = out.device().index();
  check_dev(x, dev, name);
  DeviceScope scope(dev);
  OCL_OP(name, dev);
  if (out.numel() == 0) return out;
  pvb2_tensor o = desc(out), a = desc_expanded(x, out.sizes());
  int cd = compute_code(out.scalar_type());
  if (at::isFloatingType(x.scalar_type()) && !at::isFloatingType(out.scalar_type())) cd = compute_code(x.scalar_type());
  OCL_CHECK(pvb2_unary(op, &o, &a, p0, p1, cd, stream_for(dev)));
  return out;
}

static at::Tensor unary_new(int op, const at::Tensor& x, double p0 = 0, double p1 = 0, const char* name = "unary") {
  at::Tensor out = empty(x.sizes(), x.scalar_type(), x.device().index());
  unary_out(op, x, out, p0, p1, name);
  return out;
}

// ----------------------------------------------------------------- binary
static at::Tensor& binary_out(int op, const at::Tensor& a, const at::Tensor& b, at::Tensor& out, double p0, double p1,
                              int compute, const char* name) {
  const int dev = out.device().index();
  check_dev(a, dev, name);
  check_dev(b, dev, name);
  DeviceScope scope(dev);
  OCL_OP(name, dev);
  if (out.numel() == 0) return out;
  pvb2_stream st = stream_for(dev);
  pvb2_tensor o = desc(out);
  const bool as = is_cpu_scalar(a), bs = is_cpu_scalar(b);
  if (bs && !as) {
    pvb2_tensor x = desc_expanded(a, out.sizes());
    OCL_CHECK(pvb2_binary_scalar(op, &o, &x, sc(b.item()), 0, p0, p1, compute, st));
  } else if (as && !bs) {
    pvb2_tensor y = desc_expanded(b, out.sizes());
    OCL_CHECK(pvb2_binary_scalar(op, &o, &y, sc(a.item()), 1, p0, p1, compute, st));
  } else if (as && bs) {
    // both host scalars: put one on the device
    at::Tensor ad = empty({}, a.scalar_type(), dev);
    copy_into(ad, a, false);
    pvb2_tensor x = desc_expanded(ad, out.sizes());
    OCL_CHECK(pvb2_binary_scalar(op, &o, &x, sc(b.item()), 0, p0, p1, compute, st));
  } else {
    pvb2_tensor x = desc_expanded(a, out.sizes()), y = desc_expanded(b, out.sizes());
    OCL_CHECK(pvb2_binary(op, &o, &x, &y, p0, p1, compute, st));
  }
  return out;
}

static int arith_compute(const at::Tensor& out) { return compute_code(out.scalar_type()); }

static int common_compute(const at::Tensor& a, const at::Tensor& b) {
  return compute_code(at::result_type(a, b));
}

#define BINARY_OUT(fname, OP)                                                                               \
  static at::Tensor& fname(const at::Tensor& self, const at::Tensor& other, at::Tensor& out) {              \
    return binary_out(OP, self, other, out, 1.0, 0.0, arith_compute(out), #fname);                          \
  }

// add.out / sub.out: pointwise_ops.cpp:133-172, :206-210
// (or formed by a pending convolution dgrad whose result is one operand)
static at::Tensor& add_out(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha, at::Tensor& out) {
  if (fuse_deferred_dgrad_add(self, other, alpha, out)) return out;
  return binary_out(PVB2_BIN_ADD, self, other, out, sc(alpha), 0.0, arith_compute(out), "add.out");
}
// add_.Tensor: in place through add.out (out = self), or folded into a
// pending batch-norm pass when self is its output
static at::Tensor& add_inplace(at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
  if (fuse_deferred_add(self, other, alpha) || defer_counter_increment(self, other, alpha)) return self;
  TORCH_CHECK(at::can_cast(at::result_type(self, other), self.scalar_type()), "result type ",
              at::result_type(self, other), " can't be cast to the desired output type ", self.scalar_type());
  return add_out(self, other, alpha, self);
}
static at::Tensor& sub_out(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha, at::Tensor& out) {
  return binary_out(PVB2_BIN_SUB, self, other, out, sc(alpha), 0.0, arith_compute(out), "sub.out");
}
BINARY_OUT(mul_out, PVB2_BIN_MUL)      // :407-411
BINARY_OUT(maximum_out, PVB2_BIN_MAXIMUM)
BINARY_OUT(minimum_out, PVB2_BIN_MINIMUM)
BINARY_OUT(atan2_out, PVB2_BIN_ATAN2)
BINARY_OUT(pow_tt_out, PVB2_BIN_POW)
BINARY_OUT(remainder_out, PVB2_BIN_REMAINDER)
BINARY_OUT(bitwise_and_out, PVB2_BIN_BITWISE_AND)
BINARY_OUT(bitwise_or_out, PVB2_BIN_BITWISE_OR)
BINARY_OUT(bitwise_xor_out, PVB2_BIN_BITWISE_XOR)

// div.out / div.out_mode, :318-344
static at::Tensor& div_out(const at::Tensor& self, const at::Tensor& other, at::Tensor& out) {
  return binary_out(PVB2_BIN_DIV, self, other, out, 1.0, 0.0, arith_compute(out), "div.out");
}
static at::Tensor& div_out_mode(const at::Tensor& self, const at::Tensor& other,
                                std::optional<c10::string_view> mode, at::Tensor& out) {
  int op = PVB2_BIN_DIV;
  if (mode.has_value()) {
    if (*mode == "trunc") op = PVB2_BIN_DIV_TRUNC;
    else if (*mode == "floor") op = PVB2_BIN_DIV_FLOOR;
  }
  return binary_out(op, self, other, out, 1.0, 0.0, arith_compute(out), "div.out_mode");
}

#define COMPARE_OUT(fname, OP)                                                                             \
  static at::Tensor& fname##_tensor(const at::Tensor& self, const at::Tensor& other, at::Tensor& out) {    \
    return binary_out(OP, self, other, out, 0, 0, common_compute(self, other), #fname);                   \
  }                                                                                                        \
  static at::Tensor& fname##_scalar(const at::Tensor& self, const at::Scalar& other, at::Tensor& out) {    \
    at::Tensor o = at::scalar_tensor(other, at::TensorOptions().dtype(other.type()));                     \
    return binary_out(OP, self, o, out, 0, 0, compute_code(at::result_type(self, other)), #fname);       \
  }
COMPARE_OUT(eq, PVB2_BIN_EQ)
COMPARE_OUT(ne, PVB2_BIN_NE)
COMPARE_OUT(lt, PVB2_BIN_LT)
COMPARE_OUT(le, PVB2_BIN_LE)
COMPARE_OUT(gt, PVB2_BIN_GT)
COMPARE_OUT(ge, PVB2_BIN_GE)

// threshold_backward, :437-455:  grad_input = self <= threshold ? 0 : grad
static at::Tensor& threshold_backward_out(const at::Tensor& grad, const at::Tensor& self, const at::Scalar& threshold,
                                          at::Tensor& grad_input) {
  // ReLU's gradient: left pending for a following batch-norm backward
  if (!threshold.isComplex() && threshold.toDouble() == 0.0 && is_ocl(grad) && is_ocl(self) && is_ocl(grad_input) &&
      grad_input.sizes().equals(grad.sizes()) && defer_threshold_bwd(grad, self, grad_input, 1))
    return grad_input;
  return binary_out(PVB2_BIN_THRESHOLD_BWD, grad, self, grad_input, sc(threshold), 0, arith_compute(grad_input),
                    "threshold_backward");
}

// hardtanh / ReLU6, :559-603 (mask follows CPU: strictly inside (min, max))
static at::Tensor hardtanh(const at::Tensor& self, const at::Scalar& mn, const at::Scalar& mx) {
  return unary_new(PVB2_UN_HARDTANH, self, sc(mn), sc(mx), "hardtanh");
}
static bool is_relu6(const at::Scalar& mn, const at::Scalar& mx) {
  return !mn.isComplex() && !mx.isComplex() && mn.toDouble() == 0.0 && mx.toDouble() == 6.0;
}
static at::Tensor& hardtanh_(at::Tensor& self, const at::Scalar& mn, const at::Scalar& mx) {
  if (is_relu6(mn, mx) && fuse_deferred_act(self, 2)) return self;  // joined a pending batch-norm pass
  return unary_out(PVB2_UN_HARDTANH, self, self, sc(mn), sc(mx), "hardtanh_");
}
static at::Tensor& hardtanh_out(const at::Tensor& self, const at::Scalar& mn, const at::Scalar& mx, at::Tensor& out) {
  return unary_out(PVB2_UN_HARDTANH, self, out, sc(mn), sc(mx), "hardtanh.out");
}
static at::Tensor& hardtanh_backward_out(const at::Tensor& grad, const at::Tensor& self, const at::Scalar& mn,
                                         const at::Scalar& mx, at::Tensor& grad_input) {
  // ReLU6's gradient: left pending for a following batch-norm backward
  if (is_relu6(mn, mx) && is_ocl(grad) && is_ocl(self) && is_ocl(grad_input) &&
      grad_input.sizes().equals(grad.sizes()) && defer_threshold_bwd(grad, self, grad_input, 2))
    return grad_input;
  return binary_out(PVB2_BIN_HARDTANH_BWD, grad, self, grad_input, sc(mn), sc(mx), arith_compute(grad_input),
                    "hardtanh_backward");
}
static at::Tensor hardtanh_backward(const at::Tensor& grad, const at::Tensor& self, const at::Scalar& mn,
                                    const at::Scalar& mx) {
  at::Tensor gi = empty(grad.sizes(), grad.scalar_type(), grad.device().index());
  hardtanh_backward_out(grad, self, mn, mx, gi);
  return gi;
}

// relu / relu_, :55-113
static at::Tensor relu(const at::Tensor& self) { return unary_new(PVB2_UN_RELU, self, 0, 0, "relu"); }
static at::Tensor& relu_(at::Tensor& self) {
  if (fuse_deferred_act(self, 1)) return self;  // joined a pending batch-norm pass
  return unary_out(PVB2_UN_RELU, self, self, 0, 0, "relu_");
}

// gelu / gelu_backward, :1324-1393
static at::Tensor& gelu_out(const at::Tensor& self, c10::string_view approximate, at::Tensor& out) {
  return unary_out(approximate == "tanh" ? PVB2_UN_GELU_TANH : PVB2_UN_GELU_ERF, self, out, 0, 0, "gelu");
}
static at::Tensor& gelu_backward_out(const at::Tensor& grad, const at::Tensor& self, c10::string_view approximate,
                                     at::Tensor& grad_input) {
  return binary_out(approximate == "tanh" ? PVB2_BIN_GELU_TANH_BWD : PVB2_BIN_GELU_ERF_BWD, grad, self, grad_input, 0,
                    0, arith_compute(grad_input), "gelu_backward");
}

#define UNARY_OUT(fname, OP) \
  static at::Tensor& fname(const at::Tensor& self, at::Tensor& out) { return unary_out(OP, self, out, 0, 0, #fname); }
UNARY_OUT(exp_out, PVB2_UN_EXP)
UNARY_OUT(log_out, PVB2_UN_LOG)
UNARY_OUT(sqrt_out, PVB2_UN_SQRT)
UNARY_OUT(rsqrt_out, PVB2_UN_RSQRT)
UNARY_OUT(neg_out, PVB2_UN_NEG)
UNARY_OUT(abs_out, PVB2_UN_ABS)
UNARY_OUT(sigmoid_out, PVB2_UN_SIGMOID)
UNARY_OUT(tanh_out, PVB2_UN_TANH)
UNARY_OUT(reciprocal_out, PVB2_UN_RECIPROCAL)
UNARY_OUT(silu_out, PVB2_UN_SILU)
UNARY_OUT(hardsigmoid_out, PVB2_UN_HARDSIGMOID)
UNARY_OUT(hardswish_out, PVB2_UN_HARDSWISH)
UNARY_OUT(ceil_out, PVB2_UN_CEIL)
UNARY_OUT(floor_out, PVB2_UN_FLOOR)
UNARY_OUT(trunc_out, PVB2_UN_TRUNC)
UNARY_OUT(round_out, PVB2_UN_ROUND)
UNARY_OUT(atan_out, PVB2_UN_ATAN)
UNARY_OUT(sgn_out, PVB2_UN_SGN)
static at::Tensor& bitwise_not_out(const at::Tensor& self, at::Tensor& out) {
  return unary_out(self.scalar_type() == at::kBool ? PVB2_UN_LOGICAL_NOT : PVB2_UN_BITWISE_NOT, self, out, 0, 0,
                   "bitwise_not");
}
UNARY_OUT(logical_not_out, PVB2_UN_LOGICAL_NOT)
UNARY_OUT(isposinf_out, PVB2_UN_ISPOSINF)
UNARY_OUT(isneginf_out, PVB2_UN_ISNEGINF)
UNARY_OUT(sign_out, PVB2_UN_SGN)
static at::Tensor isnan(const at::Tensor& self) {
  at::Tensor out = empty(self.sizes(), at::kBool, self.device().index());
  return unary_out(PVB2_UN_ISNAN, self, out, 0, 0, "isnan");
}
static at::Tensor& logit_out(const at::Tensor& self, std::optional<double> eps, at::Tensor& out) {
  return unary_out(PVB2_UN_LOGIT, self, out, eps.has_value() ? *eps : -1.0, 0, "logit");
}
static at::Tensor logit(const at::Tensor& self, std::optional<double> eps) {
  at::Tensor out = empty(self.sizes(), self.scalar_type(), self.device().index());
  return logit_out(self, eps, out);
}
static at::Tensor& clamp_max_out(const at::Tensor& self, const at::Scalar& mx, at::Tensor& out) {
  return unary_out(PVB2_UN_CLAMP, self, out, at::isFloatingType(out.scalar_type()) ? -INFINITY : -9.2e18, sc(mx),
                   "clamp_max");
}

static at::Tensor abs_new(const at::Tensor& self) { return unary_new(PVB2_UN_ABS, self, 0, 0, "abs"); }
static at::Tensor& hardswish_(at::Tensor& self) { return unary_out(PVB2_UN_HARDSWISH, self, self, 0, 0, "hardswish_"); }
static at::Tensor hardswish(const at::Tensor& self) { return unary_new(PVB2_UN_HARDSWISH, self, 0, 0, "hardswish"); }

static at::Tensor& pow_ts_out(const at::Tensor& self, const at::Scalar& e, at::Tensor& out) {
  return unary_out(PVB2_UN_POW, self, out, sc(e), 0, "pow");
}
static at::Tensor& clamp_out(const at::Tensor& self, const std::optional<at::Scalar>& mn,
                             const std::optional<at::Scalar>& mx, at::Tensor& out) {
  const double lo = mn.has_value() ? sc(*mn) : -INFINITY;
  const double hi = mx.has_value() ? sc(*mx) : INFINITY;
  if (!at::isFloatingType(out.scalar_type())) {
    const double l2 = mn.has_value() ? lo : -9.2e18, h2 = mx.has_value() ? hi : 9.2e18;
    return unary_out(PVB2_UN_CLAMP, self, out, l2, h2, "clamp");
  }
  return unary_out(PVB2_UN_CLAMP, self, out, lo, hi, "clamp");
}
static at::Tensor& clamp_min_out(const at::Tensor& self, const at::Scalar& mn, at::Tensor& out) {
  return unary_out(PVB2_UN_CLAMP_MIN, self, out, sc(mn), 0, "clamp_min");
}
static at::Tensor& leaky_relu_out(const at::Tensor& self, const at::Scalar& slope, at::Tensor& out) {
  return unary_out(PVB2_UN_LEAKY_RELU, self, out, sc(slope), 0, "leaky_relu");
}

#define BWD_OUT(fname, OP)                                                                                  \
  static at::Tensor& fname(const at::Tensor& grad, const at::Tensor& x, at::Tensor& gi) {                   \
    return binary_out(OP, grad, x, gi, 0, 0, arith_compute(gi), #fname);                                    \
  }
BWD_OUT(sigmoid_backward_out, PVB2_BIN_SIGMOID_BWD)
BWD_OUT(tanh_backward_out, PVB2_BIN_TANH_BWD)
BWD_OUT(silu_backward_out, PVB2_BIN_SILU_BWD)
BWD_OUT(hardsigmoid_backward_out, PVB2_BIN_HARDSIGMOID_BWD)

static at::Tensor hardswish_backward(const at::Tensor& grad, const at::Tensor& self) {
  at::Tensor gi = empty(grad.sizes(), grad.scalar_type(), grad.device().index());
  return binary_out(PVB2_BIN_HARDSWISH_BWD, grad, self, gi, 0, 0, arith_compute(gi), "hardswish_backward");
}
static at::Tensor& leaky_relu_backward_out(const at::Tensor& grad, const at::Tensor& self, const at::Scalar& slope,
                                           bool self_is_result, at::Tensor& gi) {
  return binary_out(PVB2_BIN_LEAKY_RELU_BWD, grad, self, gi, sc(slope), 0, arith_compute(gi), "leaky_relu_backward");
}

// log_sigmoid: forward returns (out, buffer); the buffer is not needed here
static std::tuple<at::Tensor&, at::Tensor&> log_sigmoid_forward_out(const at::Tensor& self, at::Tensor& out,
                                                                    at::Tensor& buffer) {
  unary_out(PVB2_UN_LOG_SIGMOID, self, out, 0, 0, "log_sigmoid");
  return {out, buffer};
}
static std::tuple<at::Tensor, at::Tensor> log_sigmoid_forward(const at::Tensor& self) {
  at::Tensor out = unary_new(PVB2_UN_LOG_SIGMOID, self, 0, 0, "log_sigmoid");
  return {out, empty({0}, self.scalar_type(), self.device().index())};
}
static at::Tensor& log_sigmoid_backward_out(const at::Tensor& grad, const at::Tensor& self, const at::Tensor& buffer,
                                            at::Tensor& gi) {
  return binary_out(PVB2_BIN_LOG_SIGMOID_BWD, grad, self, gi, 0, 0, arith_compute(gi), "log_sigmoid_backward");
}
static at::Tensor log_sigmoid_backward(const at::Tensor& grad, const at::Tensor& self, const at::Tensor& buffer) {
  at::Tensor gi = empty(grad.sizes(), grad.scalar_type(), grad.device().index());
  return log_sigmoid_backward_out(grad, self, buffer, gi);
}

static at::Tensor& lerp_out(const at::Tensor& self, const at::Tensor& end, const at::Scalar& w, at::Tensor& out) {
  return binary_out(PVB2_BIN_LERP, self, end, out, sc(w), 0, arith_compute(out), "lerp");
}

// ---------------------------------------------------------------- ternary
static at::Tensor& ternary_out(int op, const at::Tensor& a, const at::Tensor& b, const at::Tensor& c, double p0,
                               at::Tensor& out, int compute, const char* name) {
  const int dev = out.device().index();
  DeviceScope scope(dev);
  OCL_OP(name, dev);
  if (out.numel() == 0) return out;
  auto up = [&](const at::Tensor& t) {
    if (is_ocl(t)) return t;
    at::Tensor d = empty(t.sizes(), t.scalar_type(), dev);
    copy_into(d, t, false);
    return d;
  };
  at::Tensor A = up(a), B = up(b), C = up(c);
  pvb2_tensor o = desc(out), x = desc_expanded(A, out.sizes()), y = desc_expanded(B, out.sizes()),
              z = desc_expanded(C, out.sizes());
  OCL_CHECK(pvb2_ternary(op, &o, &x, &y, &z, p0, compute, stream_for(dev)));
  return out;
}
// addcmul / addcdiv, :214-234, :414-434
static at::Tensor& addcmul_out(const at::Tensor& self, const at::Tensor& t1, const at::Tensor& t2,
                               const at::Scalar& value, at::Tensor& out) {
  return ternary_out(PVB2_TER_ADDCMUL, self, t1, t2, sc(value), out, arith_compute(out), "addcmul");
}
static at::Tensor& addcdiv_out(const at::Tensor& self, const at::Tensor& t1, const at::Tensor& t2,
                               const at::Scalar& value, at::Tensor& out) {
  return ternary_out(PVB2_TER_ADDCDIV, self, t1, t2, sc(value), out, arith_compute(out), "addcdiv");
}
static at::Tensor& where_out(const at::Tensor& cond, const at::Tensor& self, const at::Tensor& other, at::Tensor& out) {
  return ternary_out(PVB2_TER_WHERE, cond, self, other, 0, out, arith_compute(out), "where");
}
static at::Tensor where_self(const at::Tensor& cond, const at::Tensor& self, const at::Tensor& other) {
  auto sizes = at::infer_size(at::infer_size(cond.sizes(), self.sizes()), other.sizes());
  const int dev = is_ocl(cond) ? cond.device().index() : (is_ocl(self) ? self.device().index() : other.device().index());
  at::Tensor out = empty(sizes, at::result_type(self, other), dev);
  return where_out(cond, self, other, out);
}

// ------------------------------------------------------------- reductions
// red_op_out, :501-555
static at::Tensor& reduce_out(int op, const at::Tensor& self, at::OptionalIntArrayRef dims_opt, bool keepdim,
                              at::Tensor& out, bool mean, const char* name) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP(name, dev);
  const int64_t nd = self.dim();
  std::vector<bool> red(std::max<int64_t>(nd, 1), false);
  bool all = !dims_opt.has_value() || dims_opt->empty();
  if (!all)
    for (int64_t d : *dims_opt) red[c10::maybe_wrap_dim(d, nd)] = true;
  else
    for (int64_t d = 0; d < nd; ++d) red[d] = true;
  // out viewed with every reduced dim present as size 1
  std::vector<int64_t> osz, ost;
  int64_t count = 1;
  int k = 0;
  for (int64_t d = 0; d < nd; ++d) {
    if (red[d]) {
      count *= self.size(d);
      osz.push_back(1);
      ost.push_back(0);
      if (keepdim) ++k;
    } else {
      osz.push_back(self.size(d));
      ost.push_back(out.dim() > k ? out.stride(k) : 0);
      ++k;
    }
  }
  if (out.numel() == 0) return out;
  pvb2_tensor o = desc(out);
  o.ndim = (int32_t)nd;
  for (int64_t d = 0; d < nd; ++d) {
    o.sizes[d] = osz[d];
    o.strides[d] = ost[d];
  }
  pvb2_tensor in = desc(self);
  if (nd == 0) {  // 0-dim input: the reduction is a copy
    o = desc(out);
    OCL_CHECK(pvb2_copy(&o, &in, stream_for(dev)));
    return out;
  }
  int cd = compute_code(out.scalar_type());
  if (op == PVB2_RED_ARGMAX || op == PVB2_RED_ARGMIN) cd = compute_code(self.scalar_type());
  const double scale = mean ? (count ? 1.0 / (double)count : NAN) : 1.0;
  const size_t wsb = pvb2_reduce_workspace_size(op, &o, &in, cd);
  if (wsb == 0) {
    OCL_CHECK(pvb2_reduce(op, &o, &in, scale, cd, stream_for(dev)));
  } else {
    Workspace ws(wsb, dev);
    OCL_CHECK(pvb2_reduce_ws(op, &o, &in, scale, cd, ws.get(), ws.bytes, stream_for(dev)));
  }
  return out;
}

static at::Tensor& sum_out(const at::Tensor& self, at::OptionalIntArrayRef dim, bool keepdim,
                           std::optional<at::ScalarType> dtype, at::Tensor& out) {
  return reduce_out(PVB2_RED_SUM, self, dim, keepdim, out, false, "sum");
}
static at::Tensor& mean_out(const at::Tensor& self, at::OptionalIntArrayRef dim, bool keepdim,
                            std::optional<at::ScalarType> dtype, at::Tensor& out) {
  return reduce_out(PVB2_RED_SUM, self, dim, keepdim, out, true, "mean");
}
static at::Tensor& prod_out(const at::Tensor& self, int64_t dim, bool keepdim, std::optional<at::ScalarType> dtype,
                            at::Tensor& out) {
  std::vector<int64_t> d{dim};
  return reduce_out(PVB2_RED_PROD, self, d, keepdim, out, false, "prod");
}
static at::Tensor& amax_out(const at::Tensor& self, at::IntArrayRef dim, bool keepdim, at::Tensor& out) {
  return reduce_out(PVB2_RED_MAX, self, dim, keepdim, out, false, "amax");
}
static at::Tensor& amin_out(const at::Tensor& self, at::IntArrayRef dim, bool keepdim, at::Tensor& out) {
  return reduce_out(PVB2_RED_MIN, self, dim, keepdim, out, false, "amin");
}
static at::Tensor& argmax_out(const at::Tensor& self, std::optional<int64_t> dim, bool keepdim, at::Tensor& out) {
  if (dim.has_value()) {
    std::vector<int64_t> d{*dim};
    return reduce_out(PVB2_RED_ARGMAX, self, d, keepdim, out, false, "argmax");
  }
  return reduce_out(PVB2_RED_ARGMAX, self.reshape({-1}), std::nullopt, keepdim, out, false, "argmax");
}
static at::Tensor& argmin_out(const at::Tensor& self, std::optional<int64_t> dim, bool keepdim, at::Tensor& out) {
  if (dim.has_value()) {
    std::vector<int64_t> d{*dim};
    return reduce_out(PVB2_RED_ARGMIN, self, d, keepdim, out, false, "argmin");
  }
  return reduce_out(PVB2_RED_ARGMIN, self.reshape({-1}), std::nullopt, keepdim, out, false, "argmin");
}
static at::Tensor max_all(const at::Tensor& self) {
  TORCH_CHECK(self.numel() > 0, "max(): expected a non-empty tensor");
  at::Tensor out = empty({}, self.scalar_type(), self.device().index());
  return reduce_out(PVB2_RED_MAX, self, std::nullopt, false, out, false, "max");
}
static at::Tensor min_all(const at::Tensor& self) {
  TORCH_CHECK(self.numel() > 0, "min(): expected a non-empty tensor");
  at::Tensor out = empty({}, self.scalar_type(), self.device().index());
  return reduce_out(PVB2_RED_MIN, self, std::nullopt, false, out, false, "min");
}
// dot, :1200-ish (sum of products)
static at::Tensor dot(const at::Tensor& a, const at::Tensor& b) {
  TORCH_CHECK(a.dim() == 1 && b.dim() == 1 && a.numel() == b.numel(), "dot: 1-D tensors of equal length expected");
  at::Tensor prod = empty(a.sizes(), a.scalar_type(), a.device().index());
  binary_out(PVB2_BIN_MUL, a, b, prod, 1, 0, arith_compute(prod), "dot");
  at::Tensor out = empty({}, a.scalar_type(), a.device().index());
  return reduce_out(PVB2_RED_SUM, prod, std::nullopt, false, out, false, "dot");
}

// arange.start_out: out[i] = start + i*step (resized like the CPU kernel)
static at::Tensor& arange_out(const at::Scalar& start, const at::Scalar& end, const at::Scalar& step, at::Tensor& out) {
  const double s = start.toDouble(), e = end.toDouble(), st = step.toDouble();
  TORCH_CHECK(st != 0.0, "arange: step must be nonzero");
  int64_t n;
  if (at::isIntegralType(out.scalar_type(), true) && start.isIntegral(true) && end.isIntegral(true) && step.isIntegral(true)) {
    const int64_t a = start.toLong(), b = end.toLong(), c = step.toLong();
    n = (b - a + c - (c > 0 ? 1 : -1)) / c;
  } else {
    n = (int64_t)std::ceil((e - s) / st);
  }
  if (n < 0) n = 0;
  if (out.numel() != n) out.resize_({n});
  const int dev = out.device().index();
  DeviceScope scope(dev);
  OCL_OP("arange", dev);
  if (n == 0) return out;
  pvb2_tensor o = desc(out);
  OCL_CHECK(pvb2_arange(&o, s, st, stream_for(dev)));
  return out;
}

// all / any: min / max over the values taken as booleans
static at::Tensor& logical_reduce(bool all, const at::Tensor& self, at::OptionalIntArrayRef dims, bool keepdim,
                                  at::Tensor& out) {
  at::Tensor b = self;
  if (self.scalar_type() != at::kBool) {
    b = empty(self.sizes(), at::kBool, self.device().index());
    pvb2_tensor bd = desc(b), sd = desc(self);
    OCL_CHECK(pvb2_copy(&bd, &sd, stream_for(self.device().index())));
  }
  if (self.numel() == 0) return out.fill_(all);
  return reduce_out(all ? PVB2_RED_MIN : PVB2_RED_MAX, b, dims, keepdim, out, false, all ? "all" : "any");
}
static at::Tensor& all_dims_out(const at::Tensor& self, at::OptionalIntArrayRef dim, bool keepdim, at::Tensor& out) {
  return logical_reduce(true, self, dim, keepdim, out);
}
static at::Tensor& all_out(const at::Tensor& self, int64_t dim, bool keepdim, at::Tensor& out) {
  std::vector<int64_t> d{dim};
  return logical_reduce(true, self, d, keepdim, out);
}
static at::Tensor& all_all_out(const at::Tensor& self, at::Tensor& out) {
  return logical_reduce(true, self, std::nullopt, false, out);
}
static at::Tensor& any_dims_out(const at::Tensor& self, at::OptionalIntArrayRef dim, bool keepdim, at::Tensor& out) {
  return logical_reduce(false, self, dim, keepdim, out);
}
static at::Tensor& any_out(const at::Tensor& self, int64_t dim, bool keepdim, at::Tensor& out) {
  std::vector<int64_t> d{dim};
  return logical_reduce(false, self, d, keepdim, out);
}
static at::Tensor& any_all_out(const at::Tensor& self, at::Tensor& out) {
  return logical_reduce(false, self, std::nullopt, false, out);
}

// masked_select / nonzero (tensor_ops.cpp:303-356): compaction on the device;
// the one host read is the selected count, needed to size the output
static int64_t select_count(const pvb2_tensor& m, int dev, Workspace& ws, at::Tensor& total) {
  OCL_CHECK(pvb2_select_count(&m, ws.get(), ws.bytes, total.data_ptr<int64_t>(), stream_for(dev)));
  return total.item<int64_t>();
}
static at::Tensor masked_select(const at::Tensor& self, const at::Tensor& mask) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("masked_select", dev);
  auto sizes = at::infer_size(self.sizes(), mask.sizes());
  pvb2_tensor sd = desc_expanded(self, sizes), md = desc_expanded(mask, sizes);
  int64_t n = 1;
  for (auto v : sizes) n *= v;
  Workspace ws(pvb2_select_workspace_size(n), dev);
  at::Tensor total = empty({}, at::kLong, dev);
  const int64_t k = select_count(md, dev, ws, total);
  at::Tensor out = empty({k}, self.scalar_type(), dev);
  if (k) OCL_CHECK(pvb2_select_gather(&sd, &md, out.data_ptr(), ws.get(), stream_for(dev)));
  return out;
}
static at::Tensor nonzero(const at::Tensor& self) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("nonzero", dev);
  pvb2_tensor md = desc(self);
  Workspace ws(pvb2_select_workspace_size(self.numel()), dev);
  at::Tensor total = empty({}, at::kLong, dev);
  const int64_t k = select_count(md, dev, ws, total);
  at::Tensor out = empty({k, self.dim()}, at::kLong, dev);
  if (k && self.dim()) OCL_CHECK(pvb2_select_gather(nullptr, &md, out.data_ptr(), ws.get(), stream_for(dev)));
  return out;
}
// masked_fill_: self = mask ? value : self
static at::Tensor& masked_fill_tensor_(at::Tensor& self, const at::Tensor& mask, const at::Tensor& value) {
  const int dev = self.device().index();
  at::Tensor v = value;
  if (!is_ocl(v)) {
    v = empty({}, self.scalar_type(), dev);
    copy_into(v, value.to(self.scalar_type()), false);
  }
  return ternary_out(PVB2_TER_WHERE, mask, v, self, 0, self, arith_compute(self), "masked_fill_");
}
static at::Tensor& masked_fill_scalar_(at::Tensor& self, const at::Tensor& mask, const at::Scalar& value) {
  return masked_fill_tensor_(self, mask, at::scalar_tensor(value, at::TensorOptions().dtype(self.scalar_type())));
}

// index.Tensor_out (advanced indexing).  Same result layout as torch's
// AdvancedIndex: boolean masks become nonzero() coordinates (on the device),
// all index tensors broadcast to one shape; if the indexed dims are not
// adjacent they move to the front; the result is
// [dims before] + index shape + [dims after], read from src with the indexed
// dims' strides.  The gather runs on the device.
static at::Tensor& index_out(const at::Tensor& self, const c10::List<std::optional<at::Tensor>>& indices,
                             at::Tensor& out) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("index", dev);
  // 1. expand masks into per-dim long indices
  std::vector<at::Tensor> idx;  // one entry per dim of self (undefined = not indexed)
  for (size_t i = 0; i < indices.size(); ++i) {
    std::optional<at::Tensor> t = indices[i];
    if (!t.has_value() || !t->defined()) {
      idx.emplace_back();
      continue;
    }
    at::Tensor ti = *t;
    if (ti.scalar_type() == at::kBool || ti.scalar_type() == at::kByte) {
      const int64_t d0 = (int64_t)idx.size();
      TORCH_CHECK(d0 + ti.dim() <= self.dim(), "index: too many indices");
      for (int64_t j = 0; j < ti.dim(); ++j)
        TORCH_CHECK(ti.size(j) == self.size(d0 + j), "index: mask shape does not match the indexed tensor");
      at::Tensor nz = is_ocl(ti) ? ti.nonzero() : ti.nonzero().to(self.device());
      for (int64_t j = 0; j < ti.dim(); ++j) idx.push_back(nz.select(1, j));
    } else {
      TORCH_CHECK(ti.scalar_type() == at::kLong || ti.scalar_type() == at::kInt, "index: tensors must be long, int or bool");
      idx.push_back(is_ocl(ti) ? ti.to(at::kLong) : ti.to(self.device(), at::kLong));
    }
  }
  while ((int64_t)idx.size() < self.dim()) idx.emplace_back();
  // 2. broadcast the defined indices
  std::vector<int64_t> bshape;
  bool first = true;
  for (auto& t : idx)
    if (t.defined()) {
      bshape = first ? t.sizes().vec() : at::infer_size(bshape, t.sizes());
      first = false;
    }
  TORCH_CHECK(!first, "index: no index tensors");
  // 3. adjacency; move indexed dims to the front when they are not adjacent
  at::Tensor src = self;
  std::vector<int64_t> dims_idx;
  for (int64_t d = 0; d < self.dim(); ++d)
    if (idx[d].defined()) dims_idx.push_back(d);
  bool adjacent = true;
  for (size_t i = 1; i < dims_idx.size(); ++i) adjacent &= dims_idx[i] == dims_idx[i - 1] + 1;
  if (!adjacent) {
    std::vector<int64_t> perm;
    std::vector<at::Tensor> nidx;
    for (int64_t d : dims_idx) {
      perm.push_back(d);
      nidx.push_back(idx[d]);
    }
    for (int64_t d = 0; d < self.dim(); ++d)
      if (!idx[d].defined()) {
        perm.push_back(d);
        nidx.emplace_back();
      }
    src = self.permute(perm);
    idx = nidx;
    dims_idx.clear();
    for (size_t i = 0; i < nidx.size(); ++i)
      if (nidx[i].defined()) dims_idx.push_back((int64_t)i);
  }
  const int64_t d_first = dims_idx.front(), d_last = dims_idx.back();
  std::vector<int64_t> osz, ost;
  std::vector<int64_t> isz, istr;
  for (int64_t d = 0; d < d_first; ++d) {
    osz.push_back(src.size(d));
    ost.push_back(src.stride(d));
  }
  const int64_t idx_pos = (int64_t)osz.size();
  for (int64_t v : bshape) {
    osz.push_back(v);
    ost.push_back(0);
  }
  for (int64_t d = d_last + 1; d < src.dim(); ++d) {
    osz.push_back(src.size(d));
    ost.push_back(src.stride(d));
  }
  for (int64_t d : dims_idx) {
    isz.push_back(src.size(d));
    istr.push_back(src.stride(d));
  }
  TORCH_CHECK(dims_idx.size() <= 4, "ocl index: at most 4 indexed dims");
  if (!out.sizes().equals(osz)) out.resize_(osz);
  if (out.numel() == 0) return out;
  at::Tensor o = out.is_contiguous() ? out : empty(out.sizes(), out.scalar_type(), dev);
  // src and indices as descriptors of the output's shape
  pvb2_tensor sd;
  memset(&sd, 0, sizeof(sd));
  sd.data = src.data_ptr();
  sd.ndim = (int32_t)osz.size();
  sd.dtype = dtype_code(src.scalar_type());
  for (size_t i = 0; i < osz.size(); ++i) {
    sd.sizes[i] = osz[i];
    sd.strides[i] = ost[i];
  }
  std::vector<pvb2_tensor> ids;
  std::vector<at::Tensor> keep;
  for (int64_t d : dims_idx) {
    at::Tensor e = idx[d].expand(bshape);
    keep.push_back(e);
    pvb2_tensor t;
    memset(&t, 0, sizeof(t));
    t.data = e.data_ptr();
    t.ndim = (int32_t)osz.size();
    t.dtype = PVB2_I64;
    for (size_t i = 0; i < osz.size(); ++i) {
      t.sizes[i] = osz[i];
      const int64_t j = (int64_t)i - idx_pos;
      t.strides[i] = (j >= 0 && j < (int64_t)bshape.size()) ? e.stride(j) : 0;
    }
    ids.push_back(t);
  }
  pvb2_tensor od = desc(o);
  OCL_CHECK(pvb2_index_gather(&od, &sd, (int)ids.size(), ids.data(), isz.data(), istr.data(), stream_for(dev)));
  write_back(out, o);
  return out;
}

// ---------------------------------------------------------------- cat.out
// cat.out, :689-705
static at::Tensor& cat_out(const at::ITensorListRef& tensors, int64_t dim, at::Tensor& out) {
  const int dev = out.device().index();
  DeviceScope scope(dev);
  OCL_OP("cat", dev);
  std::vector<pvb2_tensor> ins;
  const int64_t d = c10::maybe_wrap_dim(dim, out.dim());
  for (const at::Tensor& t : tensors) {
    if (t.dim() == 1 && t.numel() == 0 && out.dim() != 1) continue;  // legacy empty inputs
    check_dev(t, dev, "cat");
    ins.push_back(desc(t));
  }
  if (out.numel() == 0) return out;
  pvb2_tensor o = desc(out);
  OCL_CHECK(pvb2_cat(&o, ins.data(), (int)ins.size(), (int)d, stream_for(dev)));
  return out;
}

// ----------------------------------------------------------- multi-tensor
static bool mt_ok(at::TensorList ts, int dev) {
  for (const auto& t : ts)
    if (!is_ocl(t) || t.device().index() != dev || t.scalar_type() != at::kFloat || !t.is_contiguous()) return false;
  return true;
}

static void foreach_launch(int op, at::TensorList out, at::TensorList a, at::TensorList b, double scalar, double alpha) {
  if (out.empty()) return;
  const int dev = out[0].device().index();
  DeviceScope scope(dev);
  OCL_OP("_foreach", dev);
  std::vector<float*> o(out.size());
  std::vector<const float*> x(out.size()), y(b.empty() ? 0 : out.size());
  std::vector<int64_t> n(out.size());
  for (size_t i = 0; i < out.size(); ++i) {
    o[i] = out[i].numel() ? out[i].data_ptr<float>() : nullptr;
    x[i] = a[i].numel() ? a[i].data_ptr<float>() : nullptr;
    if (!b.empty()) y[i] = b[i].numel() ? b[i].data_ptr<float>() : nullptr;
    n[i] = out[i].numel();
  }
  OCL_CHECK(pvb2_foreach_binary(op, (int)out.size(), o.data(), x.data(), b.empty() ? nullptr : y.data(), n.data(),
                                scalar, alpha, stream_for(dev)));
}

static void foreach_add_list_(at::TensorList self, at::TensorList other, const at::Scalar& alpha) {
  TORCH_CHECK(self.size() == other.size(), "_foreach_add_: list sizes differ");
  if (!self.empty() && mt_ok(self, self[0].device().index()) && mt_ok(other, self[0].device().index())) {
    foreach_launch(PVB2_BIN_ADD, self, self, other, 0, sc(alpha));
    return;
  }
  for (size_t i = 0; i < self.size(); ++i) const_cast<at::Tensor&>(self[i]).add_(other[i], alpha);
}
static void foreach_sub_list_(at::TensorList self, at::TensorList other, const at::Scalar& alpha) {
  if (!self.empty() && mt_ok(self, self[0].device().index()) && mt_ok(other, self[0].device().index())) {
    foreach_launch(PVB2_BIN_SUB, self, self, other, 0, sc(alpha));
    return;
  }
  for (size_t i = 0; i < self.size(); ++i) const_cast<at::Tensor&>(self[i]).sub_(other[i], alpha);
}
static void foreach_mul_list_(at::TensorList self, at::TensorList other) {
  if (!self.empty() && mt_ok(self, self[0].device().index()) && mt_ok(other, self[0].device().index())) {
    foreach_launch(PVB2_BIN_MUL, self, self, other, 0, 1);
    return;
  }
  for (size_t i = 0; i < self.size(); ++i) const_cast<at::Tensor&>(self[i]).mul_(other[i]);
}
static void foreach_add_scalar_(at::TensorList self, const at::Scalar& s) {
  if (!self.empty() && mt_ok(self, self[0].device().index())) {
    foreach_launch(PVB2_BIN_ADD, self, self, {}, sc(s), 1);
    return;
  }
  for (auto& t : self) const_cast<at::Tensor&>(t).add_(s);
}
static void foreach_mul_scalar_(at::TensorList self, const at::Scalar& s) {
  if (!self.empty() && mt_ok(self, self[0].device().index())) {
    foreach_launch(PVB2_BIN_MUL, self, self, {}, sc(s), 1);
    return;
  }
  for (auto& t : self) const_cast<at::Tensor&>(t).mul_(s);
}
static void foreach_div_scalar_(at::TensorList self, const at::Scalar& s) {
  if (!self.empty() && mt_ok(self, self[0].device().index())) {
    foreach_launch(PVB2_BIN_DIV, self, self, {}, sc(s), 1);
    return;
  }
  for (auto& t : self) const_cast<at::Tensor&>(t).div_(s);
}
static void foreach_zero_(at::TensorList self) {
  for (auto& t : self) const_cast<at::Tensor&>(t).zero_();
}
static std::vector<at::Tensor> foreach_add_list(at::TensorList self, at::TensorList other, const at::Scalar& alpha) {
  std::vector<at::Tensor> out;
  for (auto& t : self) out.push_back(empty(t.sizes(), t.scalar_type(), t.device().index()));
  if (!self.empty() && mt_ok(self, self[0].device().index()) && mt_ok(other, self[0].device().index())) {
    foreach_launch(PVB2_BIN_ADD, out, self, other, 0, sc(alpha));
    return out;
  }
  for (size_t i = 0; i < self.size(); ++i) out[i] = self[i].add(other[i], alpha);
  return out;
}
static std::vector<at::Tensor> foreach_mul_scalar(at::TensorList self, const at::Scalar& s) {
  std::vector<at::Tensor> out;
  for (auto& t : self) out.push_back(empty(t.sizes(), t.scalar_type(), t.device().index()));
  if (!self.empty() && mt_ok(self, self[0].device().index())) {
    foreach_launch(PVB2_BIN_MUL, out, self, {}, sc(s), 1);
    return out;
  }
  for (size_t i = 0; i < self.size(); ++i) out[i] = self[i].mul(s);
  return out;
}

// _fused_sgd_: one launch for the whole parameter list (torch.optim.SGD(fused=True))
static void fused_sgd_(at::TensorList self, at::TensorList grads, at::TensorList momentum_buffer_list,
                       double weight_decay, double momentum, double lr, double dampening, bool nesterov, bool maximize,
                       bool is_first_step, const std::optional<at::Tensor>& grad_scale,
                       const std::optional<at::Tensor>& found_inf) {
  TORCH_CHECK(!grad_scale.has_value() && !found_inf.has_value(), "ocl _fused_sgd_: grad scaling is not supported");
  if (self.empty()) return;
  const int dev = self[0].device().index();
  TORCH_CHECK(mt_ok(self, dev) && mt_ok(grads, dev), "ocl _fused_sgd_: fp32 contiguous tensors on one device expected");
  if (momentum != 0.0) TORCH_CHECK(mt_ok(momentum_buffer_list, dev), "ocl _fused_sgd_: bad momentum buffers");
  DeviceScope scope(dev);
  OCL_OP("_fused_sgd_", dev);
  const size_t n = self.size();
  std::vector<float*> p(n), b(n);
  std::vector<const float*> g(n);
  std::vector<int64_t> numel(n);
  for (size_t i = 0; i < n; ++i) {
    p[i] = self[i].data_ptr<float>();
    g[i] = grads[i].data_ptr<float>();
    b[i] = momentum != 0.0 ? momentum_buffer_list[i].data_ptr<float>() : nullptr;
    numel[i] = self[i].numel();
  }
  OCL_CHECK(pvb2_sgd_multi((int)n, p.data(), g.data(), momentum != 0.0 ? b.data() : nullptr, numel.data(), lr,
                           momentum, dampening, weight_decay, nesterov ? 1 : 0, is_first_step ? 1 : 0,
                           maximize ? -1.0 : 1.0, stream_for(dev)));
}

}  // namespace ocl

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  using namespace ocl;
  m.impl("add.out", &add_out);
  m.impl("add_.Tensor", &add_inplace);
  m.impl("sub.out", &sub_out);
  m.impl("mul.out", &mul_out);
  m.impl("div.out", &div_out);
  m.impl("div.out_mode", &div_out_mode);
  m.impl("maximum.out", &maximum_out);
  m.impl("minimum.out", &minimum_out);
  m.impl("atan2.out", &atan2_out);
  m.impl("pow.Tensor_Tensor_out", &pow_tt_out);
  m.impl("pow.Tensor_Scalar_out", &pow_ts_out);
  m.impl("remainder.Tensor_out", &remainder_out);
  m.impl("bitwise_and.Tensor_out", &bitwise_and_out);
  m.impl("bitwise_or.Tensor_out", &bitwise_or_out);
  m.impl("bitwise_xor.Tensor_out", &bitwise_xor_out);
  m.impl("bitwise_not.out", &bitwise_not_out);
  m.impl("eq.Tensor_out", &eq_tensor);
  m.impl("ne.Tensor_out", &ne_tensor);
  m.impl("lt.Tensor_out", &lt_tensor);
  m.impl("le.Tensor_out", &le_tensor);
  m.impl("gt.Tensor_out", &gt_tensor);
  m.impl("ge.Tensor_out", &ge_tensor);
  m.impl("eq.Scalar_out", &eq_scalar);
  m.impl("ne.Scalar_out", &ne_scalar);
  m.impl("lt.Scalar_out", &lt_scalar);
  m.impl("le.Scalar_out", &le_scalar);
  m.impl("gt.Scalar_out", &gt_scalar);
  m.impl("ge.Scalar_out", &ge_scalar);
  m.impl("threshold_backward.grad_input", &threshold_backward_out);
  m.impl("relu", &relu);
  m.impl("relu_", &relu_);
  m.impl("hardtanh", &hardtanh);
  m.impl("hardtanh_", &hardtanh_);
  m.impl("hardtanh.out", &hardtanh_out);
  m.impl("hardtanh_backward", &hardtanh_backward);
  m.impl("hardtanh_backward.grad_input", &hardtanh_backward_out);
  m.impl("gelu.out", &gelu_out);
  m.impl("gelu_backward.grad_input", &gelu_backward_out);
  m.impl("exp.out", &exp_out);
  m.impl("log.out", &log_out);
  m.impl("sqrt.out", &sqrt_out);
  m.impl("rsqrt.out", &rsqrt_out);
  m.impl("neg.out", &neg_out);
  m.impl("abs", &abs_new);
  m.impl("abs.out", &abs_out);
  m.impl("sigmoid.out", &sigmoid_out);
  m.impl("tanh.out", &tanh_out);
  m.impl("reciprocal.out", &reciprocal_out);
  m.impl("silu.out", &silu_out);
  m.impl("hardsigmoid.out", &hardsigmoid_out);
  m.impl("hardswish", &hardswish);
  m.impl("hardswish_", &hardswish_);
  m.impl("hardswish.out", &hardswish_out);
  m.impl("ceil.out", &ceil_out);
  m.impl("floor.out", &floor_out);
  m.impl("trunc.out", &trunc_out);
  m.impl("round.out", &round_out);
  m.impl("atan.out", &atan_out);
  m.impl("sgn.out", &sgn_out);
  m.impl("clamp.out", &clamp_out);
  m.impl("clamp_min.out", &clamp_min_out);
  m.impl("leaky_relu.out", &leaky_relu_out);
  m.impl("sigmoid_backward.grad_input", &sigmoid_backward_out);
  m.impl("tanh_backward.grad_input", &tanh_backward_out);
  m.impl("silu_backward.grad_input", &silu_backward_out);
  m.impl("hardsigmoid_backward.grad_input", &hardsigmoid_backward_out);
  m.impl("hardswish_backward", &hardswish_backward);
  m.impl("leaky_relu_backward.grad_input", &leaky_relu_backward_out);
  m.impl("log_sigmoid_forward", &log_sigmoid_forward);
  m.impl("log_sigmoid_forward.output", &log_sigmoid_forward_out);
  m.impl("log_sigmoid_backward", &log_sigmoid_backward);
  m.impl("log_sigmoid_backward.grad_input", &log_sigmoid_backward_out);
  m.impl("lerp.Scalar_out", &lerp_out);
  m.impl("addcmul.out", &addcmul_out);
  m.impl("addcdiv.out", &addcdiv_out);
  m.impl("where.self", &where_self);
  m.impl("where.self_out", &where_out);
  m.impl("sum.IntList_out", &sum_out);
  m.impl("mean.out", &mean_out);
  m.impl("prod.int_out", &prod_out);
  m.impl("amax.out", &amax_out);
  m.impl("amin.out", &amin_out);
  m.impl("argmax.out", &argmax_out);
  m.impl("argmin.out", &argmin_out);
  m.impl("max", &max_all);
  m.impl("min", &min_all);
  m.impl("dot", &dot);
  m.impl("cat.out", &cat_out);
  m.impl("logical_not.out", &logical_not_out);
  m.impl("isposinf.out", &isposinf_out);
  m.impl("isneginf.out", &isneginf_out);
  m.impl("isnan", &isnan);
  m.impl("sign.out", &sign_out);
  m.impl("logit", &logit);
  m.impl("logit.out", &logit_out);
  m.impl("clamp_max.out", &clamp_max_out);
  m.impl("all.dims_out", &all_dims_out);
  m.impl("all.out", &all_out);
  m.impl("all.all_out", &all_all_out);
  m.impl("any.dims_out", &any_dims_out);
  m.impl("any.out", &any_out);
  m.impl("any.all_out", &any_all_out);
  m.impl("masked_select", &masked_select);
  m.impl("index.Tensor_out", &index_out);
  m.impl("nonzero", &nonzero);
  m.impl("masked_fill_.Scalar", &masked_fill_scalar_);
  m.impl("masked_fill_.Tensor", &masked_fill_tensor_);
  m.impl("arange.start_out", &arange_out);
  m.impl("_foreach_add_.List", &foreach_add_list_);
  m.impl("_foreach_sub_.List", &foreach_sub_list_);
  m.impl("_foreach_mul_.List", &foreach_mul_list_);
  m.impl("_foreach_add_.Scalar", &foreach_add_scalar_);
  m.impl("_foreach_mul_.Scalar", &foreach_mul_scalar_);
  m.impl("_foreach_div_.Scalar", &foreach_div_scalar_);
  m.impl("_foreach_zero_", &foreach_zero_);
  m.impl("_foreach_add.List", &foreach_add_list);
  m.impl("_foreach_mul.Scalar", &foreach_mul_scalar);
  m.impl("_fused_sgd_", &fused_sgd_);
}
