// Autograd kernels of the `ocl` device, where torch's device-independent one
// does more device work than the op needs.
//
// hardtanh_ (MobileNet-v2's ReLU6(inplace=True) reaches it through relu6_,
// ref pointwise_ops.cpp:559-603): torch's autograd kernel saves the op's
// input for hardtanh_backward, so it first clones the tensor it is about to
// overwrite, a full extra write of every ReLU6 activation.  For bounds
// min < max the gradient mask is the same read from the output: out <= min
// exactly when in <= min, out >= max exactly when in >= max.  The kernel
// below saves the output instead (as torch's relu_ does), so no clone is
// made; like relu_'s, its backward then refuses to run if the output was
// modified in place afterwards.  Every other case (a leaf or a view,
// min >= max, complex bounds) runs as copy_ of the out-of-place op on a
// clone under torch's autograd, which has the same values and gradients.
#include <torch/csrc/autograd/custom_function.h>
#include <torch/csrc/autograd/variable.h>

#include "ocl.h"

namespace ocl {
namespace {

using torch::autograd::AutogradContext;
using torch::autograd::variable_list;

struct HardtanhInplace : public torch::autograd::Function<HardtanhInplace> {
  static at::Tensor forward(AutogradContext* ctx, at::Tensor self, at::Scalar mn, at::Scalar mx) {
    {
      at::AutoDispatchBelowADInplaceOrView below;  // the device kernel (ops_pointwise.cpp)
      at::hardtanh_(self, mn, mx);
    }
    ctx->mark_dirty({self});
    ctx->save_for_backward({self});
    ctx->saved_data["min"] = mn;
    ctx->saved_data["max"] = mx;
    return self;
  }

  static variable_list backward(AutogradContext* ctx, variable_list grads) {
    const variable_list saved = ctx->get_saved_variables();
    at::Tensor gi;
    if (grads[0].defined())
      gi = at::hardtanh_backward(grads[0], saved[0], ctx->saved_data["min"].toScalar(),
                                 ctx->saved_data["max"].toScalar());
    return {gi, at::Tensor(), at::Tensor()};
  }
};

at::Tensor& hardtanh_autograd(at::Tensor& self, const at::Scalar& mn, const at::Scalar& mx) {
  if (!at::GradMode::is_enabled() || !self.requires_grad()) {
    // what torch's kernels do when no graph is recorded: the op, then the
    // version bump of an in-place op
    {
      at::AutoDispatchBelowADInplaceOrView below;
      at::hardtanh_(self, mn, mx);
    }
    torch::autograd::impl::bump_version(self);
    return self;
  }
  const bool take = self.grad_fn() != nullptr && !self.is_view() && !mn.isComplex() && !mx.isComplex() &&
                    mn.toDouble() < mx.toDouble();
  if (take) {
    HardtanhInplace::apply(self, mn, mx);
    return self;
  }
  // anything else through torch's autograd of the out-of-place op on a
  // clone (which the op saves, so the copy_ back does not invalidate it) and
  // copy_ (a view, a leaf that requires grad -- which copy_ refuses as
  // torch's hardtanh_ does --, or min >= max): torch's hardtanh_ clones too
  self.copy_(at::hardtanh(self.clone(), mn, mx));
  return self;
}

}  // namespace
}  // namespace ocl

TORCH_LIBRARY_IMPL(aten, AutogradPrivateUse1, m) { m.impl("hardtanh_", &ocl::hardtanh_autograd); }
