// Fused scaled-dot-product attention for `ocl` tensors.
//
// torch's scaled_dot_product_attention asks the device's
// _fused_sdp_choice_stub (also registered as the aten::_fused_sdp_choice op)
// which implementation to run.  For `ocl` it answers
// "overrideable" when this backend's fused kernel covers the call (4-D fp32
// q/k/v with equal batch and heads, head dim 32/64/128, no attention mask,
// no dropout) and "math" otherwise; the overrideable choice lands in
// _scaled_dot_product_fused_attention_overrideable and its backward, both
// implemented here on pvb2_sdpa_fwd / pvb2_sdpa_bwd.  The reference had no
// fused attention: ViT's attention ran as bmm + softmax (src/vision_ops.cpp:
// 541-626, src/loss_ops.cpp:137-213), which is still what "math" runs.
#include <ATen/SDPBackend.h>
#include <ATen/native/DispatchStub.h>
#include <ATen/native/transformers/attention.h>
#include <torch/extension.h>

#include <cmath>

#include "ocl.h"

namespace ocl {

static bool sdpa_covered(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                         const std::optional<at::Tensor>& mask, double dropout_p, bool enable_gqa) {
  if (!is_ocl(q) || !is_ocl(k) || !is_ocl(v)) return false;
  if (mask.has_value() && mask->defined()) return false;
  if (dropout_p != 0.0) return false;
  if (q.dim() != 4 || k.dim() != 4 || v.dim() != 4) return false;
  for (const at::Tensor* t : {&q, &k, &v})
    if (t->scalar_type() != at::kFloat) return false;
  const int64_t D = q.size(3);
  if (D != 32 && D != 64 && D != 128) return false;
  if (k.size(3) != D || v.size(3) != D) return false;
  if (k.size(0) != q.size(0) || v.size(0) != q.size(0) || k.size(1) != q.size(1) || v.size(1) != q.size(1))
    return false;  // grouped-query attention and broadcasting go to "math"
  if (k.size(2) != v.size(2)) return false;
  if (q.size(0) * q.size(1) > 65535) return false;
  (void)enable_gqa;
  return true;
}

static int64_t fused_sdp_choice(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                const std::optional<at::Tensor>& mask, double dropout_p, bool is_causal,
                                std::optional<double> scale, bool enable_gqa) {
  (void)is_causal;
  (void)scale;
  // torch.nn.attention.sdpa_kernel([...]) switches backends on and off
  const auto& ctx = at::globalContext();
  if (ctx.userEnabledOverrideableSDP() && sdpa_covered(q, k, v, mask, dropout_p, enable_gqa))
    return static_cast<int64_t>(at::SDPBackend::overrideable);
  TORCH_CHECK(ctx.userEnabledMathSDP(),
              "ocl scaled_dot_product_attention: no enabled backend covers these arguments (the fused kernel "
              "takes 4-D fp32 q/k/v with head dim 32/64/128, no mask and no dropout; math is disabled)");
  return static_cast<int64_t>(at::SDPBackend::math);
}

// rows 16-byte aligned and unit stride along the head dimension, or a copy
static at::Tensor sdpa_operand(const at::Tensor& t) {
  const bool ok = t.stride(3) == 1 && t.stride(0) % 4 == 0 && t.stride(1) % 4 == 0 && t.stride(2) % 4 == 0 &&
                  (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0;
  return ok ? t : contiguous(t);
}

static pvb2_sdpa_desc sdpa_desc(const at::Tensor& q, const at::Tensor& k, bool is_causal,
                                std::optional<double> scale) {
  pvb2_sdpa_desc d;
  d.B = (int32_t)q.size(0);
  d.H = (int32_t)q.size(1);
  d.Lq = (int32_t)q.size(2);
  d.Lk = (int32_t)k.size(2);
  d.D = (int32_t)q.size(3);
  d.scale = (float)(scale.has_value() ? *scale : 1.0 / std::sqrt((double)d.D));
  d.causal = is_causal ? 1 : 0;
  d.math = math_mode() == PVB2_MATH_FP32 ? PVB2_MATH_FP32 : PVB2_MATH_TF32;
  return d;
}

static std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, c10::SymInt, c10::SymInt, at::Tensor, at::Tensor,
                  at::Tensor>
sdpa_fwd(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
         const std::optional<at::Tensor>& attn_bias, double dropout_p, bool is_causal, bool return_debug_mask,
         std::optional<double> scale) {
  TORCH_CHECK(sdpa_covered(query, key, value, attn_bias, dropout_p, false),
              "ocl fused attention: unsupported arguments (mask, dropout, dtype or head dimension)");
  TORCH_CHECK(!return_debug_mask, "ocl fused attention: no debug mask");
  const int dev = query.device().index();
  DeviceScope scope(dev);
  OCL_OP("_scaled_dot_product_fused_attention_overrideable", dev);
  const at::Tensor q = sdpa_operand(query), k = sdpa_operand(key), v = sdpa_operand(value);
  const pvb2_sdpa_desc d = sdpa_desc(q, k, is_causal, scale);
  at::Tensor out = empty(q.sizes(), at::kFloat, dev);
  at::Tensor lse = empty({q.size(0), q.size(1), q.size(2)}, at::kFloat, dev);
  const pvb2_tensor qd = desc(q), kd = desc(k), vd = desc(v), od = desc(out);
  OCL_CHECK(pvb2_sdpa_fwd(&d, &qd, &kd, &vd, &od, lse.numel() ? lse.data_ptr<float>() : nullptr, stream_for(dev)));
  const at::Tensor none = empty({0}, at::kFloat, dev);
  return {out, lse, none, none, c10::SymInt(d.Lq), c10::SymInt(d.Lk), none, none, none};
}

static std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> sdpa_bwd(
    const at::Tensor& grad_out, const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
    const at::Tensor& attn_bias, std::array<bool, 4> grad_input_mask, const at::Tensor& out,
    const at::Tensor& logsumexp, const at::Tensor& cum_seq_q, const at::Tensor& cum_seq_k, c10::SymInt max_q,
    c10::SymInt max_k, double dropout_p, bool is_causal, const at::Tensor& philox_seed,
    const at::Tensor& philox_offset, std::optional<double> scale) {
  (void)cum_seq_q;
  (void)cum_seq_k;
  (void)max_q;
  (void)max_k;
  (void)philox_seed;
  (void)philox_offset;
  TORCH_CHECK(!attn_bias.defined() && dropout_p == 0.0, "ocl fused attention backward: no bias or dropout");
  const int dev = query.device().index();
  DeviceScope scope(dev);
  OCL_OP("_scaled_dot_product_fused_attention_overrideable_backward", dev);
  const at::Tensor q = sdpa_operand(query), k = sdpa_operand(key), v = sdpa_operand(value);
  const at::Tensor o = sdpa_operand(out), g = sdpa_operand(grad_out);
  const at::Tensor lse = contiguous(logsumexp);
  const pvb2_sdpa_desc d = sdpa_desc(q, k, is_causal, scale);
  at::Tensor dq = empty(q.sizes(), at::kFloat, dev);
  at::Tensor dk = empty(k.sizes(), at::kFloat, dev);
  at::Tensor dv = empty(v.sizes(), at::kFloat, dev);
  Workspace ws(pvb2_sdpa_bwd_workspace_size(&d), dev);
  const pvb2_tensor qd = desc(q), kd = desc(k), vd = desc(v), od = desc(o), gd = desc(g);
  const pvb2_tensor dqd = desc(dq), dkd = desc(dk), dvd = desc(dv);
  OCL_CHECK(pvb2_sdpa_bwd(&d, &qd, &kd, &vd, &od, &gd, lse.numel() ? lse.data_ptr<float>() : nullptr, &dqd, &dkd,
                          &dvd, ws.get(), ws.bytes, stream_for(dev)));
  return {grad_input_mask[0] ? dq : at::Tensor(), grad_input_mask[1] ? dk : at::Tensor(),
          grad_input_mask[2] ? dv : at::Tensor(), at::Tensor()};
}

}  // namespace ocl

namespace at::native {
REGISTER_PRIVATEUSE1_DISPATCH(_fused_sdp_choice_stub, &ocl::fused_sdp_choice);
}  // namespace at::native

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("_fused_sdp_choice", &ocl::fused_sdp_choice);
  m.impl("_scaled_dot_product_fused_attention_overrideable", &ocl::sdpa_fwd);
  m.impl("_scaled_dot_product_fused_attention_overrideable_backward", &ocl::sdpa_bwd);
}
