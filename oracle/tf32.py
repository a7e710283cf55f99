"""TF32 emulation of the device's tensor-core contractions -- TEST INFRASTRUCTURE ONLY.

In its default math mode the device runs convolutions, linear layers and
attention on TF32 tensor cores.  A TF32 product uses the top 10 explicit
mantissa bits of each fp32 operand; the products are exact in fp32 and are
accumulated in fp32.  This module restates that arithmetic on the CPU so the
oracle can be compared with the device tensor by tensor instead of through a
bound as wide as the TF32 rounding itself:

* ``cut_tf32``    -- the operand conversion of the tcgen05 convolution and
  GEMM kernels (``kind::tf32``): the fp32 value with its low 13 mantissa bits
  cleared (the tensor core reads the register as TF32);
* ``round_tf32``  -- the conversion of the fused attention kernels, which
  round each staged tile once with ``cvt.rna.tf32.f32`` (round to nearest,
  ties away from zero);
* ``Tf32Emulation`` -- a context that swaps ``torch.nn.functional.conv2d``,
  ``linear`` and ``scaled_dot_product_attention`` for autograd functions that
  convert exactly the operands the device converts, in the forward pass and
  in each backward pass (input gradient, weight gradient), and compute the
  rest in the tensors' own dtype (float64 for the ground truth, float32 for
  the CPU's own rounding-noise estimate).

Which passes run on the tensor cores is the device library's decision
(shapes, alignment, math mode).  The caller supplies it as a ``Paths``
object (the tests build one from the library's own path queries), so the
emulation follows the device's dispatch instead of restating it.

The reference (pytorch_ocl 0.2.0) has no TF32 mode: its dlprimitives kernels
are fp32 throughout (src/vision_ops.cpp:61-186, 243-351), and its validation
compares with torch-CPU fp32 (tests/validate_network.py:94-122).  This module
only models the precision the device states for its tensor-core paths.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn.functional as F

_conv2d = torch.nn.functional.conv2d
_linear = torch.nn.functional.linear
_sdpa = torch.nn.functional.scaled_dot_product_attention


def cut_tf32(t: torch.Tensor) -> torch.Tensor:
    """fp32 value of `t` with the low 13 mantissa bits cleared, in t's dtype."""
    f = t.detach().to(torch.float32).contiguous()
    r = (f.view(torch.int32) & -8192).view(torch.float32)
    return r.to(t.dtype)


def round_tf32(t: torch.Tensor) -> torch.Tensor:
    """fp32 value of `t` rounded to 10 mantissa bits, ties away from zero.
    The magnitude bits of an IEEE float are an unsigned integer, so adding
    half a TF32 unit (0x1000) and clearing the low 13 bits rounds the
    magnitude for either sign."""
    f = t.detach().to(torch.float32).contiguous()
    r = ((f.view(torch.int32) + 0x1000) & -8192).view(torch.float32)
    return r.to(t.dtype)


@dataclass
class Paths:
    """Which contraction passes the device runs on the tensor cores.

    conv(x_shape, w_shape, stride, padding, dilation, groups, which) -> bool
        which: 0 forward, 1 input gradient, 2 weight gradient
    linear(rows, in_features, out_features, which) -> bool
        which: 0 y = x W^T, 1 dX = dY W, 2 dW = dY^T X
    attention(head_dim) -> bool
    """
    conv: Callable[..., bool]
    linear: Callable[..., bool]
    attention: Callable[[int], bool]


def _pair(v):
    return tuple(v) if isinstance(v, (tuple, list)) else (v, v)


class _Conv2d(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, stride, padding, dilation, groups, tc, cut):
        ctx.save_for_backward(x, w)
        ctx.conf = (stride, padding, dilation, groups, tc, cut, b is not None)
        if tc[0]:
            return _conv2d(cut(x), cut(w), b, stride, padding, dilation, groups)
        return _conv2d(x, w, b, stride, padding, dilation, groups)

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        stride, padding, dilation, groups, tc, cut, has_b = ctx.conf
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            ww, g1 = (cut(w), cut(gy)) if tc[1] else (w, gy)
            gx = torch.nn.grad.conv2d_input(x.shape, ww, g1, stride, padding, dilation, groups)
        if ctx.needs_input_grad[1]:
            xx, g2 = (cut(x), cut(gy)) if tc[2] else (x, gy)
            gw = torch.nn.grad.conv2d_weight(xx, w.shape, g2, stride, padding, dilation, groups)
        if has_b and ctx.needs_input_grad[2]:
            gb = gy.sum((0, 2, 3))
        return gx, gw, gb, None, None, None, None, None, None


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, tc, cut):
        ctx.save_for_backward(x, w)
        ctx.conf = (tc, cut, b is not None)
        x2 = x.reshape(-1, x.shape[-1])
        y = cut(x2) @ cut(w).t() if tc[0] else x2 @ w.t()
        if b is not None:
            y = y + b
        return y.reshape(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        tc, cut, has_b = ctx.conf
        x2 = x.reshape(-1, x.shape[-1])
        g2 = gy.reshape(-1, gy.shape[-1])
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            gx = (cut(g2) @ cut(w) if tc[1] else g2 @ w).reshape(x.shape)
        if ctx.needs_input_grad[1]:
            gw = cut(g2).t() @ cut(x2) if tc[2] else g2.t() @ x2
        if has_b and ctx.needs_input_grad[2]:
            gb = g2.sum(0)
        return gx, gw, gb, None, None


class _Attention(torch.autograd.Function):
    """softmax(q k^T * scale) v over [B, H, L, D] without mask or dropout.

    The tensor-core kernels round (q * scale), k, v, the probabilities before
    P V, dO, and dS once to TF32; scores and sums stay fp32 (here: the
    tensor's dtype).  The device rounds each 64-key block's probabilities
    against the running maximum of the online softmax; the emulation rounds
    them against the row's final maximum, a difference of at most one TF32
    unit in some probabilities."""

    @staticmethod
    def forward(ctx, q, k, v, scale, tc, rnd):
        qs = q * scale
        if tc:
            qs, kr, vr = rnd(qs), rnd(k), rnd(v)
        else:
            kr, vr = k, v
        s = qs @ kr.transpose(-1, -2)
        m = s.amax(-1, keepdim=True)
        p = torch.exp(s - m)
        l = p.sum(-1, keepdim=True)
        o = ((rnd(p) if tc else p) @ vr) / l
        lse = m + torch.log(l)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.conf = (scale, tc, rnd)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        scale, tc, rnd = ctx.conf
        r = rnd if tc else (lambda t: t)
        qs, kr, vr, dor = r(q * scale), r(k), r(v), r(do)
        p = torch.exp(qs @ kr.transpose(-1, -2) - lse)
        di = (do * o).sum(-1, keepdim=True)
        dp = dor @ vr.transpose(-1, -2)
        ds = r(p * (dp - di))
        dv = r(p).transpose(-1, -2) @ dor
        dk = ds.transpose(-1, -2) @ qs
        dq = (ds @ kr) * scale
        return dq, dk, dv, None, None, None


@contextlib.contextmanager
def Tf32Emulation(paths: Optional[Paths], cut: Callable = cut_tf32, rnd: Callable = round_tf32):
    """Within the context, F.conv2d / F.linear / F.scaled_dot_product_attention
    (the functions torchvision's layers and nn.MultiheadAttention call) run
    the emulated arithmetic.  paths=None converts nothing (plain arithmetic in
    the tensors' dtype, through the same functions)."""

    def conv2d(input, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
        st, pd, dl = _pair(stride), _pair(padding), _pair(dilation)
        if paths is None:
            tc = (False, False, False)
        else:
            tc = tuple(bool(paths.conv(tuple(input.shape), tuple(weight.shape), st, pd, dl, groups, i))
                       for i in range(3))
        return _Conv2d.apply(input, weight, bias, st, pd, dl, groups, tc, cut)

    def linear(input, weight, bias=None):
        rows = input.numel() // input.shape[-1] if input.dim() else 1
        if paths is None:
            tc = (False, False, False)
        else:
            tc = tuple(bool(paths.linear(rows, weight.shape[1], weight.shape[0], i)) for i in range(3))
        return _Linear.apply(input, weight, bias, tc, cut)

    def sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, enable_gqa=False):
        if attn_mask is not None or dropout_p != 0.0 or is_causal or enable_gqa:
            raise NotImplementedError("emulated attention: no mask, dropout, causal or GQA")
        d = query.shape[-1]
        sc = scale if scale is not None else d ** -0.5
        tc = paths is not None and bool(paths.attention(d))
        return _Attention.apply(query, key, value, sc, tc, rnd)

    saved = (F.conv2d, F.linear, F.scaled_dot_product_attention)
    F.conv2d, F.linear, F.scaled_dot_product_attention = conv2d, linear, sdpa
    try:
        yield
    finally:
        F.conv2d, F.linear, F.scaled_dot_product_attention = saved
