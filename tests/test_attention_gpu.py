"""Fused scaled-dot-product attention on `ocl` (pvb2_sdpa_fwd / _bwd behind
torch's overrideable SDPA backend) against a float64 CPU computation.

The reference ran attention as bmm + softmax (vision_ops.cpp:541-626,
loss_ops.cpp:137-213) and compared networks with torch-CPU; the fused kernel
is fp32 on CUDA cores, so outputs and gradients are checked at fp32 accuracy
(1e-5 relative to each tensor's magnitude)."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "ocl:0"


def _rel(ref, got):
    # error relative to the tensor's magnitude, floored at 1 (the scale of the
    # unit-normal inputs): with one visible key dq is exactly zero in float64
    # and fp32 leaves dP - Di rounding residue of about 1e-6 there
    ref = ref.detach().double()
    return ((got.detach().cpu().double() - ref).abs().max() / max(ref.abs().max().item(), 1.0)).item()


CASES = [
    # B, H, Lq, Lk, D, causal, layout
    (2, 3, 197, 197, 64, False, "contiguous"),   # ViT-B/16 head shape
    (2, 2, 70, 130, 32, False, "contiguous"),    # Lq != Lk, partial blocks
    (1, 2, 129, 129, 128, True, "contiguous"),   # causal, D = 128
    (3, 4, 50, 50, 64, False, "heads_last"),     # q/k/v as the strided views MultiheadAttention makes
    (2, 2, 1, 65, 64, True, "contiguous"),       # a single query row
    (1, 3, 150, 90, 64, True, "contiguous"),     # causal with Lk < Lq: late rows see every key
    (2, 1, 128, 256, 128, False, "contiguous"),  # whole 64-row blocks only
    (1, 2, 257, 200, 32, True, "heads_last"),
]


def _make(B, H, L, D, layout, g):
    if layout == "heads_last":
        return torch.randn(B, L, H, D, generator=g).transpose(1, 2)
    return torch.randn(B, H, L, D, generator=g)


# exact fp32 (CUDA-core kernels) at fp32 accuracy; TF32 tensor cores (the
# default math mode, D = 32 / 64) within 5e-3 of each tensor's magnitude --
# TF32 operands carry 11 significant bits
MATH = [("fp32", 1, 1e-5), ("tf32", 0, 5e-3)]


@pytest.mark.parametrize("math_name,mode,tol", MATH, ids=[m[0] for m in MATH])
@pytest.mark.parametrize("case", CASES, ids=["-".join(map(str, c)) for c in CASES])
def test_sdpa_fused_matches_float64(ocl, case, math_name, mode, tol):
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(mode)
    try:
        _sdpa_case(case, tol)
    finally:
        torch.ocl.set_math_mode(old)


def _sdpa_case(case, tol):
    B, H, Lq, Lk, D, causal, layout = case
    g = torch.Generator().manual_seed(B * 100 + Lq)
    q, k, v = _make(B, H, Lq, D, layout, g), _make(B, H, Lk, D, layout, g), _make(B, H, Lk, D, layout, g)
    dout = torch.randn(B, H, Lq, D, generator=g)
    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    # the fused kernel is the one chosen for these arguments
    assert torch._fused_sdp_choice(qd, kd, vd, is_causal=causal) == 4
    od = F.scaled_dot_product_attention(qd, kd, vd, is_causal=causal)
    od.backward(dout.to(DEV))
    q64, k64, v64 = (t.double().requires_grad_() for t in (q, k, v))
    s = q64 @ k64.transpose(-1, -2) / math.sqrt(D)
    if causal:
        s = s.masked_fill(torch.ones(Lq, Lk, dtype=torch.bool).triu(1), float("-inf"))
    o64 = torch.softmax(s, -1) @ v64
    o64.backward(dout.double())
    assert _rel(o64, od) < tol
    assert _rel(q64.grad, qd.grad) < tol
    assert _rel(k64.grad, kd.grad) < tol
    assert _rel(v64.grad, vd.grad) < tol


def test_sdpa_unsupported_falls_back_to_math(ocl):
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(2, 2, 9, 24, generator=g) for _ in range(3))  # head dim 24: not fused
    qd, kd, vd = (t.to(DEV) for t in (q, k, v))
    assert torch._fused_sdp_choice(qd, kd, vd) == 0
    mask = torch.rand(9, 9, generator=g) > 0.3
    out = F.scaled_dot_product_attention(qd, kd, vd, attn_mask=mask.to(DEV))
    ref = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    assert (out.cpu() - ref).abs().max().item() < 1e-3


def test_multihead_attention_module(ocl):
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(1)  # exact fp32 projections: the comparison isolates attention
    try:
        _mha_check()
    finally:
        torch.ocl.set_math_mode(old)


def _mha_check():
    torch.manual_seed(0)
    mha = torch.nn.MultiheadAttention(256, 4, batch_first=True)
    x = torch.randn(3, 40, 256, generator=torch.Generator().manual_seed(1))
    y, _ = mha(x, x, x, need_weights=False)
    y.sum().backward()
    ref = {n: p.grad.clone() for n, p in mha.named_parameters()}
    mha.zero_grad(set_to_none=True)
    mha_d = mha.to(DEV)
    yd, _ = mha_d(x.to(DEV), x.to(DEV), x.to(DEV), need_weights=False)
    yd.sum().backward()
    assert _rel(y, yd) < 1e-4
    for n, p in mha_d.named_parameters():
        assert _rel(ref[n], p.grad) < 1e-4, n


def test_sdpa_kernel_context_selects_backend(ocl):
    from torch.nn.attention import SDPBackend, sdpa_kernel
    q, k, v = (torch.randn(2, 3, 40, 64, generator=torch.Generator().manual_seed(i)).to(DEV) for i in range(3))
    assert torch._fused_sdp_choice(q, k, v) == 4
    with sdpa_kernel(SDPBackend.MATH):
        assert torch._fused_sdp_choice(q, k, v) == 0
        om = F.scaled_dot_product_attention(q, k, v)
    with sdpa_kernel(SDPBackend.OVERRIDEABLE):
        of = F.scaled_dot_product_attention(q, k, v)
    assert _rel(om.cpu().double(), of) < 5e-3  # math runs its matmuls in the current (TF32) mode


def test_sdpa_backward_without_slice_workspace(ocl):
    """pvb2_sdpa_bwd through the C-ABI with the full workspace (dQ from
    per-key-block slices) and with only the D_i part (dQ recomputed per query
    block): both match float64."""
    import ctypes
    import os

    import pytorch_vulkan_b200 as p

    class T(ctypes.Structure):
        _fields_ = [("data", ctypes.c_void_p), ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8),
                    ("ndim", ctypes.c_int32), ("dtype", ctypes.c_int32)]

    class Desc(ctypes.Structure):
        _fields_ = [("B", ctypes.c_int32), ("H", ctypes.c_int32), ("Lq", ctypes.c_int32), ("Lk", ctypes.c_int32),
                    ("D", ctypes.c_int32), ("scale", ctypes.c_float), ("causal", ctypes.c_int32),
                    ("math", ctypes.c_int32)]

    def td(t):
        return T(t.data_ptr(), (ctypes.c_int64 * 8)(*t.shape), (ctypes.c_int64 * 8)(*t.stride()), t.dim(), 0)

    lib = ctypes.CDLL(os.path.join(os.path.dirname(p.__file__), "lib", "libpvb2.so"))
    lib.pvb2_sdpa_bwd_workspace_size.restype = ctypes.c_size_t
    lib.pvb2_last_error.restype = ctypes.c_char_p
    stream = ctypes.c_void_p(p._C.impl_stream_handle(0))
    B, H, Lq, Lk, D = 2, 3, 150, 197, 64
    for causal in (0, 1):
        g = torch.Generator().manual_seed(40 + causal)
        q, k, v = (torch.randn(B, H, n, D, generator=g) for n in (Lq, Lk, Lk))
        dout = torch.randn(B, H, Lq, D, generator=g)
        d = Desc(B, H, Lq, Lk, D, 1.0 / math.sqrt(D), causal, 1)  # exact fp32 kernels
        qd, kd, vd, gd = (t.to(DEV) for t in (q, k, v, dout))
        od = torch.empty_like(qd)
        lse = torch.empty(B, H, Lq, device=DEV)
        assert lib.pvb2_sdpa_fwd(ctypes.byref(d), ctypes.byref(td(qd)), ctypes.byref(td(kd)), ctypes.byref(td(vd)),
                                 ctypes.byref(td(od)), ctypes.c_void_p(lse.data_ptr()), stream) == 0
        full = lib.pvb2_sdpa_bwd_workspace_size(ctypes.byref(d))
        di_only = (B * H * Lq * 4 + 255) // 256 * 256
        assert full > di_only
        q64, k64, v64 = (t.double().requires_grad_() for t in (q, k, v))
        s = q64 @ k64.transpose(-1, -2) / math.sqrt(D)
        if causal:
            s = s.masked_fill(torch.ones(Lq, Lk, dtype=torch.bool).triu(1), float("-inf"))
        (torch.softmax(s, -1) @ v64).backward(dout.double())
        for ws_bytes in (full, di_only):
            ws = torch.empty(ws_bytes // 4, device=DEV)
            dq, dk, dv = torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)
            rc = lib.pvb2_sdpa_bwd(ctypes.byref(d), ctypes.byref(td(qd)), ctypes.byref(td(kd)),
                                   ctypes.byref(td(vd)), ctypes.byref(td(od)), ctypes.byref(td(gd)),
                                   ctypes.c_void_p(lse.data_ptr()), ctypes.byref(td(dq)), ctypes.byref(td(dk)),
                                   ctypes.byref(td(dv)), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws_bytes),
                                   stream)
            assert rc == 0, lib.pvb2_last_error()
            assert _rel(q64.grad, dq) < 1e-5
            assert _rel(k64.grad, dk) < 1e-5
            assert _rel(v64.grad, dv) < 1e-5
        too_small = torch.empty(16, device=DEV)
        rc = lib.pvb2_sdpa_bwd(ctypes.byref(d), ctypes.byref(td(qd)), ctypes.byref(td(kd)), ctypes.byref(td(vd)),
                               ctypes.byref(td(od)), ctypes.byref(td(gd)), ctypes.c_void_p(lse.data_ptr()),
                               ctypes.byref(td(dq)), ctypes.byref(td(dk)), ctypes.byref(td(dv)),
                               ctypes.c_void_p(too_small.data_ptr()), ctypes.c_size_t(64), stream)
        assert rc != 0 and b"workspace" in lib.pvb2_last_error()
