"""The staged convolution input kept from a training forward for the weight
gradient: the C-ABI pair pvb2_conv2d_fwd_staged / pvb2_conv2d_bwd_filter_staged
gives the same weight gradient, bit for bit, as the plain pvb2_conv2d_bwd_filter
(which stages x itself), and the host cache behind autograd hands the copy
only to the backward of the same input and geometry."""
import ctypes

import numpy as np
import pytest
import torch
import torch.nn as nn

import pytorch_vulkan_b200 as p
from test_capi_gpu import LIB, Conv, ok, stream, sync, td

pytestmark = pytest.mark.gpu
DEV = "ocl:0"


@pytest.fixture(scope="module")
def lib(ocl):
    L = ctypes.CDLL(LIB)
    L.pvb2_last_error.restype = ctypes.c_char_p
    L.pvb2_conv2d_workspace_size.restype = ctypes.c_size_t
    L.pvb2_conv2d_staged_input_bytes.restype = ctypes.c_size_t
    L.pvb2_conv2d_staged_grad_bytes.restype = ctypes.c_size_t
    return L


STAGED_SHAPES = [
    # N, C, H, W, K, R, S, stride, pad, dil, staged
    (2, 64, 56, 56, 64, 3, 3, 1, 1, 1, True),      # ResNet layer1 3x3: channels-last copy
    (2, 128, 28, 28, 128, 3, 3, 2, 1, 1, True),    # stride-2 3x3
    (2, 3, 64, 64, 64, 7, 7, 2, 3, 1, True),       # stem
    (2, 1, 28, 28, 32, 5, 5, 1, 0, 1, True),       # MNIST conv1: im2col columns
    (2, 3, 224, 224, 768, 16, 16, 16, 0, 1, True),  # ViT-B/16 patch embedding: im2col columns
    (2, 64, 14, 14, 128, 1, 1, 1, 0, 1, False),    # pointwise: reads NCHW, nothing staged
    (2, 64, 16, 16, 128, 1, 1, 2, 0, 1, False),    # strided 1x1: subsampled, nothing kept
    (2, 64, 14, 14, 128, 1, 1, 2, 0, 1, True),     # strided 1x1 with 49 sampled pixels: channels-last copy
]


@pytest.mark.parametrize("shape", STAGED_SHAPES, ids=["x".join(map(str, s[:10])) for s in STAGED_SHAPES])
def test_staged_wgrad_matches_plain(lib, shape):
    N, C, H, W, K, R, S, st, pd, dl, staged = shape
    P = (H + 2 * pd - dl * (R - 1) - 1) // st + 1
    Q = (W + 2 * pd - dl * (S - 1) - 1) // st + 1
    d = Conv(N, C, H, W, K, R, S, P, Q, st, st, pd, pd, dl, dl, 1, 0)
    nbytes = lib.pvb2_conv2d_staged_input_bytes(ctypes.byref(d))
    assert (nbytes > 0) == staged
    exact = Conv(N, C, H, W, K, R, S, P, Q, st, st, pd, pd, dl, dl, 1, 1)
    assert lib.pvb2_conv2d_staged_input_bytes(ctypes.byref(exact)) == 0  # exact fp32 path stages nothing
    g = torch.Generator().manual_seed(sum(shape[:10]))
    x = torch.randn(N, C, H, W, generator=g).to(DEV)
    w = (torch.randn(K, C, R, S, generator=g) * 0.1).to(DEV)
    gy = torch.randn(N, K, P, Q, generator=g).to(DEV)
    y = torch.empty(N, K, P, Q).to(DEV)
    buf = torch.empty(max(nbytes, 16), dtype=torch.uint8).to(DEV)
    ws0 = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 0), 4), dtype=torch.uint8).to(DEV)
    ws2 = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 2), 4), dtype=torch.uint8).to(DEV)
    written = ctypes.c_int(-1)
    sync()
    ok(lib, lib.pvb2_conv2d_fwd_staged(ctypes.byref(d), ctypes.byref(td(x)), ctypes.c_void_p(w.data_ptr()), None,
                                       ctypes.byref(td(y)), ctypes.c_void_p(ws0.data_ptr()),
                                       ctypes.c_size_t(ws0.numel()), ctypes.c_void_p(buf.data_ptr()),
                                       ctypes.c_size_t(nbytes), ctypes.byref(written), stream()))
    sync()
    assert written.value == (1 if staged else 0)
    y_plain = torch.empty_like(y)
    ok(lib, lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(td(x)), ctypes.c_void_p(w.data_ptr()), None,
                                ctypes.byref(td(y_plain)), ctypes.c_void_p(ws0.data_ptr()),
                                ctypes.c_size_t(ws0.numel()), stream()))
    sync()
    assert torch.equal(y.cpu(), y_plain.cpu())
    gw_plain, gw_staged = torch.empty(w.shape).to(DEV), torch.empty(w.shape).to(DEV)
    ok(lib, lib.pvb2_conv2d_bwd_filter(ctypes.byref(d), ctypes.byref(td(x)), ctypes.byref(td(gy)),
                                       ctypes.c_void_p(gw_plain.data_ptr()), None, ctypes.c_void_p(ws2.data_ptr()),
                                       ctypes.c_size_t(ws2.numel()), stream()))
    if staged:
        ok(lib, lib.pvb2_conv2d_bwd_filter_staged(
            ctypes.byref(d), ctypes.byref(td(x)), ctypes.byref(td(gy)), ctypes.c_void_p(gw_staged.data_ptr()), None,
            ctypes.c_void_p(ws2.data_ptr()), ctypes.c_size_t(ws2.numel()), ctypes.c_void_p(buf.data_ptr()),
            ctypes.c_size_t(nbytes), stream()))
        sync()
        assert torch.equal(gw_plain.cpu(), gw_staged.cpu())
    else:
        # a staged copy that this convolution never makes is refused
        st_ = lib.pvb2_conv2d_bwd_filter_staged(
            ctypes.byref(d), ctypes.byref(td(x)), ctypes.byref(td(gy)), ctypes.c_void_p(gw_staged.data_ptr()), None,
            ctypes.c_void_p(ws2.data_ptr()), ctypes.c_size_t(ws2.numel()), ctypes.c_void_p(buf.data_ptr()),
            ctypes.c_size_t(16), stream())
        sync()
        assert st_ != 0
    ref = torch.nn.grad.conv2d_weight(x.cpu().double(), w.shape, gy.cpu().double(), st, pd, dl)
    # TF32 products carry a relative error below 2^-9
    bound = 2.0 ** -9 * torch.nn.grad.conv2d_weight(x.cpu().double().abs(), w.shape,
                                                gy.cpu().double().abs(), st, pd, dl) + 1e-4
    assert bool(((gw_plain.cpu().double() - ref).abs() <= bound).all())


GRAD_SHAPES = [
    # N, C, H, W, K, R, S, stride, pad, dil, staged
    (2, 64, 56, 56, 64, 3, 3, 1, 1, 1, True),      # ResNet layer1 3x3
    (2, 128, 28, 28, 128, 3, 3, 2, 1, 1, True),    # stride-2 3x3: four input-gradient phases read the copy
    (3, 512, 7, 7, 512, 3, 3, 1, 1, 1, True),      # layer4 3x3: split-K input gradient
    (2, 512, 7, 7, 256, 1, 1, 1, 0, 1, True),      # 1x1 on 49-pixel planes: tap-box path
    (2, 20, 17, 17, 40, 7, 7, 1, 3, 1, True),      # 7x7, K padded to 40
    (2, 3, 64, 64, 64, 7, 7, 2, 3, 1, False),      # stem: the weight gradient reads NCHW dy (window path)
    (2, 64, 14, 14, 128, 1, 1, 1, 0, 1, False),    # pointwise: NCHW throughout
]


@pytest.mark.parametrize("shape", GRAD_SHAPES, ids=["x".join(map(str, s[:10])) for s in GRAD_SHAPES])
def test_staged_grad_matches_plain(lib, shape):
    """pvb2_conv2d_bwd_data_staged leaves its channels-last dy for
    pvb2_conv2d_bwd_filter_staged_grad: input and weight gradients are bit
    for bit those of the plain calls (each staging dy itself)"""
    N, C, H, W, K, R, S, st, pd, dl, staged = shape
    P = (H + 2 * pd - dl * (R - 1) - 1) // st + 1
    Q = (W + 2 * pd - dl * (S - 1) - 1) // st + 1
    d = Conv(N, C, H, W, K, R, S, P, Q, st, st, pd, pd, dl, dl, 1, 0)
    nbytes = lib.pvb2_conv2d_staged_grad_bytes(ctypes.byref(d))
    assert (nbytes > 0) == staged
    exact = Conv(N, C, H, W, K, R, S, P, Q, st, st, pd, pd, dl, dl, 1, 1)
    assert lib.pvb2_conv2d_staged_grad_bytes(ctypes.byref(exact)) == 0
    g = torch.Generator().manual_seed(sum(shape[:10]) + 1)
    x = torch.randn(N, C, H, W, generator=g).to(DEV)
    w = (torch.randn(K, C, R, S, generator=g) * 0.1).to(DEV)
    gy = torch.randn(N, K, P, Q, generator=g).to(DEV)
    buf = torch.empty(max(nbytes, 16), dtype=torch.uint8).to(DEV)
    ws1 = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 1), 4), dtype=torch.uint8).to(DEV)
    ws2 = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 2), 4), dtype=torch.uint8).to(DEV)
    gx_plain, gx_staged = torch.empty(x.shape).to(DEV), torch.empty(x.shape).to(DEV)
    gw_plain, gw_staged = torch.empty(w.shape).to(DEV), torch.empty(w.shape).to(DEV)
    wp = ctypes.c_void_p(w.data_ptr())
    sync()
    ok(lib, lib.pvb2_conv2d_bwd_data(ctypes.byref(d), ctypes.byref(td(gy)), wp, ctypes.byref(td(gx_plain)),
                                     ctypes.c_void_p(ws1.data_ptr()), ctypes.c_size_t(ws1.numel()), stream()))
    ok(lib, lib.pvb2_conv2d_bwd_filter(ctypes.byref(d), ctypes.byref(td(x)), ctypes.byref(td(gy)),
                                       ctypes.c_void_p(gw_plain.data_ptr()), None, ctypes.c_void_p(ws2.data_ptr()),
                                       ctypes.c_size_t(ws2.numel()), stream()))
    written = ctypes.c_int(-1)
    ok(lib, lib.pvb2_conv2d_bwd_data_staged(ctypes.byref(d), ctypes.byref(td(gy)), wp, ctypes.byref(td(gx_staged)),
                                            ctypes.c_void_p(ws1.data_ptr()), ctypes.c_size_t(ws1.numel()),
                                            ctypes.c_void_p(buf.data_ptr()), ctypes.c_size_t(nbytes),
                                            ctypes.byref(written), stream()))
    sync()
    assert written.value == (1 if staged else 0)
    assert torch.equal(gx_plain.cpu(), gx_staged.cpu())
    st_ = lib.pvb2_conv2d_bwd_filter_staged_grad(
        ctypes.byref(d), ctypes.byref(td(x)), ctypes.byref(td(gy)), ctypes.c_void_p(gw_staged.data_ptr()), None,
        ctypes.c_void_p(ws2.data_ptr()), ctypes.c_size_t(ws2.numel()), None, ctypes.c_size_t(0),
        ctypes.c_void_p(buf.data_ptr()), ctypes.c_size_t(max(nbytes, 16)), stream())
    sync()
    if staged:
        ok(lib, st_)
        assert torch.equal(gw_plain.cpu(), gw_staged.cpu())
    else:
        assert st_ != 0  # a staged dy that this convolution never makes is refused
    ref = torch.nn.grad.conv2d_input(x.shape, w.cpu().double(), gy.cpu().double(), st, pd, dl)
    bound = 2.0 ** -9 * torch.nn.grad.conv2d_input(x.shape, w.cpu().double().abs(), gy.cpu().double().abs(), st,
                                                   pd, dl) + 1e-4
    assert bool(((gx_plain.cpu().double() - ref).abs() <= bound).all())


def test_autograd_backward_keeps_staged_grad(ocl):
    """through autograd (convolution_backward passing the staged dy from the
    input gradient to the weight gradient) the gradients equal those of the
    exact path within the TF32 bound, for a 3x3 and a 7x7-plane 1x1 layer"""
    old = torch.ocl.get_math_mode()
    try:
        for (C, K, R, hw) in [(32, 48, 3, 20), (64, 96, 1, 7)]:
            torch.manual_seed(11)
            conv = nn.Conv2d(C, K, R, padding=R // 2, bias=False).to(DEV)
            x0 = torch.randn(4, C, hw, hw)
            g0 = torch.randn(4, K, hw, hw)
            grads = []
            for mode in (0, 1):
                torch.ocl.set_math_mode(mode)
                conv.zero_grad()
                x = x0.to(DEV).requires_grad_()
                conv(x).backward(g0.to(DEV))
                grads.append((x.grad.cpu().double(), conv.weight.grad.cpu().double()))
            for a, b in zip(*grads):
                assert (a - b).abs().max().item() <= 2e-3 * max(1.0, b.abs().max().item())
    finally:
        torch.ocl.set_math_mode(old)


def _grads(conv, xs, clear_between):
    conv.zero_grad()
    ys = [conv(x) for x in xs]
    if clear_between:
        torch.ocl.empty_cache()
    loss = sum((y * (i + 1)).sum() for i, y in enumerate(ys))
    loss.backward()
    torch.ocl.synchronize()
    return conv.weight.grad.cpu().clone()


@pytest.mark.parametrize("spec", [(16, 32, 3, 1, 1, 20), (3, 16, 7, 2, 3, 32), (1, 32, 5, 1, 0, 28)],
                         ids=["3x3", "7x7s2", "5x5"])
def test_autograd_cache_hands_copy_to_matching_backward(ocl, spec):
    """Two inputs through one convolution, their backwards in reverse order:
    each weight-gradient term must read its own input's copy.  The result is
    bit-identical to the run whose copies were dropped before the backward
    (the weight gradient staged each input again), and matches the CPU."""
    C, K, R, st, pd, hw = spec
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(0)
    try:
        torch.manual_seed(7)
        ref = nn.Conv2d(C, K, R, stride=st, padding=pd, bias=False)
        conv = nn.Conv2d(C, K, R, stride=st, padding=pd, bias=False).to(DEV)
        conv.load_state_dict(ref.state_dict())
        xs_cpu = [torch.randn(2, C, hw, hw), torch.randn(2, C, hw, hw)]
        xs = [x.to(DEV) for x in xs_cpu]
        torch.ocl.empty_cache()
        with torch.no_grad():
            conv(xs[0])
        assert p._C.impl_staged_input_bytes() == 0  # nothing kept without grad mode
        conv.zero_grad()
        ys = [conv(x) for x in xs]
        assert p._C.impl_staged_input_bytes() > 0
        sum((y * (i + 1)).sum() for i, y in enumerate(ys)).backward()
        assert p._C.impl_staged_input_bytes() == 0  # each backward took its copy
        g_cached = conv.weight.grad.cpu().clone()
        g_restaged = _grads(conv, xs, clear_between=True)
        assert torch.equal(g_cached, g_restaged)
        ys_ref = [ref(x) for x in xs_cpu]
        sum((y * (i + 1)).sum() for i, y in enumerate(ys_ref)).backward()
        err = (g_cached.double() - ref.weight.grad.double()).abs().max().item()
        assert err <= 2e-3 + 5e-3 * ref.weight.grad.abs().max().item()
    finally:
        torch.ocl.set_math_mode(old)


def test_autograd_cache_ignores_changed_or_freed_inputs(ocl):
    """A copy is used only for the very input it was made from: a
    non-contiguous input is staged from a temporary that the forward frees,
    so its backward stages again and still gets the CPU's gradient; a copy
    whose input is freed without a backward is dropped on the next forward."""
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(0)
    try:
        torch.manual_seed(3)
        ref = nn.Conv2d(8, 16, 3, padding=1, bias=False)
        conv = nn.Conv2d(8, 16, 3, padding=1, bias=False).to(DEV)
        conv.load_state_dict(ref.state_dict())
        torch.ocl.empty_cache()
        xc = torch.randn(2, 20, 20, 8)
        x = xc.to(DEV).permute(0, 3, 1, 2)  # non-contiguous: the forward stages a temporary copy
        conv(x).sum().backward()
        ref(xc.permute(0, 3, 1, 2)).sum().backward()
        err = (conv.weight.grad.cpu().double() - ref.weight.grad.double()).abs().max().item()
        assert err <= 2e-3 + 5e-3 * ref.weight.grad.abs().max().item()
        torch.ocl.empty_cache()
        assert p._C.impl_staged_input_bytes() == 0
        # an entry whose input was never used by a backward goes when the
        # input's storage is freed (checked on the next forward)
        a = torch.randn(2, 8, 20, 20).to(DEV)
        conv(a)
        kept = p._C.impl_staged_input_bytes()
        assert kept > 0
        del a
        b = torch.randn(2, 8, 20, 20).to(DEV)
        conv(b)
        assert p._C.impl_staged_input_bytes() == kept
        # an input modified in place after its forward: its copy can never
        # be used again and goes on the next forward
        b.add_(1.0)
        c = torch.randn(2, 8, 20, 20).to(DEV)
        conv(c)
        assert p._C.impl_staged_input_bytes() == kept
        torch.ocl.empty_cache()
        assert p._C.impl_staged_input_bytes() == 0
    finally:
        torch.ocl.set_math_mode(old)
