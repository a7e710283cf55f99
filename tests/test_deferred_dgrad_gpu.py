"""Input gradient of a 1x1 stride-1 convolution summed in the dgrad's
epilogue: pvb2_conv2d_bwd_data_acc gives dgrad + addend rounded once (the
separate add's result, bit for bit), and the host defers such a dgrad so
that the autograd engine's sum of a residual block's two input gradients
joins it (csrc/host/deferred.cpp).  Every other reader of the gradient sees
the plain dgrad."""
import csv
import ctypes
import os
import tempfile

import pytest
import torch
import torch.nn as nn

from test_capi_gpu import LIB, Conv, ok, stream, sync, td

pytestmark = pytest.mark.gpu
DEV = "ocl:0"


@pytest.fixture(scope="module")
def lib(ocl):
    L = ctypes.CDLL(LIB)
    L.pvb2_last_error.restype = ctypes.c_char_p
    L.pvb2_conv2d_workspace_size.restype = ctypes.c_size_t
    return L


ACC_SHAPES = [
    # N, C, H, W, K
    (2, 64, 56, 56, 256),   # ResNet layer1 bottleneck conv1 (its dgrad: 256 -> 64 channels)
    (3, 36, 12, 12, 40),    # channel tails, 144-pixel planes (part-empty slots)
    (2, 128, 28, 28, 512),  # layer2 conv1
    (4, 256, 14, 14, 64),
]


@pytest.mark.parametrize("inplace", [False, True], ids=["out", "inplace"])
@pytest.mark.parametrize("shape", ACC_SHAPES, ids=["x".join(map(str, s)) for s in ACC_SHAPES])
def test_dgrad_acc_capi_is_dgrad_plus_addend(lib, shape, inplace):
    N, C, H, W, K = shape
    d = Conv(N, C, H, W, K, 1, 1, H, W, 1, 1, 0, 0, 1, 1, 1, 0)
    g = torch.Generator().manual_seed(sum(shape))
    gy = torch.randn(N, K, H, W, generator=g).to(DEV)
    w = (torch.randn(K, C, 1, 1, generator=g) * 0.1).to(DEV)
    addend = torch.randn(N, C, H, W, generator=g).to(DEV)
    plain = torch.empty(N, C, H, W).to(DEV)
    ws = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 1), 4), dtype=torch.uint8).to(DEV)
    sync()
    ok(lib, lib.pvb2_conv2d_bwd_data(ctypes.byref(d), ctypes.byref(td(gy)), ctypes.c_void_p(w.data_ptr()),
                                     ctypes.byref(td(plain)), ctypes.c_void_p(ws.data_ptr()),
                                     ctypes.c_size_t(ws.numel()), stream()))
    out = addend.clone() if inplace else torch.empty(N, C, H, W).to(DEV)
    src = out if inplace else addend
    sync()
    assert lib.pvb2_conv2d_bwd_data_acc_ok(ctypes.byref(d), ctypes.c_void_p(gy.data_ptr()),
                                           ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                           ctypes.c_void_p(src.data_ptr())) == 1
    ok(lib, lib.pvb2_conv2d_bwd_data_acc(ctypes.byref(d), ctypes.byref(td(gy)), ctypes.c_void_p(w.data_ptr()),
                                         ctypes.byref(td(out)), ctypes.byref(td(src)), stream()))
    sync()
    expect = plain.cpu() + addend.cpu()  # fp32 add, rounded once
    assert torch.equal(out.cpu(), expect)


def test_dgrad_acc_refuses_other_convolutions(lib):
    d = Conv(2, 64, 14, 14, 64, 3, 3, 14, 14, 1, 1, 1, 1, 1, 1, 1, 0)  # 3x3
    t = torch.empty(2, 64, 14, 14).to(DEV)
    w = torch.empty(64, 64, 3, 3).to(DEV)
    p = ctypes.c_void_p(t.data_ptr())
    assert lib.pvb2_conv2d_bwd_data_acc_ok(ctypes.byref(d), p, ctypes.c_void_p(w.data_ptr()), p, p) == 0
    st = lib.pvb2_conv2d_bwd_data_acc(ctypes.byref(d), ctypes.byref(td(t)), ctypes.c_void_p(w.data_ptr()),
                                      ctypes.byref(td(t)), ctypes.byref(td(t)), stream())
    assert st == 2  # PVB2_ERR_UNSUPPORTED
    exact = Conv(2, 64, 14, 14, 64, 1, 1, 14, 14, 1, 1, 0, 0, 1, 1, 1, 1)  # exact fp32 math: SIMT path
    assert lib.pvb2_conv2d_bwd_data_acc_ok(ctypes.byref(exact), p, ctypes.c_void_p(w.data_ptr()), p, p) == 0
    # 7x7 planes: rows of 49 floats are not 16-byte runs, so the 1x1 dgrad is
    # not a pointwise GEMM there
    seven = Conv(2, 512, 7, 7, 2048, 1, 1, 7, 7, 1, 1, 0, 0, 1, 1, 1, 0)
    assert lib.pvb2_conv2d_bwd_data_acc_ok(ctypes.byref(seven), p, ctypes.c_void_p(w.data_ptr()), p, p) == 0


class _Block(nn.Module):
    """x -> 1x1 conv -> 3x3 conv, plus the identity: the input gradient is
    the 1x1 conv's dgrad + the identity's gradient.  (No ReLU between: under
    TF32 a few pre-activations near zero change sign against the CPU's, and
    the gradient through them with it.)"""

    def __init__(self, C, M):
        super().__init__()
        self.a = nn.Conv2d(C, M, 1, bias=False)
        self.b = nn.Conv2d(M, C, 3, padding=1, bias=False)

    def forward(self, x):
        return x + self.b(self.a(x))


def _op_names(fn):
    path = os.path.join(tempfile.mkdtemp(), "prof.csv")
    with torch.ocl.profile(DEV, path):
        fn()
        torch.ocl.synchronize()
    with open(path) as f:
        return [r["kernel"] for r in csv.DictReader(f)]


def test_residual_input_gradient_joins_dgrad(ocl):
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(0)
    try:
        torch.manual_seed(11)
        ref = _Block(64, 32)
        blk = _Block(64, 32).to(DEV)
        blk.load_state_dict(ref.state_dict())
        xc = torch.randn(4, 64, 16, 16)
        gyc = torch.randn(4, 64, 16, 16)
        x = xc.to(DEV).requires_grad_()
        gy = gyc.to(DEV)
        y = blk(x)
        names = _op_names(lambda: y.backward(gy))
        assert "convolution_backward+add" in names
        # the same sum from separate steps: the 1x1 dgrad alone (read back
        # before anything adds to it), then an fp32 add on the host
        x2 = xc.to(DEV).requires_grad_()
        h = blk.a(x2)
        (gh,) = torch.autograd.grad(blk.b(h), h, gy)
        (g1,) = torch.autograd.grad(blk.a(x2), x2, gh)
        g1c = g1.cpu()
        assert torch.equal(x.grad.cpu(), gyc + g1c)
        # a kept gradient that an add consumed is still written: g1 + gy
        # forms the sum in the dgrad, and g1 itself reads back unchanged
        (g2,) = torch.autograd.grad(blk.a(x2), x2, gh)
        s2 = g2 + gy
        assert torch.equal(s2.cpu(), gyc + g1c)
        assert torch.equal(g2.cpu(), g1c)
        xr = xc.clone().requires_grad_()
        ref(xr).backward(gyc)
        err = (x.grad.cpu().double() - xr.grad.double()).abs().max().item()
        assert err <= 2e-3 + 5e-3 * xr.grad.abs().max().item()
    finally:
        torch.ocl.set_math_mode(old)


def test_pending_dgrad_read_directly(ocl):
    """autograd.grad of the 1x1 conv alone: no add follows, so the pending
    dgrad is launched as it is before anyone reads it."""
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(0)
    try:
        torch.manual_seed(12)
        ref = nn.Conv2d(64, 128, 1, bias=False)
        conv = nn.Conv2d(64, 128, 1, bias=False).to(DEV)
        conv.load_state_dict(ref.state_dict())
        xc, gyc = torch.randn(2, 64, 8, 8), torch.randn(2, 128, 8, 8)
        x = xc.to(DEV).requires_grad_()
        (gx,) = torch.autograd.grad(conv(x), x, gyc.to(DEV))
        xr = xc.clone().requires_grad_()
        (gr,) = torch.autograd.grad(ref(xr), xr, gyc)
        assert (gx.cpu() - gr).abs().max().item() <= 2e-3 + 5e-3 * gr.abs().max().item()
        # accumulating into an existing .grad over two backwards
        x.grad = None
        for _ in range(2):
            conv(x).backward(gyc.to(DEV))
        assert (x.grad.cpu() - 2 * gr).abs().max().item() <= 4e-3 + 1e-2 * gr.abs().max().item()
    finally:
        torch.ocl.set_math_mode(old)
