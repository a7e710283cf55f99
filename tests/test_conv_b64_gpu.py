"""Every distinct convolution of ResNet-50 at the benchmark's batch of 64,
through the C-ABI in TF32 math, against the TF32-emulating float64 oracle.

The tile, split-K, phase and staging plans of the tensor-core convolutions
are chosen from N*P*Q and the channel counts, so the plans the benchmark runs
are the ones a batch-64 test has to exercise.  For each geometry:

* forward, input gradient (dgrad) and weight gradient (wgrad) through
  pvb2_conv2d_fwd / _bwd_data / _bwd_filter;
* the staged pair (pvb2_conv2d_fwd_staged keeps the channels-last / im2col
  copy, pvb2_conv2d_bwd_filter_staged reads it): bit-identical to the plain
  forward and weight gradient;
* the accumulating dgrad (pvb2_conv2d_bwd_data_acc) where the geometry
  allows it: bit-identical to the plain dgrad plus the addend in fp32.

Oracle: float64 convolution of operands cut to TF32 (``oracle.tf32.cut_tf32``,
the tensor core's conversion), so the device's only remaining error is its
fp32 accumulation; the elementwise bound is 2^-17 x the same convolution of
the absolute values (the TF32 rounding bound of the per-op tests,
test_capi_gpu.py, is 2^-9; the largest error measured on a B200 is 1.2e-6
of |x||w|, 0.16 of this bound, while plain fp32 arithmetic without the TF32
cut lands 13-95x above it, so the bound tells the two apart).  To keep the CPU side to seconds the forward and
dgrad are checked on three whole images (0, 37, 63: each image's output
depends only on its own input) and the weight gradient on eight output
channels spread over K (each reduces over all 64 images).
"""
import ctypes
import json
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle.tf32 import cut_tf32
from test_capi_gpu import LIB, Conv, ok, stream, sync, td

pytestmark = pytest.mark.gpu
DEV = "ocl:0"
BOUND = 2.0 ** -17
IMAGES = [0, 37, 63]

# N, C, H, W, K, R, stride, pad  (every distinct geometry of torchvision's resnet50, batch 64)
R50 = [
    (64, 3, 224, 224, 64, 7, 2, 3),      # stem (im2col columns)
    (64, 64, 56, 56, 64, 1, 1, 0),       # layer1.0.conv1
    (64, 64, 56, 56, 64, 3, 1, 1),       # layer1 3x3
    (64, 64, 56, 56, 256, 1, 1, 0),      # layer1 conv3, layer1.0.downsample
    (64, 256, 56, 56, 64, 1, 1, 0),      # layer1.1/2.conv1
    (64, 256, 56, 56, 128, 1, 1, 0),     # layer2.0.conv1
    (64, 128, 56, 56, 128, 3, 2, 1),     # layer2.0.conv2 (strided 3x3)
    (64, 128, 28, 28, 512, 1, 1, 0),     # layer2 conv3
    (64, 256, 56, 56, 512, 1, 2, 0),     # layer2.0.downsample (strided 1x1)
    (64, 512, 28, 28, 128, 1, 1, 0),     # layer2.1-3.conv1
    (64, 128, 28, 28, 128, 3, 1, 1),     # layer2 3x3
    (64, 512, 28, 28, 256, 1, 1, 0),     # layer3.0.conv1
    (64, 256, 28, 28, 256, 3, 2, 1),     # layer3.0.conv2
    (64, 256, 14, 14, 1024, 1, 1, 0),    # layer3 conv3
    (64, 512, 28, 28, 1024, 1, 2, 0),    # layer3.0.downsample
    (64, 1024, 14, 14, 256, 1, 1, 0),    # layer3.1-5.conv1
    (64, 256, 14, 14, 256, 3, 1, 1),     # layer3 3x3
    (64, 1024, 14, 14, 512, 1, 1, 0),    # layer4.0.conv1
    (64, 512, 14, 14, 512, 3, 2, 1),     # layer4.0.conv2
    (64, 512, 7, 7, 2048, 1, 1, 0),      # layer4 conv3
    (64, 1024, 14, 14, 2048, 1, 2, 0),   # layer4.0.downsample
    (64, 2048, 7, 7, 512, 1, 1, 0),      # layer4.1-2.conv1
    (64, 512, 7, 7, 512, 3, 1, 1),       # layer4 3x3
]


@pytest.fixture(scope="module")
def lib(ocl):
    L = ctypes.CDLL(LIB)
    L.pvb2_last_error.restype = ctypes.c_char_p
    L.pvb2_conv2d_workspace_size.restype = ctypes.c_size_t
    L.pvb2_conv2d_staged_input_bytes.restype = ctypes.c_size_t
    return L


def _ws(lib, d, which):
    return torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), which), 16), dtype=torch.uint8).to(DEV)


def _check(name, got, ref, scale, geom):
    err = (got - ref).abs()
    ratio = (err / (BOUND * scale + 1e-30)).max().item()
    path = os.environ.get("PVB2_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"test": f"conv_b64_{name}", "geom": geom, "max_ratio_to_bound": ratio,
                                "max_rel_to_abs_conv": (err / (scale + 1e-30)).max().item()}) + "\n")
    assert ratio <= 1.0, f"{name}: error {ratio:.3g}x the bound 2^-17 * |x||w| (geometry {geom})"


@pytest.mark.parametrize("geom", R50, ids=["x".join(map(str, g)) for g in R50])
def test_resnet50_conv_b64(lib, geom):
    N, C, H, W, K, R, st, pd = geom
    P = (H + 2 * pd - R) // st + 1
    d = Conv(N, C, H, W, K, R, R, P, P, st, st, pd, pd, 1, 1, 1, 0)
    assert lib.pvb2_conv2d_path(ctypes.byref(d), 0) == 1
    assert lib.pvb2_conv2d_path(ctypes.byref(d), 1) == 1
    assert lib.pvb2_conv2d_path(ctypes.byref(d), 2) == 1
    g = torch.Generator().manual_seed(sum(geom))
    x = torch.randn(N, C, H, W, generator=g)
    w = torch.randn(K, C, R, R, generator=g) * (2.0 / (C * R * R)) ** 0.5
    gy = torch.randn(N, K, P, P, generator=g)
    xd, wd, gyd = x.to(DEV), w.to(DEV), gy.to(DEV)
    y = torch.empty(N, K, P, P).to(DEV)
    gx = torch.empty(N, C, H, W).to(DEV)
    gw = torch.empty(K, C, R, R).to(DEV)
    ws0, ws1, ws2 = _ws(lib, d, 0), _ws(lib, d, 1), _ws(lib, d, 2)
    sync()
    s = stream()
    ok(lib, lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(td(xd)), ctypes.c_void_p(wd.data_ptr()), None,
                                ctypes.byref(td(y)), ctypes.c_void_p(ws0.data_ptr()), ctypes.c_size_t(ws0.numel()), s))
    ok(lib, lib.pvb2_conv2d_bwd_data(ctypes.byref(d), ctypes.byref(td(gyd)), ctypes.c_void_p(wd.data_ptr()),
                                     ctypes.byref(td(gx)), ctypes.c_void_p(ws1.data_ptr()),
                                     ctypes.c_size_t(ws1.numel()), s))
    ok(lib, lib.pvb2_conv2d_bwd_filter(ctypes.byref(d), ctypes.byref(td(xd)), ctypes.byref(td(gyd)),
                                       ctypes.c_void_p(gw.data_ptr()), None, ctypes.c_void_p(ws2.data_ptr()),
                                       ctypes.c_size_t(ws2.numel()), s))
    sync()

    # staged pair: same bits as the plain forward and weight gradient
    nb = lib.pvb2_conv2d_staged_input_bytes(ctypes.byref(d))
    if nb:
        buf = torch.empty(nb, dtype=torch.uint8).to(DEV)
        y2 = torch.empty_like(y)
        gw2 = torch.empty_like(gw)
        written = ctypes.c_int(-1)
        ok(lib, lib.pvb2_conv2d_fwd_staged(ctypes.byref(d), ctypes.byref(td(xd)), ctypes.c_void_p(wd.data_ptr()),
                                           None, ctypes.byref(td(y2)), ctypes.c_void_p(ws0.data_ptr()),
                                           ctypes.c_size_t(ws0.numel()), ctypes.c_void_p(buf.data_ptr()),
                                           ctypes.c_size_t(nb), ctypes.byref(written), s))
        ok(lib, lib.pvb2_conv2d_bwd_filter_staged(ctypes.byref(d), ctypes.byref(td(xd)), ctypes.byref(td(gyd)),
                                                  ctypes.c_void_p(gw2.data_ptr()), None,
                                                  ctypes.c_void_p(ws2.data_ptr()), ctypes.c_size_t(ws2.numel()),
                                                  ctypes.c_void_p(buf.data_ptr()), ctypes.c_size_t(nb), s))
        sync()
        assert written.value == 1
        assert torch.equal(y2.cpu(), y.cpu()), "staged forward differs from the plain forward"
        assert torch.equal(gw2.cpu(), gw.cpu()), "weight gradient from the staged copy differs from the plain one"

    # accumulating dgrad: dgrad + addend rounded once, as a separate fp32 add
    if lib.pvb2_conv2d_bwd_data_acc_ok(ctypes.byref(d), ctypes.c_void_p(gyd.data_ptr()),
                                       ctypes.c_void_p(wd.data_ptr()), ctypes.c_void_p(gx.data_ptr()),
                                       ctypes.c_void_p(gx.data_ptr())):
        addend = torch.randn(N, C, H, W, generator=g).to(DEV)
        acc = torch.empty_like(gx)
        ok(lib, lib.pvb2_conv2d_bwd_data_acc(ctypes.byref(d), ctypes.byref(td(gyd)), ctypes.c_void_p(wd.data_ptr()),
                                             ctypes.byref(td(acc)), ctypes.byref(td(addend)), s))
        sync()
        assert torch.equal(acc.cpu(), gx.cpu() + addend.cpu()), "accumulating dgrad differs from dgrad + addend"

    # oracle: float64 on TF32-cut operands
    xt, wt, gt = cut_tf32(x).double(), cut_tf32(w).double(), cut_tf32(gy).double()
    im = torch.tensor(IMAGES)
    yref = F.conv2d(xt[im], wt, None, st, pd)
    yabs = F.conv2d(xt[im].abs(), wt.abs(), None, st, pd)
    _check("fwd", y.cpu()[im].double(), yref, yabs, geom)
    gxref = torch.nn.grad.conv2d_input((len(IMAGES), C, H, W), wt, gt[im], st, pd)
    gxabs = torch.nn.grad.conv2d_input((len(IMAGES), C, H, W), wt.abs(), gt[im].abs(), st, pd)
    _check("dgrad", gx.cpu()[im].double(), gxref, gxabs, geom)
    ks = torch.linspace(0, K - 1, 8).round().long().unique()
    gwref = torch.nn.grad.conv2d_weight(xt, (len(ks), C, R, R), gt[:, ks], st, pd)
    gwabs = torch.nn.grad.conv2d_weight(xt.abs(), (len(ks), C, R, R), gt[:, ks].abs(), st, pd)
    _check("wgrad", gw.cpu()[ks].double(), gwref, gwabs, geom)


def test_tensor_core_operand_conversion_is_truncation(lib):
    """The oracle's TF32 conversion is the hardware's: a GEMM on the tensor
    cores of A = 1 + 0.75 * 2^-10 (three quarters of a TF32 unit above 1)
    against B = 1 gives K * 1 (truncation), not K * (1 + 2^-10) (rounding)."""
    M = N = K = 256
    ulp = 2.0 ** -10
    a = torch.full((1, M, K), 1.0 + 0.75 * ulp).to(DEV)
    b = torch.ones(1, K, N).to(DEV)
    c = torch.empty(1, M, N).to(DEV)
    A, B, Cd = td(a), td(b), td(c)
    assert lib.pvb2_gemm_path(ctypes.byref(A), ctypes.byref(B), ctypes.byref(Cd), 0) == 1
    sync()
    ok(lib, lib.pvb2_gemm(ctypes.byref(A), ctypes.byref(B), ctypes.byref(Cd), None, 1, ctypes.c_double(1.0),
                          ctypes.c_double(0.0), 0, stream()))
    sync()
    assert torch.equal(c.cpu(), torch.full((1, M, N), float(K)))
    # the same through a 1x1 convolution (pointwise tensor-core path)
    d = Conv(1, 64, 32, 32, 256, 1, 1, 32, 32, 1, 1, 0, 0, 1, 1, 1, 0)
    assert lib.pvb2_conv2d_path(ctypes.byref(d), 0) == 1
    x = torch.full((1, 64, 32, 32), 1.0 + 0.75 * ulp).to(DEV)
    w = torch.ones(256, 64, 1, 1).to(DEV)
    y = torch.empty(1, 256, 32, 32).to(DEV)
    ws = _ws(lib, d, 0)
    sync()
    ok(lib, lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(td(x)), ctypes.c_void_p(w.data_ptr()), None,
                                ctypes.byref(td(y)), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()),
                                stream()))
    sync()
    assert torch.equal(y.cpu(), torch.full((1, 256, 32, 32), 64.0))
    np.testing.assert_array_equal(y.cpu().numpy(), 64.0)
