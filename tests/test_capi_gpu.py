"""Parity through the C-ABI (libpvb2.so via ctypes, no torch dispatcher): each
entry point is called with raw device pointers and checked against the
oracle (numpy restatements in oracle.npref / torch-CPU) on seeded inputs,
including edge cases (empty tensors, ragged sizes, ties in max-pool)."""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import npref

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "pytorch_vulkan_b200", "lib", "libpvb2.so")
DEV = "ocl:0"


class T(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8),
                ("ndim", ctypes.c_int32), ("dtype", ctypes.c_int32)]


DT = {torch.float32: 0, torch.float64: 1, torch.int64: 4, torch.int32: 5, torch.uint8: 8, torch.bool: 9}


def td(t):
    return T(t.data_ptr() if t.numel() else None, (ctypes.c_int64 * 8)(*t.shape), (ctypes.c_int64 * 8)(*t.stride()),
             t.dim(), DT[t.dtype])


class Conv(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ["N", "C", "H", "W", "K", "R", "S", "P", "Q", "stride_h", "stride_w",
                                             "pad_h", "pad_w", "dil_h", "dil_w", "groups", "math"]]


class Pool(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ["kh", "kw", "sh", "sw", "ph", "pw", "dh", "dw", "ceil_mode",
                                             "count_include_pad", "divisor_override"]]


@pytest.fixture(scope="module")
def lib(ocl):
    L = ctypes.CDLL(LIB)
    L.pvb2_last_error.restype = ctypes.c_char_p
    L.pvb2_conv2d_workspace_size.restype = ctypes.c_size_t
    L.pvb2_batch_norm_workspace_size.restype = ctypes.c_size_t
    return L


def stream():
    import pytorch_vulkan_b200 as p

    return ctypes.c_void_p(p._C.impl_stream_handle(0))


def sync():
    torch.ocl.synchronize()


def ok(lib, status):
    assert status == 0, lib.pvb2_last_error().decode()


def dev(x):
    return torch.as_tensor(x).to(DEV)


CONV_SHAPES = [
    # N, C, H, W, K, R, S, stride, pad, dil, groups
    (2, 8, 9, 11, 12, 3, 3, 1, 1, 1, 1),
    (2, 6, 10, 20, 8, 3, 5, 2, 2, 1, 2),
    (3, 16, 7, 7, 32, 1, 1, 1, 0, 1, 1),
    (1, 3, 23, 23, 16, 7, 7, 2, 3, 1, 1),
    (2, 64, 14, 14, 64, 3, 3, 1, 1, 1, 1),
    (2, 128, 8, 8, 256, 1, 1, 2, 0, 1, 1),
    (2, 4, 9, 9, 4, 3, 3, 1, 2, 2, 1),
    # ResNet-50 layer shapes (small batch) that take the tensor-core paths
    (2, 3, 64, 64, 64, 7, 7, 2, 3, 1, 1),        # stem: C=3 padded to 4 channels
    (2, 64, 56, 56, 64, 3, 3, 1, 1, 1, 1),       # layer1 3x3
    (2, 64, 56, 56, 256, 1, 1, 1, 0, 1, 1),      # layer1 1x1 expand
    (2, 128, 28, 28, 128, 3, 3, 2, 1, 1, 1),     # layer2 stride-2 3x3
    (2, 1024, 14, 14, 256, 1, 1, 1, 0, 1, 1),    # layer3 1x1 reduce
    (3, 512, 7, 7, 512, 3, 3, 1, 1, 1, 1),       # layer4 3x3: tiles span two images; split-K fwd / dgrad
    (2, 128, 14, 14, 256, 3, 3, 2, 1, 1, 1),     # strided, few tiles: split-K in every dgrad phase
    (2, 256, 56, 56, 512, 1, 1, 2, 0, 1, 1),     # strided 1x1 projection: pointwise over sampled pixels
    (3, 64, 15, 15, 128, 1, 1, 2, 0, 1, 1),      # strided 1x1 with 8 x 8 = 64 sampled pixels per image
    (2, 64, 14, 14, 128, 1, 1, 2, 0, 1, 1),      # strided 1x1 with 49 sampled pixels: staged path
    (2, 32, 26, 26, 64, 3, 3, 1, 0, 1, 1),       # MNIST conv2
    # weight packing: 49 taps (phase packs of 5 channels), strided 5x5 phases,
    # a channel count padded inside its last 64-channel chunk
    (2, 22, 17, 17, 40, 7, 7, 1, 3, 1, 1),
    (2, 12, 15, 15, 36, 5, 5, 2, 2, 1, 1),
    (2, 66, 9, 9, 20, 3, 3, 1, 1, 1, 1),
    (2, 16, 12, 12, 32, 1, 1, 3, 0, 1, 1),       # strided 1x1 at stride 3: the scatter's runtime-stride form
    # pointwise (1x1, stride 1) paths that read NCHW directly
    (4, 36, 12, 12, 40, 1, 1, 1, 0, 1, 1),       # channel tails, 144-pixel images (part-empty slots)
    (3, 64, 20, 20, 64, 1, 1, 1, 0, 1, 1),       # 13 slots per image: last tile only partly used
    (2, 256, 28, 28, 512, 1, 1, 1, 0, 1, 1),     # layer2 1x1 expand
    (2, 512, 7, 7, 2048, 1, 1, 1, 0, 1, 1),      # 49-pixel images: staged path, direct stores
    # few input channels: GEMMs over im2col columns
    (2, 1, 28, 28, 32, 5, 5, 1, 0, 1, 1),        # MNIST conv1
    (3, 3, 30, 30, 24, 3, 3, 1, 1, 2, 1),        # dilated
    (2, 4, 40, 40, 20, 5, 5, 2, 2, 1, 1),        # strided, 100 columns, output-channel tail
    (2, 3, 224, 224, 768, 16, 16, 16, 0, 1, 1),  # ViT-B/16 patch embedding: 768 columns, stride 16
    # epilogue store boxes
    (4, 64, 14, 14, 100, 3, 3, 1, 1, 1, 1),      # 14-wide rows stored as whole-row runs; output-channel tail
    (2, 16, 112, 112, 24, 3, 3, 1, 1, 1, 1),     # two 64-wide pixel blocks per row
    # many tiles per CTA with fewer output channels than the tile: chunks without a store
    (4, 3, 224, 224, 32, 3, 3, 1, 1, 1, 1),
    (16, 64, 56, 56, 32, 1, 1, 1, 0, 1, 1),
    # depthwise (groups = C = K): MobileNet-v2's 3x3 layers through the direct kernels
    (2, 32, 112, 112, 32, 3, 3, 1, 1, 1, 32),    # 16-byte loads and stores
    (2, 96, 112, 112, 96, 3, 3, 2, 1, 1, 96),    # stride 2: sub-pixel input gradient, 16-byte paths
    (3, 144, 56, 56, 144, 3, 3, 1, 1, 1, 144),
    (2, 192, 28, 28, 192, 3, 3, 2, 1, 1, 192),   # 14-wide outputs: scalar paths
    (4, 576, 14, 14, 576, 3, 3, 2, 1, 1, 576),
    (4, 960, 7, 7, 960, 3, 3, 1, 1, 1, 960),
    (2, 24, 15, 13, 24, 3, 3, 2, 1, 1, 24),      # odd planes at stride 2 (last dX row has one phase)
    (2, 8, 10, 12, 8, 3, 3, 2, 0, 1, 8),         # stride 2 pad 0: tiled input gradient
    (2, 8, 9, 10, 8, 3, 3, 1, 0, 1, 8),          # stride 1 pad 0 (input gradient with pad 2)
    (2, 8, 9, 10, 8, 3, 3, 1, 2, 1, 8),          # stride 1 pad 2 (input gradient with pad 0)
    (2, 16, 20, 20, 16, 5, 5, 1, 2, 1, 16),      # 5x5
    (2, 8, 9, 11, 8, 3, 3, 1, 1, 2, 8),          # dilation 2, odd plane
    (3, 8, 13, 13, 8, 7, 7, 1, 3, 1, 8),         # 7x7 filter: direct kernels
]


@pytest.mark.parametrize("math", [1, 0])
@pytest.mark.parametrize("shape", CONV_SHAPES, ids=["x".join(map(str, s)) for s in CONV_SHAPES])
def test_conv_fwd_bwd_capi(lib, shape, math):
    """fwd / dgrad / wgrad / bias grad through the C-ABI.  Exact-fp32 math is
    checked against the float64 restatement at fp32 accuracy; TF32 math
    against the elementwise bound 2^-9 * (the same conv on |x|, |w|, |dy|),
    since each TF32 product carries a relative error below 2^-9."""
    N, C, H, W, K, R, S, st, pd, dl, g = shape
    rng = np.random.default_rng(sum(shape))
    x = rng.standard_normal((N, C, H, W)).astype(np.float32)
    w = (rng.standard_normal((K, C // g, R, S)) * 0.2).astype(np.float32)
    b = rng.standard_normal(K).astype(np.float32)
    xt = torch.from_numpy(x).double().requires_grad_()
    wt = torch.from_numpy(w).double().requires_grad_()
    yt = torch.nn.functional.conv2d(xt, wt, torch.from_numpy(b).double(), st, pd, dl, g)
    gy = torch.from_numpy(rng.standard_normal(yt.shape).astype(np.float32))
    yt.backward(gy.double())
    # absolute-value run: elementwise error scales
    xa = xt.detach().abs().requires_grad_()
    wa = wt.detach().abs().requires_grad_()
    ya = torch.nn.functional.conv2d(xa, wa, None, st, pd, dl, g)
    ya.backward(gy.double().abs())
    yref = yt.detach().numpy()
    P, Q = yref.shape[2], yref.shape[3]
    d = Conv(N, C, H, W, K, R, S, P, Q, st, st, pd, pd, dl, dl, g, math)
    xd, wd, bd = dev(x), dev(w), dev(b)
    yd = torch.empty((N, K, P, Q)).to(DEV)
    ws = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 0), 4), dtype=torch.uint8).to(DEV)
    sync()
    ok(lib, lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(td(xd)), ctypes.c_void_p(wd.data_ptr()),
                                ctypes.c_void_p(bd.data_ptr()), ctypes.byref(td(yd)), ctypes.c_void_p(ws.data_ptr()),
                                ctypes.c_size_t(ws.numel()), stream()))
    gyd = gy.to(DEV)
    gxd = torch.empty(x.shape).to(DEV)
    gwd = torch.empty(w.shape).to(DEV)
    gbd = torch.empty(K).to(DEV)
    ws1 = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 1), 4), dtype=torch.uint8).to(DEV)
    ws2 = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 2), 4), dtype=torch.uint8).to(DEV)
    sync()
    ok(lib, lib.pvb2_conv2d_bwd_data(ctypes.byref(d), ctypes.byref(td(gyd)), ctypes.c_void_p(wd.data_ptr()),
                                     ctypes.byref(td(gxd)), ctypes.c_void_p(ws1.data_ptr()),
                                     ctypes.c_size_t(ws1.numel()), stream()))
    ok(lib, lib.pvb2_conv2d_bwd_filter(ctypes.byref(d), ctypes.byref(td(xd)), ctypes.byref(td(gyd)),
                                       ctypes.c_void_p(gwd.data_ptr()), ctypes.c_void_p(gbd.data_ptr()),
                                       ctypes.c_void_p(ws2.data_ptr()), ctypes.c_size_t(ws2.numel()), stream()))
    sync()
    rel = 2.0 ** -9 if math == 0 else 2.0 ** -20 * (C // g * R * S + 16)
    relw = 2.0 ** -9 if math == 0 else 2.0 ** -30 * 64
    ybound = rel * ya.detach().numpy() + 1e-5
    assert np.all(np.abs(yd.cpu().numpy() - yref) <= ybound), "forward"
    gx_bound = (2.0 ** -9 if math == 0 else 2.0 ** -20 * (K // g * R * S + 16)) * xa.grad.numpy() + 1e-5
    assert np.all(np.abs(gxd.cpu().double().numpy() - xt.grad.numpy()) <= gx_bound), "dgrad"
    gw_bound = (2.0 ** -9 if math == 0 else 2.0 ** -22 * 64) * wa.grad.numpy() + 1e-4
    assert np.all(np.abs(gwd.cpu().double().numpy() - wt.grad.numpy()) <= gw_bound), "wgrad"
    gb_ref = gy.double().sum((0, 2, 3))
    assert (gbd.cpu().double() - gb_ref).abs().max().item() <= 1e-5 * gy.abs().sum().item() / K + 1e-5


@pytest.mark.parametrize("M,N,K,batch", [(1, 1, 1, 1), (7, 13, 5, 2), (64, 1000, 2048, 1), (128, 128, 128, 3),
                                         (300, 257, 129, 1), (64, 9216, 128, 1)])
@pytest.mark.parametrize("math", [1, 0])
def test_gemm_capi(lib, M, N, K, batch, math):
    rng = np.random.default_rng(M * N + K)
    a = rng.standard_normal((batch, M, K)).astype(np.float32)
    b = rng.standard_normal((batch, K, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    ref = np.einsum("bmk,bkn->bmn", a.astype(np.float64), b.astype(np.float64)) * 0.5 + bias
    ad, bd, bsd = dev(a), dev(b), dev(bias)
    cd = torch.empty((batch, M, N)).to(DEV)
    sync()
    ok(lib, lib.pvb2_gemm(ctypes.byref(td(ad)), ctypes.byref(td(bd)), ctypes.byref(td(cd)),
                          ctypes.c_void_p(bsd.data_ptr()), 1, ctypes.c_double(0.5), ctypes.c_double(0.0), math,
                          stream()))
    sync()
    err = np.abs(cd.cpu().numpy() - ref)
    # elementwise bound: fp32 accumulation (math=1) or TF32 operands, whose 10
    # mantissa bits give each product a relative error below 2^-9 (math=0)
    absref = np.einsum("bmk,bkn->bmn", np.abs(a).astype(np.float64), np.abs(b).astype(np.float64)) * 0.5
    rel = 2.0 ** -20 * K if math == 1 else 2.0 ** -9
    assert np.all(err <= rel * absref + 1e-5), float((err / (absref + 1e-30)).max())


def test_gemm_transposed_operands_capi(lib):
    """B given as a transposed view (linear's W^T): strides carried through the C-ABI."""
    rng = np.random.default_rng(9)
    x = rng.standard_normal((64, 512)).astype(np.float32)
    w = rng.standard_normal((1000, 512)).astype(np.float32)
    xd, wd = dev(x), dev(w)
    out = torch.empty((64, 1000)).to(DEV)
    A, B, C = xd.unsqueeze(0), wd.t().unsqueeze(0), out.unsqueeze(0)
    sync()
    ok(lib, lib.pvb2_gemm(ctypes.byref(td(A)), ctypes.byref(td(B)), ctypes.byref(td(C)), None, 1,
                          ctypes.c_double(1.0), ctypes.c_double(0.0), 0, stream()))
    sync()
    ref = x.astype(np.float64) @ w.T.astype(np.float64)
    absref = np.abs(x).astype(np.float64) @ np.abs(w.T).astype(np.float64)
    assert np.all(np.abs(out.cpu().numpy() - ref) <= 2.0 ** -9 * absref + 1e-5)


GEMM_OUTPUTS = [
    # layout of C, batch, M, N, K, bias_dim, beta
    ("rows", 1, 300, 200, 96, 1, 0.0),           # row-major C, ragged edges: TMA row boxes, clipped
    ("rows_padded", 2, 130, 96, 256, 0, 0.0),     # row stride N + 4, batched, bias per row
    ("cols", 1, 200, 160, 192, 1, 0.0),          # C a transposed view: column boxes
    ("rows_odd_stride", 1, 150, 90, 512, 1, 0.0),  # row stride N + 1: per-element stores
    ("rows_beta", 1, 256, 256, 128, 1, 0.75),    # beta != 0 reads C: per-element stores
]


@pytest.mark.parametrize("case", GEMM_OUTPUTS, ids=[c[0] for c in GEMM_OUTPUTS])
def test_gemm_output_layouts_capi(lib, case):
    """TF32 GEMM epilogue for each output layout (TMA row / column boxes,
    per-element fallback) against float64; every case is above the size
    where small products stay on the exact SIMT kernel."""
    layout, batch, M, N, K, bias_dim, beta = case
    rng = np.random.default_rng(M + N)
    a = rng.standard_normal((batch, M, K)).astype(np.float32)
    b = rng.standard_normal((batch, K, N)).astype(np.float32)
    c0 = rng.standard_normal((batch, M, N)).astype(np.float32)
    bias = rng.standard_normal(N if bias_dim == 1 else M).astype(np.float32)
    ref = np.einsum("bmk,bkn->bmn", a.astype(np.float64), b.astype(np.float64)) * 1.5 + beta * c0
    ref = ref + (bias[None, None, :] if bias_dim == 1 else bias[None, :, None])
    absref = np.einsum("bmk,bkn->bmn", np.abs(a).astype(np.float64), np.abs(b).astype(np.float64)) * 1.5
    if layout == "cols":
        store = torch.from_numpy(np.ascontiguousarray(c0.transpose(0, 2, 1))).to(DEV)
        cd = store.transpose(1, 2)
    elif layout in ("rows_padded", "rows_odd_stride"):
        pad = 4 if layout == "rows_padded" else 1
        store = torch.zeros((batch, M, N + pad)).to(DEV)
        cd = store[:, :, :N]
        cd.copy_(torch.from_numpy(c0).to(DEV))
    else:
        cd = torch.from_numpy(c0).to(DEV)
    ad, bd, bsd = dev(a), dev(b), dev(bias)
    sync()
    ok(lib, lib.pvb2_gemm(ctypes.byref(td(ad)), ctypes.byref(td(bd)), ctypes.byref(td(cd)),
                          ctypes.c_void_p(bsd.data_ptr()), bias_dim, ctypes.c_double(1.5), ctypes.c_double(beta), 0,
                          stream()))
    sync()
    got = cd.cpu().numpy()
    assert np.all(np.abs(got - ref) <= 2.0 ** -9 * absref + 1e-4)
    if layout in ("rows_padded", "rows_odd_stride"):
        assert store[:, :, N:].abs().max().item() == 0.0  # padding untouched


SPLITK = [
    # batch, M, N, K, A transposed (dY^T), beta
    (1, 768, 768, 6304, True, 0.0),   # a linear layer's weight gradient: 18 tiles, K = tokens
    (1, 200, 300, 4000, False, 0.5),  # ragged tiles, beta != 0 (C read in the reduction)
    (2, 130, 250, 2048, True, 0.0),   # batched
]


@pytest.mark.parametrize("case", SPLITK, ids=["x".join(map(str, c[:4])) for c in SPLITK])
def test_gemm_split_k_capi(lib, case):
    """Split-K TF32 GEMM (few output tiles, long K) with its workspace, and the
    same product unsplit without one, both against float64."""
    batch, M, N, K, at, beta = case
    lib.pvb2_gemm_workspace_size.restype = ctypes.c_size_t
    rng = np.random.default_rng(M + K)
    a = rng.standard_normal((batch, M, K)).astype(np.float32)
    b = rng.standard_normal((batch, K, N)).astype(np.float32)
    c0 = rng.standard_normal((batch, M, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    ref = np.einsum("bmk,bkn->bmn", a.astype(np.float64), b.astype(np.float64)) + beta * c0 + bias
    absref = np.einsum("bmk,bkn->bmn", np.abs(a).astype(np.float64), np.abs(b).astype(np.float64))
    ad = dev(np.ascontiguousarray(a.transpose(0, 2, 1))).transpose(1, 2) if at else dev(a)
    bd, bsd = dev(b), dev(bias)
    outs = []
    for use_ws in (True, False):
        cd = dev(c0)
        wsz = lib.pvb2_gemm_workspace_size(ctypes.byref(td(ad)), ctypes.byref(td(bd)), ctypes.byref(td(cd)), 0)
        assert wsz > 0
        ws = torch.empty(wsz // 4 if use_ws else 4).to(DEV)
        sync()
        ok(lib, lib.pvb2_gemm_ws(ctypes.byref(td(ad)), ctypes.byref(td(bd)), ctypes.byref(td(cd)),
                                 ctypes.c_void_p(bsd.data_ptr()), 1, ctypes.c_double(1.0), ctypes.c_double(beta), 0,
                                 ctypes.c_void_p(ws.data_ptr() if use_ws else None),
                                 ctypes.c_size_t(wsz if use_ws else 0), stream()))
        sync()
        got = cd.cpu().numpy()
        assert np.all(np.abs(got - ref) <= 2.0 ** -9 * absref + 1e-4), use_ws
        outs.append(got)
    # the split partials are summed in a fixed order: repeatable bit for bit
    cd = dev(c0)
    ws = torch.empty(wsz // 4).to(DEV)
    ok(lib, lib.pvb2_gemm_ws(ctypes.byref(td(ad)), ctypes.byref(td(bd)), ctypes.byref(td(cd)),
                             ctypes.c_void_p(bsd.data_ptr()), 1, ctypes.c_double(1.0), ctypes.c_double(beta), 0,
                             ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(wsz), stream()))
    sync()
    assert np.array_equal(cd.cpu().numpy(), outs[0])


@pytest.mark.parametrize("shape", [(4, 3, 5, 6), (64, 64, 56, 56), (2, 8, 7, 7), (3, 5, 1, 1), (0, 4, 3, 3)])
def test_batch_norm_capi(lib, shape):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(shape) * 3 + 2).astype(np.float32)
    C = shape[1]
    gam, bet = rng.standard_normal(C).astype(np.float32), rng.standard_normal(C).astype(np.float32)
    rm, rv = np.zeros(C, np.float32), np.ones(C, np.float32)
    xd, gd, bd, rmd, rvd = dev(x), dev(gam), dev(bet), dev(rm), dev(rv)
    yd = torch.empty(shape).to(DEV)
    md, isd = torch.empty(C).to(DEV), torch.empty(C).to(DEV)
    wsz = lib.pvb2_batch_norm_workspace_size(ctypes.byref(td(xd)))
    ws = torch.empty(max(wsz, 4), dtype=torch.uint8).to(DEV)
    sync()
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    ok(lib, lib.pvb2_batch_norm_fwd_train(ctypes.byref(td(xd)), ptr(gd), ptr(bd), ptr(rmd), ptr(rvd),
                                          ctypes.c_double(0.1), ctypes.c_double(1e-5), ctypes.byref(td(yd)), ptr(md),
                                          ptr(isd), ptr(ws), ctypes.c_size_t(ws.numel()), stream()))
    sync()
    if shape[0] == 0:
        return
    y, mean, invstd, nrm, nrv = npref.batch_norm_train(x, gam, bet, rm, rv, 0.1, 1e-5)
    assert np.abs(yd.cpu().numpy() - y).max() < 1e-4
    assert np.abs(md.cpu().numpy() - mean).max() < 1e-5
    assert np.abs(rmd.cpu().numpy() - nrm).max() < 1e-5
    assert np.abs(rvd.cpu().numpy() - nrv).max() < 1e-4
    dy = rng.standard_normal(shape).astype(np.float32)
    dyd = dev(dy)
    dxd, dgd, dbd = torch.empty(shape).to(DEV), torch.empty(C).to(DEV), torch.empty(C).to(DEV)
    sync()
    ok(lib, lib.pvb2_batch_norm_bwd(ctypes.byref(td(dyd)), ctypes.byref(td(xd)), ptr(gd), ptr(md), ptr(isd), 1,
                                    ctypes.byref(td(dxd)), ptr(dgd), ptr(dbd), ptr(ws), ctypes.c_size_t(ws.numel()),
                                    stream()))
    sync()
    dx, dg, db = npref.batch_norm_backward(dy, x, gam, mean, invstd)
    m = x.size // C
    assert np.abs(dxd.cpu().numpy() - dx).max() < 1e-4
    assert np.abs(dgd.cpu().numpy() - dg).max() < 1e-5 * m
    assert np.abs(dbd.cpu().numpy() - db).max() < 1e-5 * m


@pytest.mark.parametrize("cfg", [(3, 2, 1, False), (2, 2, 0, False), (3, 2, 0, True)])
def test_max_pool_capi_bit_exact(lib, cfg):
    k, s, p, ceil = cfg
    rng = np.random.default_rng(2)
    x = rng.integers(0, 3, (2, 5, 13, 13)).astype(np.float32)  # ties everywhere
    y, ind = npref.max_pool2d(x, k, s, p, 1, ceil)
    xd = dev(x)
    yd = torch.empty(y.shape).to(DEV)
    indd = torch.empty(y.shape, dtype=torch.int64).to(DEV)
    pdsc = Pool(k, k, s, s, p, p, 1, 1, int(ceil), 0, 0)
    sync()
    ok(lib, lib.pvb2_max_pool2d_fwd(ctypes.byref(pdsc), ctypes.byref(td(xd)), ctypes.byref(td(yd)),
                                    ctypes.c_void_p(indd.data_ptr()), stream()))
    sync()
    assert np.array_equal(yd.cpu().numpy(), y)
    assert np.array_equal(indd.cpu().numpy(), ind)  # bit-exact indices
    dy = rng.standard_normal(y.shape).astype(np.float32)
    dyd = dev(dy)
    dxd = torch.empty(x.shape).to(DEV)
    sync()
    ok(lib, lib.pvb2_max_pool2d_bwd(ctypes.byref(pdsc), ctypes.byref(td(dyd)), ctypes.c_void_p(indd.data_ptr()),
                                    ctypes.byref(td(dxd)), stream()))
    sync()
    assert np.abs(dxd.cpu().numpy() - npref.max_pool2d_backward(dy, ind, x.shape)).max() < 1e-6


@pytest.mark.parametrize("N,C", [(64, 1000), (1, 10), (7, 3), (300, 4097)])
def test_log_softmax_nll_capi(lib, N, C):
    rng = np.random.default_rng(N + C)
    x = (rng.standard_normal((N, C)) * 4).astype(np.float32)
    t = rng.integers(0, C, N).astype(np.int64)
    if N > 2:
        t[1] = -100  # ignore_index
    xd, tdv = dev(x), dev(t)
    lp = torch.empty((N, C)).to(DEV)
    out, tw = torch.empty(()).to(DEV), torch.empty(()).to(DEV)
    sync()
    ok(lib, lib.pvb2_softmax_fwd(1, ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(lp.data_ptr()),
                                 ctypes.c_int64(N), ctypes.c_int64(C), ctypes.c_int64(1), stream()))
    ok(lib, lib.pvb2_nll_loss_fwd(ctypes.c_void_p(lp.data_ptr()), ctypes.c_void_p(tdv.data_ptr()), None,
                                  ctypes.c_int64(N), ctypes.c_int64(C), 1, ctypes.c_int64(-100),
                                  ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(tw.data_ptr()), stream()))
    sync()
    ref_lp = npref.log_softmax(x, 1)
    assert np.abs(lp.cpu().numpy() - ref_lp).max() < 1e-5
    assert abs(out.item() - npref.nll_loss(ref_lp, t, "mean", -100)) < 1e-5


def test_sgd_multi_capi(lib):
    rng = np.random.default_rng(4)
    sizes = [1, 3, 8193, 100000, 5]
    ps = [rng.standard_normal(n).astype(np.float32) for n in sizes]
    gs = [rng.standard_normal(n).astype(np.float32) for n in sizes]
    pd_ = [dev(p) for p in ps]
    gd = [dev(g) for g in gs]
    bd = [torch.empty(n).to(DEV) for n in sizes]
    arr = lambda ts: (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
    numel = (ctypes.c_int64 * len(sizes))(*sizes)
    bufs = [None] * len(sizes)
    ref = list(ps)
    for it in range(3):
        sync()
        ok(lib, lib.pvb2_sgd_multi(len(sizes), arr(pd_), arr(gd), arr(bd), numel, ctypes.c_double(0.1),
                                   ctypes.c_double(0.9), ctypes.c_double(0.0), ctypes.c_double(1e-4), 0,
                                   1 if it == 0 else 0, ctypes.c_double(1.0), stream()))
        sync()
        for i in range(len(sizes)):
            ref[i], bufs[i] = npref.sgd_momentum(ref[i], gs[i], bufs[i], 0.1, 0.9, 0.0, 1e-4)
    for p, r in zip(pd_, ref):
        assert np.abs(p.cpu().numpy() - r).max() < 1e-5


def test_invalid_arguments_are_reported(lib):
    d = Conv(2, 3, 8, 8, 4, 3, 3, 99, 99, 1, 1, 1, 1, 1, 1, 1, 0)  # inconsistent output size
    x = torch.empty((2, 3, 8, 8)).to(DEV)
    y = torch.empty((2, 4, 8, 8)).to(DEV)
    w = torch.empty((4, 3, 3, 3)).to(DEV)
    st = lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(td(x)), ctypes.c_void_p(w.data_ptr()), None,
                             ctypes.byref(td(y)), None, ctypes.c_size_t(0), stream())
    assert st == 1 and b"output size" in lib.pvb2_last_error()


@pytest.mark.parametrize("residual,relu", [(False, False), (False, True), (True, True), (True, False)])
def test_batch_norm_split_fwd_capi(lib, residual, relu):
    """pvb2_batch_norm_fwd_stats + pvb2_batch_norm_fwd_apply (with the fused
    residual / ReLU epilogue) against the numpy restatement."""
    rng = np.random.default_rng(21)
    shape = (6, 24, 13, 11)
    x = (rng.standard_normal(shape) * 2 + 1).astype(np.float32)
    r = rng.standard_normal(shape).astype(np.float32)
    C = shape[1]
    gam, bet = rng.standard_normal(C).astype(np.float32), rng.standard_normal(C).astype(np.float32)
    rm, rv = np.zeros(C, np.float32), np.ones(C, np.float32)
    xd, rd, gd, bd, rmd, rvd = dev(x), dev(r), dev(gam), dev(bet), dev(rm), dev(rv)
    yd = torch.empty(shape).to(DEV)
    md, isd = torch.empty(C).to(DEV), torch.empty(C).to(DEV)
    assert lib.pvb2_batch_norm_fwd_split_ok(ctypes.byref(td(xd))) == 1
    wsz = lib.pvb2_batch_norm_workspace_size(ctypes.byref(td(xd)))
    ws = torch.empty(max(wsz, 4), dtype=torch.uint8).to(DEV)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    sync()
    ok(lib, lib.pvb2_batch_norm_fwd_stats(ctypes.byref(td(xd)), ptr(ws), ctypes.c_size_t(ws.numel()), stream()))
    ok(lib, lib.pvb2_batch_norm_fwd_apply(ctypes.byref(td(xd)), ptr(gd), ptr(bd), ptr(rmd), ptr(rvd),
                                          ctypes.c_double(0.1), ctypes.c_double(1e-5), ctypes.byref(td(yd)), ptr(md),
                                          ptr(isd), ctypes.byref(td(rd)) if residual else None, int(relu), None,
                                          ptr(ws), ctypes.c_size_t(ws.numel()), stream()))
    sync()
    y, mean, invstd, nrm, nrv = npref.batch_norm_train(x, gam, bet, rm, rv, 0.1, 1e-5)
    if residual:
        y = y + r
    if relu:
        y = np.maximum(y, 0)
    assert np.abs(yd.cpu().numpy() - y).max() < 1e-4
    assert np.abs(md.cpu().numpy() - mean).max() < 1e-5
    assert np.abs(rmd.cpu().numpy() - nrm).max() < 1e-5
    assert np.abs(rvd.cpu().numpy() - nrv).max() < 1e-4


def test_batch_norm_relu6_capi(lib):
    """ReLU6 through the split batch norm: pvb2_batch_norm_fwd_apply with
    act = 2 and sum_out (plain values to y, clamped ones to sum_out, no
    residual), then pvb2_batch_norm_bwd_act with act = 2 (the hardtanh
    gradient (out <= 0 || out >= 6) ? 0 : g formed in the first pass),
    against the numpy restatements; act values other than 0-2 are refused."""
    rng = np.random.default_rng(23)
    shape = (4, 16, 12, 10)
    x = (rng.standard_normal(shape) * 2 + 1).astype(np.float32)
    C = shape[1]
    gam = rng.uniform(2.0, 4.0, C).astype(np.float32)  # a good share of the outputs past 6
    bet = rng.standard_normal(C).astype(np.float32)
    rm, rv = np.zeros(C, np.float32), np.ones(C, np.float32)
    xd, gd, bd, rmd, rvd = dev(x), dev(gam), dev(bet), dev(rm), dev(rv)
    yd, od = torch.empty(shape).to(DEV), torch.empty(shape).to(DEV)
    md, isd = torch.empty(C).to(DEV), torch.empty(C).to(DEV)
    wsz = lib.pvb2_batch_norm_workspace_size(ctypes.byref(td(xd)))
    ws = torch.empty(max(wsz, 4), dtype=torch.uint8).to(DEV)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    sync()
    ok(lib, lib.pvb2_batch_norm_fwd_stats(ctypes.byref(td(xd)), ptr(ws), ctypes.c_size_t(ws.numel()), stream()))
    apply = lambda act: lib.pvb2_batch_norm_fwd_apply(
        ctypes.byref(td(xd)), ptr(gd), ptr(bd), ptr(rmd), ptr(rvd), ctypes.c_double(0.1), ctypes.c_double(1e-5),
        ctypes.byref(td(yd)), ptr(md), ptr(isd), None, act, ctypes.byref(td(od)), ptr(ws),
        ctypes.c_size_t(ws.numel()), stream())
    assert apply(3) == 1 and b"activation" in lib.pvb2_last_error()
    ok(lib, apply(2))
    sync()
    y, mean, invstd, _, _ = npref.batch_norm_train(x, gam, bet, rm, rv, 0.1, 1e-5)
    out = np.clip(y, 0.0, 6.0)
    assert (out == 6.0).any() and (out == 0.0).any()
    assert np.abs(yd.cpu().numpy() - y).max() < 1e-4
    assert np.abs(od.cpu().numpy() - out).max() < 1e-4

    g = rng.standard_normal(shape).astype(np.float32)
    gdv = dev(g)
    dyd, dxd = torch.empty(shape).to(DEV), torch.empty(shape).to(DEV)
    dgam, dbet = torch.empty(C).to(DEV), torch.empty(C).to(DEV)
    outd = od.clone()
    sync()
    ok(lib, lib.pvb2_batch_norm_bwd_act(2, ctypes.byref(td(gdv)), ctypes.byref(td(outd)), ctypes.byref(td(xd)),
                                        ptr(gd), ptr(md), ptr(isd), ctypes.byref(td(dyd)), ctypes.byref(td(dxd)),
                                        ptr(dgam), ptr(dbet), ptr(ws), ctypes.c_size_t(ws.numel()), stream()))
    assert lib.pvb2_batch_norm_bwd_act(3, ctypes.byref(td(gdv)), ctypes.byref(td(outd)), ctypes.byref(td(xd)),
                                       ptr(gd), ptr(md), ptr(isd), ctypes.byref(td(dyd)), ctypes.byref(td(dxd)),
                                       ptr(dgam), ptr(dbet), ptr(ws), ctypes.c_size_t(ws.numel()), stream()) == 1
    sync()
    o = od.cpu().numpy()
    dy = np.where((o <= 0.0) | (o >= 6.0), 0.0, g).astype(np.float32)
    assert np.array_equal(dyd.cpu().numpy(), dy)
    dx, dgr, dbr = npref.batch_norm_backward(dy, x, gam, md.cpu().numpy(), isd.cpu().numpy())
    scale = np.abs(dx).max()
    assert np.abs(dxd.cpu().numpy() - dx).max() < 1e-4 * scale
    assert np.abs(dgam.cpu().numpy() - dgr).max() < 1e-3 * np.abs(dgr).max()
    assert np.abs(dbet.cpu().numpy() - dbr).max() < 1e-3 * np.abs(dbr).max()


@pytest.mark.parametrize("act", [1, 2])
@pytest.mark.parametrize("shape", [(4, 16, 12, 10), (8, 32, 14, 14), (3, 5, 7, 7)], ids=["odd_hw", "vec", "tiny"])
def test_batch_norm_act_from_x_capi(lib, act, shape):
    """pvb2_batch_norm_fwd_apply_ab hands out the pass's (a, b): its
    activated output is act(fmaf(x, a, b)) bit for bit, and
    pvb2_batch_norm_bwd_act_ab, which forms the mask from x and ab, gives
    exactly what pvb2_batch_norm_bwd_act (reading that output) gives: the
    gradient below the activation, dx, dgamma, dbeta; dy may be omitted."""
    rng = np.random.default_rng(29 + act)
    x = (rng.standard_normal(shape) * 2 + 1).astype(np.float32)
    C = shape[1]
    gam = rng.uniform(1.5, 4.0, C).astype(np.float32)
    bet = rng.standard_normal(C).astype(np.float32)
    xd, gd, bd = dev(x), dev(gam), dev(bet)
    rmd, rvd = dev(np.zeros(C, np.float32)), dev(np.ones(C, np.float32))
    yd, abd = torch.empty(shape).to(DEV), torch.empty(2 * C).to(DEV)
    md, isd = torch.empty(C).to(DEV), torch.empty(C).to(DEV)
    wsz = lib.pvb2_batch_norm_workspace_size(ctypes.byref(td(xd)))
    ws = torch.empty(max(wsz, 4), dtype=torch.uint8).to(DEV)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    sync()
    ok(lib, lib.pvb2_batch_norm_fwd_stats(ctypes.byref(td(xd)), ptr(ws), ctypes.c_size_t(ws.numel()), stream()))
    ok(lib, lib.pvb2_batch_norm_fwd_apply_ab(
        ctypes.byref(td(xd)), ptr(gd), ptr(bd), ptr(rmd), ptr(rvd), ctypes.c_double(0.1), ctypes.c_double(1e-5),
        ctypes.byref(td(yd)), ptr(md), ptr(isd), None, act, None, ptr(ws), ctypes.c_size_t(ws.numel()),
        ptr(abd), stream()))
    sync()
    a, b = abd.cpu()[:C].view(1, C, 1, 1).double(), abd.cpu()[C:].view(1, C, 1, 1).double()
    v = (torch.from_numpy(x).double() * a + b).float()  # x * a exact in float64, then rounded: fmaf
    ref = v.clamp(min=0.0) if act == 1 else v.clamp(0.0, 6.0)
    assert torch.equal(yd.cpu(), ref)
    g = dev(rng.standard_normal(shape).astype(np.float32))
    outs = []
    for use_ab in (False, True):
        dyd, dxd = torch.full(shape, 7.0).to(DEV), torch.empty(shape).to(DEV)
        dgam, dbet = torch.empty(C).to(DEV), torch.empty(C).to(DEV)
        if use_ab:
            ok(lib, lib.pvb2_batch_norm_bwd_act_ab(
                act, ctypes.byref(td(g)), ctypes.byref(td(xd)), ptr(abd), ptr(gd), ptr(md), ptr(isd),
                ctypes.byref(td(dyd)), ctypes.byref(td(dxd)), ptr(dgam), ptr(dbet), ptr(ws),
                ctypes.c_size_t(ws.numel()), stream()))
        else:
            ok(lib, lib.pvb2_batch_norm_bwd_act(
                act, ctypes.byref(td(g)), ctypes.byref(td(yd)), ctypes.byref(td(xd)), ptr(gd), ptr(md), ptr(isd),
                ctypes.byref(td(dyd)), ctypes.byref(td(dxd)), ptr(dgam), ptr(dbet), ptr(ws),
                ctypes.c_size_t(ws.numel()), stream()))
        sync()
        outs.append([t.cpu() for t in (dyd, dxd, dgam, dbet)])
    for p_, q_ in zip(*outs):
        assert torch.equal(p_, q_)
    # without dy: the same dx, dgamma, dbeta, and dy left untouched
    dyd, dxd = torch.full(shape, 7.0).to(DEV), torch.empty(shape).to(DEV)
    dgam, dbet = torch.empty(C).to(DEV), torch.empty(C).to(DEV)
    ok(lib, lib.pvb2_batch_norm_bwd_act_ab(
        act, ctypes.byref(td(g)), ctypes.byref(td(xd)), ptr(abd), ptr(gd), ptr(md), ptr(isd), None,
        ctypes.byref(td(dxd)), ptr(dgam), ptr(dbet), ptr(ws), ctypes.c_size_t(ws.numel()), stream()))
    sync()
    assert torch.equal(dxd.cpu(), outs[0][1]) and torch.equal(dgam.cpu(), outs[0][2])
    assert torch.equal(dbet.cpu(), outs[0][3]) and bool((dyd.cpu() == 7.0).all())
    assert lib.pvb2_batch_norm_bwd_act_ab(
        act, ctypes.byref(td(g)), ctypes.byref(td(xd)), None, ptr(gd), ptr(md), ptr(isd), None,
        ctypes.byref(td(dxd)), ptr(dgam), ptr(dbet), ptr(ws), ctypes.c_size_t(ws.numel()), stream()) != 0
