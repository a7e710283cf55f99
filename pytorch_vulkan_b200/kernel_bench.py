"""Per-kernel timing through the C-ABI (libpvb2.so via ctypes, device memory
from the `ocl` backend), for looking at one launch alone under a profiler.

    python -m pytorch_vulkan_b200.kernel_bench dgrad_acc [--n 32] [--c 256] [--hw 56] [--k 64]
    python -m pytorch_vulkan_b200.kernel_bench conv --which fwd|dgrad|wgrad [--n 32] [--c 64] [--hw 56]
           [--k 64] [--r 3] [--stride 1] [--pad 1]

`dgrad_acc`: the 1x1 stride-1 convolution input gradient dX[n, c] =
sum_k W[k, c] dY[n, k] (a residual block's first convolution), first plain
(`pvb2_conv2d_bwd_data`), then with the other input gradient summed in its
epilogue (`pvb2_conv2d_bwd_data_acc`).  Each is run 3 times untimed, then 10
times between device events; the line printed per variant gives the mean
launch time and the algorithmic bytes (dY read, dX written, addend read) per
second.  Launch order: 13 plain, then 13 accumulating.

`conv`: one convolution pass (TF32) through `pvb2_conv2d_fwd`,
`pvb2_conv2d_bwd_data` or `pvb2_conv2d_bwd_filter`, 3 untimed and 10 timed
calls (each call may launch staging / packing / reduction kernels beside the
tensor-core one); prints the mean time per call and its TFLOP/s.

`dw`: MobileNet-v2's depthwise 3x3 convolutions at batch --n (default 128),
each pass timed as `conv` does, with algorithmic GB/s (input read + output
written once; the filter is negligible) against the measured HBM copy rate.

`bn`: the batch-norm passes of ResNet-50's activation shapes at batch --n
(default 64): statistics, normalising pass with ReLU, and the backward's
reduce and apply passes with the ReLU gradient (pvb2_batch_norm_fwd_stats,
pvb2_batch_norm_fwd_apply, pvb2_batch_norm_bwd_relu), each timed alone, with
the bytes each pass moves and its algorithmic bytes per element (8 forward,
16 backward with the ReLU mask).

`r50`: every distinct convolution of ResNet-50 at batch --n (default 64),
each pass timed as `conv` does, with the number of times the geometry occurs
in one training step; prints per pass the time, TFLOP/s and algorithmic
GB/s (input read + output written once), and the step's weighted totals.
`mbv2`: the same for MobileNet-v2's dense convolutions (stem, 1x1 expansions
and projections) at batch --n (default 128).
"""
from __future__ import annotations

import argparse
import ctypes
import os

import torch

import pytorch_vulkan_b200 as _pkg

_LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libpvb2.so")


class _Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8),
                ("ndim", ctypes.c_int32), ("dtype", ctypes.c_int32)]


class _Conv(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ["N", "C", "H", "W", "K", "R", "S", "P", "Q", "stride_h", "stride_w",
                                             "pad_h", "pad_w", "dil_h", "dil_w", "groups", "math"]]


def _desc(t: torch.Tensor) -> _Tensor:
    assert t.dtype == torch.float32
    return _Tensor(t.data_ptr(), (ctypes.c_int64 * 8)(*t.shape), (ctypes.c_int64 * 8)(*t.stride()), t.dim(), 0)


def _time(fn, dev: int) -> float:
    for _ in range(3):
        fn()
    torch.ocl.synchronize()
    e0, e1 = _pkg._C.impl_event_create(True), _pkg._C.impl_event_create(True)
    _pkg._C.impl_event_record(e0, dev)
    for _ in range(10):
        fn()
    _pkg._C.impl_event_record(e1, dev)
    torch.ocl.synchronize()
    ms = _pkg._C.impl_event_elapsed_ms(e0, e1) / 10
    _pkg._C.impl_event_destroy(e0)
    _pkg._C.impl_event_destroy(e1)
    return ms


def dgrad_acc(n: int, c: int, hw: int, k: int, dev: int = 0) -> None:
    lib = ctypes.CDLL(_LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p
    lib.pvb2_conv2d_workspace_size.restype = ctypes.c_size_t
    d = _Conv(n, c, hw, hw, k, 1, 1, hw, hw, 1, 1, 0, 0, 1, 1, 1, 0)  # TF32 math
    name = f"ocl:{dev}"
    g = torch.Generator().manual_seed(0)
    gy = torch.randn(n, k, hw, hw, generator=g).to(name)
    w = (torch.randn(k, c, 1, 1, generator=g) * 0.1).to(name)
    addend = torch.randn(n, c, hw, hw, generator=g).to(name)
    out = torch.empty(n, c, hw, hw).to(name)
    ws = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 1), 4), dtype=torch.uint8).to(name)
    stream = ctypes.c_void_p(_pkg._C.impl_stream_handle(dev))
    gyd, outd, addd = _desc(gy), _desc(out), _desc(addend)
    wp = ctypes.c_void_p(w.data_ptr())

    def check(status):
        if status != 0:
            raise RuntimeError(lib.pvb2_last_error().decode())

    def plain():
        check(lib.pvb2_conv2d_bwd_data(ctypes.byref(d), ctypes.byref(gyd), wp, ctypes.byref(outd),
                                       ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()), stream))

    def acc():
        check(lib.pvb2_conv2d_bwd_data_acc(ctypes.byref(d), ctypes.byref(gyd), wp, ctypes.byref(outd),
                                           ctypes.byref(addd), stream))

    pixels = n * hw * hw
    for label, fn, planes in (("plain", plain, k + c), ("acc", acc, k + 2 * c)):
        ms = _time(fn, dev)
        gbs = pixels * planes * 4 / (ms * 1e-3) / 1e9
        print(f"{label}: {ms * 1e3:.1f} us per launch, {gbs:.0f} GB/s algorithmic "
              f"(N={n}, {k} -> {c} channels, {hw}x{hw})")


def conv(which: str, n: int, c: int, hw: int, k: int, r: int, stride: int, pad: int, dev: int = 0) -> None:
    lib = ctypes.CDLL(_LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p
    lib.pvb2_conv2d_workspace_size.restype = ctypes.c_size_t
    p = (hw + 2 * pad - r) // stride + 1
    d = _Conv(n, c, hw, hw, k, r, r, p, p, stride, stride, pad, pad, 1, 1, 1, 0)  # TF32 math
    name = f"ocl:{dev}"
    g = torch.Generator().manual_seed(0)
    x = torch.randn(n, c, hw, hw, generator=g).to(name)
    w = (torch.randn(k, c, r, r, generator=g) * 0.1).to(name)
    y = torch.randn(n, k, p, p, generator=g).to(name)
    dx = torch.empty(n, c, hw, hw).to(name)
    dw = torch.empty(k, c, r, r).to(name)
    slot = {"fwd": 0, "dgrad": 1, "wgrad": 2}[which]
    ws = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), slot), 4), dtype=torch.uint8).to(name)
    stream = ctypes.c_void_p(_pkg._C.impl_stream_handle(dev))
    xd, yd, dxd = _desc(x), _desc(y), _desc(dx)
    wsp, wsn = ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel())

    def run():
        if which == "fwd":
            st = lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(xd), ctypes.c_void_p(w.data_ptr()), None,
                                     ctypes.byref(yd), wsp, wsn, stream)
        elif which == "dgrad":
            st = lib.pvb2_conv2d_bwd_data(ctypes.byref(d), ctypes.byref(yd), ctypes.c_void_p(w.data_ptr()),
                                          ctypes.byref(dxd), wsp, wsn, stream)
        else:
            st = lib.pvb2_conv2d_bwd_filter(ctypes.byref(d), ctypes.byref(xd), ctypes.byref(yd),
                                            ctypes.c_void_p(dw.data_ptr()), None, wsp, wsn, stream)
        if st != 0:
            raise RuntimeError(lib.pvb2_last_error().decode())

    ms = _time(run, dev)
    flop = 2.0 * n * p * p * k * c * r * r
    print(f"conv {which}: {ms * 1e3:.1f} us per call, {flop / (ms * 1e-3) / 1e12:.1f} TFLOP/s "
          f"(N={n}, {c} -> {k} channels, {hw}x{hw}, {r}x{r} stride {stride} pad {pad})")


# N-independent ResNet-50 geometries: (C, H, K, R, stride, pad, count per step, input gradient needed)
R50 = [
    (3, 224, 64, 7, 2, 3, 1, False), (64, 56, 64, 1, 1, 0, 1, True), (64, 56, 64, 3, 1, 1, 3, True),
    (64, 56, 256, 1, 1, 0, 4, True), (256, 56, 64, 1, 1, 0, 2, True), (256, 56, 128, 1, 1, 0, 1, True),
    (128, 56, 128, 3, 2, 1, 1, True), (128, 28, 512, 1, 1, 0, 4, True), (256, 56, 512, 1, 2, 0, 1, True),
    (512, 28, 128, 1, 1, 0, 3, True), (128, 28, 128, 3, 1, 1, 3, True), (512, 28, 256, 1, 1, 0, 1, True),
    (256, 28, 256, 3, 2, 1, 1, True), (256, 14, 1024, 1, 1, 0, 6, True), (512, 28, 1024, 1, 2, 0, 1, True),
    (1024, 14, 256, 1, 1, 0, 5, True), (256, 14, 256, 3, 1, 1, 5, True), (1024, 14, 512, 1, 1, 0, 1, True),
    (512, 14, 512, 3, 2, 1, 1, True), (512, 7, 2048, 1, 1, 0, 3, True), (1024, 14, 2048, 1, 2, 0, 1, True),
    (2048, 7, 512, 1, 1, 0, 2, True), (512, 7, 512, 3, 1, 1, 2, True),
]


# MobileNet-v2's dense convolutions (the stem and every 1x1 expansion and
# projection; the depthwise ones are in MBV2_DW), same fields as R50
MBV2 = [
    (3, 224, 32, 3, 2, 1, 1, False), (32, 112, 16, 1, 1, 0, 1, True), (16, 112, 96, 1, 1, 0, 1, True),
    (96, 56, 24, 1, 1, 0, 1, True), (24, 56, 144, 1, 1, 0, 2, True), (144, 56, 24, 1, 1, 0, 1, True),
    (144, 28, 32, 1, 1, 0, 1, True), (32, 28, 192, 1, 1, 0, 3, True), (192, 28, 32, 1, 1, 0, 2, True),
    (192, 14, 64, 1, 1, 0, 1, True), (64, 14, 384, 1, 1, 0, 4, True), (384, 14, 64, 1, 1, 0, 3, True),
    (384, 14, 96, 1, 1, 0, 1, True), (96, 14, 576, 1, 1, 0, 3, True), (576, 14, 96, 1, 1, 0, 2, True),
    (576, 7, 160, 1, 1, 0, 1, True), (160, 7, 960, 1, 1, 0, 3, True), (960, 7, 160, 1, 1, 0, 2, True),
    (960, 7, 320, 1, 1, 0, 1, True), (320, 7, 1280, 1, 1, 0, 1, True),
]


def r50(n: int, dev: int = 0, table=None) -> None:
    table = R50 if table is None else table
    lib = ctypes.CDLL(_LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p
    lib.pvb2_conv2d_workspace_size.restype = ctypes.c_size_t
    name = f"ocl:{dev}"
    stream = ctypes.c_void_p(_pkg._C.impl_stream_handle(dev))
    tot = {"fwd": 0.0, "dgrad": 0.0, "wgrad": 0.0}
    flops = 0.0
    print(f"{'C':>5} {'HW':>4} {'K':>5} {'R':>2} {'s':>2} {'x':>2} | "
          f"{'fwd us':>8} {'TF/s':>6} {'GB/s':>6} | {'dgrad us':>8} {'TF/s':>6} {'GB/s':>6} | "
          f"{'wgrad us':>8} {'TF/s':>6} {'GB/s':>6}")
    for (c, hw, k, r, st, pd, cnt, need_dx) in table:
        p = (hw + 2 * pd - r) // st + 1
        d = _Conv(n, c, hw, hw, k, r, r, p, p, st, st, pd, pd, 1, 1, 1, 0)
        g = torch.Generator().manual_seed(0)
        x = torch.randn(n, c, hw, hw, generator=g).to(name)
        w = (torch.randn(k, c, r, r, generator=g) * 0.1).to(name)
        y = torch.randn(n, k, p, p, generator=g).to(name)
        dx = torch.empty(n, c, hw, hw).to(name)
        dw = torch.empty(k, c, r, r).to(name)
        ws = [torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), i), 4), dtype=torch.uint8).to(name)
              for i in range(3)]
        xd, yd, dxd = _desc(x), _desc(y), _desc(dx)
        wp = ctypes.c_void_p(w.data_ptr())
        calls = {
            "fwd": lambda: lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(xd), wp, None, ctypes.byref(yd),
                                               ctypes.c_void_p(ws[0].data_ptr()), ctypes.c_size_t(ws[0].numel()),
                                               stream),
            "dgrad": lambda: lib.pvb2_conv2d_bwd_data(ctypes.byref(d), ctypes.byref(yd), wp, ctypes.byref(dxd),
                                                      ctypes.c_void_p(ws[1].data_ptr()),
                                                      ctypes.c_size_t(ws[1].numel()), stream),
            "wgrad": lambda: lib.pvb2_conv2d_bwd_filter(ctypes.byref(d), ctypes.byref(xd), ctypes.byref(yd),
                                                        ctypes.c_void_p(dw.data_ptr()), None,
                                                        ctypes.c_void_p(ws[2].data_ptr()),
                                                        ctypes.c_size_t(ws[2].numel()), stream),
        }
        fl = 2.0 * n * p * p * k * c * r * r
        xb, yb, wb = 4.0 * n * c * hw * hw, 4.0 * n * k * p * p, 4.0 * k * c * r * r
        bytes_ = {"fwd": xb + wb + yb, "dgrad": yb + wb + xb, "wgrad": xb + yb + wb}
        cols = []
        for which in ("fwd", "dgrad", "wgrad"):
            if which == "dgrad" and not need_dx:
                cols.append(f"{'-':>8} {'-':>6} {'-':>6}")
                continue

            def run(f=calls[which]):
                st_ = f()
                if st_ != 0:
                    raise RuntimeError(lib.pvb2_last_error().decode())

            ms = _time(run, dev)
            tot[which] += ms * cnt
            flops += fl * cnt
            cols.append(f"{ms * 1e3:8.1f} {fl / (ms * 1e-3) / 1e12:6.1f} {bytes_[which] / (ms * 1e-3) / 1e9:6.0f}")
        print(f"{c:5d} {hw:4d} {k:5d} {r:2d} {st:2d} {cnt:2d} | " + " | ".join(cols))
    ms = sum(tot.values())
    print(f"step total (weighted by count): fwd {tot['fwd']:.3f} ms, dgrad {tot['dgrad']:.3f} ms, "
          f"wgrad {tot['wgrad']:.3f} ms; {ms:.3f} ms, {flops / (ms * 1e-3) / 1e12:.1f} TFLOP/s over "
          f"{flops / 1e9:.1f} GFLOP")


# MobileNet-v2 depthwise layers: (channels, input size, stride, count per step)
MBV2_DW = [(32, 112, 1, 1), (96, 112, 2, 1), (144, 56, 1, 1), (144, 56, 2, 1), (192, 28, 1, 2), (192, 28, 2, 1),
           (384, 14, 1, 4), (576, 14, 1, 2), (576, 14, 2, 1), (960, 7, 1, 3)]


def depthwise(n: int, dev: int = 0) -> None:
    lib = ctypes.CDLL(_LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p
    lib.pvb2_conv2d_workspace_size.restype = ctypes.c_size_t
    name = f"ocl:{dev}"
    stream = ctypes.c_void_p(_pkg._C.impl_stream_handle(dev))
    try:
        import json
        peak = json.load(open(os.path.join(os.path.dirname(os.path.dirname(_LIB)), "..", "MEASURED_PEAKS.json")))[
            "hbm_gbs"]
    except Exception:
        peak = 6650.0
    tot = {"fwd": 0.0, "dgrad": 0.0, "wgrad": 0.0}
    byts = {"fwd": 0.0, "dgrad": 0.0, "wgrad": 0.0}
    print(f"{'C':>5} {'HW':>4} {'s':>2} {'x':>2} | {'fwd us':>8} {'GB/s':>6} | {'dgrad us':>8} {'GB/s':>6} | "
          f"{'wgrad us':>8} {'GB/s':>6}")
    for (c, hw, st, cnt) in MBV2_DW:
        p = (hw + 2 - 3) // st + 1
        d = _Conv(n, c, hw, hw, c, 3, 3, p, p, st, st, 1, 1, 1, 1, c, 0)
        g = torch.Generator().manual_seed(0)
        x = torch.randn(n, c, hw, hw, generator=g).to(name)
        w = torch.randn(c, 1, 3, 3, generator=g).to(name)
        y = torch.randn(n, c, p, p, generator=g).to(name)
        dx = torch.empty(n, c, hw, hw).to(name)
        dw = torch.empty(c, 1, 3, 3).to(name)
        ws = torch.empty(max(lib.pvb2_conv2d_workspace_size(ctypes.byref(d), 2), 4), dtype=torch.uint8).to(name)
        xd, yd, dxd = _desc(x), _desc(y), _desc(dx)
        wp = ctypes.c_void_p(w.data_ptr())
        calls = {
            "fwd": lambda: lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(xd), wp, None, ctypes.byref(yd), None,
                                               ctypes.c_size_t(0), stream),
            "dgrad": lambda: lib.pvb2_conv2d_bwd_data(ctypes.byref(d), ctypes.byref(yd), wp, ctypes.byref(dxd), None,
                                                      ctypes.c_size_t(0), stream),
            "wgrad": lambda: lib.pvb2_conv2d_bwd_filter(ctypes.byref(d), ctypes.byref(xd), ctypes.byref(yd),
                                                        ctypes.c_void_p(dw.data_ptr()), None,
                                                        ctypes.c_void_p(ws.data_ptr()),
                                                        ctypes.c_size_t(ws.numel()), stream),
        }
        b = 4.0 * n * c * (hw * hw + p * p)
        cols = []
        for which in ("fwd", "dgrad", "wgrad"):
            def run(f=calls[which]):
                if f() != 0:
                    raise RuntimeError(lib.pvb2_last_error().decode())

            ms = _time(run, dev)
            tot[which] += ms * cnt
            byts[which] += b * cnt
            cols.append(f"{ms * 1e3:8.1f} {b / (ms * 1e-3) / 1e9:6.0f}")
        print(f"{c:5d} {hw:4d} {st:2d} {cnt:2d} | " + " | ".join(cols))
    for k in tot:
        print(f"{k}: {tot[k]:.3f} ms per step, {byts[k] / (tot[k] * 1e-3) / 1e9:.0f} GB/s algorithmic "
              f"= {byts[k] / (tot[k] * 1e-3) / 1e9 / peak:.2f} of {peak:.0f} GB/s")


# ResNet-50 batch-norm inputs: (channels, plane size, count per step)
R50_BN = [(64, 112, 1), (64, 56, 6), (256, 56, 4), (128, 56, 1), (128, 28, 7), (512, 28, 5), (256, 28, 1),
          (256, 14, 11), (1024, 14, 7), (512, 14, 1), (512, 7, 5), (2048, 7, 4)]


def batch_norm(n: int, dev: int = 0) -> None:
    lib = ctypes.CDLL(_LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p
    lib.pvb2_batch_norm_workspace_size.restype = ctypes.c_size_t
    name = f"ocl:{dev}"
    stream = ctypes.c_void_p(_pkg._C.impl_stream_handle(dev))
    p_ = lambda t: ctypes.c_void_p(t.data_ptr())
    tot = {"stats": 0.0, "apply": 0.0, "bwd": 0.0}
    alg = {"fwd": 0.0, "bwd": 0.0}
    print(f"{'C':>5} {'HW':>4} {'x':>2} | {'stats us':>8} {'GB/s':>6} | {'apply us':>8} {'GB/s':>6} | "
          f"{'bwd us':>8} {'GB/s':>6}")
    for (c, hw, cnt) in R50_BN:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(n, c, hw, hw, generator=g).to(name)
        y = torch.empty_like(x)
        dy = torch.randn(n, c, hw, hw, generator=g).to(name)
        dyo = torch.empty_like(x)
        dx = torch.empty_like(x)
        gam, bet = torch.ones(c).to(name), torch.zeros(c).to(name)
        rm, rv, mean, inv = (torch.zeros(c).to(name) for _ in range(4))
        dg, db = torch.empty(c).to(name), torch.empty(c).to(name)
        xd, yd, dyd, dyod, dxd = (_desc(t) for t in (x, y, dy, dyo, dx))
        ws = torch.empty(max(lib.pvb2_batch_norm_workspace_size(ctypes.byref(xd)), 16), dtype=torch.uint8).to(name)
        wsp, wsn = p_(ws), ctypes.c_size_t(ws.numel())

        def chk(st):
            if st != 0:
                raise RuntimeError(lib.pvb2_last_error().decode())

        stats = lambda: chk(lib.pvb2_batch_norm_fwd_stats(ctypes.byref(xd), wsp, wsn, stream))
        apply = lambda: chk(lib.pvb2_batch_norm_fwd_apply(ctypes.byref(xd), p_(gam), p_(bet), p_(rm), p_(rv),
                                                          ctypes.c_double(0.1), ctypes.c_double(1e-5),
                                                          ctypes.byref(yd), p_(mean), p_(inv), None, 1, None, wsp,
                                                          wsn, stream))
        bwd = lambda: chk(lib.pvb2_batch_norm_bwd_relu(ctypes.byref(dyd), ctypes.byref(yd), ctypes.byref(xd),
                                                       p_(gam), p_(mean), p_(inv), ctypes.byref(dyod),
                                                       ctypes.byref(dxd), p_(dg), p_(db), wsp, wsn, stream))
        stats()
        apply()
        e = x.numel()
        ms = {k: _time(f, dev) for k, f in (("stats", stats), ("apply", apply), ("bwd", bwd))}
        moved = {"stats": 4.0 * e, "apply": 8.0 * e, "bwd": 28.0 * e}
        for k in tot:
            tot[k] += ms[k] * cnt
        alg["fwd"] += 8.0 * e * cnt
        alg["bwd"] += 16.0 * e * cnt
        print(f"{c:5d} {hw:4d} {cnt:2d} | " + " | ".join(
            f"{ms[k] * 1e3:8.1f} {moved[k] / (ms[k] * 1e-3) / 1e9:6.0f}" for k in ("stats", "apply", "bwd")))
    fwd = tot["stats"] + tot["apply"]
    print(f"step: stats {tot['stats']:.3f} ms, apply {tot['apply']:.3f} ms, backward {tot['bwd']:.3f} ms; "
          f"forward {alg['fwd'] / (fwd * 1e-3) / 1e9:.0f} GB/s algorithmic, backward "
          f"{alg['bwd'] / (tot['bwd'] * 1e-3) / 1e9:.0f} GB/s algorithmic")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["dgrad_acc", "conv", "r50", "mbv2", "dw", "bn"])
    ap.add_argument("--which", choices=["fwd", "dgrad", "wgrad"], default="fwd")
    ap.add_argument("--n", type=int, default=None, help="batch (default 32; 64 for r50)")
    ap.add_argument("--c", type=int, default=None)
    ap.add_argument("--hw", type=int, default=56)
    ap.add_argument("--k", type=int, default=64)
    ap.add_argument("--r", type=int, default=3)
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--pad", type=int, default=None)
    a = ap.parse_args()
    torch.ocl.set_device(0)
    if a.kernel == "r50":
        r50(64 if a.n is None else a.n)
        return
    if a.kernel == "mbv2":
        r50(128 if a.n is None else a.n, table=MBV2)
        return
    if a.kernel == "dw":
        depthwise(128 if a.n is None else a.n)
        return
    if a.kernel == "bn":
        batch_norm(64 if a.n is None else a.n)
        return
    n = 32 if a.n is None else a.n
    if a.kernel == "dgrad_acc":
        dgrad_acc(n, 256 if a.c is None else a.c, a.hw, a.k)
    else:
        conv(a.which, n, 64 if a.c is None else a.c, a.hw, a.k, a.r, a.stride, a.r // 2 if a.pad is None else a.pad)


if __name__ == "__main__":
    main()
