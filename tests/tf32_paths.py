"""Which contraction passes the device runs on TF32 tensor cores, asked of the
device library itself (pvb2_conv2d_path / pvb2_gemm_path, host-only logic),
packaged as the oracle's ``oracle.tf32.Paths``.

The linear layer's three products are described the way torch's autograd
hands them to the GEMM entry point: y = x W^T with W^T a transposed view,
dX = dY W, and dW = dY^T X with dY^T a transposed view (torch's
mm_mat2_backward keeps a transposed weight's gradient column-major).  The
data pointers are any 256-byte aligned value: the queries only check
alignment."""
import ctypes
import os

from oracle.tf32 import Paths

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "pytorch_vulkan_b200", "lib", "libpvb2.so")
_ALIGNED = 256


class T(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8),
                ("ndim", ctypes.c_int32), ("dtype", ctypes.c_int32)]


class Conv(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ["N", "C", "H", "W", "K", "R", "S", "P", "Q", "stride_h", "stride_w",
                                             "pad_h", "pad_w", "dil_h", "dil_w", "groups", "math"]]


def _lib():
    return ctypes.CDLL(LIB)


def _mat(rows, cols, srow, scol):
    """a [1, rows, cols] fp32 operand as the host's as3d() describes a 2-D tensor"""
    return T(_ALIGNED, (ctypes.c_int64 * 8)(1, rows, cols), (ctypes.c_int64 * 8)(0, srow, scol), 3, 0)


def conv_desc(x_shape, w_shape, stride, padding, dilation, groups, math=0):
    N, C, H, W = x_shape
    K, _, R, S = w_shape
    P = (H + 2 * padding[0] - dilation[0] * (R - 1) - 1) // stride[0] + 1
    Q = (W + 2 * padding[1] - dilation[1] * (S - 1) - 1) // stride[1] + 1
    return Conv(N, C, H, W, K, R, S, P, Q, stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1],
                groups, math)


def device_paths(math=0):
    lib = _lib()

    def conv(x_shape, w_shape, stride, padding, dilation, groups, which):
        d = conv_desc(x_shape, w_shape, stride, padding, dilation, groups, math)
        r = lib.pvb2_conv2d_path(ctypes.byref(d), which)
        assert r >= 0, "invalid convolution descriptor"
        return r == 1

    def linear(rows, fin, fout, which):
        if which == 0:    # y[rows, fout] = x[rows, fin] @ W^T[fin, fout]
            a, b, c = _mat(rows, fin, fin, 1), _mat(fin, fout, 1, fin), _mat(rows, fout, fout, 1)
        elif which == 1:  # dX[rows, fin] = dY[rows, fout] @ W[fout, fin]
            a, b, c = _mat(rows, fout, fout, 1), _mat(fout, fin, fin, 1), _mat(rows, fin, fin, 1)
        else:             # dW[fout, fin] = dY^T[fout, rows] @ X[rows, fin]
            a, b, c = _mat(fout, rows, 1, fout), _mat(rows, fin, fin, 1), _mat(fout, fin, fin, 1)
        r = lib.pvb2_gemm_path(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), math)
        assert r >= 0, "invalid GEMM descriptor"
        return r == 1

    def attention(d):
        # the fused attention runs its tile products on TF32 tensor cores for
        # head dimensions 32 and 64 (sdpa_fwd_tc_kernel / sdpa_bwd_kv_tc_kernel)
        return math == 0 and d in (32, 64)

    return Paths(conv=conv, linear=linear, attention=attention)
