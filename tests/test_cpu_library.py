"""CPU-only checks of the native libraries: the C-ABI library loads and exports
every entry point that include/pvb2.h declares, status/error reporting works
without a GPU, and the torch host extension imports and registers the `ocl`
device module with the reference's API (python/pytorch_ocl/__init__.py)."""
import ctypes
import os
import re

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "pytorch_vulkan_b200", "lib", "libpvb2.so")
HDR = os.path.join(REPO, "include", "pvb2.h")


def declared_symbols():
    text = open(HDR).read()
    return sorted(set(re.findall(r"PVB2_API\s+[\w\s\*]+?\b(pvb2_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) > 50
    for must in ["pvb2_conv2d_fwd", "pvb2_conv2d_bwd_data", "pvb2_conv2d_bwd_filter", "pvb2_gemm",
                 "pvb2_batch_norm_fwd_train", "pvb2_batch_norm_bwd", "pvb2_layer_norm_fwd", "pvb2_max_pool2d_fwd",
                 "pvb2_softmax_fwd", "pvb2_nll_loss_fwd", "pvb2_sgd_multi", "pvb2_philox_fill",
                 "pvb2_nccl_allreduce"]:
        assert must in syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"not exported: {missing}"


def test_library_status_without_gpu():
    lib = ctypes.CDLL(LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p
    n = ctypes.c_int(-1)
    assert lib.pvb2_device_count(ctypes.byref(n)) == 0
    assert n.value >= 0
    assert lib.pvb2_version() >= 1
    if n.value == 0:
        # an invalid request is reported as a status code with a message, never an abort
        assert lib.pvb2_set_device(7) != 0
        assert len(lib.pvb2_last_error()) > 0


def test_launcher_argument_checks_need_no_gpu():
    """Shape validation happens on the host before any launch."""
    lib = ctypes.CDLL(LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p

    class T(ctypes.Structure):
        _fields_ = [("data", ctypes.c_void_p), ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8),
                    ("ndim", ctypes.c_int32), ("dtype", ctypes.c_int32)]

    a = T(None, (ctypes.c_int64 * 8)(2, 3, 4), (ctypes.c_int64 * 8)(12, 4, 1), 3, 0)
    b = T(None, (ctypes.c_int64 * 8)(2, 5, 4), (ctypes.c_int64 * 8)(20, 4, 1), 3, 0)
    c = T(None, (ctypes.c_int64 * 8)(2, 3, 4), (ctypes.c_int64 * 8)(12, 4, 1), 3, 0)
    st = lib.pvb2_gemm(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None, 1, ctypes.c_double(1.0),
                       ctypes.c_double(0.0), 0, None)
    assert st == 1  # PVB2_ERR_INVALID: K mismatch (4 vs 5)
    assert b"shape mismatch" in lib.pvb2_last_error()


class _Conv(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ["N", "C", "H", "W", "K", "R", "S", "P", "Q", "stride_h", "stride_w",
                                             "pad_h", "pad_w", "dil_h", "dil_w", "groups", "math"]]


def _conv(N, C, H, W, K, R, st, pd, math=0):
    P = (H + 2 * pd - R) // st + 1
    return _Conv(N, C, H, W, K, R, R, P, P, st, st, pd, pd, 1, 1, 1, math)


def test_conv_path_queries_need_no_gpu():
    """Which tensor-core path a convolution takes is host logic: the size of
    the staged input a training forward can keep for its weight gradient
    (channels-last copy, im2col columns, or none), and whether a dgrad can
    also form a sum in its epilogue (1x1 stride 1, 16-byte planes, TF32)."""
    lib = ctypes.CDLL(LIB)
    lib.pvb2_conv2d_staged_input_bytes.restype = ctypes.c_size_t
    q = lambda d: lib.pvb2_conv2d_staged_input_bytes(ctypes.byref(d))
    assert q(_conv(64, 64, 56, 56, 64, 3, 1, 1)) == 64 * 56 * 56 * 64 * 4       # channels-last copy
    assert q(_conv(64, 3, 224, 224, 64, 7, 2, 3)) == 64 * 230 * 230 * 16       # stem: padded 4-channel row windows
    assert q(_conv(64, 256, 56, 56, 64, 1, 1, 0)) == 0                          # pointwise: reads NCHW
    assert q(_conv(64, 64, 56, 56, 64, 3, 1, 1, math=1)) == 0                   # exact fp32: SIMT path
    al = ctypes.c_void_p(1 << 20)
    ok = lambda d, p=al: lib.pvb2_conv2d_bwd_data_acc_ok(ctypes.byref(d), p, p, p, p)
    assert ok(_conv(64, 256, 56, 56, 64, 1, 1, 0)) == 1
    assert ok(_conv(64, 256, 56, 56, 64, 1, 1, 0), ctypes.c_void_p((1 << 20) + 4)) == 0  # not 16-byte aligned
    assert ok(_conv(64, 2048, 7, 7, 512, 1, 1, 0)) == 0    # 49-pixel planes
    assert ok(_conv(64, 64, 56, 56, 64, 3, 1, 1)) == 0     # 3x3
    assert ok(_conv(64, 256, 56, 56, 64, 1, 1, 0, math=1)) == 0


def test_package_registers_ocl_module():
    import pytorch_vulkan_b200 as pkg

    assert torch._C._get_privateuse1_backend_name() == "ocl"
    for name in ["synchronize", "manual_seed_all", "empty_cache", "profile", "enable_profiling", "device",
                 "_is_in_bad_fork", "is_available", "device_count"]:
        assert hasattr(torch.ocl, name), name
    for name in ["impl_custom_device", "impl_seed_all", "impl_synchronize_device", "impl_is_bad_fork",
                 "impl_empty_cache", "impl_enable_profiling", "impl_start_profiling", "impl_stop_profiling"]:
        assert hasattr(pkg, name), name
    assert hasattr(torch.Tensor, "is_ocl")


def test_no_cpu_fallback_without_device():
    """Without a device the backend raises instead of silently computing on the CPU."""
    import pytorch_vulkan_b200  # noqa: F401

    if torch.ocl.is_available():
        pytest.skip("a device is visible")
    with pytest.raises(RuntimeError):
        torch.empty(3, device="ocl")


def test_reference_package_name_imports():
    """`import pytorch_ocl` works unchanged (python/pytorch_ocl/__init__.py:1-2):
    the package re-exports the reference's pt_ocl `impl_*` names and helpers."""
    import pytorch_ocl
    from pytorch_ocl import pt_ocl

    for name in ["impl_custom_device", "impl_seed_all", "impl_synchronize_device", "impl_is_bad_fork",
                 "impl_empty_cache", "impl_enable_profiling", "impl_start_profiling", "impl_stop_profiling"]:
        assert callable(getattr(pt_ocl, name)), name
        assert getattr(pytorch_ocl, name) is getattr(pt_ocl, name)
    for name in ["synchronize", "manual_seed_all", "empty_cache"]:
        assert callable(getattr(pytorch_ocl, name)), name
    assert torch._C._get_privateuse1_backend_name() == "ocl"
    assert pytorch_ocl._device_index("ocl:3") == 3


def test_unimplemented_math_mode_is_rejected():
    """3xTF32 (math mode 2) is not implemented: the host refuses it and the
    C-ABI convolution / GEMM entry points return PVB2_ERR_UNSUPPORTED."""
    import pytorch_vulkan_b200  # noqa: F401

    with pytest.raises(RuntimeError):
        torch.ocl.set_math_mode(2)
    assert torch.ocl.get_math_mode() in (0, 1)
    lib = ctypes.CDLL(LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p

    class T(ctypes.Structure):
        _fields_ = [("data", ctypes.c_void_p), ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8),
                    ("ndim", ctypes.c_int32), ("dtype", ctypes.c_int32)]

    a = T(None, (ctypes.c_int64 * 8)(1, 3, 4), (ctypes.c_int64 * 8)(12, 4, 1), 3, 0)
    b = T(None, (ctypes.c_int64 * 8)(1, 4, 5), (ctypes.c_int64 * 8)(20, 5, 1), 3, 0)
    c = T(None, (ctypes.c_int64 * 8)(1, 3, 5), (ctypes.c_int64 * 8)(15, 5, 1), 3, 0)
    assert lib.pvb2_gemm(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None, 1, ctypes.c_double(1.0),
                         ctypes.c_double(0.0), 2, None) == 2
    x = T(None, (ctypes.c_int64 * 8)(1, 4, 8, 8), (ctypes.c_int64 * 8)(256, 64, 8, 1), 4, 0)
    y = T(None, (ctypes.c_int64 * 8)(1, 4, 8, 8), (ctypes.c_int64 * 8)(256, 64, 8, 1), 4, 0)
    d = _conv(1, 4, 8, 8, 4, 3, 1, 1, math=2)
    assert lib.pvb2_conv2d_fwd(ctypes.byref(d), ctypes.byref(x), None, None, ctypes.byref(y), None,
                               ctypes.c_size_t(0), None) == 2
    assert b"math mode 2" in lib.pvb2_last_error()


def test_graph_api_host_side():
    """torch.ocl.Graph refuses replay() before a capture and reports no
    kernels; the C-ABI graph calls check their arguments before touching a
    device (a NULL graph is refused, destroying NULL is a no-op)."""
    import pytorch_vulkan_b200  # noqa: F401

    g = torch.ocl.Graph(0)
    assert g.kernels == 0 and g.device == 0
    with pytest.raises(RuntimeError):
        g.replay()
    g.reset()
    lib = ctypes.CDLL(LIB)
    lib.pvb2_last_error.restype = ctypes.c_char_p
    assert lib.pvb2_graph_launch(None, None) != 0
    assert b"graph" in lib.pvb2_last_error()
    n = ctypes.c_int64(-1)
    assert lib.pvb2_graph_kernel_count(None, ctypes.byref(n)) != 0
    assert lib.pvb2_graph_destroy(None) == 0
    assert lib.pvb2_graph_capture_begin(None) != 0
