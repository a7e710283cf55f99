"""B200 `ocl` device backend for PyTorch.

Drop-in for the reference's ``pytorch_ocl`` package
(python/pytorch_ocl/__init__.py): importing it renames torch's PrivateUse1
backend to ``ocl`` and registers ``torch.ocl`` with the same API
(``synchronize``, ``manual_seed_all``, ``empty_cache``, ``profile``,
``enable_profiling``, ``device``, ``_is_in_bad_fork``) plus the usual
device-module helpers (``is_available``, ``device_count``,
``current_device``, ``set_device``, memory statistics).

All device arithmetic runs in hand-written sm_100a CUDA kernels
(``lib/libpvb2.so``, C-ABI in ``include/pvb2.h``) reached from the C++ host
extension ``_C``.  There is no CPU fallback: an op without a device kernel
raises ``NotImplementedError``.
"""
from __future__ import annotations

import os

import torch

try:
    from . import _C
except ImportError as e:  # the product path must fail loudly without its native code
    raise ImportError(
        "pytorch_vulkan_b200: native extension not built "
        "(run `python pytorch_vulkan_b200/_build.py`): " + str(e)
    ) from e

from ._C import (  # noqa: F401  (same impl_* names as the reference's pt_ocl module)
    impl_custom_device,
    impl_empty_cache,
    impl_enable_profiling,
    impl_is_bad_fork,
    impl_seed_all,
    impl_start_profiling,
    impl_stop_profiling,
    impl_synchronize_device,
)

MATH_TF32, MATH_FP32, MATH_3XTF32 = 0, 1, 2


def _device_index(device) -> int:
    """python/pytorch_ocl/__init__.py:4-13"""
    if isinstance(device, int):
        return device
    if isinstance(device, str):
        device = torch.device(device)
    if isinstance(device, torch.device):
        if device.index is None:
            return _C.impl_current_device()
        return device.index
    return -1


class _OCL:
    """The ``torch.ocl`` device module (python/pytorch_ocl/__init__.py:17-71)."""

    class profile:
        """Per-op device timing written as CSV (section,kernel,start,end,duration).

        Same contract as the reference's ``torch.ocl.profile(device, path)``:
        profiling is active only when ``path`` is not None.
        """

        def __init__(self, device, path=None):
            self._device_id = _device_index(device)
            self._path = path

        def __enter__(self):
            if self._path is not None:
                _C.impl_start_profiling(self._device_id)
            return self

        def __exit__(self, type, value, traceback):
            if self._path is not None:
                _C.impl_stop_profiling(self._device_id, self._path)
            return False

    @staticmethod
    def enable_profiling(device):
        return _C.impl_enable_profiling(_device_index(device))

    class device:
        """Context manager that makes `device` current (the reference's was a no-op)."""

        def __init__(self, device):
            self.idx = _device_index(device)
            self.prev = -1

        def __enter__(self):
            self.prev = _C.impl_current_device()
            if self.idx >= 0:
                _C.impl_set_device(self.idx)
            return self

        def __exit__(self, type, value, traceback):
            if self.prev >= 0:
                _C.impl_set_device(self.prev)
            return False

    @staticmethod
    def synchronize(dev=None):
        _C.impl_synchronize_device(-1 if dev is None else _device_index(dev))

    @staticmethod
    def manual_seed_all(seed: int):
        _C.impl_seed_all(int(seed) & 0xFFFFFFFFFFFFFFFF)

    @staticmethod
    def manual_seed(seed: int):
        _OCL.manual_seed_all(seed)

    @staticmethod
    def _is_in_bad_fork():
        return _C.impl_is_bad_fork()

    @staticmethod
    def empty_cache():
        _C.impl_empty_cache()

    # --- device-module helpers torch and user code expect
    @staticmethod
    def is_available() -> bool:
        return _C.impl_device_count() > 0

    @staticmethod
    def device_count() -> int:
        return _C.impl_device_count()

    @staticmethod
    def current_device() -> int:
        return _C.impl_current_device()

    @staticmethod
    def set_device(device):
        _C.impl_set_device(_device_index(device))

    @staticmethod
    def get_device_name(device=None) -> str:
        return _C.impl_device_name(_device_index(device if device is not None else _C.impl_current_device()))

    @staticmethod
    def is_initialized() -> bool:
        return True

    @staticmethod
    def memory_stats(device=None) -> dict:
        return _C.impl_memory_stats(_device_index(device if device is not None else _C.impl_current_device()))

    @staticmethod
    def memory_allocated(device=None) -> int:
        return _OCL.memory_stats(device)["allocated_bytes"]

    @staticmethod
    def max_memory_allocated(device=None) -> int:
        return _OCL.memory_stats(device)["peak_allocated_bytes"]

    @staticmethod
    def memory_reserved(device=None) -> int:
        return _OCL.memory_stats(device)["reserved_bytes"]

    @staticmethod
    def reset_peak_memory_stats(device=None):
        _C.impl_reset_peak_memory_stats(_device_index(device if device is not None else _C.impl_current_device()))

    @staticmethod
    def set_math_mode(mode: int):
        """0 = TF32 tensor cores (default), 1 = exact fp32 (SIMT); other values raise."""
        _C.impl_set_math_mode(int(mode))

    @staticmethod
    def get_math_mode() -> int:
        return _C.impl_get_math_mode()

    @staticmethod
    def kernel_launch_count() -> int:
        """Kernels launched by libpvb2 in this process (all devices)."""
        return _C.impl_launch_count()


from .graphs import Graph  # noqa: E402

_OCL.Graph = Graph


def synchronize(dev=None):
    """Module-level synchronize (the reference's referenced an undefined name, __init__.py:73-74)."""
    _OCL.synchronize(dev)


def manual_seed_all(seed):
    _OCL.manual_seed_all(seed)


def empty_cache():
    _OCL.empty_cache()


def is_available() -> bool:
    return _OCL.is_available()


def device_count() -> int:
    return _OCL.device_count()


def set_math_mode(mode: int):
    _OCL.set_math_mode(mode)


def get_math_mode() -> int:
    return _OCL.get_math_mode()


def _register():
    """python/pytorch_ocl/__init__.py:80-86"""
    if torch._C._get_privateuse1_backend_name() != "ocl":
        torch.utils.rename_privateuse1_backend("ocl")
    if not hasattr(torch, "ocl"):
        torch._register_device_module("ocl", _OCL)
    if not hasattr(torch.Tensor, "is_ocl"):
        torch.utils.generate_methods_for_privateuse1_backend(
            for_tensor=True, for_module=True, for_packed_sequence=True, for_storage=True
        )


_register()
