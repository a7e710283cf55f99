"""``import pytorch_ocl`` for code written against the reference's package
(python/pytorch_ocl/__init__.py:1-86).

Importing it loads the B200 backend (``pytorch_vulkan_b200``): torch's
PrivateUse1 backend becomes ``ocl``, ``torch.ocl`` is registered, and the
module-level helpers (``synchronize``, ``manual_seed_all``, ``empty_cache``)
and the ``impl_*`` functions of the reference's ``pt_ocl`` extension module
(src/python_iface.cpp:79-88) are reachable here under the same names, so
scripts such as the reference's tests/validate_network.py run unchanged.
"""
import pytorch_vulkan_b200 as _backend

from .pt_ocl import *  # noqa: F401,F403  (as the reference's __init__.py:2)
from .pt_ocl import __all__ as _impl_names

_device_index = _backend._device_index
_OCL = _backend._OCL
synchronize = _backend.synchronize
manual_seed_all = _backend.manual_seed_all
empty_cache = _backend.empty_cache
is_available = _backend.is_available
device_count = _backend.device_count

__all__ = list(_impl_names) + ["synchronize", "manual_seed_all", "empty_cache", "is_available", "device_count"]
