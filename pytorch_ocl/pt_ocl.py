"""The reference's ``pt_ocl`` extension module (src/python_iface.cpp:79-88):
every ``impl_*`` function of the B200 host extension under its own name."""
from pytorch_vulkan_b200 import _C as _ext

__all__ = sorted(n for n in dir(_ext) if n.startswith("impl_"))
globals().update({n: getattr(_ext, n) for n in __all__})
