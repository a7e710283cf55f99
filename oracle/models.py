"""The workload definitions (test infrastructure view).

The builders, seeded inputs and losses live in
``pytorch_vulkan_b200/workloads.py``, a definitions-only module shared with
the benchmark; it is loaded here by file path so that importing the oracle
never loads the backend's native libraries.
"""
import importlib.util as _ilu
import os as _os

_path = _os.path.join(_os.path.dirname(_os.path.dirname(_os.path.abspath(__file__))), "pytorch_vulkan_b200",
                      "workloads.py")
_spec = _ilu.spec_from_file_location("_pvb2_workloads", _path)
_mod = _ilu.module_from_spec(_spec)
_spec.loader.exec_module(_mod)

MnistCNN = _mod.MnistCNN
CONFIGS = _mod.CONFIGS
GFLOP_PER_IMAGE = _mod.GFLOP_PER_IMAGE
build = _mod.build
make_inputs = _mod.make_inputs
loss_fn = _mod.loss_fn
