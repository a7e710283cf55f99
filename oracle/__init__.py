"""Oracle for the `ocl` training hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker / the timed
CPU reference.  The product path (``pytorch_vulkan_b200``) never imports,
calls or falls back to anything here.

What the oracle is
------------------
The reference (pytorch_ocl 0.2.0) validates its device kernels by running the
same step on torch-CPU ATen and comparing (tests/validate_network.py:94-106,
tests/test_op.py:22-104).  Its device arithmetic lives in the external
``dlprimitives`` library, which is absent from the reference tree (empty git
submodule), so dlprimitives itself cannot be run: parity against dlprimitives
is *unpinned*.  The arbiter is therefore exactly the reference's own:

* ``oracle.step``   -- the torch-CPU fp32 training step of the five workloads
  (same seeded weights and synthetic inputs as the device run);
* ``oracle.models`` -- the workload definitions (MNIST-shaped CNN as
  specified for the benchmark, torchvision ResNet-18/50, MobileNet-v2,
  ViT-B/16);
* ``oracle.npref``  -- independent numpy restatements of the semantics the
  kernels must reproduce (batch-norm statistics and running-stat update,
  max-pool argmax with first-index ties, NLL mean, log-softmax, GELU,
  hardtanh mask, SGD-momentum), cross-checked against torch-CPU in the CPU
  test suite so that the arbiter itself is pinned.

The committed fixtures under ``tests/golden/`` (made by
``tests/golden/make_golden.py`` from this oracle) pin the oracle's outputs
for small cases across torch versions.
"""

from . import models, npref, step  # noqa: F401
