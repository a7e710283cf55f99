"""The reference's own network validation, on its own images.

tests/validate_network.py:15-38 builds a batch of four real images
(tests/samples/{cat,dog,parrot,goldfish}.ppm, ImageNet-normalised in float32,
labels 281 / 207 / 87 / 1), runs one step on the device and on torch-CPU
(:62-106; LogSoftmax + NLLLoss, no optimizer step, training mode except the
networks it validates in eval mode), and passes when the largest absolute
difference over the output and every parameter gradient is <= 1e-2
(:109-122).  The images come from tests/golden/ppm_samples.pt (made by
tests/golden/make_ppm_fixture.py from those files).

Differences from the reference's run: the weights are random (its pretrained
ImageNet weights need a network), so ViT-B/16's zero-initialised head gets
random weights for gradients to reach the encoder.

Criteria:
* exact-fp32 math (math=1): the reference's max-abs <= 1e-2 against torch-CPU
  fp32 for ResNet-18, MobileNet-v2 (eval, as the reference validates it) and
  ViT-B/16.  ResNet-50 with random weights is too ill-conditioned for an
  absolute criterion (torch-CPU fp32 itself is 0.27 away from float64 on the
  stem's weight gradient, whose entries reach 19), so it is held, per tensor,
  to 10x torch-CPU fp32's own error against float64 plus the floors below.
* TF32 math (math=0): every network per tensor against the TF32-emulating
  float64 oracle, within 10x the emulated fp32 CPU run's error plus a floor.
The floors are those of test_network_gpu.py: 1e-5 for the output, 2e-2 for
each gradient (a few ReLU-mask or max-pool-argmax decisions taken the other
way on values within an ulp of the threshold move a layer's gradient by
about 1% relative; the ResNet-18 run here shows one such event on the
device, at layer4, and torch-CPU fp32 one at layer3).
"""
import copy
import json
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import tf32_paths
from oracle import models
from oracle.tf32 import Tf32Emulation

pytestmark = pytest.mark.gpu
DEV = "ocl:0"
HERE = os.path.dirname(os.path.abspath(__file__))
FLOOR_FWD, FLOOR = 1e-5, 2e-2


def floor_for(key):
    return FLOOR_FWD if key == "output" else FLOOR


def ppm_batch():
    """validate_network.py:15-38 make_batch('standard') from the fixture"""
    d = torch.load(os.path.join(HERE, "golden", "ppm_samples.pt"))
    img = d["images"].numpy().astype(np.float32) * (1.0 / 255)
    mean = np.array([0.485, 0.456, 0.406]).astype(np.float32)
    std = np.array([0.229, 0.224, 0.225]).astype(np.float32)
    fact = 1.0 / np.array(std)
    off = -np.array(mean) * fact
    data = np.zeros((4, 3, 224, 224)).astype(np.float32)
    for k in range(3):
        data[:, k, :, :] = img[:, :, :, k] * fact[k] + off[k]
    return torch.from_numpy(data), d["labels"].clone()


def _model(name):
    m = models.build(name, 0)
    if name == "vit_b_16":
        g = torch.Generator().manual_seed(1)
        with torch.no_grad():
            m.heads.head.weight.copy_(torch.randn(m.heads.head.weight.shape, generator=g) * 0.02)
    return m


def one_step(model, x, y, train):
    """validate_network.py:58-92 step() with opt_steps = 0: output and gradients"""
    model.train(train)
    out = model(x)
    loss = F.nll_loss(F.log_softmax(out, dim=1), y)
    loss.backward()
    r = {"output": out.detach().to("cpu", torch.float64)}
    for n, p in model.named_parameters():
        if p.grad is not None:
            r[n] = p.grad.detach().to("cpu", torch.float64)
    return r


def cpu_step(model, x, y, train, dtype):
    m = copy.deepcopy(model).to(dtype)
    return one_step(m, x.to(dtype), y, train)


def rel(a, truth):
    return {k: (a[k] - t).norm().item() / max(t.norm().item(), 1e-30) for k, t in truth.items()}


# (network, training mode) as the reference's --all list validates them
NETS = [("resnet18", True), ("resnet50", True), ("mobilenet_v2", False), ("vit_b_16", True)]


@pytest.mark.parametrize("math", [1, 0])
@pytest.mark.parametrize("name,train", NETS, ids=[n for n, _ in NETS])
def test_reference_images(ocl, name, train, math):
    x, y = ppm_batch()
    model = _model(name)
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(math)
    try:
        got = one_step(copy.deepcopy(model).to(DEV), x.to(DEV), y.to(DEV), train)
    finally:
        torch.ocl.set_math_mode(old)
    ref32 = cpu_step(model, x, y, train, torch.float32)  # the reference's comparison run
    max_abs = max((got[k] - ref32[k]).abs().max().item() for k in ref32)
    paths = tf32_paths.device_paths() if math == 0 else None
    with Tf32Emulation(paths):
        t64 = cpu_step(model, x, y, train, torch.float64)
        t32 = cpu_step(model, x, y, train, torch.float32)
    e_dev, e_cpu = rel(got, t64), rel(t32, t64)
    bad = {k: (e_dev[k], e_cpu[k]) for k in t64 if e_dev[k] > 10 * e_cpu[k] + floor_for(k)}
    path = os.environ.get("PVB2_PARITY_LOG")
    if path:
        worst = max(t64, key=lambda k: e_dev[k] / (10 * e_cpu[k] + floor_for(k)))
        with open(path, "a") as f:
            f.write(json.dumps({"test": f"ppm_{name}_math{math}", "max_abs_vs_cpu_fp32": max_abs,
                                "worst_key": worst, "worst_dev_err": e_dev[worst],
                                "worst_cpu_err": e_cpu[worst]}) + "\n")
    assert not bad, f"{name}: {len(bad)} tensors off (dev err, cpu err): {list(bad.items())[:5]}"
    if math == 1 and name != "resnet50":
        assert max_abs <= 1e-2, f"{name}: max abs diff {max_abs} against torch-CPU fp32 (reference criterion 1e-2)"
