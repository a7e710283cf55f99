"""Network-level parity of whole training steps on the `ocl` device against the
torch-CPU oracle -- the reference's tests/validate_network.py:62-122 harness
(same weights and inputs; output, loss, every parameter gradient and the
state after an SGD-momentum step are compared).

Exact-fp32 math (math=1): each tensor is compared as described below.  With
TF32 tensor cores (math=0) the comparison has to account for how sensitive
the step is: truncating the weights to TF32 alone (mantissa cut to 10 bits)
moves ResNet-50's fp64 gradients by ~100% (median, batch 2), MobileNet-v2's
by ~75% and ResNet-18's by ~20% at random init.  So in TF32 mode the
device's global relative gradient error (all gradients concatenated) and its
output / loss errors must be within 3x of that TF32-truncated-weights fp64
run's (plus 1e-3).

The reference's pass criterion is max abs diff <= 1e-2 (validate_network.py:119,
with pretrained weights and real images).  With random-init weights and the
small batches a CPU-side test can afford, training-mode batch norm makes deep
gradients ill-conditioned: torch-CPU fp32 run with 1 and with 8 threads
disagrees by up to 0.18 abs / 14% relative on ResNet-50's gradients.  So each
tensor is measured against a float64 CPU run of the same step (the ground
truth): the device's relative Frobenius error must be within 10x torch-CPU
fp32's own error plus a floor: 2e-2 with TF32 tensor cores; 1e-3 in exact-fp32
math, because a last-bit difference in an activation can flip a ReLU sign or
a max-pool argmax and route a whole gradient element elsewhere (on the
MNIST net only the gradients upstream of the pool move, while conv2.bias,
the routing-invariant sum of dy, matches to 1e-7).  The reference's max-abs
figure is reported alongside.

Batch sizes are reduced so the CPU side finishes in seconds; the layer
shapes are those of the benchmark configurations.  MobileNet-v2's classifier
dropout is set to p=0 for the comparison (the device draws its own Philox
stream); ViT-B/16's dropout is 0 by default."""
import copy

import pytest
import torch

from oracle import models, step

pytestmark = pytest.mark.gpu
DEV = "ocl:0"
FLOOR = {0: 2e-2, 1: 1e-3}


def tf32_truncated(model):
    """copy of `model` with every floating parameter's mantissa cut to TF32's 10 bits"""
    m = copy.deepcopy(model)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_((p.detach().view(torch.int32) & ~0x1FFF).view(torch.float32))
    return m


def global_rel(a, truth, prefix="grad."):
    keys = [k for k in truth if k.startswith(prefix) and k in a]
    num = sum(((a[k] - truth[k]) ** 2).sum().item() for k in keys)
    den = sum((truth[k] ** 2).sum().item() for k in keys)
    return (num / max(den, 1e-300)) ** 0.5


def run_parity(name, batch, math=0, steps=1, prep=None):
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(math)
    try:
        model = models.build(name, 0)
        if prep:
            prep(model)
        dev_model = copy.deepcopy(model).to(DEV)
        _, ref64 = step.cpu_reference(name, batch, steps=steps, model=copy.deepcopy(model), dtype=torch.float64)
        if math == 0:
            _, pert64 = step.cpu_reference(name, batch, steps=steps, model=tf32_truncated(model), dtype=torch.float64)
        _, ref32 = step.cpu_reference(name, batch, steps=steps, model=model)
        x, y = models.make_inputs(name, batch, 1234)
        opt = torch.optim.SGD(dev_model.parameters(), lr=0.01, momentum=0.9)
        dev_model.train()
        for _ in range(steps):
            out, l = step.train_step(dev_model, x.to(DEV), y.to(DEV), models.loss_fn(name), opt)
        got = step.snapshot(dev_model, out, l, with_state=True)
        assert set(ref32) == set(got)
        worst_abs = step.max_abs_diff(ref32, got)
        e_dev = step.frob_rel(got, ref64)
        if math == 0:
            e_pert = step.frob_rel(pert64, ref64)
            g_dev, g_pert = global_rel(got, ref64), global_rel(pert64, ref64)
            assert g_dev <= 3 * g_pert + 1e-3, f"{name}: gradient error {g_dev} vs TF32-weights {g_pert}"
            for k in ("output", "loss"):
                assert e_dev[k] <= 3 * e_pert[k] + 1e-3, f"{name}: {k} error {e_dev[k]} vs TF32-weights {e_pert[k]}"
            return g_dev, worst_abs
        e_cpu = step.frob_rel(ref32, ref64)
        bad = {k: (e_dev[k], e_cpu[k]) for k in e_dev if e_dev[k] > 10 * e_cpu[k] + FLOOR[math]}
        worst_rel = max(e_dev.items(), key=lambda kv: kv[1])
        assert not bad, f"{name}: {len(bad)} tensors off (dev err, cpu err): {list(bad.items())[:5]}; " \
                        f"max abs vs cpu fp32 {worst_abs}"
        return worst_rel, worst_abs
    finally:
        torch.ocl.set_math_mode(old)


@pytest.mark.parametrize("math", [0, 1])
def test_mnist_step(ocl, math):
    run_parity("mnist", 64, math=math, steps=2)
    # the reference's own criterion holds for this well-conditioned net
    model = models.build("mnist", 0)
    dm = copy.deepcopy(model).to(DEV)
    _, ref = step.cpu_reference("mnist", 64, steps=2, model=model)
    x, y = models.make_inputs("mnist", 64, 1234)
    opt = torch.optim.SGD(dm.parameters(), lr=0.01, momentum=0.9)
    for _ in range(2):
        out, l = step.train_step(dm, x.to(DEV), y.to(DEV), torch.nn.functional.nll_loss, opt)
    assert step.max_abs_diff(ref, step.snapshot(dm, out, l, with_state=True))[0] <= 1e-2


@pytest.mark.parametrize("math", [0, 1])
def test_resnet18_step(ocl, math):
    run_parity("resnet18", 4, math=math)


@pytest.mark.parametrize("math", [0, 1])
def test_resnet50_step(ocl, math):
    run_parity("resnet50", 2, math=math)


@pytest.mark.parametrize("math", [0, 1])
def test_mobilenet_v2_step(ocl, math):
    def no_dropout(m):
        m.classifier[0].p = 0.0

    run_parity("mobilenet_v2", 4, math=math, prep=no_dropout)


@pytest.mark.parametrize("math", [0, 1])
def test_vit_b_16_step(ocl, math):
    run_parity("vit_b_16", 2, math=math)


def test_resnet50_full_batch_properties(ocl):
    """At the benchmark batch (64) the CPU oracle is too slow per test; check
    size-independent properties instead: the loss is finite and near ln(1000)
    at init, BN running stats moved, and two identical runs are bit-identical
    (deterministic kernels)."""
    losses = []
    for _ in range(2):
        model = models.build("resnet50", 0).to(DEV)
        x, y = models.make_inputs("resnet50", 64, 1234)
        xd, yd = x.to(DEV), y.to(DEV)
        opt = torch.optim.SGD(model.parameters(), lr=0.05, momentum=0.9)
        l0 = step.train_step(model, xd, yd, torch.nn.functional.cross_entropy, opt)[1].item()
        l1 = step.train_step(model, xd, yd, torch.nn.functional.cross_entropy, opt)[1].item()
        losses.append((l0, l1))
        assert abs(l0 - 6.9) < 1.0 and l1 == l1
        assert model.bn1.running_mean.abs().sum().item() > 0
    assert losses[0] == losses[1]
