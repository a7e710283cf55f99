"""CUDA-graph capture and replay of `ocl` work (pytorch_vulkan_b200/graphs.py,
csrc/host/backend.cpp): a replay runs exactly the captured kernels, so a
training step replayed from a graph must give the same losses and
parameters, bit for bit, as the same steps run eagerly from the same state
(the deferred batch-norm epilogues, the pending num_batches_tracked
increment, the staged convolution copies and the activation masks formed
from x all take part, decided once at capture)."""
import copy

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu
DEV = "ocl:0"


def test_graph_replays_captured_ops(ocl):
    x = torch.zeros(3, 1000).to(DEV)
    g = torch.ocl.Graph()
    with g.capture():
        y = torch.relu(x * 2.0 + 1.0)
        z = y.sum(dim=1)
    assert g.kernels > 0
    for k in range(3):
        src = torch.randn(3, 1000, generator=torch.Generator().manual_seed(k))
        x.copy_(src.to(DEV))
        n0 = torch.ocl.kernel_launch_count()
        g.replay()
        assert torch.ocl.kernel_launch_count() - n0 == g.kernels
        ref = torch.relu(src * 2.0 + 1.0)
        assert torch.equal(y.cpu(), ref)
        assert torch.allclose(z.cpu(), ref.sum(dim=1), rtol=1e-5, atol=1e-4)
    g.reset()


class _Block(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.conv1 = nn.Conv2d(c, c, 3, padding=1, bias=False)
        self.bn1 = nn.BatchNorm2d(c)
        self.conv2 = nn.Conv2d(c, c, 3, padding=1, bias=False)
        self.bn2 = nn.BatchNorm2d(c)
        self.relu = nn.ReLU(inplace=True)

    def forward(self, x):
        out = self.relu(self.bn1(self.conv1(x)))
        out = self.bn2(self.conv2(out))
        out += x
        return self.relu(out)


def _net():
    torch.manual_seed(5)
    return nn.Sequential(nn.Conv2d(3, 32, 3, padding=1, bias=False), nn.BatchNorm2d(32), nn.ReLU(inplace=True),
                         _Block(32), _Block(32), nn.AdaptiveAvgPool2d(1), nn.Flatten(), nn.Linear(32, 10))


def test_graph_training_step_matches_eager(ocl):
    model = _net().to(DEV).train()
    opt = torch.optim.SGD(model.parameters(), lr=0.05, momentum=0.9, fused=True)
    g_in = torch.Generator().manual_seed(6)
    x = torch.randn(8, 3, 16, 16, generator=g_in).to(DEV)
    y = torch.randint(0, 10, (8,), generator=g_in).to(DEV)
    loss_fn = nn.CrossEntropyLoss()

    def step():
        opt.zero_grad(set_to_none=True)
        loss = loss_fn(model(x), y)
        loss.backward()
        opt.step()
        return loss

    for _ in range(2):  # momentum buffers exist before the snapshot
        step()
    torch.ocl.synchronize()
    state = copy.deepcopy({k: v.cpu() for k, v in model.state_dict().items()})
    moms = [opt.state[p]["momentum_buffer"].cpu() for p in model.parameters()]

    def restore():
        with torch.no_grad():
            for k, v in model.state_dict().items():
                v.copy_(state[k].to(DEV))
            for p, m in zip(model.parameters(), moms):
                opt.state[p]["momentum_buffer"].copy_(m.to(DEV))
        torch.ocl.synchronize()

    eager_losses = [step().item() for _ in range(3)]
    eager_state = {k: v.cpu() for k, v in model.state_dict().items()}
    restore()
    graph = torch.ocl.Graph()
    with graph.capture():
        loss = step()
    graph_losses = []
    for _ in range(3):
        graph.replay()
        graph_losses.append(loss.item())
    graph_state = {k: v.cpu() for k, v in model.state_dict().items()}
    assert graph_losses == eager_losses
    for k in eager_state:
        assert torch.equal(eager_state[k], graph_state[k]), k
    graph.reset()
    # eager steps still run after the graph is gone
    step()
    torch.ocl.synchronize()
