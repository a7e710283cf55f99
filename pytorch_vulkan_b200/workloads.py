"""Workload definitions of the training hot path: model builders, seeded
synthetic inputs and losses, shared by the benchmark and the oracle.

The five configurations of the benchmark: an MNIST-shaped CNN, ResNet-18,
ResNet-50, MobileNet-v2 and ViT-B/16, all fp32, random-initialised from a
seed (pretrained weights need a network and are not used).  The torchvision
builders are the same models the reference validates in
tests/validate_network.py:249-292.

This module holds definitions only (no arithmetic of its own) and depends on
nothing in this package, so the oracle loads it by path without loading the
backend.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class MnistCNN(nn.Module):
    """conv 1->32 3x3 -> ReLU -> conv 32->64 3x3 -> ReLU -> maxpool 2 ->
    flatten 9216 -> linear 128 -> ReLU -> linear 10 -> log_softmax.
    (Differs from the reference's mnist.py:12-44 net on purpose: this is the
    benchmark's MNIST-shaped configuration.)"""

    def __init__(self):
        super().__init__()
        self.conv1 = nn.Conv2d(1, 32, 3, 1)
        self.conv2 = nn.Conv2d(32, 64, 3, 1)
        self.fc1 = nn.Linear(9216, 128)
        self.fc2 = nn.Linear(128, 10)

    def forward(self, x):
        x = F.relu(self.conv1(x))
        x = F.relu(self.conv2(x))
        x = F.max_pool2d(x, 2)
        x = torch.flatten(x, 1)
        x = F.relu(self.fc1(x))
        return F.log_softmax(self.fc2(x), dim=1)


# name -> (builder, input shape (C,H,W), classes, default per-GPU batch, loss)
CONFIGS = {
    "mnist": (lambda: MnistCNN(), (1, 28, 28), 10, 64, "nll"),
    "resnet18": (lambda: __import__("torchvision").models.resnet18(), (3, 224, 224), 1000, 64, "ce"),
    "resnet50": (lambda: __import__("torchvision").models.resnet50(), (3, 224, 224), 1000, 64, "ce"),
    "mobilenet_v2": (lambda: __import__("torchvision").models.mobilenet_v2(), (3, 224, 224), 1000, 128, "ce"),
    "vit_b_16": (lambda: __import__("torchvision").models.vit_b_16(), (3, 224, 224), 1000, 32, "ce"),
}

# algorithmic work per image, fwd+bwd (2*MAC of conv/linear/bmm)
GFLOP_PER_IMAGE = {"mnist": 0.072, "resnet18": 10.65, "resnet50": 24.30, "mobilenet_v2": 1.81, "vit_b_16": 100.9}


def build(name: str, seed: int = 0) -> nn.Module:
    """Weights from torch.manual_seed(seed) with the default (Kaiming-uniform) init, on CPU."""
    torch.manual_seed(seed)
    return CONFIGS[name][0]()


def make_inputs(name: str, batch: int, seed: int = 1234):
    """Seeded synthetic inputs: MNIST x~U[0,1), labels 0-9; ImageNet-shaped x~N(0,1), labels 0-999."""
    _, shape, classes, _, _ = CONFIGS[name]
    g = torch.Generator().manual_seed(seed)
    if name == "mnist":
        x = torch.rand((batch, *shape), generator=g)
    else:
        x = torch.randn((batch, *shape), generator=g)
    y = torch.randint(0, classes, (batch,), generator=g)
    return x, y


def loss_fn(name: str):
    return F.nll_loss if CONFIGS[name][4] == "nll" else F.cross_entropy
