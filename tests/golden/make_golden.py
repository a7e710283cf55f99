"""Regenerate the golden fixtures of the oracle (torch-CPU, the reference's
validation path).  Run from the repository root:

    python tests/golden/make_golden.py

mnist_step.pt : output/loss/gradients/state after 2 SGD-momentum steps of the
                MNIST-shaped CNN (batch 8, weight seed 0, input seed 1234).
ops.pt        : a seeded input, its 3x3/s2/p1 max-pool indices and log-softmax.
"""
import os
import sys

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import step  # noqa: E402


def main():
    _, snap = step.cpu_reference("mnist", batch=8, steps=2)
    keep = {k: v for k, v in snap.items() if k in ("loss", "output") or k.startswith("grad.fc2") or
            k.startswith("grad.conv1") or k.startswith("state.conv1")}
    torch.save(keep, os.path.join(HERE, "mnist_step.pt"))
    g = torch.Generator().manual_seed(7)
    x = torch.randn(4, 3, 8, 8, generator=g)
    _, ind = F.max_pool2d(x, 3, 2, 1, return_indices=True)
    torch.save({"seed": torch.tensor(7), "x": x, "maxpool_ind": ind, "log_softmax": F.log_softmax(x.flatten(1), 1)},
               os.path.join(HERE, "ops.pt"))
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
