"""The torch-CPU training step: the reference's own validation path
(tests/validate_network.py:62-106: deep-copy the state, run the step on the
device, restore the state, re-run the same step on CPU and compare output,
every parameter gradient and, with optimizer steps, the updated state).
Test infrastructure only.
"""
from __future__ import annotations

import copy
import time

import torch

from . import models


def train_step(model, x, y, loss, optimizer=None):
    """One step: zero_grad, forward, loss, backward, optional optimizer step.
    Returns (output, loss) detached."""
    if optimizer is not None:
        optimizer.zero_grad(set_to_none=True)
    out = model(x)
    l = loss(out, y)
    l.backward()
    if optimizer is not None:
        optimizer.step()
    return out.detach(), l.detach()


def snapshot(model, out=None, loss=None, with_state=False):
    """Output, loss, every parameter gradient (and optionally the state) as CPU float64 tensors."""
    r = {}
    if out is not None:
        r["output"] = out.detach().to("cpu", torch.float64)
    if loss is not None:
        r["loss"] = loss.detach().to("cpu", torch.float64)
    for n, p in model.named_parameters():
        if p.grad is not None:
            r["grad." + n] = p.grad.detach().to("cpu", torch.float64)
    if with_state:
        for n, t in model.state_dict().items():
            if t.is_floating_point():
                r["state." + n] = t.detach().to("cpu", torch.float64)
    return r


def cpu_reference(name: str, batch: int, steps: int = 1, lr: float = 0.01, momentum: float = 0.9, seed: int = 0,
                  input_seed: int = 1234, model=None, dtype=torch.float32):
    """Run `steps` SGD steps of workload `name` on CPU; return (model, snapshot of the last step).
    dtype=torch.float64 gives the ground truth that fp32 results are measured against."""
    if model is None:
        model = models.build(name, seed)
    model = model.to(dtype)
    x, y = models.make_inputs(name, batch, input_seed)
    x = x.to(dtype)
    opt = torch.optim.SGD(model.parameters(), lr=lr, momentum=momentum, foreach=False)
    loss = models.loss_fn(name)
    model.train()
    out = l = None
    for _ in range(steps):
        out, l = train_step(model, x, y, loss, opt)
    return model, snapshot(model, out, l, with_state=True)


def max_abs_diff(a: dict, b: dict):
    """max |a-b| over common keys; returns (worst value, worst key)."""
    worst, key = 0.0, None
    for k in a:
        if k not in b:
            continue
        d = (a[k] - b[k]).abs().max().item() if a[k].numel() else 0.0
        if d > worst or key is None:
            worst, key = d, k
    return worst, key


def rel_diff(a: dict, b: dict):
    """per-key max|a-b| / max(max|a|, tiny) -- scale-free comparison."""
    out = {}
    for k in a:
        if k in b and a[k].numel():
            scale = max(a[k].abs().max().item(), 1e-12)
            out[k] = (a[k] - b[k]).abs().max().item() / scale
    return out


def time_cpu_steps(name: str, batch: int, steps: int, warmup: int = 1, threads: int | None = None):
    """Time the torch-CPU training step (the reference's CPU path) on this host.
    Returns (seconds per step, threads used)."""
    if threads:
        torch.set_num_threads(threads)
    model = models.build(name, 0)
    x, y = models.make_inputs(name, batch, 1234)
    opt = torch.optim.SGD(model.parameters(), lr=0.01, momentum=0.9)
    loss = models.loss_fn(name)
    model.train()
    for _ in range(warmup):
        train_step(model, x, y, loss, opt)
    t0 = time.perf_counter()
    for _ in range(steps):
        train_step(model, x, y, loss, opt)
    dt = (time.perf_counter() - t0) / max(steps, 1)
    return dt, torch.get_num_threads()


def frob_rel(a: dict, truth: dict):
    """per-key ||a - truth||_F / ||truth||_F (keys of `truth` present in `a`)."""
    out = {}
    for k, t in truth.items():
        if k in a and t.numel():
            n = t.norm().item()
            out[k] = (a[k] - t).norm().item() / max(n, 1e-30)
    return out


def clone_model(model):
    return copy.deepcopy(model)
