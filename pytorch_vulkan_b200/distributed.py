"""Data-parallel training for `ocl` devices: one process per GPU, the batch
sharded across ranks, gradients averaged with an NCCL all-reduce over
NVLink / NVSwitch before the optimizer step.

The reference has no multi-device code at all; this is the one exchange
step of the data-parallel training path.  Host-side plumbing (rendezvous,
unique-id exchange, barriers, timing reductions) uses torch.distributed with
the gloo backend; the gradient traffic runs on the backend's own streams
through libpvb2's NCCL entry points.

Gradient buckets (about 25 MB, filled in reverse registration order, which
is close to the order backward produces them) are flattened into one buffer
by a single multi-tensor kernel as soon as their last gradient is
accumulated, then all-reduced (average) on a separate communication stream
while the rest of backward runs.  The bucket of the first-registered
parameters, which backward finishes last, is kept small (about 2 MB), so
the all-reduce left after backward ends is short; ``exposed_comm_ms`` reports
how long the communication stream ran past the end of backward in the last
step (device events), and ``params_agree`` checks that every rank holds
bit-identical parameters.  After backward the compute stream waits
for the communication stream and every parameter's ``.grad`` is pointed at
its slice of the reduced bucket, so the optimizer reads the averaged
gradients with no copy back.

For parameters on the CPU (the gloo test path) the same bucketing runs with
``torch.distributed.all_reduce`` on the flat buffer.
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch
import torch.distributed as dist

from . import _C

AVG = 1
SUM = 0


class Communicator:
    """An NCCL communicator bound to one `ocl` device (one rank per GPU)."""

    def __init__(self, rank: int, world: int, device: int, group=None):
        self.rank, self.world, self.device = rank, world, device
        obj = [_C.impl_nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        self.handle = _C.impl_nccl_init(world, obj[0], rank, device)
        self.stream = _C.impl_new_stream(device, -1)  # high-priority comm stream

    def allreduce_(self, t: torch.Tensor, op: int = AVG, stream: Optional[int] = None):
        _C.impl_nccl_allreduce(self.handle, t, op, self.stream if stream is None else stream)

    def broadcast_(self, t: torch.Tensor, root: int = 0, stream: Optional[int] = None):
        _C.impl_nccl_broadcast(self.handle, t, root, self.stream if stream is None else stream)

    def close(self, abort: bool = False):
        if self.handle:
            (_C.impl_nccl_abort if abort else _C.impl_nccl_destroy)(self.handle)
            self.handle = 0


def init_process_group(timeout_s: float = 120.0):
    """Initialise torch.distributed (gloo, host plumbing) from the torchrun
    environment and create the NCCL communicator for this rank's device.
    Returns (rank, world, local_rank, Communicator or None)."""
    import datetime

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1:
        return rank, world, local, None
    if not dist.is_initialized():
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
    torch.ocl.set_device(local)
    comm = Communicator(rank, world, local)
    return rank, world, local, comm


class _Bucket:
    def __init__(self, params: List[torch.nn.Parameter], device):
        self.params = params
        self.numel = sum(p.numel() for p in params)
        self.offsets = []
        off = 0
        for p in params:
            self.offsets.append(off)
            off += p.numel()
        self.flat = torch.empty(self.numel, dtype=torch.float32, device=device)
        self.pending = set()

    def reset(self):
        self.pending = {id(p) for p in self.params}


class DistributedDataParallel(torch.nn.Module):
    """Minimal DDP for `ocl` (and CPU/gloo) modules: broadcast of the initial
    state from rank 0, bucketed gradient averaging overlapped with backward."""

    def __init__(self, module: torch.nn.Module, comm: Optional[Communicator] = None, bucket_cap_mb: float = 25.0,
                 group=None, last_bucket_cap_mb: float = 2.0):
        super().__init__()
        self.module = module
        self.comm = comm
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        params = [p for p in module.parameters() if p.requires_grad]
        self.device = params[0].device if params else torch.device("cpu")
        self.on_ocl = self.device.type == "ocl"
        cap = int(bucket_cap_mb * 1024 * 1024 / 4)
        first_cap = int(last_bucket_cap_mb * 1024 * 1024 / 4)
        # groups in registration order, the first one small; reduced last-first
        groups: List[List[torch.nn.Parameter]] = []
        cur: List[torch.nn.Parameter] = []
        size = 0
        for p in params:
            cur.append(p)
            size += p.numel()
            if size >= (first_cap if not groups else cap):
                groups.append(cur)
                cur, size = [], 0
        if cur:
            groups.append(cur)
        self.buckets: List[_Bucket] = [_Bucket(list(reversed(g)), self.device) for g in reversed(groups)]
        self._owner = {}
        for b in self.buckets:
            for p in b.params:
                self._owner[id(p)] = b
                p.register_post_accumulate_grad_hook(self._hook)
        self._queued = False
        self._launched: List[_Bucket] = []
        self._ev = None
        if self.on_ocl and self.world > 1:
            self._ev = (_C.impl_event_create(True), _C.impl_event_create(True))
        self._timed = False
        self._broadcast_state()

    # -- initial state: every rank starts from rank 0's weights and buffers
    def _broadcast_state(self):
        if self.world == 1:
            return
        with torch.no_grad():
            for t in list(self.module.parameters()) + list(self.module.buffers()):
                if self.on_ocl and t.is_floating_point() and t.is_contiguous():
                    self.comm.broadcast_(t, 0, stream=0)
                else:
                    tmp = t.detach().cpu()
                    dist.broadcast(tmp, 0, group=self.group)
                    t.copy_(tmp)
        if self.on_ocl:
            torch.ocl.synchronize(self.device)

    def forward(self, *args, **kwargs):
        for b in self.buckets:
            b.reset()
        self._queued = False
        self._launched = []
        return self.module(*args, **kwargs)

    def _hook(self, p):
        if self.world == 1:
            return
        if not self._queued:
            torch.autograd.Variable._execution_engine.queue_callback(self._finish)
            self._queued = True
        b = self._owner[id(p)]
        b.pending.discard(id(p))
        if not b.pending:
            self._launch(b)

    def _launch(self, b: _Bucket):
        grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in b.params]
        if self.on_ocl:
            dev = self.device.index or 0
            _C.impl_flatten_multi([g.contiguous() for g in grads], b.flat, 0, 1.0)
            # the comm stream must see the flattened bucket before reducing it
            _C.impl_stream_wait_stream(dev, self.comm.stream, _C.impl_get_stream(dev))
            _C.impl_record_stream(b.flat, self.comm.stream)
            self.comm.allreduce_(b.flat, AVG)
        else:
            torch.cat([g.reshape(-1) for g in grads], out=b.flat)
            dist.all_reduce(b.flat, group=self.group)
            b.flat.div_(self.world)
        self._launched.append(b)

    def _finish(self):
        for b in self.buckets:  # buckets whose hooks never fired (unused params)
            if b not in self._launched:
                self._launch(b)
        if self.on_ocl:
            dev = self.device.index or 0
            # backward's last kernel vs the communication stream's last all-reduce
            _C.impl_event_record_stream(self._ev[0], dev, _C.impl_get_stream(dev))
            _C.impl_event_record_stream(self._ev[1], dev, self.comm.stream)
            self._timed = True
            _C.impl_stream_wait_stream(dev, _C.impl_get_stream(dev), self.comm.stream)
        for b in self.buckets:
            for p, off in zip(b.params, b.offsets):
                p.grad = b.flat[off:off + p.numel()].view_as(p)

    def exposed_comm_ms(self) -> float:
        """Device time the gradient all-reduces ran past the end of the last
        backward (0 when they finished first); synchronises on the events."""
        if not self._timed:
            return 0.0
        return max(0.0, _C.impl_event_elapsed_ms(self._ev[0], self._ev[1]))

    def params_agree(self) -> bool:
        """True when every rank's parameters equal rank 0's bit for bit (rank
        0's flat copy broadcast, the per-rank maximum differences summed).
        Buffers are not compared: batch-norm running statistics follow each
        rank's own batches, as with DDP's broadcast_buffers=False."""
        if self.world == 1:
            return True
        ts = [p.detach() for p in self.module.parameters()]
        if self.on_ocl:
            flat = torch.empty(sum(t.numel() for t in ts), dtype=torch.float32, device=self.device)
            _C.impl_flatten_multi([t.contiguous() for t in ts], flat, 0, 1.0)
            ref = flat.clone()
            self.comm.broadcast_(ref, 0, stream=0)
            d = (flat - ref).abs().max().reshape(1)
            self.comm.allreduce_(d, SUM, stream=0)  # any nonzero difference anywhere stays nonzero
            torch.ocl.synchronize(self.device)
            return d.item() == 0.0
        flat = torch.cat([t.reshape(-1).float() for t in ts])
        ref = flat.clone()
        dist.broadcast(ref, 0, group=self.group)
        d = (flat - ref).abs().max().reshape(1)
        dist.all_reduce(d, op=dist.ReduceOp.MAX, group=self.group)
        return d.item() == 0.0
