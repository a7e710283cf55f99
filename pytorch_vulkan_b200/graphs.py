"""CUDA graphs for `ocl` work: capture a sequence of ops once, replay it with
one launch.

A training step through this backend costs host time for every op -- the
Python model code, the autograd engine, dispatch into the backend, each
kernel's planning and launch -- and for ResNet-50 at batch 64 on one B200
that host time is within a millisecond of the device time.  Captured once,
the step's kernels replay from a CUDA graph with microseconds of host work:

    g = torch.ocl.Graph()
    with g.capture():
        loss = step(x, y)          # nothing runs on the device here
    for batch in loader:
        x.copy_(batch)             # inputs go into the captured tensors
        g.replay()                 # the whole step, one launch
        print(loss.item())         # outputs are the captured tensors

What replays is exactly what the capture issued: the same kernels with the
same pointers and arguments.  So the captured code must do the same work on
every replay (no host-side decisions that depend on data), must not read
anything back to the host or synchronise while capturing, and must take its
inputs from tensors that outlive the graph.  Memory that the captured work
allocates comes from a pool reserved for the graph; tensors created during
the capture (the loss, gradients set to None before it and produced by its
backward) keep pointing into that pool and are rewritten by each replay.
Random numbers drawn while capturing are drawn once: a replay repeats them.

Multi-GPU data parallel steps are not captured here (their all-reduces and
timing events run on a second stream).
"""
from __future__ import annotations

import contextlib
import sys

import torch

from . import _C


class Graph:
    """A captured sequence of `ocl` work on one device (a CUDA graph)."""

    def __init__(self, device=None):
        if device is None:
            device = _C.impl_current_device()
        elif isinstance(device, torch.device):
            device = device.index if device.index is not None else _C.impl_current_device()
        elif isinstance(device, str):
            device = torch.device(device).index or 0
        self.device = int(device)
        self._h = 0

    @contextlib.contextmanager
    def capture(self):
        """Capture the ops issued in the `with` block on this device's current
        stream.  Pending device work is finished first; nothing inside the
        block runs until replay()."""
        if self._h:
            raise RuntimeError("ocl graphs: this Graph already holds a capture (reset() it first)")
        torch.ocl.synchronize(self.device)
        h = _C.impl_graph_capture_begin(self.device)
        try:
            yield self
        except BaseException:
            try:
                _C.impl_graph_capture_end(h)
            except Exception:
                pass
            _C.impl_graph_destroy(h)
            raise
        try:
            _C.impl_graph_capture_end(h)
        except BaseException:
            _C.impl_graph_destroy(h)
            raise
        self._h = h

    def replay(self):
        """Launch the captured work on the device's current stream."""
        if not self._h:
            raise RuntimeError("ocl graphs: nothing captured")
        _C.impl_graph_replay(self._h)

    @property
    def kernels(self) -> int:
        """Kernels one replay launches."""
        return _C.impl_graph_kernels(self._h) if self._h else 0

    def reset(self):
        """Release the graph and the memory reserved for it (after waiting for
        its replays to finish)."""
        if self._h:
            h, self._h = self._h, 0
            _C.impl_graph_destroy(h)

    def __del__(self):
        # not at interpreter shutdown: the device runtime may be gone by then,
        # and the process's memory is released with it anyway
        if self._h and not sys.is_finalizing():
            try:
                self.reset()
            except Exception:
                pass
