#!/usr/bin/env python
"""Benchmark: fp32 training throughput of ResNet-50 (batch 64 per GPU,
synthetic 3x224x224 inputs, cross-entropy, SGD momentum 0.9) on the `ocl`
backend, data-parallel over N GPUs (one process per GPU, launched by torchrun).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line (rank 0).  `value` is whole-job images/s with inputs
resident in HBM (device-timed with events on the backend stream, max over
ranks); `e2e` is the same metric through the public API with each step's
batch copied from pinned host memory (on a copy stream, overlapping the
previous step) and every step's loss copied back to pinned host memory and
read by the host after it has enqueued the next step.  The roofline
object covers the dominant kernel class (the convolutions, fwd+bwd); the CPU
baseline is the torch-CPU step (the reference's validation path) timed on
this host at the configuration's batch (2 warm-up + 3 timed steps).  A second
roofline object, `roofline_bn`, covers the batch-norm class (forward with its
fused residual add / ReLU, backward with its fused ReLU gradient) against the
measured HBM copy bandwidth.

On one GPU the step is captured once as a CUDA graph (`torch.ocl.Graph`,
`--graph auto`, the default) and every timed step, in both measurements,
replays it: the same kernels as the eager step, issued with one launch
instead of by Python, the autograd engine and the backend op by op (the
eager step's host time is within a millisecond of its device time).  Before
timing, one eager step and the first replay run from the same saved state
and must give the same loss bit for bit.  If the capture fails or the
losses differ, the bench times eager steps and says so (`config.step`), as
it does for steps that draw random numbers (dropout), which a replay would
repeat; `--graph off` forces eager steps.  Data-parallel runs step eagerly.

`--impl reference` times the reference's CPU path (torch-CPU ATen, as its
tests/validate_network.py runs it) for the same workload on all host cores;
under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

MODEL = "resnet50"
GFLOP_PER_IMAGE = 24.30  # fwd+bwd conv/linear 2*MAC, torch.utils.flop_counter


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--model", default=MODEL)
    ap.add_argument("--attention", default="fused", choices=["fused", "math"],
                    help="scaled_dot_product_attention backend for vit_b_16 (math = bmm + softmax + bmm)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--graph", default="auto", choices=["auto", "off"],
                    help="auto: one-GPU runs capture the step as a CUDA graph and replay it (eager if capture fails)")
    ap.add_argument("--deadline-s", type=float, default=600.0,
                    help="multi-GPU runs abort the NCCL communicator and exit 3 after this many seconds")
    return ap.parse_args()


def env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.samples.append([s.strip() for s in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit())
        mx = max((float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for n, v in zip(names, s[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(self.samples)}


# --------------------------------------------------------- reference arm
def run_reference(a):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from oracle import step as ostep

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # every step is the full per-GPU batch of the configuration; the step
    # count is bounded so the run stays within a few minutes on the host cores
    sample = a.batch
    steps = max(1, min(a.steps, 10))
    warm = max(1, min(a.warmup, 2))
    dt, used = ostep.time_cpu_steps(a.model, sample, steps, warm, threads)
    v = sample / dt
    line = {
        "impl": "reference", "metric": "train images/sec (fp32)", "value": round(v, 3), "unit": "images/s",
        "n_gpus": a.gpus, "steps": steps, "warmup": warm, "ms_per_step": round(dt * 1000, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{a.model} fp32 train step (fwd+bwd+SGD m0.9), batch {a.batch}/GPU, 3x224x224",
                   "global_batch": a.batch, "sample": f"{sample} images per step (the full per-GPU batch)",
                   "path": "torch-CPU ATen (reference CPU validation path)"},
        "cpu_baseline": {"value": round(v, 3), "unit": "images/s", "cores": used, "kind": "port",
                         "cpu": cpu_model(),
                         "sample": f"{warm} warm-up + {steps} timed steps x {sample} images of the {a.model} "
                                   f"workload on torch-CPU"},
        "e2e": {"value": round(v, 3), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- ours arm
def conv_flops_per_step(model, x):
    """Algorithmic conv+linear FLOPs (2*MAC) of one fwd+bwd, from the shapes."""
    from torch.utils.flop_counter import FlopCounterMode

    m = model.to("cpu")
    with FlopCounterMode(display=False) as fc:
        m(x[:1].cpu()).sum().backward()
    m.zero_grad(set_to_none=True)
    total = fc.get_total_flops()
    conv = sum(v for k, v in fc.get_flop_counts()["Global"].items() if "convolution" in str(k))
    return total * x.shape[0], conv * x.shape[0]


def bn_roofline(rows, bn_numel, hbm_gbs, measured):
    """HBM roofline of the batch-norm class in one profiled step.

    Device time: every op row whose name holds "batch_norm" (statistics,
    normalising passes with their fused residual add / ReLU, backward passes
    with their fused ReLU gradient).  Algorithmic bytes per element of a
    layer's input: forward 8 (read x, write y) + 4 when the residual add is
    fused (read the other summand); backward 12 (read dy and x, write dx) + 4
    when the ReLU / ReLU6 gradient is fused and read from the activation's
    output (not when its mask is formed from x).  The normalising
    passes run in forward call order and the backward passes in reverse, so
    row i of each kind belongs to batch norm i (resp. n-1-i)."""
    ms = sum(d for k, d in rows if "batch_norm" in k)
    if not bn_numel or ms <= 0:
        return None
    n = len(bn_numel)
    # a forward batch norm appears as one row, or as a statistics row followed
    # (later) by its deferred normalising row "native_batch_norm.apply[+...]"
    applies = [k for k, _ in rows if k.startswith("native_batch_norm.apply")]
    bwd = [k for k, _ in rows if "native_batch_norm_backward" in k]
    fwd_b = sum(8 * e for e in bn_numel)
    if len(applies) == n:
        fwd_b += sum(4 * e for e, k in zip(bn_numel, applies) if "+add_" in k)
    bwd_b = sum(12 * e for e in bn_numel)
    if len(bwd) == n:
        bwd_b += sum(4 * e for e, k in zip(reversed(bn_numel), bwd) if _reads_act_out(k))
    total = fwd_b + bwd_b
    achieved = total / (ms / 1000.0) / 1e9
    return {"bound": "hbm", "kernel": "batch norm fwd+bwd (all batch-norm launches of one step)",
            "achieved": round(achieved, 1), "peak": round(hbm_gbs, 1), "unit": "GB/s",
            "frac": round(achieved / hbm_gbs, 4),
            "peak_note": "measured HBM copy (MEASURED_PEAKS.json)" if measured else "fallback 6650 GB/s",
            "traffic": None, "bn_ms_per_step": round(ms, 3), "bn_layers": n,
            "algorithmic_gb_per_step": round(total / 1e9, 3), "fused_adds": sum("+add_" in k for k in applies),
            "fused_relu_grads": sum(_act_grad_fused(k) for k in bwd),
            "act_masks_from_x": sum("@x+" in k for k in bwd)}


def _act_grad_fused(name):
    """a batch-norm backward row that also formed the ReLU / ReLU6 gradient"""
    return "threshold_backward" in name or "hardtanh_backward" in name


def _reads_act_out(name):
    """such a row that read the activation's output for the mask (rather than
    forming it from x and the forward's (a, b): the "@x" rows)"""
    return _act_grad_fused(name) and "@x+" not in name


def _watchdog(comm, seconds):
    """Multi-GPU runs: if the whole run has not finished after `seconds`, abort
    the NCCL communicator (unblocking any collective waiting for a peer) and
    exit with status 3 instead of waiting forever."""
    def fire():
        sys.stderr.write(f"bench: no completion after {seconds:.0f} s, aborting the NCCL communicator\n")
        try:
            comm.close(abort=True)
        finally:
            os._exit(3)

    t = threading.Timer(seconds, fire)
    t.daemon = True
    t.start()


def run_ours(a):
    import pytorch_vulkan_b200 as pvb2  # noqa: F401
    from pytorch_vulkan_b200 import _C
    from pytorch_vulkan_b200 import workloads
    from pytorch_vulkan_b200.distributed import DistributedDataParallel, init_process_group

    rank, world, local, comm = init_process_group()
    if world == 1:
        torch.ocl.set_device(0)
    else:
        _watchdog(comm, a.deadline_s)
    dev = f"ocl:{local}"
    if a.attention == "math":
        from torch.nn.attention import SDPBackend, sdpa_kernel

        a.sdpa_ctx = sdpa_kernel(SDPBackend.MATH)  # kept alive: closing it restores the backends
        a.sdpa_ctx.__enter__()
    torch.manual_seed(0)
    model = workloads.build(a.model, 0)
    x_cpu, y_cpu = workloads.make_inputs(a.model, a.batch, 1234 + rank)
    total_flops, conv_flops = conv_flops_per_step(model, x_cpu) if rank == 0 else (0, 0)
    model = model.to(dev)
    model.train()
    net = DistributedDataParallel(model, comm) if world > 1 else model
    opt = torch.optim.SGD(model.parameters(), lr=0.1, momentum=0.9, fused=True)
    loss_fn = workloads.loss_fn(a.model)
    x = x_cpu.to(dev)
    y = y_cpu.to(dev)

    def step(xb, yb):
        opt.zero_grad(set_to_none=True)
        out = net(xb)
        l = loss_fn(out, yb)
        l.backward()
        opt.step()
        return l

    def barrier():
        torch.ocl.synchronize(local)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for _ in range(a.warmup):
        step(x, y)
    barrier()

    # one-GPU runs: the step captured once, replayed as one launch
    graph = None
    l_graph = None
    graph_note = "eager"
    # a replay repeats the random numbers drawn at capture: steps that draw
    # some (dropout) stay eager
    draws = any(isinstance(m_, torch.nn.Dropout) and m_.p > 0 for m_ in model.modules())
    if world == 1 and a.graph == "auto" and draws:
        graph_note = "eager (the step draws random numbers)"
    elif world == 1 and a.graph == "auto":
        try:
            from pytorch_vulkan_b200.graphs import Graph

            # checked on this workload: from one saved state, the first
            # replay's loss must equal an eager step's bit for bit
            with torch.no_grad():
                saved = [t.detach().clone() for t in model.state_dict().values()]
                saved_m = [(st_["momentum_buffer"], st_["momentum_buffer"].clone()) for st_ in opt.state.values()
                           if st_.get("momentum_buffer") is not None]

            def restore():
                with torch.no_grad():
                    for t, v in zip(model.state_dict().values(), saved):
                        t.copy_(v)
                    for t, v in saved_m:
                        t.copy_(v)

            eager_loss = step(x, y).item()
            restore()
            graph = Graph(local)
            with graph.capture():
                l_graph = step(x, y)
            graph.replay()
            replay_loss = l_graph.item()
            del saved, saved_m
            if replay_loss != eager_loss:
                raise RuntimeError(f"replayed step's loss {replay_loss!r} differs from the eager step's {eager_loss!r}")
            for _ in range(a.warmup):
                graph.replay()
            graph_note = f"cuda_graph ({graph.kernels} kernels per replay, first replay's loss equal to eager)"
        except Exception as e:  # the eager step is the same work, issued op by op
            sys.stderr.write(f"bench: graph capture unavailable ({e}); timing eager steps\n")
            if graph is not None:
                graph.reset()
            graph = None
            graph_note = "eager (graph capture failed)"

    def run_step(xb=None, yb=None):
        if graph is None:
            return step(x if xb is None else xb, y if yb is None else yb)
        if xb is not None:  # the captured step reads x and y: the batch goes there
            x.copy_(xb)
            y.copy_(yb)
        graph.replay()
        return l_graph

    # ---------------------------------------------------------- timed region
    e0, e1 = _C.impl_event_create(True), _C.impl_event_create(True)
    l0 = _C.impl_launch_count()
    with ClockSampler(local) as clk:
        barrier()
        _C.impl_event_record(e0, local)
        for _ in range(a.steps):
            run_step()
        _C.impl_event_record(e1, local)
        barrier()
    launches = _C.impl_launch_count() - l0
    ms = _C.impl_event_elapsed_ms(e0, e1) / a.steps
    ms = max_over_ranks(ms)
    value = a.batch * world / (ms / 1000.0)

    # ----------------------------------------------- end to end (public API)
    e2e = None
    if not a.no_e2e:
        # A data-loader-style pipeline: each step's batch is copied from
        # pinned host memory on a copy stream into one of two device
        # buffers while the previous step computes; the compute stream
        # waits for its batch's copy, and each step's loss is read back.
        xp, yp = x_cpu.pin_memory(), y_cpu.pin_memory()
        bufs = [(torch.empty_like(x), torch.empty_like(y)) for _ in range(2)]
        copy_s = torch.Stream(device=dev)
        ready = [torch.Event(device=dev) for _ in range(2)]
        free = [torch.Event(device=dev) for _ in range(2)]

        def load(i):
            with copy_s:
                if i >= 2:
                    free[i % 2].wait()  # the step that last read this buffer
                bufs[i % 2][0].copy_(xp, non_blocking=True)
                bufs[i % 2][1].copy_(yp, non_blocking=True)
                ready[i % 2].record()

        # each step's loss goes to pinned host memory on the compute stream
        # right after the step; the host reads it once the next step is
        # enqueued (a training loop that logs the loss one step behind), so
        # the device is never left waiting for the host between steps
        loss_h = [torch.empty((), dtype=torch.float32, pin_memory=True) for _ in range(2)]
        loss_ev = [torch.Event(device=dev) for _ in range(2)]
        losses = []

        def run_e2e(n):
            losses.clear()
            load(0)
            for i in range(n):
                ready[i % 2].wait()
                l = run_step(*bufs[i % 2])
                free[i % 2].record()
                loss_h[i % 2].copy_(l.detach(), non_blocking=True)
                loss_ev[i % 2].record()
                if i + 1 < n:
                    load(i + 1)
                if i > 0:
                    loss_ev[(i - 1) % 2].synchronize()
                    losses.append(loss_h[(i - 1) % 2].item())
            loss_ev[(n - 1) % 2].synchronize()
            losses.append(loss_h[(n - 1) % 2].item())

        run_e2e(2)
        barrier()
        _C.impl_event_record(e0, local)
        run_e2e(a.steps)
        _C.impl_event_record(e1, local)
        barrier()
        ems = max_over_ranks(_C.impl_event_elapsed_ms(e0, e1) / a.steps)
        e2e = {"value": round(a.batch * world / (ems / 1000.0), 2), "unit": "images/s",
               "h2d_bytes_per_step": int(x.numel() * x.element_size() + y.numel() * y.element_size()),
               "d2h_bytes_per_step": 4, "ms_per_step": round(ems, 3)}

    # ------------------------------- data parallel: exposure and agreement
    # the last step's gradient all-reduce time past the end of backward, and
    # a bit-for-bit comparison of every rank's parameters with rank 0's (a
    # run whose ranks diverged is not a data-parallel run and fails)
    dp = None
    if world > 1:
        exposed = max_over_ranks(net.exposed_comm_ms())
        agree = net.params_agree()
        dp = {"exposed_comm_ms_last_step": round(exposed, 4), "params_agree_across_ranks": bool(agree),
              "buckets": len(net.buckets)}
        if not agree:
            sys.stderr.write("bench: ranks hold different parameters after the timed steps\n")
            sys.exit(4)

    # --------------------------------------- dominant kernel class roofline
    # every rank runs this step (its gradient all-reduces must be matched on
    # all ranks); rank 0 records it under the profiler
    roof = roof_bn = None
    if rank != 0:
        step(x, y)
        torch.ocl.synchronize(local)
    else:
        import csv
        import tempfile

        # element counts of every batch norm's input, in call order
        bn_numel = []
        hooks = [m.register_forward_hook(lambda mod, inp, out: bn_numel.append(inp[0].numel()))
                 for m in model.modules() if isinstance(m, torch.nn.modules.batchnorm._BatchNorm)]
        path = os.path.join(tempfile.mkdtemp(), "prof.csv")
        with torch.ocl.profile(local, path):
            step(x, y)
            torch.ocl.synchronize(local)
        for h in hooks:
            h.remove()
        conv_ms = 0.0
        n_conv = 0
        per_op = {}
        rows = []
        with open(path) as f:
            for r in csv.DictReader(f):
                d = float(r["duraion(ms)"])
                if r["section"] == "":
                    rows.append((r["kernel"], d))
                    per_op[r["kernel"]] = per_op.get(r["kernel"], 0.0) + d
                    if r["kernel"].startswith("convolution"):  # + the dgrad launches that also form an add
                        conv_ms += d
                        n_conv += 1
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))
        except Exception:
            pass
        bf16 = peaks.get("bf16_tflops", 1590.0)
        hbm = peaks.get("hbm_gbs", 6650.0)
        tf32_peak = bf16 / 2.0
        achieved = conv_flops / (conv_ms / 1000.0) / 1e12 if conv_ms > 0 else 0.0
        roof = {"bound": "tensor", "kernel": "convolution fwd+bwd (all conv launches of one step)",
                "achieved": round(achieved, 2), "peak": round(tf32_peak, 1), "unit": "TFLOP/s",
                "frac": round(achieved / tf32_peak, 4),
                "peak_note": ("TF32 dense = 1/2 of measured burst bf16 (MEASURED_PEAKS.json)" if peaks
                              else "TF32 dense = 1/2 of the fallback bf16 1590 TFLOP/s"),
                # per-launch DRAM traffic is captured per kernel variant under ncu
                # (profiles/); the per-step sum of those captures is not formed here
                "traffic": None,
                "conv_ms_per_step": round(conv_ms, 3), "conv_launch_groups": n_conv,
                "conv_gflop_per_step": round(conv_flops / 1e9, 1),
                "top_ops_ms": dict(sorted(per_op.items(), key=lambda kv: -kv[1])[:8])}
        roof_bn = bn_roofline(rows, bn_numel, hbm, bool(peaks))

    # ------------------------------------------------------- CPU baseline
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        from oracle import step as ostep

        threads = os.cpu_count() or 1
        sample = a.batch
        dt, used = ostep.time_cpu_steps(a.model, sample, 3, 2, threads)
        cpu = {"value": round(sample / dt, 3), "unit": "images/s", "cores": used, "kind": "port", "cpu": cpu_model(),
               "sample": f"2 warm-up + 3 timed steps x {sample} images of {a.model} on torch-CPU ATen "
                         f"(reference CPU path)"}

    if rank == 0:
        line = {
            "metric": "train images/sec (fp32)", "value": round(value, 2), "unit": "images/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{a.model} fp32 train step (fwd+bwd+SGD m0.9), batch {a.batch}/GPU, 3x224x224",
                       "global_batch": a.batch * world, "parallelism": f"dp{world}", "step": graph_note,
                       "math": ["tf32", "fp32", "3xtf32"][torch.ocl.get_math_mode()],
                       **({"attention": a.attention} if "vit" in a.model else {}),
                       "l2": "inputs/activations larger than L2 (126 MB) every step",
                       "gflop_per_step": round(total_flops / 1e9, 1)},
            "e2e": e2e, "gpu_launches": int(launches), "roofline": roof, "roofline_bn": roof_bn, "cpu_baseline": cpu,
            **({"dp": dp} if dp else {}),
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        graph.reset()
    if comm is not None:
        comm.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
