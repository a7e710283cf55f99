"""Data-parallel host logic on CPU ranks (gloo, world size 2).

pytorch_vulkan_b200.distributed.DistributedDataParallel buckets gradients,
reduces each bucket as soon as its last gradient is accumulated and points
every .grad at its slice of the averaged bucket.  On CPU tensors the same
bucketing runs with torch.distributed.all_reduce, so the logic is checked
here without a GPU:
  * the averaged gradients of 2 ranks x 4 samples equal the gradients of one
    process on all 8 samples (mean loss), with many small buckets;
  * rank 0's initial weights reach rank 1;
  * the first-registered parameters form the last, small bucket, and
    params_agree() reports equal parameters after an SGD step and a
    difference once one rank's weights move;
  * a rank that raises before the exchange makes the other rank's collective
    fail within the process-group timeout instead of hanging.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _net():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Conv2d(1, 4, 3), torch.nn.ReLU(), torch.nn.Flatten(),
                               torch.nn.Linear(4 * 6 * 6, 10))


def _data():
    g = torch.Generator().manual_seed(3)
    return torch.randn(8, 1, 8, 8, generator=g), torch.randint(0, 10, (8,), generator=g)


def _worker(rank, world, port, out, mode):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from pytorch_vulkan_b200.distributed import DistributedDataParallel

    model = _net()
    if rank == 1:
        with torch.no_grad():  # rank 1 starts from different weights: DDP must broadcast rank 0's
            for p in model.parameters():
                p.add_(1.0)
    ddp = DistributedDataParallel(model, None, bucket_cap_mb=0.0005, last_bucket_cap_mb=0.0002)  # many small buckets
    x, y = _data()
    xs, ys = x[rank * 4:(rank + 1) * 4], y[rank * 4:(rank + 1) * 4]
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        loss = torch.nn.functional.cross_entropy(ddp(xs), ys)
        loss.backward()
        out[rank] = {n: p.grad.clone() for n, p in model.named_parameters()}
        out[f"w{rank}"] = {n: p.detach().clone() for n, p in model.named_parameters()}
        # bucket order: the last bucket holds the first-registered parameter
        out[f"last{rank}"] = [tuple(p.shape) for p in ddp.buckets[-1].params]
        torch.optim.SGD(model.parameters(), lr=0.1).step()
        out[f"agree{rank}"] = ddp.params_agree()
        if rank == 1:
            with torch.no_grad():
                next(model.parameters()).add_(1e-3)
        out[f"disagree{rank}"] = not ddp.params_agree()
    except Exception as e:  # noqa: BLE001
        out[f"err{rank}"] = type(e).__name__ + ": " + str(e)[:200]
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _spawn(mode):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out, mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    return dict(out)


def test_bucketed_average_equals_full_batch():
    out = _spawn("ok")
    assert 0 in out and 1 in out, out
    model = _net()
    x, y = _data()
    torch.nn.functional.cross_entropy(model(x), y).backward()
    for n, p in model.named_parameters():
        assert torch.allclose(out[0][n], p.grad, atol=1e-6), n
        assert torch.allclose(out[1][n], p.grad, atol=1e-6), n
        assert torch.equal(out["w0"][n], out["w1"][n]), n  # rank 0's weights broadcast
    first = tuple(next(model.parameters()).shape)
    assert first in out["last0"] and out["last0"] == out["last1"]
    assert out["agree0"] and out["agree1"]
    assert out["disagree0"] and out["disagree1"]


def test_failed_rank_is_reported_not_hung():
    out = _spawn("fail")
    assert "err1" in out
    assert "err0" in out, "rank 0 should see its collective fail when rank 1 never joins"
