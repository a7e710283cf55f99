"""Deferred batch-norm pass: a training batch norm leaves its normalising
pass pending and an in-place residual add / ReLU / ReLU6 of its output joins it
(csrc/host/deferred.cpp).  Every way the output can be read before, between
or instead of those ops must see exactly what the three separate ops give;
checked against torch-CPU on the same inputs (the reference's own arbiter,
tests/test_op.py:14-150 of the reference)."""
import copy

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu
DEV = "ocl:0"


def _bn_pair(C, seed):
    torch.manual_seed(seed)
    cpu = nn.BatchNorm2d(C)
    with torch.no_grad():
        cpu.weight.uniform_(0.5, 1.5)
        cpu.bias.uniform_(-0.5, 0.5)
    dev = nn.BatchNorm2d(C).to(DEV)
    dev.load_state_dict(cpu.state_dict())
    return cpu.train(), dev.train()


def _x(shape, seed):
    return torch.randn(shape, generator=torch.Generator().manual_seed(seed)) * 2 + 0.3


def _close(a, b, tol=2e-5):
    return (a.detach().double() - b.detach().cpu().double()).abs().max().item() <= tol * max(1.0, a.abs().max().item())


def _check_bn_state(cpu, dev):
    assert _close(cpu.running_mean, dev.running_mean)
    assert _close(cpu.running_var, dev.running_var)


SHAPES = [(8, 64, 28, 28), (4, 32, 7, 7), (2, 3, 5, 6)]


@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
def test_bn_relu_inplace(ocl, shape):
    cpu, dev = _bn_pair(shape[1], 1)
    x = _x(shape, 2)
    ref = torch.relu_(cpu(x))
    got = torch.relu_(dev(x.to(DEV)))
    assert _close(ref, got)
    _check_bn_state(cpu, dev)


@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
def test_bn_add_relu_inplace(ocl, shape):
    cpu, dev = _bn_pair(shape[1], 3)
    x, r = _x(shape, 4), _x(shape, 5)
    y = cpu(x)
    y += r
    ref = torch.relu_(y)
    yd = dev(x.to(DEV))
    yd += r.to(DEV)
    got = torch.relu_(yd)
    assert _close(ref, got)
    _check_bn_state(cpu, dev)


def test_bn_output_read_before_relu(ocl):
    cpu, dev = _bn_pair(16, 6)
    x = _x((4, 16, 9, 9), 7)
    y = cpu(x)
    yd = dev(x.to(DEV))
    assert _close(y, yd.cpu())          # the copy to the host launches the pending pass
    assert _close(torch.relu_(y), torch.relu_(yd))


def test_bn_add_then_other_op(ocl):
    cpu, dev = _bn_pair(16, 8)
    x, r = _x((4, 16, 9, 9), 9), _x((4, 16, 9, 9), 10)
    y = cpu(x)
    y += r
    yd = dev(x.to(DEV))
    yd += r.to(DEV)
    assert _close(y * 2, yd * 2)        # another op flushes with the residual folded in


def test_bn_out_of_place_relu(ocl):
    cpu, dev = _bn_pair(8, 11)
    x = _x((2, 8, 10, 10), 12)
    y = cpu(x)
    yd = dev(x.to(DEV))
    assert _close(torch.relu(y), torch.relu(yd))
    assert _close(y, yd)                # y itself keeps the batch-norm values


def test_bn_self_add_and_view_relu(ocl):
    cpu, dev = _bn_pair(8, 13)
    x = _x((2, 8, 10, 10), 14)
    y = cpu(x)
    y += y                              # aliasing residual: not folded
    yd = dev(x.to(DEV))
    yd += yd
    assert _close(y, yd)
    cpu2, dev2 = _bn_pair(8, 15)
    y = cpu2(x)
    yd = dev2(x.to(DEV))
    torch.relu_(y[:1])                  # ReLU of a view: not folded
    torch.relu_(yd[:1])
    assert _close(y, yd)


def test_bn_then_synchronize_and_stats(ocl):
    cpu, dev = _bn_pair(32, 16)
    x = _x((8, 32, 6, 6), 17)
    y = cpu(x)
    yd = dev(x.to(DEV))
    torch.ocl.synchronize()
    _check_bn_state(cpu, dev)
    assert _close(y, yd)


def test_bottleneck_forward_backward(ocl):
    """conv -> bn -> relu_ -> conv -> bn -> += identity -> relu_, forward and
    backward, in exact-fp32 math so that only the fusion is under test."""
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(1)
    try:
        torch.manual_seed(18)
        C = 32
        blk = nn.ModuleDict({"c1": nn.Conv2d(C, C, 3, padding=1, bias=False), "b1": nn.BatchNorm2d(C),
                             "c2": nn.Conv2d(C, C, 3, padding=1, bias=False), "b2": nn.BatchNorm2d(C)})

        def run(m, x):
            out = torch.relu_(m["b1"](m["c1"](x)))
            out = m["b2"](m["c2"](out))
            out += x
            return torch.relu_(out)

        dev = copy.deepcopy(blk).to(DEV)
        x = _x((4, C, 14, 14), 19)
        xc, xd = x.clone().requires_grad_(), x.to(DEV).requires_grad_()
        yc, yd = run(blk, xc), run(dev, xd)
        assert _close(yc, yd, 1e-4)
        g = _x(yc.shape, 20)
        yc.backward(g)
        yd.backward(g.to(DEV))
        assert _close(xc.grad, xd.grad, 1e-4)
        for (n, p), (_, q) in zip(blk.named_parameters(), dev.named_parameters()):
            assert _close(p.grad, q.grad, 1e-4), n
    finally:
        torch.ocl.set_math_mode(old)


def test_relu_grad_into_bn_backward(ocl):
    """threshold_backward left pending and formed inside the batch-norm
    backward; and the same when the batch-norm output also has a second
    consumer (its gradient is then a sum, and the pending op runs alone)."""
    for second_use in (False, True):
        cpu, dev = _bn_pair(24, 30 + second_use)
        x = _x((4, 24, 10, 10), 31)
        g1, g2 = _x((4, 24, 10, 10), 32), _x((4, 24, 10, 10), 33)
        grads = []
        for m, d in ((cpu, "cpu"), (dev, DEV)):
            xx = x.detach().clone().to(d).requires_grad_()
            y = m(xx)
            loss = (torch.relu(y) * g1.to(d)).sum()
            if second_use:
                loss = loss + (y * g2.to(d)).sum()
            loss.backward()
            grads.append((xx.grad, m.weight.grad, m.bias.grad))
        for a, b in zip(*grads):
            assert _close(a, b, 1e-4)


@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
def test_identity_bn_add_relu(ocl, shape):
    """`out += identity; relu_(out)` where identity is the pending batch norm
    (a downsampling projection): folded with a separate output; identity keeps
    its own values."""
    cpu, dev = _bn_pair(shape[1], 60)
    x, o = _x(shape, 61), _x(shape, 62)
    ident = cpu(x)
    out = o.clone()
    out += ident
    ref = torch.relu_(out)
    ident_d = dev(x.to(DEV))
    out_d = o.to(DEV)
    out_d += ident_d
    got = torch.relu_(out_d)
    assert _close(ref, got)
    assert _close(ident, ident_d)
    _check_bn_state(cpu, dev)


def _bn_pair_wide(C, seed):
    """gamma in [2, 4] so that a good share of the outputs pass 6 and ReLU6
    clamps (and masks the gradient) at both ends"""
    cpu, dev = _bn_pair(C, seed)
    with torch.no_grad():
        cpu.weight.uniform_(2.0, 4.0)
        dev.weight.copy_(cpu.weight)
    return cpu, dev


@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
def test_bn_relu6_inplace(ocl, shape):
    """MobileNet-v2's batch norm -> ReLU6(inplace=True): hardtanh_(y, 0, 6)
    joins the pending pass"""
    cpu, dev = _bn_pair_wide(shape[1], 70)
    x = _x(shape, 71)
    ref = nn.functional.relu6(cpu(x), inplace=True)
    got = nn.functional.relu6(dev(x.to(DEV)), inplace=True)
    assert (ref == 6).any() and (ref == 0).any()
    assert _close(ref, got)
    _check_bn_state(cpu, dev)


def test_bn_hardtanh_other_bounds_not_folded(ocl):
    cpu, dev = _bn_pair_wide(16, 72)
    x = _x((4, 16, 9, 9), 73)
    ref = nn.functional.hardtanh(cpu(x), -1.0, 2.0, inplace=True)
    got = nn.functional.hardtanh(dev(x.to(DEV)), -1.0, 2.0, inplace=True)
    assert _close(ref, got)


def test_relu6_grad_into_bn_backward(ocl):
    """hardtanh_backward(.., 0, 6) left pending and formed inside the
    batch-norm backward; with a second consumer of the batch-norm output the
    pending op runs alone"""
    for second_use in (False, True):
        cpu, dev = _bn_pair_wide(24, 74 + second_use)
        x = _x((4, 24, 10, 10), 76)
        g1, g2 = _x((4, 24, 10, 10), 77), _x((4, 24, 10, 10), 78)
        grads = []
        for m, d in ((cpu, "cpu"), (dev, DEV)):
            xx = x.detach().clone().to(d).requires_grad_()
            y = m(xx)
            a = nn.functional.relu6(y, inplace=not second_use)
            loss = (a * g1.to(d)).sum()
            if second_use:
                loss = loss + (y * g2.to(d)).sum()
            loss.backward()
            grads.append((xx.grad, m.weight.grad, m.bias.grad))
        for a, b in zip(*grads):
            assert _close(a, b, 1e-4)


def test_inverted_residual_forward_backward(ocl):
    """MobileNet-v2's inverted residual (1x1 expand -> bn -> ReLU6 -> 3x3
    depthwise -> bn -> ReLU6 -> 1x1 project -> bn, + x), forward and backward
    in exact-fp32 math"""
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(1)
    try:
        torch.manual_seed(79)
        C, E = 24, 96
        blk = nn.Sequential(nn.Conv2d(C, E, 1, bias=False), nn.BatchNorm2d(E), nn.ReLU6(inplace=True),
                            nn.Conv2d(E, E, 3, padding=1, groups=E, bias=False), nn.BatchNorm2d(E),
                            nn.ReLU6(inplace=True), nn.Conv2d(E, C, 1, bias=False), nn.BatchNorm2d(C))
        with torch.no_grad():
            for m in blk:
                if isinstance(m, nn.BatchNorm2d):
                    m.weight.uniform_(1.0, 4.0)
        dev = copy.deepcopy(blk).to(DEV)
        x = _x((4, C, 14, 14), 80)
        xc, xd = x.clone().requires_grad_(), x.to(DEV).requires_grad_()
        yc, yd = xc + blk(xc), xd + dev(xd)
        assert _close(yc, yd, 1e-4)
        g = _x(yc.shape, 81)
        yc.backward(g)
        yd.backward(g.to(DEV))
        assert _close(xc.grad, xd.grad, 1e-4)
        for (n, p), (_, q) in zip(blk.named_parameters(), dev.named_parameters()):
            assert _close(p.grad, q.grad, 1e-4), n
    finally:
        torch.ocl.set_math_mode(old)


@pytest.mark.parametrize("then", ["relu_", "relu6_", "add_", "mul", "none"])
def test_bn_clone_joins_pass(ocl, then):
    """a clone of the pending output (what autograd takes before an in-place
    activation) joins the pass; the clone keeps the plain values whatever
    happens to the output next"""
    cpu, dev = _bn_pair_wide(16, 82)
    x, r = _x((4, 16, 9, 9), 83), _x((4, 16, 9, 9), 84)

    def run(m, d):
        y = m(x.to(d))
        c = y.clone()
        if then == "relu_":
            torch.relu_(y)
        elif then == "relu6_":
            nn.functional.relu6(y, inplace=True)
        elif then == "add_":
            y += r.to(d)
        elif then == "mul":
            y = y * 2
        return y, c

    (y0, c0), (y1, c1) = run(cpu, "cpu"), run(dev, DEV)
    assert _close(c0, c1) and _close(y0, y1)
    _check_bn_state(cpu, dev)


def _relu6_grads(make, dev):
    """forward + backward of make(x) on `dev`: (output, x.grad)"""
    x = _x((2, 8, 6, 6), 90).to(dev).requires_grad_()
    y = make(x)
    y.backward(_x(y.shape, 91).to(dev))
    return y.detach().cpu(), x.grad.cpu()


def test_relu6_inplace_saves_output_not_a_clone(ocl, tmp_path):
    """hardtanh_ under autograd (csrc/host/ops_autograd.cpp) saves its output:
    the batch norm's pending pass takes the ReLU6 with no clone folded in, and
    the gradients equal torch-CPU's (whose kernel clones the input)"""
    cpu, dev = _bn_pair_wide(8, 92)
    path = str(tmp_path / "prof.csv")
    x = _x((4, 8, 9, 9), 93)
    xc, xd = x.clone().requires_grad_(), x.to(DEV).requires_grad_()
    yc = nn.functional.relu6(cpu(xc), inplace=True)
    with torch.ocl.profile(DEV, path):
        yd = nn.functional.relu6(dev(xd), inplace=True)
        torch.ocl.synchronize()
    ops = [line.split(",")[1] for line in open(path).read().splitlines()[1:]]
    assert "native_batch_norm.apply+hardtanh_" in ops, ops
    assert not any("copy" in o for o in ops), ops
    g = _x(yc.shape, 94)
    yc.backward(g)
    yd.backward(g.to(DEV))
    assert _close(yc, yd) and _close(xc.grad, xd.grad, 1e-4)
    for p, q in zip(cpu.parameters(), dev.parameters()):
        assert _close(p.grad, q.grad, 1e-4)


@pytest.mark.parametrize("case", ["view", "min_ge_max", "no_grad_input"])
def test_hardtanh_inplace_other_cases_follow_torch(ocl, case):
    """the cases the output-saving kernel leaves to torch's own autograd
    kernel give torch-CPU's results"""
    def make(x):
        y = x * 1.5 + 0.5
        if case == "view":
            nn.functional.hardtanh(y[:, :4], 0.0, 6.0, inplace=True)
        elif case == "min_ge_max":
            nn.functional.hardtanh(y, 1.0, 1.0, inplace=True)
        else:
            y = y + x.detach()
            nn.functional.relu6(y, inplace=True)
        return y

    (y0, g0), (y1, g1) = _relu6_grads(make, "cpu"), _relu6_grads(make, DEV)
    assert _close(y0, y1) and _close(g0, g1, 1e-5)


def test_hardtanh_inplace_no_grad_and_leaf(ocl):
    x = _x((3, 5), 95).to(DEV)
    with torch.no_grad():
        v = x._version
        nn.functional.relu6(x, inplace=True)
        assert x._version == v + 1
    assert _close(nn.functional.relu6(_x((3, 5), 95)), x)
    leaf = _x((3, 5), 96).to(DEV).requires_grad_()
    with pytest.raises(RuntimeError):
        nn.functional.relu6(leaf, inplace=True)


def test_relu6_output_modified_before_backward_raises(ocl):
    """like relu_, the saved output must not change before backward"""
    x = _x((2, 4, 5, 5), 97).to(DEV).requires_grad_()
    y = nn.functional.relu6(x * 2.0, inplace=True)
    y.add_(1.0)
    with pytest.raises(RuntimeError):
        y.sum().backward()


@pytest.mark.parametrize("shape", SHAPES + [(16, 24)], ids=["x".join(map(str, s)) for s in SHAPES + [(16, 24)]])
@pytest.mark.parametrize("momentum", [0.1, None], ids=["m0.1", "cumulative"])
def test_num_batches_tracked_joins_stats(ocl, shape, momentum, tmp_path):
    """the module's num_batches_tracked += 1 is applied by the following
    training batch norm's statistics kernel (no launch of its own); the
    count and the running statistics equal torch-CPU's, with momentum=None
    (which reads the count on the host) too"""
    C = shape[1]
    mk = nn.BatchNorm2d if len(shape) == 4 else nn.BatchNorm1d
    torch.manual_seed(98)
    cpu = mk(C, momentum=momentum).train()
    dev = mk(C, momentum=momentum).to(DEV).train()
    dev.load_state_dict(cpu.state_dict())
    path = str(tmp_path / "prof.csv")
    with torch.ocl.profile(DEV, path):
        for i in range(4):
            x = _x(shape, 99 + i)
            assert _close(cpu(x), dev(x.to(DEV)))
        torch.ocl.synchronize()
    ops = [line.split(",")[1] for line in open(path).read().splitlines()[1:]]
    if momentum is not None:
        assert not any(o.startswith("add") for o in ops), ops
    assert dev.num_batches_tracked.item() == cpu.num_batches_tracked.item() == 4
    _check_bn_state(cpu, dev)


def test_pending_count_read_or_followed_by_other_ops(ocl):
    """a pending count is applied before anything else reads it"""
    cpu, dev = _bn_pair(8, 103)
    x = _x((2, 8, 4, 4), 104)
    cpu(x), dev(x.to(DEV))
    dev.num_batches_tracked.add_(1)
    assert dev.num_batches_tracked.item() == 2
    dev.num_batches_tracked.add_(1)
    t = dev.num_batches_tracked * 10  # another op on the counter itself
    assert t.item() == 30
    dev.num_batches_tracked.add_(1)
    dev.eval()(x.to(DEV))  # an eval batch norm does not take it
    assert dev.num_batches_tracked.item() == 4
    dev.train()
    dev.num_batches_tracked.add_(2)  # not an increment by one: a plain add
    dev.num_batches_tracked.add_(1, alpha=3)
    assert dev.num_batches_tracked.item() == 9
    c = dev.num_batches_tracked.clone()
    dev.num_batches_tracked.add_(1)
    c.add_(1)  # another counter: the first one is launched first
    dev(x.to(DEV))
    assert (dev.num_batches_tracked.item(), c.item()) == (11, 10)


@pytest.mark.parametrize("act", ["relu", "relu6"])
def test_act_grad_kept_by_hook_is_written(ocl, act):
    """the batch-norm backward forms the activation gradient from x and does
    not store it; a hook that keeps that gradient (the batch norm's output
    gradient) still sees the right values, written by the next flush"""
    cpu, dev = _bn_pair_wide(16, 105) if act == "relu6" else _bn_pair(16, 105)
    f = (lambda t: nn.functional.relu6(t, inplace=True)) if act == "relu6" else (lambda t: torch.relu_(t))
    x = _x((4, 16, 10, 10), 106)
    g = _x((4, 16, 10, 10), 107)
    res = []
    for m, d in ((cpu, "cpu"), (dev, DEV)):
        xi = x.detach().to(d).requires_grad_()
        kept = []
        y = m(xi)
        y.register_hook(lambda t: kept.append(t))
        z = f(y)
        z.backward(g.to(d))
        res.append((kept[0].cpu(), xi.grad.cpu()))
    assert _close(res[0][0], res[1][0], 1e-6) and _close(res[0][1], res[1][1], 1e-4)


@pytest.mark.parametrize("act", ["relu", "relu6"])
def test_act_grad_from_x_twice_with_retained_graph(ocl, act):
    """a second backward through a retained graph (the (a, b) record is
    consumed by the first) reads the activation output instead, with the
    same result, bit for bit"""
    _, dev = _bn_pair_wide(8, 108) if act == "relu6" else _bn_pair(8, 108)
    f = (lambda t: nn.functional.relu6(t, inplace=True)) if act == "relu6" else (lambda t: torch.relu_(t))
    x = _x((4, 8, 12, 12), 109).to(DEV).requires_grad_()
    z = f(dev(x))
    g = _x((4, 8, 12, 12), 110).to(DEV)
    (g1,) = torch.autograd.grad(z, x, g, retain_graph=True)
    (g2,) = torch.autograd.grad(z, x, g)
    assert torch.equal(g1.cpu(), g2.cpu())
