"""Op-level parity on the `ocl` device against torch-CPU (the reference's own
differential harness, tests/test_op.py:14-150, with fixed seeds).

Tolerances follow the reference: forward-only ops <= 1e-6 abs, forward +
backward <= 1e-3 abs (test_op.py:39,103,149), mm / bmm / cat bit-exact
(test_op.py:190,236,479).  Contractions are checked in both math modes:
exact fp32 (SIMT, reference tolerances) and TF32 tensor cores (abs 1e-3 +
rel 5e-3 of each compared tensor's magnitude, the stated TF32 tolerance)."""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "ocl:0"


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _inputs(specs, seed, randgen="randn"):
    g = _gen(seed)
    xs = []
    for shape, limit in specs:
        if limit <= 0:
            x = torch.randn(shape, generator=g) if randgen == "randn" else torch.rand(shape, generator=g)
        else:
            x = torch.randint(limit, shape, generator=g)
        xs.append(x)
    return xs


def _diff(a, b):
    return (a.detach().double() - b.detach().to("cpu").double()).abs().max().item() if a.numel() else 0.0


def check_fwd(specs, call, tol=1e-6, seed=0):
    xs = _inputs(specs, seed)
    with torch.no_grad():
        y_cpu = call(*xs)
        y_dev = call(*[x.to(DEV) for x in xs])
    assert y_dev.device.type == "ocl"
    d = _diff(y_cpu, y_dev)
    assert d <= tol, f"forward diff {d} > {tol}"


def check_fwd_bwd(specs, call, tol=1e-3, seed=0, randgen="randn"):
    xs_cpu = _inputs(specs, seed, randgen)
    xs_dev = []
    for (shape, limit), x in zip(specs, xs_cpu):
        xd = x.to(DEV)
        if limit <= 0:
            x.requires_grad_()
            xd.requires_grad_()
        xs_dev.append(xd)
    y_cpu = call(*xs_cpu)
    y_dev = call(*xs_dev)
    if y_cpu.dim():
        dy = torch.randn(y_cpu.shape, generator=_gen(seed + 1))
        y_cpu.backward(dy)
        y_dev.backward(dy.to(DEV))
    else:
        y_cpu.backward()
        y_dev.backward()
    diffs = {"y": _diff(y_cpu, y_dev)}
    for i, (x, xd) in enumerate(zip(xs_cpu, xs_dev)):
        if x.grad is not None:
            diffs[f"x{i}"] = _diff(x.grad, xd.grad)
    worst = max(diffs.values())
    assert worst <= tol, f"diffs {diffs} > {tol}"


def check_module(specs, module, tol=1e-3, seed=0, paramgen=None, rel=0.0):
    torch.manual_seed(seed)
    if paramgen is not None:
        with torch.no_grad():
            for p in module.parameters():
                p.copy_(paramgen(p.shape, generator=_gen(seed + 7)))
    xs_cpu = _inputs(specs, seed)
    for x in xs_cpu:
        if x.is_floating_point():
            x.requires_grad_()
    y_cpu = module(*xs_cpu)
    dy = torch.randn(y_cpu.shape, generator=_gen(seed + 1))
    y_cpu.backward(dy)
    grads_cpu = {n: p.grad.clone() for n, p in module.named_parameters()}
    module.zero_grad(set_to_none=True)
    dev_mod = module.to(DEV)
    xs_dev = [x.detach().to(DEV).requires_grad_() if x.is_floating_point() else x.to(DEV) for x in xs_cpu]
    y_dev = dev_mod(*xs_dev)
    y_dev.backward(dy.to(DEV))
    # per tensor: abs tolerance plus `rel` times that tensor's own magnitude
    pairs = {"y": (y_cpu, y_dev)}
    for i, (x, xd) in enumerate(zip(xs_cpu, xs_dev)):
        if x.grad is not None:
            pairs[f"x{i}"] = (x.grad, xd.grad)
    for n, p in dev_mod.named_parameters():
        pairs["p_" + n] = (grads_cpu[n], p.grad)
    bad = {}
    for k, (ref, got) in pairs.items():
        d = _diff(ref, got)
        lim = tol + rel * max(ref.abs().max().item(), 1.0)
        if d > lim:
            bad[k] = (d, lim)
    assert not bad, f"off: {bad}"


# ------------------------------------------------------------ reductions
REDUCTIONS = [
    ("mean_1d", lambda x: torch.mean(x, dim=0, keepdim=True)),
    ("mean_2d", lambda x: torch.mean(x, dim=(1, 2), keepdim=True)),
    ("mean_1d_squeeze", lambda x: torch.mean(x, dim=0, keepdim=False)),
    ("mean_2d_squeeze", lambda x: torch.mean(x, dim=(0, 2), keepdim=False)),
    ("mean_all", lambda x: torch.mean(x)),
    ("sum_1d", lambda x: torch.sum(x, dim=0, keepdim=True)),
    ("sum_2d", lambda x: torch.sum(x, dim=(1, 2), keepdim=True)),
    ("sum_1d_squeeze", lambda x: torch.sum(x, dim=0, keepdim=False)),
    ("sum_2d_squeeze", lambda x: torch.sum(x, dim=(0, 2), keepdim=False)),
    ("prod_1d", lambda x: torch.prod(x, dim=1, keepdim=True)),
    ("prod_1d_squeeze", lambda x: torch.prod(x, dim=1, keepdim=False)),
]


@pytest.mark.parametrize("name,fn", REDUCTIONS, ids=[r[0] for r in REDUCTIONS])
def test_reductions(ocl, name, fn):
    check_fwd_bwd([([2, 3, 4], -1)], fn)


# ------------------------------------------------------- pointwise / acts
ACTS = [
    ("logsoftmax_2d", [([4, 3], -1)], nn.LogSoftmax(dim=1)),
    ("logsoftmax_3d_last", [([4, 3, 5], -1)], nn.LogSoftmax(dim=-1)),
    ("logsoftmax_3d_mid", [([4, 3, 5], -1)], nn.LogSoftmax(dim=1)),
    ("logsoftmax_3d_first", [([4, 3, 5], -1)], nn.LogSoftmax(dim=0)),
    ("softmax", [([4, 3], -1)], nn.Softmax(dim=1)),
    ("nllloss", [([4, 3], -1), ([4], 3)], nn.NLLLoss()),
    ("aapool2d", [([4, 8, 2, 2], -1)], nn.AdaptiveAvgPool2d((1, 1))),
    ("aapool2d_general", [([2, 3, 7, 9], -1)], nn.AdaptiveAvgPool2d((3, 4))),
    ("abs", [([4, 3], -1)], torch.abs),
    ("abs_", [([4, 3], -1)], lambda x: torch.abs_(x * 1.0)),
    ("hardtanh", [([4, 3], -1)], nn.Hardtanh()),
    ("hardtanh_", [([4, 3], -1)], lambda x: nn.Hardtanh(inplace=True)(x * 1.0)),
    ("relu6", [([4, 30], -1)], lambda x: nn.ReLU6(inplace=True)(x * 4.0)),
    ("sigmoid", [([4, 3], -1)], nn.Sigmoid()),
    ("sigmoid_", [([4, 3], -1)], lambda x: torch.sigmoid_(x * 1.0)),
    ("hardsigmoid", [([4, 3], -1)], nn.Hardsigmoid()),
    ("relu", [([4, 3], -1)], nn.ReLU()),
    ("relu_", [([4, 3], -1)], lambda x: nn.ReLU(inplace=True)(x * 1.0)),
    ("leaky_relu", [([4, 3], -1)], nn.LeakyReLU()),
    ("tanh", [([4, 3], -1)], nn.Tanh()),
    ("tanh_", [([4, 3], -1)], lambda x: torch.tanh_(x * 1.0)),
    ("silu", [([4, 3], -1)], nn.SiLU()),
    ("gelu", [([4, 3], -1)], nn.GELU()),
    ("gelu_tanh", [([4, 3], -1)], lambda x: nn.GELU(approximate="tanh")(x * 1.0)),
    ("log_sigmoid", [([2, 4], -1)], nn.LogSigmoid()),
    ("amax", [([2, 3, 4, 5], -1)], lambda x: torch.amax(x, (1, -1))),
    ("amax_keepdim", [([2, 3, 4, 5], -1)], lambda x: torch.amax(x, (1, -1), keepdim=True)),
    ("amin", [([2, 3, 4, 5], -1)], lambda x: torch.amin(x, (1, -1))),
    ("add_broadcast", [([4, 3, 5], -1), ([3, 1], -1)], lambda a, b: a + 2.5 * b),
    ("mul_div", [([4, 3, 5], -1), ([5], -1)], lambda a, b: a * b / (b.abs() + 1)),
    ("maxpool_3_2_1", [([2, 4, 11, 11], -1)], lambda x: F.max_pool2d(x, 3, 2, 1)),
    ("maxpool_2", [([2, 4, 12, 12], -1)], lambda x: F.max_pool2d(x, 2)),
    ("maxpool_ceil", [([2, 4, 11, 11], -1)], lambda x: F.max_pool2d(x, 3, 2, 0, ceil_mode=True)),
    ("avgpool", [([2, 4, 11, 11], -1)], lambda x: F.avg_pool2d(x, 3, 2, 1)),
    ("avgpool_nopad", [([2, 4, 11, 11], -1)], lambda x: F.avg_pool2d(x, 3, 2, 1, count_include_pad=False)),
    ("cross_entropy", [([6, 10], -1), ([6], 10)], lambda x, t: F.cross_entropy(x, t)),
    ("batch_norm_train", [([4, 3, 5, 6], -1)],
     lambda x: F.batch_norm(x, None, None, torch.ones(3, device=x.device), torch.zeros(3, device=x.device), True)),
    ("layer_norm", [([2, 3, 4, 30], -1)], lambda x: F.layer_norm(x, (4, 30))),
]


@pytest.mark.parametrize("name,specs,fn", ACTS, ids=[a[0] for a in ACTS])
def test_fwd_bwd_ops(ocl, name, specs, fn):
    check_fwd_bwd(specs, fn)


FWD = [
    ("atan", [([4, 3, 5], -1)], torch.atan),
    ("min", [([4, 3, 5], -1)], torch.min),
    ("max", [([4, 3, 5], -1)], torch.max),
    ("lerp", [([4, 3, 5], -1), ([4, 3, 1], -1)], lambda x, y: torch.lerp(x, y, 0.1)),
    ("dot", [([16], -1), ([16], -1)], torch.dot),
    ("clamp1", [([4, 3, 5], -1)], lambda x: torch.clamp(x, min=-0.2, max=0.3)),
    ("clamp2", [([4, 3, 5], -1)], lambda x: torch.clamp(x, min=-0.2)),
    ("clamp3", [([4, 3, 5], -1)], lambda x: torch.clamp(x, max=0.3)),
    ("pow2", [([2, 4], -1)], lambda a: torch.abs(a) ** 2.0),
    ("pow13", [([2, 4], -1)], lambda a: torch.abs(a) ** 1.3),
    ("exp_log", [([2, 4], -1)], lambda a: torch.log(torch.exp(a) + 1)),
    ("argmax", [([4, 7], -1)], lambda a: torch.argmax(a, 1)),
    ("where", [([4, 7], -1)], lambda a: torch.where(a > 0, a, a * 0.5)),
    ("addcmul", [([4, 3], -1), ([4, 3], -1), ([4, 3], -1)], lambda a, b, c: torch.addcmul(a, b, c, value=0.5)),
    ("addcdiv", [([4, 3], -1), ([4, 3], -1), ([4, 3], -1)],
     lambda a, b, c: torch.addcdiv(a, b, c.abs() + 1, value=0.5)),
]


@pytest.mark.parametrize("name,specs,fn", FWD, ids=[a[0] for a in FWD])
def test_fwd_ops(ocl, name, specs, fn):
    check_fwd(specs, fn)


# ------------------------------------------------------- comparisons / logic
@pytest.mark.parametrize("op", [torch.eq, torch.ne, torch.gt, torch.lt, torch.ge, torch.le, torch.maximum,
                                torch.minimum])
def test_compare(ocl, op):
    """test_op.py:521-557"""
    check_fwd([([20, 30], -1), ([1, 30], -1)],
              lambda a, b: op(torch.round(a) * 10, torch.round(b) * 10).to(torch.float))
    if op not in (torch.maximum, torch.minimum):
        check_fwd([([20, 30], -1)], lambda a: op(torch.round(a) * 10, 5).to(torch.float))
    check_fwd([([20, 30], -1)], lambda a: op(torch.round(a) * 10, torch.tensor(5.0)).to(torch.float))


@pytest.mark.parametrize("sym", ["&", "|", "^", "~"])
def test_logical(ocl, sym):
    ops = {"&": lambda a, b: a & b, "|": lambda a, b: a | b, "^": lambda a, b: a ^ b, "~": lambda a, b: ~a}
    op = ops[sym]
    check_fwd([([20, 30], 10), ([1, 30], 10)], lambda a, b: op(a - 5, a - 5))
    check_fwd([([20, 30], 10), ([1, 30], 10)], lambda a, b: op(a > 5, a > 5).to(torch.float32))


# ----------------------------------------------------------- contractions
@pytest.mark.parametrize("math", ["fp32", "tf32"])
def test_linear(ocl, math):
    mode = 1 if math == "fp32" else 0
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(mode)
    try:
        tol, rel = (1e-3, 0.0) if math == "fp32" else (1e-3, 5e-3)
        check_module([([8, 10], -1)], nn.Linear(10, 5), tol=tol, rel=rel)
        check_module([([2, 6, 10], -1)], nn.Linear(10, 5), tol=tol, rel=rel)
        check_module([([64, 300], -1)], nn.Linear(300, 130), tol=tol, rel=rel)
    finally:
        torch.ocl.set_math_mode(old)


CONVS = [
    ("conv_groups", [([2, 6, 10, 20], -1)], lambda: nn.Conv2d(6, 8, [3, 5], stride=[1, 2], padding=[1, 2], groups=2)),
    ("conv_3x3", [([2, 16, 14, 14], -1)], lambda: nn.Conv2d(16, 32, 3, padding=1, bias=False)),
    ("conv_1x1", [([2, 64, 7, 7], -1)], lambda: nn.Conv2d(64, 32, 1, bias=False)),
    ("conv_1x1_s2", [([2, 32, 14, 14], -1)], lambda: nn.Conv2d(32, 64, 1, stride=2, bias=False)),
    ("conv_7x7_s2", [([2, 3, 32, 32], -1)], lambda: nn.Conv2d(3, 16, 7, stride=2, padding=3, bias=False)),
    ("conv_3x3_s2", [([2, 16, 15, 15], -1)], lambda: nn.Conv2d(16, 16, 3, stride=2, padding=1, bias=False)),
    ("conv_dilated", [([2, 8, 16, 16], -1)], lambda: nn.Conv2d(8, 8, 3, padding=2, dilation=2)),
    ("depthwise", [([2, 32, 14, 14], -1)], lambda: nn.Conv2d(32, 32, 3, padding=1, groups=32, bias=False)),
    ("depthwise_s2", [([2, 32, 15, 15], -1)], lambda: nn.Conv2d(32, 32, 3, stride=2, padding=1, groups=32)),
    ("mnist_conv1", [([4, 1, 28, 28], -1)], lambda: nn.Conv2d(1, 32, 3)),
    ("convtr", [([2, 6, 10, 20], -1)],
     lambda: nn.ConvTranspose2d(6, 8, [3, 5], stride=[1, 2], padding=[1, 2], dilation=1, groups=2)),
    ("convtr_pad", [([2, 6, 10, 20], -1)],
     lambda: nn.ConvTranspose2d(6, 8, [3, 5], stride=[1, 2], padding=[1, 2], output_padding=[0, 1], groups=2)),
    ("convtr_nobias", [([2, 6, 10, 20], -1)],
     lambda: nn.ConvTranspose2d(6, 8, [3, 5], stride=[1, 2], padding=[1, 2], groups=1, bias=False)),
]


@pytest.mark.parametrize("math", ["fp32", "tf32"])
@pytest.mark.parametrize("name,specs,mk", CONVS, ids=[c[0] for c in CONVS])
def test_conv(ocl, name, specs, mk, math):
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(1 if math == "fp32" else 0)
    try:
        # TF32: each product carries up to 2^-9 relative error; 5e-3 of the
        # tensor's magnitude covers the reductions of these shapes
        tol, rel = (1e-3, 0.0) if math == "fp32" else (2e-3, 5e-3)
        check_module(specs, mk(), tol=tol, rel=rel)
    finally:
        torch.ocl.set_math_mode(old)


def test_batch_norm_module(ocl):
    check_module([([4, 5, 7, 7], -1)], nn.BatchNorm2d(5), paramgen=torch.randn)
    # running statistics are updated on the device like on the CPU (unbiased var)
    ref, bn = nn.BatchNorm2d(5), nn.BatchNorm2d(5).to(DEV)
    x = _inputs([([4, 5, 7, 7], -1)], 0)[0]
    for _ in range(3):
        ref(x)
        bn(x.to(DEV))
    assert _diff(ref.running_mean, bn.running_mean) < 1e-6
    assert _diff(ref.running_var, bn.running_var) < 1e-6
    assert bn.num_batches_tracked.item() == 3
    bn.eval()
    ref.eval()
    assert _diff(ref(x), bn(x.to(DEV))) < 1e-5


BN_SHAPES = [
    [3, 7, 7, 7],       # one CTA per channel, 49-pixel planes (scalar loads)
    [16, 8, 56, 56],    # channel split over a 2-CTA cluster
    [64, 4, 56, 56],    # 8-CTA clusters; the backward needs the one-CTA-per-SM budget
    [32, 4, 45, 45],    # odd plane size across a cluster
    [2, 3, 512, 512],   # channels too large for a cluster: two-pass kernels
]


@pytest.mark.parametrize("shape", BN_SHAPES, ids=["x".join(map(str, s)) for s in BN_SHAPES])
def test_batch_norm_shapes(ocl, shape):
    C = shape[1]
    check_module([(shape, -1)], nn.BatchNorm2d(C), paramgen=torch.randn, tol=2e-4, rel=2e-5)
    ref, bn = nn.BatchNorm2d(C), nn.BatchNorm2d(C).to(DEV)
    x = _inputs([(shape, -1)], 3)[0] * 3 + 1
    for _ in range(2):
        ref(x)
        bn(x.to(DEV))
    assert _diff(ref.running_mean, bn.running_mean) < 1e-5
    assert _diff(ref.running_var, bn.running_var) < 1e-4


def test_masked_select_nonzero_print(ocl):
    g = _gen(11)
    x = torch.randn(7, 33, generator=g)
    m = x > 0.3
    xd, md = x.to(DEV), m.to(DEV)
    assert torch.equal(torch.masked_select(xd, md).cpu(), torch.masked_select(x, m))
    assert torch.equal(xd[md].cpu(), x[m])
    assert torch.equal(torch.nonzero(md).cpu(), torch.nonzero(m))
    big = torch.randn(100003, generator=g)
    assert torch.equal(big.to(DEV)[big.to(DEV) > 1].cpu(), big[big > 1])
    y = xd.clone()
    y.masked_fill_(md, -1.0)
    assert torch.equal(y.cpu(), x.masked_fill(m, -1.0))
    assert "ocl" in repr(xd) and str(round(x[0, 0].item(), 4))[:5] in repr(xd)
    assert torch.equal(md.all(1).cpu(), m.all(1)) and torch.equal(md.any(0).cpu(), m.any(0))
    assert torch.equal(torch.isneginf(torch.tensor([1.0, -float("inf")]).to(DEV)).cpu(), torch.tensor([False, True]))


def test_layer_norm_affine(ocl):
    check_module([([2, 3, 4, 30], -1)], nn.LayerNorm((4, 30), elementwise_affine=False))
    check_module([([2, 3, 4, 30], -1)], nn.LayerNorm((4, 30), elementwise_affine=True), paramgen=torch.randn)
    check_module([([3, 197, 768], -1)], nn.LayerNorm(768), paramgen=torch.randn)


def _mat(D0, D1, d, ind):
    """test_op.py:153-170: transposed / offset / non-contiguous operands"""
    tr, offset, non_cont = ind % 2, 0 if ind < 2 else 5, ind >= 4
    if tr:
        D0, D1 = D1, D0
    tmp = torch.arange(0, 400, device=d, dtype=torch.float32)
    size = D0 * D1 * (4 if non_cont else 1)
    tmp = tmp[offset:offset + size]
    tmp = tmp.view(D0 * 2, D1 * 2)[::2, ::2] if non_cont else tmp.view(D0, D1)
    return tmp.T if tr else tmp


@pytest.mark.parametrize("math", [0, 1])
def test_mm_exact(ocl, math):
    """test_op.py:172-192: bit-exact over 6x6x6 operand layouts"""
    old = torch.ocl.get_math_mode()
    torch.ocl.set_math_mode(math)
    try:
        M, N, K = 4, 10, 6
        for Ct in range(6):
            for At in range(6):
                for Bt in range(6):
                    outs = []
                    for d in ["cpu", DEV]:
                        A, B, C = _mat(M, K, d, At), _mat(K, N, d, Bt), _mat(M, N, d, Ct)
                        torch.mm(A, B, out=C)
                        outs.append(C)
                    assert _diff(outs[0], outs[1]) == 0, (At, Bt, Ct)
    finally:
        torch.ocl.set_math_mode(old)


def _bmat(B, D0, D1, d, ind):
    tr, offset, non_cont = ind % 2, 0 if ind < 2 else 5, ind >= 4
    if tr:
        D0, D1 = D1, D0
    tmp = torch.arange(0, 10 + B * D0 * D1 * 4, device=d, dtype=torch.float32)
    size = B * D0 * D1 * (4 if non_cont else 1)
    tmp = tmp[offset:offset + size]
    tmp = tmp.view(B, D0 * 2, D1 * 2)[:, ::2, ::2] if non_cont else tmp.view(B, D0, D1)
    return torch.transpose(tmp, 2, 1) if tr else tmp


def test_bmm_exact(ocl):
    """test_op.py:194-239"""
    Bc, M, N, K = 3, 4, 10, 6
    for Ba, Bb in [(Bc, Bc), (1, Bc), (Bc, 1)]:
        for Ct in range(2):
            for At in range(6):
                for Bt in range(6):
                    outs = []
                    for d in ["cpu", DEV]:
                        A, B, C = _bmat(Ba, M, K, d, At), _bmat(Bb, K, N, d, Bt), _bmat(Bc, M, N, d, Ct)
                        if Ba < Bc:
                            A = A.expand(Bc, M, K)
                        if Bb < Bc:
                            B = B.expand(Bc, K, N)
                        torch.bmm(A, B, out=C)
                        outs.append(C)
                    assert _diff(outs[0], outs[1]) == 0, (Ba, Bb, At, Bt, Ct)


@pytest.mark.parametrize("beta,alpha", [(0.0, 1.0), (1.0, 1.0), (1.0, 0.5), (0.5, 0.5)])
def test_addmm(ocl, math_fp32, beta, alpha):
    """test_op.py:400-416 (including a transposed `out`)"""
    check_fwd([([2, 4], -1), ([2, 3], -1), ([3, 4], -1)], lambda a, b, c: torch.addmm(a, b, c, beta=beta, alpha=alpha))
    check_fwd([([2, 4], -1), ([2, 3], -1), ([3, 4], -1), ([4, 2], -1)],
              lambda a, b, c, o: torch.addmm(a, b, c, beta=beta, alpha=alpha, out=o.T))


def test_cat_exact(ocl):
    """test_op.py:456-483"""
    g = _gen(0)
    x1, x2 = torch.randn(5, 10, generator=g), torch.randn(5, 20, generator=g)
    y1 = torch.cat((x1, x2), dim=1)
    y3s = torch.zeros(10, 30)
    torch.cat((x1, x2), dim=1, out=y3s[::2, :])
    x1d, x2d = x1.to(DEV), x2.to(DEV)
    y1d = torch.cat((x1d, x2d), dim=1)
    y3sd = torch.zeros(10, 30).to(DEV)
    torch.cat((x1d, x2d), dim=1, out=y3sd[::2, :])
    assert _diff(y1, y1d) == 0
    assert _diff(y3s, y3sd) == 0


def test_rng_and_dropout(ocl):
    """test_op.py:492-518"""
    torch.ocl.manual_seed_all(10)
    x1 = torch.randn(10, device=DEV).cpu()
    x2 = torch.randn(10, device=DEV).cpu()
    torch.ocl.manual_seed_all(10)
    x3 = torch.randn(10, device=DEV).cpu()
    assert (x1 - x2).abs().max().item() > 0
    assert (x1 - x3).abs().max().item() == 0
    big = torch.randn(100000, device=DEV).cpu()
    assert abs(big.mean().item()) < 0.02 and abs(big.std().item() - 1) < 0.02
    u = torch.empty(100000, device=DEV).uniform_(2, 3).cpu()
    assert u.min() >= 2 and u.max() < 3
    x = torch.randn(1000, device=DEV, requires_grad=True)
    y = F.dropout(x, p=0.25, training=False)
    assert (x - y).abs().max().item() == 0
    x = torch.rand(1000, device=DEV, requires_grad=True)
    y = F.dropout(x, p=0.25, training=True)
    assert abs((y > 0).float().mean().item() - 0.75) < 0.1
    assert (x.mean() - y.mean()).abs().item() < 0.05
    y.backward(torch.ones(1000, device=DEV))
    assert abs((x.grad > 0).float().mean().item() - 0.75) < 0.1


def test_copies_and_views(ocl):
    g = _gen(3)
    x = torch.randn(4, 5, 6, generator=g)
    xd = x.to(DEV)
    assert torch.equal(xd.cpu(), x)
    assert torch.equal(xd.permute(2, 0, 1).contiguous().cpu(), x.permute(2, 0, 1).contiguous())
    assert torch.equal(xd[:, 1:4, ::2].cpu(), x[:, 1:4, ::2])
    assert torch.equal(xd.double().cpu(), x.double())
    assert torch.equal(xd.to(torch.int64).cpu(), x.to(torch.int64))
    assert torch.equal(xd.transpose(0, 2).cpu(), x.transpose(0, 2))
    y = torch.zeros(6, 4, 5).to(DEV)
    y.copy_(xd.permute(2, 0, 1))
    assert torch.equal(y.cpu(), x.permute(2, 0, 1))
    assert xd.sum().item() == pytest.approx(x.sum().item(), rel=1e-5)
    z = torch.full((3, 3), 2.5, device=DEV)
    assert torch.equal(z.cpu(), torch.full((3, 3), 2.5))
    i = torch.arange(10, device=DEV)
    assert torch.equal(i.cpu(), torch.arange(10))
    r = torch.empty(0, device=DEV)
    r.resize_(10)
    assert r.numel() == 10
    p = x.pin_memory()
    assert torch.equal(p.to(DEV, non_blocking=True).cpu(), x)


def test_sgd_foreach_and_fused(ocl):
    g = _gen(5)
    params = [torch.randn(s, generator=g) for s in [(10, 3), (7,), (4, 4, 4)]]
    grads = [torch.randn(p.shape, generator=g) for p in params]
    for kw in [dict(foreach=True), dict(fused=True), dict(foreach=False)]:
        pc = [p.clone().requires_grad_() for p in params]
        pd = [p.clone().to(DEV).requires_grad_() for p in params]
        oc = torch.optim.SGD(pc, lr=0.1, momentum=0.9)
        od = torch.optim.SGD(pd, lr=0.1, momentum=0.9, **kw)
        for _ in range(3):
            for a, b, gr in zip(pc, pd, grads):
                a.grad = gr.clone()
                b.grad = gr.to(DEV)
            oc.step()
            od.step()
        for a, b in zip(pc, pd):
            assert _diff(a, b) < 1e-6, kw


def test_profile_csv(ocl, tmp_path):
    """torch.ocl.profile writes the reference's CSV log (CLTensor.cpp:95-140)"""
    path = str(tmp_path / "prof.csv")
    x = torch.randn(64, 64).to(DEV)
    with torch.ocl.profile(DEV, path):
        y = torch.relu(x @ x)
        torch.ocl.synchronize()
    lines = open(path).read().strip().split("\n")
    assert lines[0] == "section,kernel,start (ms),end (ms),duraion(ms)"
    assert any("mm" in l for l in lines[1:])


# upsample and MSE / BCE losses: ops the reference ran on its CPU fallback
UPSAMPLES = [
    ("nearest_x2", lambda x: F.interpolate(x, scale_factor=2, mode="nearest")),
    ("nearest_size", lambda x: F.interpolate(x, size=(11, 13), mode="nearest")),
    ("nearest_down", lambda x: F.interpolate(x, size=(3, 4), mode="nearest")),
    ("nearest_exact", lambda x: F.interpolate(x, size=(11, 13), mode="nearest-exact")),
    ("bilinear_x2", lambda x: F.interpolate(x, scale_factor=2, mode="bilinear", align_corners=False)),
    ("bilinear_align", lambda x: F.interpolate(x, size=(11, 13), mode="bilinear", align_corners=True)),
    ("bilinear_down", lambda x: F.interpolate(x, size=(4, 3), mode="bilinear", align_corners=False)),
    ("bilinear_frac", lambda x: F.interpolate(x, scale_factor=1.7, mode="bilinear", align_corners=False)),
]


@pytest.mark.parametrize("name,call", UPSAMPLES, ids=[u[0] for u in UPSAMPLES])
def test_upsample(ocl, name, call):
    check_fwd_bwd([([2, 3, 6, 7], -1)], call, tol=1e-5)


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
def test_mse_loss(ocl, reduction):
    check_fwd_bwd([([4, 5, 6], -1), ([4, 5, 6], -1)], lambda a, b: F.mse_loss(a, b, reduction=reduction), tol=1e-4)


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
def test_bce_loss(ocl, reduction):
    g = _gen(5)
    p = torch.rand(4, 7, generator=g) * 0.98 + 0.01
    t = torch.rand(4, 7, generator=g)
    w = torch.rand(4, 7, generator=g)
    for weight in (None, w):
        pc = p.clone().requires_grad_()
        pd = p.to(DEV).requires_grad_()
        yc = F.binary_cross_entropy(pc, t, weight=weight, reduction=reduction)
        yd = F.binary_cross_entropy(pd, t.to(DEV), weight=None if weight is None else weight.to(DEV),
                                    reduction=reduction)
        assert _diff(yc, yd) <= 1e-5
        gy = torch.randn(yc.shape, generator=g) if yc.dim() else torch.tensor(1.0)
        yc.backward(gy)
        yd.backward(gy.to(DEV))
        assert _diff(pc.grad, pd.grad) <= 1e-4


# reductions at training sizes: split column sums (bias gradients), warp and
# split-block row reductions, merged dims, strided inputs, NaN propagation
BIG_REDUCTIONS = [
    ("bias_grad", [6304, 768], lambda x: x.sum(0)),
    ("bias_grad_3d", [32, 197, 768], lambda x: x.sum((0, 1))),
    ("col_narrow", [50000, 8], lambda x: x.sum(0)),
    ("col_mean", [4096, 1000], lambda x: x.mean(0, keepdim=True)),
    ("col_max", [3000, 300], lambda x: x.amax(0)),
    ("col_min", [3000, 300], lambda x: x.amin(0)),
    ("row_short", [6304, 197], lambda x: x.sum(-1)),
    ("row_long", [12, 60000], lambda x: x.sum(-1)),
    ("row_max", [64, 5000], lambda x: x.amax(-1)),
    ("all", [3, 1000, 1000], lambda x: x.sum()),
    ("all_mean", [257, 1031], lambda x: x.mean()),
    ("sumsq", [2048, 512], lambda x: (x * x).sum(0)),
    ("prod", [64, 300], lambda x: (1 + 0.01 * x).prod(0)),
    ("transposed", [768, 6304], lambda x: x.t().sum(0)),
    ("nchw_channels", [16, 64, 28, 28], lambda x: x.sum((0, 2, 3))),
]


@pytest.mark.parametrize("name,shape,call", BIG_REDUCTIONS, ids=[r[0] for r in BIG_REDUCTIONS])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64], ids=["f32", "f64"])
def test_big_reduction(ocl, name, shape, call, dtype):
    x = torch.randn(shape, generator=_gen(11), dtype=torch.float64).to(dtype)
    ref = call(x.double())
    got = call(x.to(DEV)).cpu()
    assert got.dtype == dtype and got.shape == ref.shape
    # fp32 summation error grows like sqrt(n) * eps * |terms|; 1e-5 of the
    # sum of magnitudes bounds it for every shape here
    bound = call(x.double().abs()).abs().max().item() if name not in ("col_max", "col_min", "row_max") else 1.0
    tol = (1e-5 if dtype == torch.float32 else 1e-12) * max(bound, 1.0)
    assert _diff(ref, got) <= tol


def test_reduction_nan_propagates(ocl):
    x = torch.randn(4096, 64, generator=_gen(12))
    x[1000, 5] = float("nan")
    x[3, 63] = float("nan")
    xd = x.to(DEV)
    for call in (lambda t: t.amax(0), lambda t: t.amin(0), lambda t: t.sum(0), lambda t: t.amax(-1)):
        ref, got = call(x), call(xd).cpu()
        assert torch.equal(ref.isnan(), got.isnan())
        m = ~ref.isnan()
        assert _diff(ref[m], got[m]) <= 1e-3


def test_reduction_deterministic(ocl):
    xd = torch.randn(6304, 768, generator=_gen(13)).to(DEV)
    a, b = xd.sum(0).cpu(), xd.sum(0).cpu()
    assert torch.equal(a, b)


# permuted copies with a unit-stride inner dim (row copies in 16/8/4-byte words)
ROW_COPIES = [
    ("qkv_split", torch.float32, [197, 8, 3 * 96], lambda x: x.unflatten(-1, (3, 96)).transpose(0, -2).contiguous()),
    ("head_merge", torch.float32, [4, 12, 197, 64], lambda x: x.permute(2, 0, 1, 3).contiguous()),
    ("batch_first", torch.float32, [8, 197, 768], lambda x: x.transpose(0, 1).contiguous()),
    ("odd_inner", torch.float32, [5, 7, 33], lambda x: x.transpose(0, 1).contiguous()),
    ("odd_offset", torch.float32, [6, 5, 40], lambda x: x[:, :, 1:37].transpose(0, 1).contiguous()),
    ("int64", torch.int64, [6, 5, 24], lambda x: x.transpose(0, 1).contiguous()),
    ("half", torch.float16, [6, 5, 48], lambda x: x.transpose(0, 1).contiguous()),
    ("bytes", torch.uint8, [6, 5, 160], lambda x: x.transpose(0, 1).contiguous()),
    ("expanded", torch.float32, [1, 5, 64], lambda x: x.expand(4, 5, 64).transpose(0, 1).contiguous()),
    ("long_rows", torch.float32, [3, 70004], lambda x: x[:, 2:70002].contiguous()),
]


@pytest.mark.parametrize("name,dtype,shape,call", ROW_COPIES, ids=[r[0] for r in ROW_COPIES])
def test_row_copy(ocl, name, dtype, shape, call):
    x = (torch.randn(shape, generator=_gen(14)) * 50).to(dtype)
    ref = call(x)
    got = call(x.to(DEV)).cpu()
    assert got.is_contiguous() and torch.equal(ref, got)


# fp32 binary ops on strided operands whose inner dim is unit-stride or
# broadcast (the row-run kernel): transposed residual adds, row / column
# broadcasts, strided outputs
ROW_BINARIES = [
    ("add_transposed", [197, 8, 96], [8, 197, 96], lambda a, b: a.transpose(0, 1) + b),
    ("sub_both_transposed", [197, 8, 96], [197, 8, 96], lambda a, b: a.transpose(0, 1) - b.transpose(0, 1)),
    ("mul_col_broadcast", [300, 70], [300, 1], lambda a, b: a * b),
    ("div_sliced", [40, 130], [40, 100], lambda a, b: a[:, 10:110] / (b.abs() + 0.5)),
    ("gelu_bwd_transposed", [64, 33, 48], [33, 64, 48],
     lambda a, b: torch.ops.aten.gelu_backward(a.transpose(0, 1), b)),
    ("add_alpha", [50, 3, 40], [3, 50, 40], lambda a, b: torch.add(a.transpose(0, 1), b, alpha=-2.5)),
    ("pos_embedding", [32, 197, 768], [1, 197, 768], lambda a, b: a + b),  # few rows of 151296 elements
]


@pytest.mark.parametrize("name,sa,sb,call", ROW_BINARIES, ids=[r[0] for r in ROW_BINARIES])
def test_row_binary(ocl, name, sa, sb, call):
    g = _gen(15)
    a, b = torch.randn(sa, generator=g), torch.randn(sb, generator=g)
    ref = call(a, b)
    got = call(a.to(DEV), b.to(DEV)).cpu()
    assert _diff(ref, got) <= 1e-6 * max(1.0, ref.abs().max().item())


# layer norm over rows of 128 * k floats (vectorised kernels, fused parameter
# gradients) and other widths (per-element kernels), against float64
@pytest.mark.parametrize("rows,n,affine", [(6304, 768, True), (100, 1024, True), (37, 128, False), (513, 256, True),
                                           (50, 100, True), (8, 2048, True)])
def test_layer_norm_rows(ocl, rows, n, affine):
    g = _gen(40)
    x = torch.randn(rows, n, generator=g) * 3 + 1
    gy = torch.randn(rows, n, generator=g)
    ln = nn.LayerNorm(n, elementwise_affine=affine)
    if affine:
        with torch.no_grad():
            ln.weight.copy_(torch.randn(n, generator=g))
            ln.bias.copy_(torch.randn(n, generator=g))
    ref = nn.LayerNorm(n, elementwise_affine=affine).double()
    ref.load_state_dict(ln.state_dict())
    dev = ln.to(DEV)
    xr, xd = x.double().requires_grad_(), x.to(DEV).requires_grad_()
    yr, yd = ref(xr), dev(xd)
    yr.backward(gy.double())
    yd.backward(gy.to(DEV))
    assert _diff(yr, yd) <= 1e-5 * max(1.0, yr.abs().max().item())
    assert _diff(xr.grad, xd.grad) <= 1e-4 * max(1.0, xr.grad.abs().max().item())
    if affine:
        for pr, pd in ((ref.weight, dev.weight), (ref.bias, dev.bias)):
            assert _diff(pr.grad, pd.grad) <= 1e-5 * max(1.0, pr.grad.abs().sum().item() / n)


# max-pool forward bit-exact (values and, through the gradient routing,
# indices) also with ties (integer inputs), padding, dilation, ceil mode; the
# backward adds overlapping windows' gradients in its own fixed order
@pytest.mark.parametrize("k,s,p,d,ceil", [(3, 2, 1, 1, False), (3, 1, 1, 1, False), (2, 2, 0, 1, False),
                                          (3, 2, 0, 2, True), (5, 3, 2, 1, True)])
def test_max_pool_ties_dilation_ceil(ocl, k, s, p, d, ceil):
    g = _gen(50)
    x = torch.randint(0, 4, (3, 5, 17, 19), generator=g).float()
    xc, xd = x.clone().requires_grad_(), x.to(DEV).requires_grad_()
    yc = F.max_pool2d(xc, k, s, p, d, ceil_mode=ceil)
    yd = F.max_pool2d(xd, k, s, p, d, ceil_mode=ceil)
    gy = torch.randn(yc.shape, generator=g)
    yc.backward(gy)
    yd.backward(gy.to(DEV))
    assert torch.equal(yc, yd.cpu())
    assert _diff(xc.grad, xd.grad) <= 1e-5


def test_copy_stream_pipeline(ocl):
    """Host-to-device copies on a second stream ordered against compute on
    the current one with events: the pipeline bench.py's end-to-end figure
    uses (each batch copied while the previous step computes)."""
    xs = [torch.randn(4, 3, 64, 64, generator=_gen(s)).pin_memory() for s in range(4)]
    bufs = [torch.empty(4, 3, 64, 64, device=DEV) for _ in range(2)]
    copy_s = torch.Stream(device=DEV)
    ready = [torch.Event(device=DEV) for _ in range(2)]
    free = [torch.Event(device=DEV) for _ in range(2)]
    conv = nn.Conv2d(3, 8, 3, padding=1).to(DEV)
    ref = nn.Conv2d(3, 8, 3, padding=1)
    ref.load_state_dict({k: v.cpu() for k, v in conv.state_dict().items()})

    def load(i):
        with copy_s:
            if i >= 2:
                free[i % 2].wait()
            bufs[i % 2].copy_(xs[i], non_blocking=True)
            ready[i % 2].record()

    load(0)
    outs = []
    for i in range(len(xs)):
        ready[i % 2].wait()
        with torch.no_grad():
            y = conv(bufs[i % 2]).sum((1, 2, 3))
        free[i % 2].record()
        if i + 1 < len(xs):
            load(i + 1)
        outs.append(y.cpu())
    for i, x in enumerate(xs):
        with torch.no_grad():
            r = ref(x).sum((1, 2, 3))
        assert (outs[i] - r).abs().max().item() <= 1e-2 * r.abs().max().item() + 1e-3
