"""CPU-only checks that pin the oracle: the numpy restatements (oracle.npref)
agree with torch-CPU ATen (the reference's arbiter, tests/validate_network.py
and tests/test_op.py), and the oracle reproduces the committed golden
fixtures (tests/golden/*.pt made by tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import models, npref, step

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_batch_norm_restatement_matches_torch():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 3, 5, 6, generator=g) * 2 + 1
    w, b = torch.randn(3, generator=g), torch.randn(3, generator=g)
    rm, rv = torch.zeros(3), torch.ones(3)
    y = F.batch_norm(x, rm, rv, w, b, training=True, momentum=0.1, eps=1e-5)
    ny, mean, invstd, nrm, nrv = npref.batch_norm_train(x.numpy(), w.numpy(), b.numpy(), np.zeros(3), np.ones(3),
                                                        0.1, 1e-5)
    assert np.abs(ny - y.numpy()).max() < 1e-5
    assert np.abs(nrm - rm.numpy()).max() < 1e-6
    assert np.abs(nrv - rv.numpy()).max() < 1e-6  # unbiased running variance
    xr = x.clone().requires_grad_()
    wr = w.clone().requires_grad_()
    br = b.clone().requires_grad_()
    out = F.batch_norm(xr, None, None, wr, br, training=True, eps=1e-5)
    dy = torch.randn(out.shape, generator=g)
    out.backward(dy)
    dx, dgam, dbet = npref.batch_norm_backward(dy.numpy(), x.numpy(), w.numpy(), mean, invstd)
    assert np.abs(dx - xr.grad.numpy()).max() < 1e-4
    assert np.abs(dgam - wr.grad.numpy()).max() < 1e-4
    assert np.abs(dbet - br.grad.numpy()).max() < 1e-4


@pytest.mark.parametrize("k,s,p,ceil", [(2, 2, 0, False), (3, 2, 1, False), (3, 2, 0, True), (3, 1, 1, False)])
def test_max_pool_restatement_matches_torch(k, s, p, ceil):
    g = torch.Generator().manual_seed(1)
    x = torch.randint(0, 4, (2, 3, 9, 9), generator=g).float()  # many ties
    y, ind = F.max_pool2d(x, k, s, p, ceil_mode=ceil, return_indices=True)
    ny, nind = npref.max_pool2d(x.numpy(), k, s, p, 1, ceil)
    assert np.array_equal(ny, y.numpy())
    assert np.array_equal(nind, ind.numpy())  # first index on ties, bit-exact
    dy = torch.randn(y.shape, generator=g)
    dx = torch.ops.aten.max_pool2d_with_indices_backward(dy, x, [k, k], [s, s], [p, p], [1, 1], ceil, ind)
    assert np.abs(npref.max_pool2d_backward(dy.numpy(), nind, x.shape) - dx.numpy()).max() < 1e-6


def test_max_pool_nan_wins():
    x = torch.tensor([[[[1.0, float("nan")], [3.0, 2.0]]]])
    y, ind = F.max_pool2d(x, 2, 2, return_indices=True)
    ny, nind = npref.max_pool2d(x.numpy(), 2, 2, 0)
    assert np.isnan(y.item()) and np.isnan(ny.item())
    assert ind.item() == nind.item() == 1


def test_softmax_nll_gelu_hardtanh_sgd_restatements():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(8, 11, generator=g) * 3
    t = torch.randint(0, 11, (8,), generator=g)
    t[3] = -100
    lp = F.log_softmax(x, 1)
    assert np.abs(npref.log_softmax(x.numpy(), 1) - lp.numpy()).max() < 1e-5
    for red in ["mean", "sum", "none"]:
        ref = F.nll_loss(lp, t, reduction=red, ignore_index=-100).numpy()
        assert np.abs(npref.nll_loss(lp.numpy(), t.numpy(), red, -100) - ref).max() < 1e-5
    for approx in ["none", "tanh"]:
        assert np.abs(npref.gelu(x.numpy(), approx) - F.gelu(x, approximate=approx).numpy()).max() < 1e-5
    xr = x.clone().requires_grad_()
    F.hardtanh(xr, 0.0, 6.0).backward(torch.ones_like(x))
    xe = torch.tensor([0.0, 6.0, 3.0, -1.0, 7.0]).requires_grad_()
    F.hardtanh(xe, 0.0, 6.0).backward(torch.ones(5))
    assert np.array_equal(npref.hardtanh_backward(np.ones(5), xe.detach().numpy(), 0.0, 6.0), xe.grad.numpy())
    p = torch.randn(5, generator=g)
    gr = torch.randn(5, generator=g)
    pt = p.clone().requires_grad_()
    opt = torch.optim.SGD([pt], lr=0.1, momentum=0.9)
    buf = None
    pn = p.numpy()
    for _ in range(3):
        pt.grad = gr.clone()
        opt.step()
        pn, buf = npref.sgd_momentum(pn, gr.numpy(), buf, 0.1, 0.9)
    assert np.abs(pn - pt.detach().numpy()).max() < 1e-6


@pytest.mark.parametrize("groups,stride,pad,dil", [(1, (1, 1), (0, 0), (1, 1)), (2, (1, 2), (1, 2), (1, 1)),
                                                   (1, (2, 2), (3, 3), (1, 1)), (1, (1, 1), (2, 2), (2, 2))])
def test_conv_restatement_matches_torch(groups, stride, pad, dil):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 6, 10, 12, generator=g)
    w = torch.randn(8, 6 // groups, 3, 5, generator=g)
    b = torch.randn(8, generator=g)
    y = F.conv2d(x, w, b, stride, pad, dil, groups)
    ny = npref.conv2d(x.numpy(), w.numpy(), b.numpy(), stride, pad, dil, groups)
    assert np.abs(ny - y.numpy()).max() < 1e-4


def test_oracle_matches_golden_fixtures():
    path = os.path.join(GOLDEN, "mnist_step.pt")
    gold = torch.load(path)
    _, snap = step.cpu_reference("mnist", batch=8, steps=2)
    for k, v in gold.items():
        assert k in snap, k
        assert torch.allclose(snap[k], v, rtol=1e-5, atol=1e-6), k


def test_golden_ops_fixture():
    gold = torch.load(os.path.join(GOLDEN, "ops.pt"))
    g = torch.Generator().manual_seed(gold["seed"].item())
    x = torch.randn(4, 3, 8, 8, generator=g)
    assert torch.equal(x, gold["x"])
    y, ind = F.max_pool2d(x, 3, 2, 1, return_indices=True)
    assert torch.equal(ind, gold["maxpool_ind"])
    assert torch.allclose(F.log_softmax(x.flatten(1), 1), gold["log_softmax"], atol=1e-6)


def test_workload_inputs_are_seeded():
    x1, y1 = models.make_inputs("resnet50", 2)
    x2, y2 = models.make_inputs("resnet50", 2)
    assert torch.equal(x1, x2) and torch.equal(y1, y2)
    x, y = models.make_inputs("mnist", 4)
    assert x.min() >= 0 and x.max() < 1 and y.max() < 10


# ------------------------------------------------------ TF32 emulation
def test_tf32_conversions():
    """cut_tf32 clears the low 13 mantissa bits; round_tf32 rounds to 10
    mantissa bits with ties away from zero (cvt.rna.tf32.f32)."""
    from oracle.tf32 import cut_tf32, round_tf32

    ulp = 2.0 ** -10  # one TF32 unit at 1.0
    x = torch.tensor([1.0 + 0.75 * ulp, -(1.0 + 0.75 * ulp), 1.0 + 0.5 * ulp, -(1.0 + 0.5 * ulp), 1.0 + 0.25 * ulp,
                      3.0, 0.0, 1.0 + ulp], dtype=torch.float32)
    assert cut_tf32(x).tolist() == [1.0, -1.0, 1.0, -1.0, 1.0, 3.0, 0.0, 1.0 + ulp]
    assert round_tf32(x).tolist() == [1.0 + ulp, -(1.0 + ulp), 1.0 + ulp, -(1.0 + ulp), 1.0, 3.0, 0.0, 1.0 + ulp]
    g = torch.Generator().manual_seed(3)
    y = torch.randn(10000, generator=g)
    for f in (cut_tf32, round_tf32):
        z = f(y)
        assert ((z.view(torch.int32) & 0x1FFF) == 0).all()
        assert ((z - y).abs() <= y.abs() * 2.0 ** -10).all()
    assert ((round_tf32(y) - y).abs() <= y.abs() * 2.0 ** -11 * (1 + 1e-6)).all()
    # float64 input: the fp32 value is converted, the result comes back in float64
    assert cut_tf32(y.double()).dtype == torch.float64
    assert torch.equal(cut_tf32(y.double()).float(), cut_tf32(y))


def test_tf32_emulation_identity_and_cut():
    """Tf32Emulation(None) reproduces plain torch through the same autograd
    functions; with every pass on the tensor cores the forward and both
    gradients equal the plain ops applied to cut operands."""
    from oracle.tf32 import Paths, Tf32Emulation, cut_tf32

    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 8, 9, 9, generator=g, dtype=torch.float64)
    w = torch.randn(6, 8, 3, 3, generator=g, dtype=torch.float64)
    b = torch.randn(6, generator=g, dtype=torch.float64)
    dy = torch.randn(2, 6, 5, 5, generator=g, dtype=torch.float64)

    def run(paths):
        xr, wr, br = (t.clone().requires_grad_() for t in (x, w, b))
        with Tf32Emulation(paths):
            y = F.conv2d(xr, wr, br, 2, 1)
        y.backward(dy)
        return y.detach(), xr.grad, wr.grad, br.grad

    plain = F.conv2d(x, w, b, 2, 1)
    y0, gx0, gw0, gb0 = run(None)
    assert torch.equal(y0, plain)
    allp = Paths(conv=lambda *a: True, linear=lambda *a: True, attention=lambda d: True)
    y1, gx1, gw1, gb1 = run(allp)
    assert torch.allclose(y1, F.conv2d(cut_tf32(x), cut_tf32(w), b, 2, 1), rtol=1e-12, atol=1e-12)
    assert torch.allclose(gx1, torch.nn.grad.conv2d_input(x.shape, cut_tf32(w), cut_tf32(dy), 2, 1), rtol=1e-12,
                          atol=1e-12)
    assert torch.allclose(gw1, torch.nn.grad.conv2d_weight(cut_tf32(x), w.shape, cut_tf32(dy), 2, 1), rtol=1e-12,
                          atol=1e-12)
    assert torch.equal(gb1, dy.sum((0, 2, 3)))
    assert not torch.equal(y1, y0)
    # linear: y = x W^T + b, dX = dY W, dW = dY^T X, each with cut operands
    xl = torch.randn(3, 5, 16, generator=g, dtype=torch.float64, requires_grad=True)
    wl = torch.randn(7, 16, generator=g, dtype=torch.float64, requires_grad=True)
    with Tf32Emulation(allp):
        yl = F.linear(xl, wl)
    dyl = torch.randn(3, 5, 7, generator=g, dtype=torch.float64)
    yl.backward(dyl)
    assert torch.allclose(yl, cut_tf32(xl) @ cut_tf32(wl).t(), rtol=1e-12, atol=1e-12)
    assert torch.allclose(xl.grad, cut_tf32(dyl) @ cut_tf32(wl), rtol=1e-12, atol=1e-12)
    assert torch.allclose(wl.grad, cut_tf32(dyl).reshape(-1, 7).t() @ cut_tf32(xl).reshape(-1, 16), rtol=1e-12,
                          atol=1e-12)


def test_tf32_emulated_attention_matches_torch_without_rounding():
    """The emulated attention (exact branch) is softmax(q k^T s) v with its
    gradients; the rounded branch stays within the TF32 rounding of it."""
    from oracle.tf32 import Paths, Tf32Emulation

    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(2, 3, 11, 8, generator=g, dtype=torch.float64) for _ in range(3))
    do = torch.randn(2, 3, 11, 8, generator=g, dtype=torch.float64)
    out = []
    for paths in (None, Paths(conv=None, linear=None, attention=lambda d: True)):
        qr, kr, vr = (t.clone().requires_grad_() for t in (q, k, v))
        with Tf32Emulation(paths):
            o = F.scaled_dot_product_attention(qr, kr, vr)
        o.backward(do)
        out.append((o.detach(), qr.grad, kr.grad, vr.grad))
    qr, kr, vr = (t.clone().requires_grad_() for t in (q, k, v))
    ref = torch.softmax(qr @ kr.transpose(-1, -2) / 8 ** 0.5, -1) @ vr
    ref.backward(do)
    for a, b in zip(out[0], (ref.detach(), qr.grad, kr.grad, vr.grad)):
        assert torch.allclose(a, b, rtol=1e-10, atol=1e-10)
    for a, b in zip(out[1], out[0]):
        assert (a - b).norm() <= 2e-3 * b.norm()


def test_ppm_fixture():
    """The reference's validation images (tests/golden/ppm_samples.pt) are the
    raw RGB bytes of tests/samples/*.ppm; where the reference tree is present
    the fixture is re-read from it and compared byte for byte."""
    import importlib.util

    d = torch.load(os.path.join(GOLDEN, "ppm_samples.pt"))
    assert d["images"].shape == (4, 224, 224, 3) and d["images"].dtype == torch.uint8
    assert d["labels"].tolist() == [281, 207, 87, 1]
    assert d["names"] == ["cat", "dog", "parrot", "goldfish"]
    ref = "/root/reference/tests/samples"
    if os.path.isdir(ref):
        spec = importlib.util.spec_from_file_location("mkppm", os.path.join(GOLDEN, "make_ppm_fixture.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        for i, n in enumerate(d["names"]):
            assert torch.equal(mod.read_ppm(os.path.join(ref, n + ".ppm")), d["images"][i]), n
