"""Independent numpy restatements of the hot-path semantics (test infrastructure only).

Each function states, in float64 numpy, what the device kernel must compute,
following the reference's op glue and torch-CPU (the reference's arbiter).
They are cross-checked against torch-CPU in the CPU test suite and used as a
second, torch-free check of the device results on small inputs.
"""
from __future__ import annotations

import math

import numpy as np


def batch_norm_train(x, gamma, beta, running_mean, running_var, momentum, eps):
    """native_batch_norm in training mode (src/norm_ops.cpp:19-84): batch statistics
    over (N, H, W) per channel; normalise with the biased variance; update the running
    variance with the unbiased one (M/(M-1), norm_ops.cpp:64-69).
    Returns y, mean, invstd, new_running_mean, new_running_var."""
    x = np.asarray(x, np.float64)
    axes = (0,) + tuple(range(2, x.ndim))
    m = x.size // x.shape[1]
    mean = x.mean(axis=axes)
    var = ((x - mean.reshape((1, -1) + (1,) * (x.ndim - 2))) ** 2).mean(axis=axes)
    invstd = 1.0 / np.sqrt(var + eps)
    shp = (1, -1) + (1,) * (x.ndim - 2)
    y = (x - mean.reshape(shp)) * invstd.reshape(shp)
    if gamma is not None:
        y = y * np.asarray(gamma, np.float64).reshape(shp)
    if beta is not None:
        y = y + np.asarray(beta, np.float64).reshape(shp)
    rm = rv = None
    if running_mean is not None:
        rm = (1 - momentum) * np.asarray(running_mean, np.float64) + momentum * mean
        rv = (1 - momentum) * np.asarray(running_var, np.float64) + momentum * var * m / max(m - 1, 1)
    return y, mean, invstd, rm, rv


def batch_norm_backward(dy, x, gamma, mean, invstd):
    """native_batch_norm_backward with batch statistics (src/norm_ops.cpp:87-164)."""
    dy = np.asarray(dy, np.float64)
    x = np.asarray(x, np.float64)
    axes = (0,) + tuple(range(2, x.ndim))
    shp = (1, -1) + (1,) * (x.ndim - 2)
    m = x.size // x.shape[1]
    xhat = (x - mean.reshape(shp)) * invstd.reshape(shp)
    dbeta = dy.sum(axis=axes)
    dgamma = (dy * xhat).sum(axis=axes)
    g = np.ones(x.shape[1]) if gamma is None else np.asarray(gamma, np.float64)
    dx = (g * invstd).reshape(shp) * (dy - dbeta.reshape(shp) / m - xhat * dgamma.reshape(shp) / m)
    return dx, dgamma, dbeta


def _pool_out(n, k, s, p, d, ceil_mode):
    o = (n + 2 * p - d * (k - 1) - 1 + (s - 1 if ceil_mode else 0)) // s + 1
    if ceil_mode and (o - 1) * s >= n + p:
        o -= 1
    return o


def max_pool2d(x, k, s, p, d=1, ceil_mode=False):
    """max_pool2d with torch's flat (h*W + w) indices: the first maximum in
    row-major window order wins ties, a NaN always wins (src/vision_ops.cpp:353-410,
    CPU semantics).  x: [N, C, H, W]."""
    x = np.asarray(x)
    N, C, H, W = x.shape
    P, Q = _pool_out(H, k, s, p, d, ceil_mode), _pool_out(W, k, s, p, d, ceil_mode)
    y = np.empty((N, C, P, Q), x.dtype)
    ind = np.empty((N, C, P, Q), np.int64)
    for i in range(P):
        for j in range(Q):
            h0, w0 = i * s - p, j * s - p
            hs = [h for h in range(h0, min(h0 + (k - 1) * d + 1, H), d) if h >= 0]
            ws = [w for w in range(w0, min(w0 + (k - 1) * d + 1, W), d) if w >= 0]
            best = np.full((N, C), -np.inf)
            bi = np.full((N, C), hs[0] * W + ws[0], np.int64)
            for h in hs:
                for w in ws:
                    v = x[:, :, h, w]
                    upd = (v > best) | np.isnan(v)
                    best = np.where(upd, v, best)
                    bi = np.where(upd, h * W + w, bi)
            y[:, :, i, j] = best
            ind[:, :, i, j] = bi
    return y, ind


def max_pool2d_backward(dy, ind, in_shape):
    """Gradient scattered to the recorded argmax positions (summed where windows overlap)."""
    N, C, H, W = in_shape
    dx = np.zeros((N, C, H * W), np.float64)
    dyf = np.asarray(dy, np.float64).reshape(N, C, -1)
    indf = np.asarray(ind).reshape(N, C, -1)
    for n in range(N):
        for c in range(C):
            np.add.at(dx[n, c], indf[n, c], dyf[n, c])
    return dx.reshape(N, C, H, W)


def log_softmax(x, axis=-1):
    """_log_softmax (src/loss_ops.cpp:137-175): x - max - log(sum(exp(x - max)))."""
    x = np.asarray(x, np.float64)
    m = x.max(axis=axis, keepdims=True)
    return x - m - np.log(np.exp(x - m).sum(axis=axis, keepdims=True))


def nll_loss(logp, target, reduction="mean", ignore_index=-100, weight=None):
    """nll_loss_forward (src/loss_ops.cpp:23-44): -sum(w[t] * logp[i, t]) / sum(w[t])."""
    logp = np.asarray(logp, np.float64)
    target = np.asarray(target)
    w = np.ones(logp.shape[1]) if weight is None else np.asarray(weight, np.float64)
    keep = target != ignore_index
    tsafe = np.where(keep, target, 0)
    terms = -logp[np.arange(len(target)), tsafe] * w[tsafe] * keep
    if reduction == "none":
        return terms
    if reduction == "sum":
        return terms.sum()
    return terms.sum() / (w[tsafe] * keep).sum()


def gelu(x, approximate="none"):
    """gelu (src/pointwise_ops.cpp:1324-1357): exact erf form or the tanh approximation."""
    x = np.asarray(x, np.float64)
    if approximate == "tanh":
        return 0.5 * x * (1 + np.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))
    erf = np.vectorize(math.erf)
    return 0.5 * x * (1 + erf(x / math.sqrt(2)))


def hardtanh_backward(grad, x, lo, hi):
    """ReLU6 / hardtanh backward with torch-CPU's exclusive mask lo < x < hi
    (the reference's OpenCL expression used an inclusive mask, pointwise_ops.cpp:600;
    the CPU is the arbiter)."""
    x = np.asarray(x)
    return np.where((x > lo) & (x < hi), grad, 0.0)


def sgd_momentum(p, g, buf, lr, momentum, dampening=0.0, weight_decay=0.0, nesterov=False):
    """torch.optim.SGD update for one tensor; buf None means the first step."""
    p = np.asarray(p, np.float64)
    d = np.asarray(g, np.float64) + weight_decay * p
    if momentum:
        buf = d.copy() if buf is None else momentum * np.asarray(buf, np.float64) + (1 - dampening) * d
        d = d + momentum * buf if nesterov else buf
    return p - lr * d, buf


def conv2d(x, w, b=None, stride=(1, 1), pad=(0, 0), dil=(1, 1), groups=1):
    """Direct 2-D cross-correlation in float64 (convolution_overrideable, src/vision_ops.cpp:61-113)."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    N, C, H, W = x.shape
    K, Cg, R, S = w.shape
    P = (H + 2 * pad[0] - dil[0] * (R - 1) - 1) // stride[0] + 1
    Q = (W + 2 * pad[1] - dil[1] * (S - 1) - 1) // stride[1] + 1
    xp = np.zeros((N, C, H + 2 * pad[0], W + 2 * pad[1]))
    xp[:, :, pad[0]:pad[0] + H, pad[1]:pad[1] + W] = x
    y = np.zeros((N, K, P, Q))
    Kg = K // groups
    for g in range(groups):
        for r in range(R):
            for s in range(S):
                hs = r * dil[0]
                ws = s * dil[1]
                patch = xp[:, g * Cg:(g + 1) * Cg, hs:hs + stride[0] * (P - 1) + 1:stride[0],
                           ws:ws + stride[1] * (Q - 1) + 1:stride[1]]
                y[:, g * Kg:(g + 1) * Kg] += np.einsum("nchw,kc->nkhw", patch, w[g * Kg:(g + 1) * Kg, :, r, s])
    if b is not None:
        y += np.asarray(b, np.float64).reshape(1, -1, 1, 1)
    return y
