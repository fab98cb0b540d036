"""CPU restatement of the reference's YOLO26 convolution blocks — TEST
INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker; the library never
calls it.

What it restates (float64 numpy, NCHW, groups = 1):

* ``conv2d``      — Conv2d(k, s, padding k/2, bias=False) as in
  ``src/models/yolo/yolo26/blocks/conv.rs:31-46`` (``conv``) and ``:53-69``
  (``conv_bn``): y[b,o,oy,ox] = Σ_{c,ky,kx} w[o,c,ky,kx]·x[b,c,s·oy+ky−p,s·ox+kx−p]
  with zero padding p = k/2.
* ``conv_block``  — ``conv`` (Conv2d → BN → SiLU) with BN in eval mode
  (running statistics), or without SiLU for ``conv_bn``.
* ``conv_block_train`` — the same with BN in training mode (biased batch
  variance over B·H·W), which is how the reference's stem fixture
  ``tests/fixtures/conv_yolo26/generate.py:36-47`` was produced.
* ``bottleneck``  — ``bottleneck_std`` (3×3 c→c/2, 3×3 c/2→c,
  ``bottleneck.rs:37-47``) and ``bottleneck_3x3`` (3×3 c→c twice,
  ``bottleneck.rs:53-63``), with the residual add when ``shortcut``.
* ``c3k``         — ``c3k_inner`` (``c3k2.rs:46-61``): cv3(cat(m1(m0(cv1(x))), cv2(x))).
* ``c3k2``        — ``c3k2.rs:94-127``: h = cv1(x); [y0, y1] = chunk(h, 2);
  parts += b(last) per inner block; cv2(cat(parts)).

Parity pin: ``tests/test_oracle_golden.py`` runs these on the reference's
fixtures (``conv_yolo26`` stem, ``c3k2_yolo26`` variants) copied into
``tests/golden/`` and matches their expected outputs to ≤ 1e-5.
"""
from __future__ import annotations

import numpy as np


def _f64(a):
    return np.asarray(a, dtype=np.float64)


def conv2d(x, w, stride: int = 1, bias=None):
    """Conv2d with padding k/2, groups = 1 (conv.rs:36-38)."""
    x, w = _f64(x), _f64(w)
    B, C, H, W = x.shape
    O, Ci, k, k2 = w.shape
    assert Ci == C and k == k2
    p = k // 2
    Ho, Wo = (H + 2 * p - k) // stride + 1, (W + 2 * p - k) // stride + 1
    xp = np.zeros((B, C, H + 2 * p, W + 2 * p))
    xp[:, :, p:p + H, p:p + W] = x
    y = np.zeros((B, O, Ho, Wo))
    for ky in range(k):
        for kx in range(k):
            patch = xp[:, :, ky:ky + stride * (Ho - 1) + 1:stride, kx:kx + stride * (Wo - 1) + 1:stride]
            y += np.einsum("bchw,oc->bohw", patch, w[:, :, ky, kx])
    if bias is not None:
        y += _f64(bias)[None, :, None, None]
    return y


def silu(x):
    x = _f64(x)
    return x / (1.0 + np.exp(-x))


def fold_bn(w, gamma, beta, mean, var, eps):
    """(w·s, β − μ·s) with s = γ/√(var + eps): BN folded into the conv."""
    s = _f64(gamma) / np.sqrt(_f64(var) + eps)
    return _f64(w) * s.reshape(-1, *([1] * (np.ndim(w) - 1))), _f64(beta) - _f64(mean) * s


def conv_block(x, prm, stride: int = 1, eps: float = 1e-5, act: bool = True):
    """``conv`` / ``conv_bn`` with BN in eval mode; prm = (w, γ, β, μ, σ²)."""
    w, b = fold_bn(*prm, eps)
    y = conv2d(x, w, stride, b)
    return silu(y) if act else y


def conv_block_train(x, prm, stride: int = 1, eps: float = 1e-5, act: bool = True):
    """``conv`` with BN in training mode: batch mean and biased variance over
    (B, H, W) replace the running statistics."""
    w, gamma, beta = prm[0], prm[1], prm[2]
    y = conv2d(x, w, stride)
    mu = y.mean(axis=(0, 2, 3), keepdims=True)
    var = y.var(axis=(0, 2, 3), keepdims=True)
    y = (y - mu) / np.sqrt(var + eps) * _f64(gamma)[None, :, None, None] + _f64(beta)[None, :, None, None]
    return silu(y) if act else y


def bottleneck(x, prm: dict, prefix: str, shortcut: bool, eps: float = 1e-5):
    """Two 3×3 ``conv`` blocks ``{prefix}cv1``, ``{prefix}cv2`` (+ x)."""
    y = conv_block(conv_block(x, prm[prefix + "cv1"], 1, eps), prm[prefix + "cv2"], 1, eps)
    return _f64(x) + y if shortcut else y


def c3k(x, prm: dict, prefix: str, shortcut: bool, eps: float = 1e-5):
    """C3k(c, c, n=2, e=0.5): the fixture names its convs {prefix}icv1/2/3
    and its bottlenecks {prefix}m0_, {prefix}m1_."""
    a = conv_block(x, prm[prefix + "icv1"], 1, eps)
    a = bottleneck(a, prm, prefix + "m0_", shortcut, eps)
    a = bottleneck(a, prm, prefix + "m1_", shortcut, eps)
    b = conv_block(x, prm[prefix + "icv2"], 1, eps)
    return conv_block(np.concatenate([a, b], axis=1), prm[prefix + "icv3"], 1, eps)


def c3k2(x, prm: dict, c3k_inner: bool, shortcut: bool, eps: float = 1e-5):
    """C3k2 with n = 1 (the fixtures' case): prm maps stage names (cv1, cv2,
    m0_cv1, … or m0_icv1, …) to (w, γ, β, μ, σ²)."""
    h = conv_block(x, prm["cv1"], 1, eps)
    c = h.shape[1] // 2
    y0, y1 = h[:, :c], h[:, c:]
    last = c3k(y1, prm, "m0_", shortcut, eps) if c3k_inner else bottleneck(y1, prm, "m0_", shortcut, eps)
    return conv_block(np.concatenate([y0, y1, last], axis=1), prm["cv2"], 1, eps)


def conv_synthetic(B, Cin, H, W, Cout, k, seed=0):
    """Seeded input, weight and BN-folded bias for a conv test case."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, Cin, H, W))
    w = rng.standard_normal((Cout, Cin, k, k)) / np.sqrt(Cin * k * k)
    b = rng.standard_normal(Cout) * 0.1
    return x, w, b
