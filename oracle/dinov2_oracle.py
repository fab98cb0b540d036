"""CPU restatement of DINOv2 backbone self-attention with the packed QKV Linear.

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA kernels in
``vision_rs_b200``; only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU legs may import it.

The reference (spinorml/vision-rs) has no DINOv2 code (a tree-wide search
finds no dinov2 / windowed-attention source), so there is no reference
implementation, fixture or test to pin against: parity is unpinned by the
reference.  This module restates the published operator — ViT multi-head
self-attention as used by DINOv2 (Dosovitskiy et al., ICLR 2021; Oquab et al.,
"DINOv2", 2023):

    qkv = x · W_qkvᵀ + b            W_qkv [3·hidden, hidden] (nn.Linear layout)
    q, k, v = qkv split into 3 sections of `hidden` features, each split into
              `heads` heads of 64 features (head-major inside a section)
    O_h = softmax(q_h · k_hᵀ / √64) · v_h,    O = concat_h O_h   [n, hidden]

over independent sequences (global layers: one image = 1 cls + H·W patches;
windowed layers: one window).  Windowed layers partition the patch grid into
win×win windows and prepend the cls token to every window (1 + win² tokens);
un-partitioning restores raster patch order and averages the windows' cls
outputs — the cls handling this repository chose (BASELINE leaves it open).

``dinov2_attention`` computes in float64; ``dinov2_attention_torch`` is the
same operator through ``torch.nn.functional.scaled_dot_product_attention``
(an independent formulation used to cross-check the restatement, and the
timed CPU baseline).
"""
from __future__ import annotations

import numpy as np

HEAD_DIM = 64


def qkv_linear(x, w, b):
    """x [..., hidden], w [3·hidden, hidden], b [3·hidden] → [..., 3·hidden] (float64)."""
    return np.asarray(x, np.float64) @ np.asarray(w, np.float64).T + np.asarray(b, np.float64)


def dinov2_attention(x, w, b, heads):
    """x [S, n, hidden] → O [S, n, hidden] (float64)."""
    x = np.asarray(x, np.float64)
    S, n, hidden = x.shape
    assert heads * HEAD_DIM == hidden
    qkv = qkv_linear(x, w, b).reshape(S, n, 3, heads, HEAD_DIM).transpose(2, 0, 3, 1, 4)  # [3,S,h,n,64]
    q, k, v = qkv[0], qkv[1], qkv[2]
    s = q @ k.transpose(0, 1, 3, 2) / np.sqrt(HEAD_DIM)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = p @ v                                                                  # [S,h,n,64]
    return o.transpose(0, 2, 1, 3).reshape(S, n, hidden)


def window_partition(x, gh, gw, win):
    """x [B, 1 + gh·gw, C] → [B·nw, 1 + win², C]; window w = wy·(gw/win) + wx,
    cls copied to token 0 of every window, patches row-major inside a window."""
    x = np.asarray(x)
    B, ntok, C = x.shape
    assert ntok == 1 + gh * gw and gh % win == 0 and gw % win == 0
    nwy, nwx = gh // win, gw // win
    p = x[:, 1:].reshape(B, nwy, win, nwx, win, C).transpose(0, 1, 3, 2, 4, 5).reshape(B * nwy * nwx, win * win, C)
    cls = np.repeat(x[:, :1], nwy * nwx, axis=0)
    return np.concatenate([cls, p], axis=1)


def window_unpartition(xw, B, gh, gw, win):
    """Inverse of ``window_partition``; the cls output is the mean over windows."""
    xw = np.asarray(xw)
    nwy, nwx = gh // win, gw // win
    C = xw.shape[-1]
    xw = xw.reshape(B, nwy * nwx, 1 + win * win, C)
    cls = xw[:, :, 0].astype(np.float64).mean(axis=1, keepdims=True)
    p = xw[:, :, 1:].reshape(B, nwy, nwx, win, win, C).transpose(0, 1, 3, 2, 4, 5).reshape(B, gh * gw, C)
    return np.concatenate([cls, p.astype(np.float64)], axis=1)


def dinov2_attention_torch(x, w, b, heads):
    """torch tensors x [S, n, hidden], w, b → O [S, n, hidden] via SDPA (CPU)."""
    import torch
    import torch.nn.functional as Fn
    S, n, hidden = x.shape
    qkv = (x @ w.T + b).reshape(S, n, 3, heads, HEAD_DIM).permute(2, 0, 3, 1, 4)
    o = Fn.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2])
    return o.transpose(1, 2).reshape(S, n, hidden)


def dinov2_synthetic(S=2, n=1601, hidden=384, seed=0):
    """Seeded inputs with cfg4's distributions: activations N(0,1), weights
    N(0, 0.02), biases N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((S, n, hidden)).astype(np.float32)
    w = (rng.standard_normal((3 * hidden, hidden)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(3 * hidden) * 0.02).astype(np.float32)
    return x, w, b
