"""CPU restatement of multi-scale deformable attention (MSDeformAttn).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA kernels in
``vision_rs_b200``; only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU legs may import it.

The reference (spinorml/vision-rs) has no deformable attention: a tree-wide
search finds no MSDeformAttn, RF-DETR or Deformable-DETR code, so there is no
reference implementation, fixture or test to pin against.  This module
restates the published operator (Zhu et al., "Deformable DETR", ICLR 2021,
eq. 3 — the multi-scale deformable attention core) as ``north_star`` defines
it for RF-DETR's decoder:

    out[b, q, h, :] = Σ_l Σ_p A[b,q,h,l,p] · bilinear(V_l[b, :, :, h, :],
                                                     x = loc_x·W_l − 0.5,
                                                     y = loc_y·H_l − 0.5)

with ``V_l`` the level-l slice of ``value[b, S, nh, dh]`` (rows
``level_start[l] .. +H_l·W_l``, row-major H×W), bilinear interpolation with
zero padding outside the map (PyTorch ``grid_sample(align_corners=False,
padding_mode='zeros')`` semantics), A softmaxed over L·P by the caller.

``msdeform_attn_forward`` / ``msdeform_attn_backward`` compute in float64.
``msdeform_attn_torch`` is the same operator composed from torch-CPU
``grid_sample`` per level — an independent formulation used to cross-check
the numpy restatement and its hand-derived backward (autograd), and as the
timed CPU baseline.
"""
from __future__ import annotations

import numpy as np


def _bilinear_corners(lx, ly, H, W):
    """Corner indices and weights of the align_corners=False sample at
    normalised (lx, ly): pixel coords x = lx·W − 0.5, y = ly·H − 0.5."""
    x = lx * W - 0.5
    y = ly * H - 0.5
    x0 = np.floor(x)
    y0 = np.floor(y)
    fx = x - x0
    fy = y - y0
    x0 = x0.astype(np.int64)
    y0 = y0.astype(np.int64)
    out = []
    for dy, wy in ((0, 1 - fy), (1, fy)):
        for dx, wx in ((0, 1 - fx), (1, fx)):
            xi, yi = x0 + dx, y0 + dy
            valid = (xi >= 0) & (xi < W) & (yi >= 0) & (yi < H)
            out.append((yi, xi, wy * wx, valid, dx, dy))
    return out, fx, fy


def msdeform_attn_forward(value, spatial_shapes, level_start, loc, attn):
    """value [B,S,nh,dh], spatial_shapes [L,2] (H,W), level_start [L],
    loc [B,Q,nh,L,P,2] (x,y in [0,1]), attn [B,Q,nh,L,P] → out [B,Q,nh*dh]."""
    value = np.asarray(value, np.float64)
    loc = np.asarray(loc, np.float64)
    attn = np.asarray(attn, np.float64)
    B, S, nh, dh = value.shape
    _, Q, _, L, P, _ = loc.shape
    out = np.zeros((B, Q, nh, dh))
    bidx = np.arange(B)[:, None, None, None]
    hidx = np.arange(nh)[None, None, :, None]
    for l in range(L):
        H, W = int(spatial_shapes[l][0]), int(spatial_shapes[l][1])
        s0 = int(level_start[l])
        corners, _, _ = _bilinear_corners(loc[:, :, :, l, :, 0], loc[:, :, :, l, :, 1], H, W)
        for yi, xi, w, valid, _, _ in corners:
            pix = np.where(valid, yi * W + xi, 0) + s0                     # [B,Q,nh,P]
            v = value[bidx, pix, hidx, :]                                  # [B,Q,nh,P,dh]
            coef = (attn[:, :, :, l, :] * w * valid)[..., None]
            out += (coef * v).sum(axis=3)
    return out.reshape(B, Q, nh * dh)


def msdeform_attn_backward(value, spatial_shapes, level_start, loc, attn, grad_out):
    """Gradients of ``msdeform_attn_forward``: (grad_value, grad_loc, grad_attn)."""
    value = np.asarray(value, np.float64)
    loc = np.asarray(loc, np.float64)
    attn = np.asarray(attn, np.float64)
    B, S, nh, dh = value.shape
    _, Q, _, L, P, _ = loc.shape
    go = np.asarray(grad_out, np.float64).reshape(B, Q, nh, dh)
    gv = np.zeros_like(value)
    gloc = np.zeros_like(loc)
    gattn = np.zeros_like(attn)
    bidx = np.arange(B)[:, None, None, None]
    hidx = np.arange(nh)[None, None, :, None]
    for l in range(L):
        H, W = int(spatial_shapes[l][0]), int(spatial_shapes[l][1])
        s0 = int(level_start[l])
        lx, ly = loc[:, :, :, l, :, 0], loc[:, :, :, l, :, 1]
        corners, fx, fy = _bilinear_corners(lx, ly, H, W)
        a = attn[:, :, :, l, :]
        samp = np.zeros(lx.shape + (dh,))
        gx = np.zeros(lx.shape)
        gy = np.zeros(lx.shape)
        for yi, xi, w, valid, dx, dy in corners:
            pix = np.where(valid, yi * W + xi, 0) + s0
            v = value[bidx, pix, hidx, :] * valid[..., None]               # [B,Q,nh,P,dh]
            samp += w[..., None] * v
            # d w / d fx, d w / d fy for this corner
            dwx = (fy if dy else 1 - fy) * (1 if dx else -1)
            dwy = (fx if dx else 1 - fx) * (1 if dy else -1)
            g_dot_v = (go[:, :, :, None, :] * v).sum(-1)                   # [B,Q,nh,P]
            gx += dwx * g_dot_v
            gy += dwy * g_dot_v
            contrib = (a * w * valid)[..., None] * go[:, :, :, None, :]   # [B,Q,nh,P,dh]
            np.add.at(gv, (np.broadcast_to(bidx, pix.shape), pix, np.broadcast_to(hidx, pix.shape)), contrib)
        gattn[:, :, :, l, :] = (go[:, :, :, None, :] * samp).sum(-1)
        gloc[:, :, :, l, :, 0] = a * gx * W
        gloc[:, :, :, l, :, 1] = a * gy * H
    return gv, gloc, gattn


def msdeform_attn_torch(value, spatial_shapes, level_start, loc, attn):
    """The same operator composed from torch-CPU ``grid_sample`` per level
    (autograd-differentiable); takes and returns torch tensors."""
    import torch
    import torch.nn.functional as Fn
    B, S, nh, dh = value.shape
    _, Q, _, L, P, _ = loc.shape
    outs = []
    for l in range(L):
        H, W = int(spatial_shapes[l][0]), int(spatial_shapes[l][1])
        s0 = int(level_start[l])
        v = value[:, s0:s0 + H * W].reshape(B, H, W, nh, dh).permute(0, 3, 4, 1, 2).reshape(B * nh, dh, H, W)
        grid = loc[:, :, :, l].permute(0, 2, 1, 3, 4).reshape(B * nh, Q, P, 2) * 2 - 1
        samp = Fn.grid_sample(v, grid, mode="bilinear", padding_mode="zeros", align_corners=False)  # [B*nh,dh,Q,P]
        outs.append(samp)
    samp = torch.stack(outs, dim=-2)                                       # [B*nh,dh,Q,L,P]
    a = attn.permute(0, 2, 1, 3, 4).reshape(B * nh, 1, Q, L, P)
    out = (samp * a).sum(dim=(-1, -2))                                     # [B*nh,dh,Q]
    return out.reshape(B, nh, dh, Q).permute(0, 3, 1, 2).reshape(B, Q, nh * dh)


def msdeform_synthetic(B=8, Q=300, nh=16, dh=16, shapes=((80, 80), (40, 40), (20, 20)), P=4, seed=0):
    """Seeded inputs with cfg3's distributions: value N(0,1), reference points
    U(0,1), offsets N(0,2) pixels, attention logits N(0,1) softmaxed over L·P."""
    rng = np.random.default_rng(seed)
    L = len(shapes)
    shapes = np.asarray(shapes, np.int64)
    S = int((shapes[:, 0] * shapes[:, 1]).sum())
    level_start = np.concatenate([[0], np.cumsum(shapes[:, 0] * shapes[:, 1])[:-1]]).astype(np.int64)
    value = rng.standard_normal((B, S, nh, dh)).astype(np.float32)
    ref = rng.uniform(0, 1, (B, Q, 1, 1, 1, 2))
    off = rng.standard_normal((B, Q, nh, L, P, 2)) * 2.0
    wh = np.stack([shapes[:, 1], shapes[:, 0]], -1).astype(np.float64)     # (W, H) per level
    loc = (ref + off / wh[None, None, None, :, None, :]).astype(np.float32)
    logits = rng.standard_normal((B, Q, nh, L * P))
    a = np.exp(logits - logits.max(-1, keepdims=True))
    attn = (a / a.sum(-1, keepdims=True)).reshape(B, Q, nh, L, P).astype(np.float32)
    grad_out = rng.standard_normal((B, Q, nh * dh)).astype(np.float32)
    return dict(value=value, spatial_shapes=shapes, level_start=level_start, loc=loc, attn=attn, grad_out=grad_out)
