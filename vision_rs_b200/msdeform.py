"""Multi-scale deformable attention (RF-DETR decoder) on the B200 kernels.

``MSDeformAttnFunction.apply``-style functional API over the C ABI
(``va_msdeform_attn_*``): value ``[B,S,nh,dh]``, spatial_shapes ``[L,2]``,
level_start ``[L]`` (int64, on the device), sampling_locations
``[B,Q,nh,L,P,2]``, attention_weights ``[B,Q,nh,L,P]`` → ``[B,Q,nh*dh]``.
f32 or bf16 value; locations and weights f32.  No CPU path.
"""
from __future__ import annotations

import torch

from . import _lib
from .psa import _p, _sfx, _stream


def _dims(value, loc):
    B, S, nh, dh = value.shape
    _, Q, _, L, P, _ = loc.shape
    return B, S, nh, dh, L, Q, P


def msdeform_attn_forward(value, spatial_shapes, level_start, loc, attn, out=None, stream=None):
    B, S, nh, dh, L, Q, P = _dims(value, loc)
    if out is None:
        out = torch.empty(B, Q, nh * dh, device=value.device, dtype=value.dtype)
    _lib.call(f"va_msdeform_attn_fwd_{_sfx(value)}", _p(value), _p(spatial_shapes), _p(level_start), _p(loc),
              _p(attn), _p(out), B, S, nh, dh, L, Q, P, _stream(stream))
    return out


def msdeform_attn_workspace_bytes(B, nh, L, Q, P) -> int:
    return int(_lib.lib().va_msdeform_attn_bwd_workspace_bytes(B, nh, L, Q, P))


def msdeform_attn_backward(value, spatial_shapes, level_start, loc, attn, grad_out, workspace=None, stream=None,
                           out=None):
    """Returns ``(grad_value, grad_loc, grad_attn)`` (deterministic, no atomics);
    ``out`` may supply those three tensors."""
    B, S, nh, dh, L, Q, P = _dims(value, loc)
    need = msdeform_attn_workspace_bytes(B, nh, L, Q, P)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=value.device)
    if out is not None:
        gv, gl, ga = out
    else:
        gv = torch.empty_like(value)
        gl = torch.empty_like(loc)
        ga = torch.empty_like(attn)
    _lib.call(f"va_msdeform_attn_bwd_{_sfx(value)}", _p(value), _p(spatial_shapes), _p(level_start), _p(loc),
              _p(attn), _p(grad_out), _p(gv), _p(gl), _p(ga), B, S, nh, dh, L, Q, P, _p(workspace),
              workspace.numel(), _stream(stream))
    return gv, gl, ga
