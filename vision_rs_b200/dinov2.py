"""DINOv2 backbone attention (packed QKV Linear + multi-head attention, head
dim 64) on the B200 kernels, over the C ABI (``va_dinov2_*``).

``DinoV2Attention`` is the attention of one backbone layer without its output
projection: ``x [S, n, hidden]`` bf16 → ``O [S, n, hidden]`` bf16 with
``O = concat_h softmax(q_h k_hᵀ / 8) v_h`` and ``qkv = x W_qkvᵀ + b``.  Global
layers pass whole images (S = images, n = 1 + H·W); windowed layers pass
windows from ``window_partition`` (S = images·windows, n = 1 + win², the cls
token copied into every window).  No CPU path.
"""
from __future__ import annotations

import torch

from . import _lib
from .psa import _p, _stream


def _check(t, dtype, name):
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor")


def dinov2_attention_workspace_bytes(num_seqs: int, seq_len: int, hidden: int) -> int:
    return int(_lib.lib().va_dinov2_attention_workspace_bytes(num_seqs, seq_len, hidden))


def qkv_linear(x, w_qkv, b_qkv, out=None, stream=None):
    """Packed QKV Linear: ``[..., hidden] → [..., 3·hidden]`` bf16 (f32 bias)."""
    _check(x, torch.bfloat16, "x")
    _check(w_qkv, torch.bfloat16, "w_qkv")
    _check(b_qkv, torch.float32, "b_qkv")
    hidden = x.shape[-1]
    tokens = x.numel() // hidden
    if out is None:
        out = torch.empty(*x.shape[:-1], 3 * hidden, device=x.device, dtype=torch.bfloat16)
    _lib.call("va_dinov2_qkv_linear_bf16", _p(x), _p(w_qkv), _p(b_qkv), _p(out), tokens, hidden, _stream(stream))
    return out


def window_partition(x, grid_h: int, grid_w: int, win: int, out=None, stream=None):
    """``[B, 1 + gh·gw, C] → [B·nw, 1 + win², C]`` (cls copied into every window)."""
    _check(x, torch.bfloat16, "x")
    B, _, C = x.shape
    nw = (grid_h // win) * (grid_w // win)
    if out is None:
        out = torch.empty(B * nw, 1 + win * win, C, device=x.device, dtype=x.dtype)
    _lib.call("va_dinov2_window_partition_bf16", _p(x), _p(out), B, grid_h, grid_w, win, C, _stream(stream))
    return out


def window_unpartition(xw, B: int, grid_h: int, grid_w: int, win: int, out=None, stream=None):
    """Inverse of ``window_partition``; the cls output is the mean over the windows."""
    _check(xw, torch.bfloat16, "xw")
    C = xw.shape[-1]
    if out is None:
        out = torch.empty(B, 1 + grid_h * grid_w, C, device=xw.device, dtype=xw.dtype)
    _lib.call("va_dinov2_window_unpartition_bf16", _p(xw), _p(out), B, grid_h, grid_w, win, C, _stream(stream))
    return out


class DinoV2Attention:
    """Attention of one DINOv2 layer (bf16 weights ``[3·hidden, hidden]``, f32 bias)."""

    def __init__(self, w_qkv, b_qkv, num_heads: int):
        _check(w_qkv, torch.bfloat16, "w_qkv")
        _check(b_qkv, torch.float32, "b_qkv")
        self.w_qkv, self.b_qkv, self.num_heads = w_qkv, b_qkv, num_heads
        self.hidden = w_qkv.shape[1]
        self._ws = None

    def workspace_bytes(self, num_seqs: int, seq_len: int) -> int:
        return dinov2_attention_workspace_bytes(num_seqs, seq_len, self.hidden)

    def forward_into(self, x, out, stream=None):
        _check(x, torch.bfloat16, "x")
        S, n, hidden = x.shape
        need = self.workspace_bytes(S, n)
        if self._ws is None or self._ws.numel() < need or self._ws.device != x.device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        _lib.call("va_dinov2_attention_fwd_bf16", _p(x), _p(self.w_qkv), _p(self.b_qkv), _p(out), S, n, hidden,
                  self.num_heads, _p(self._ws), self._ws.numel(), _stream(stream))
        return out

    def __call__(self, x, stream=None):
        out = torch.empty_like(x)
        return self.forward_into(x, out, stream)
