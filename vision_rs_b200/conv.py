"""The reference's YOLO26 convolution blocks as NHWC bf16 ops.

``conv(c_in, c_out, k, s)`` (Conv2d → BN(eps 1e-3) → SiLU) and
``conv_bn(c_in, c_out, k, s, 1)`` (Conv2d → BN) of
``src/models/yolo/yolo26/blocks/conv.rs:31-69`` become one
``va_conv_nhwc_bf16`` launch each: BN folded into the weights and a bias,
the implicit GEMM on the tensor cores, SiLU and the bf16 rounding in the
epilogue.  Activations are NHWC ([B, H, W, C]) bf16 tensors; weights are
kept on the device in OHWI order.

There is no CPU path: every call goes through the C ABI and raises if the
library is missing or refuses the arguments.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .psa import _p, _stream


def out_size(h: int, k: int, s: int) -> int:
    """Output extent for padding k/2 (conv.rs:37)."""
    return (h + 2 * (k // 2) - k) // s + 1


def conv_nhwc(x: torch.Tensor, w_ohwi: torch.Tensor, bias: torch.Tensor, stride: int = 1, act: bool = True,
              out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """y = act(conv(x, w) + bias); x [B, H, W, Cin] bf16, w [Cout, k, k, Cin]
    bf16, bias [Cout] f32 → y [B, Ho, Wo, Cout] bf16."""
    B, H, W, Cin = x.shape
    Cout, k, k2, Ci = w_ohwi.shape
    if Ci != Cin or k != k2:
        raise ValueError(f"weight {tuple(w_ohwi.shape)} does not match input channels {Cin}")
    Ho, Wo = out_size(H, k, stride), out_size(W, k, stride)
    if out is None:
        out = torch.empty(B, Ho, Wo, Cout, dtype=torch.bfloat16, device=x.device)
    _lib.call("va_conv_nhwc_bf16", _p(x), _p(w_ohwi), _p(bias), _p(out), B, H, W, Cin, Cout, k, stride,
              1 if act else 0, _stream(stream))
    return out


def weight_ohwi(w_oihw: torch.Tensor, stream=None) -> torch.Tensor:
    """OIHW bf16 (the reference's Conv2d weight layout) → OHWI on the device."""
    Cout, Cin, k, _ = w_oihw.shape
    out = torch.empty(Cout, k, k, Cin, dtype=torch.bfloat16, device=w_oihw.device)
    _lib.call("va_conv_weight_ohwi_bf16", _p(w_oihw), _p(out), Cout, Cin, k, _stream(stream))
    return out


class ConvBnAct:
    """One ``conv`` / ``conv_bn`` block with BN already folded: w [Cout, Cin,
    k, k] and b [Cout] (f32, host or device), stride s, SiLU when ``act``."""

    def __init__(self, w, b, stride: int = 1, act: bool = True, device="cuda"):
        w = torch.as_tensor(np.asarray(w, np.float32) if not torch.is_tensor(w) else w)
        self.w = weight_ohwi(w.to(device, torch.bfloat16).contiguous())
        self.b = torch.as_tensor(np.asarray(b, np.float32) if not torch.is_tensor(b) else b).to(
            device, torch.float32).contiguous()
        self.stride, self.act = stride, act
        self.c_out, self.k, _, self.c_in = self.w.shape

    @classmethod
    def from_safetensors(cls, st, prefix: str, stride: int = 1, act: bool = True, eps: float = 1e-3,
                         device="cuda"):
        """Folded from ``{prefix}.conv.weight`` + ``{prefix}.bn.*`` of an open
        :class:`vision_rs_b200.weights.SafeTensors` (eps 1e-3, conv.rs:39,64)."""
        w, b = st.fold_conv_bn(prefix, eps)
        return cls(w, b, stride, act, device)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        return conv_nhwc(x, self.w, self.b, self.stride, self.act, out, stream)
