"""Checkpoint weights for the PSA / C2PSA ops: safetensors reading and BN
folding through the C ABI (``va_safetensors_*``), and the C2PSA op built
from a checkpoint.

The reference loads YOLO26 checkpoints from safetensors and folds every
conv+BN pair with eps = 1e-3 (examples/yolo26.rs:3403-3470, conv.rs:39,64).
Key names follow the checkpoint's module paths, e.g. for the C2PSA at
``model.10``: ``model.10.cv1``, ``model.10.m.0.attn.qkv``,
``model.10.m.0.attn.pe``, ``model.10.m.0.attn.proj``, ``model.10.m.0.ffn.0``,
``model.10.m.0.ffn.1``, ``model.10.cv2`` — each with ``.conv.weight`` and
``.bn.{weight,bias,running_mean,running_var}``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .psa import _p, _stream

YOLO26_BN_EPS = 1e-3
BLOCK_STAGES = {"qkv": "attn.qkv", "pe": "attn.pe", "proj": "attn.proj", "ffn0": "ffn.0", "ffn1": "ffn.1"}


class SafeTensors:
    """A safetensors file opened by the library's reader (host memory)."""

    def __init__(self, path: str):
        self._h = C.c_void_p()
        _lib.call("va_safetensors_open", str(path).encode(), C.byref(self._h))

    def close(self):
        if self._h:
            _lib.lib().va_safetensors_close(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def info(self, key: str):
        """(dtype code VA_ST_*, shape) of one tensor."""
        dt, rank = C.c_int(), C.c_int()
        shape = (C.c_int64 * 8)()
        _lib.call("va_safetensors_tensor_info", self._h, key.encode(), C.byref(dt), shape, C.byref(rank))
        return dt.value, tuple(shape[i] for i in range(rank.value))

    def read_f32(self, key: str) -> np.ndarray:
        _, shape = self.info(key)
        out = np.empty(shape, np.float32)
        _lib.call("va_safetensors_read_f32", self._h, key.encode(), out.ctypes.data, out.size)
        return out

    def fold_conv_bn(self, prefix: str, eps: float = YOLO26_BN_EPS):
        """Folded (w [c_out][...], b [c_out]) of ``{prefix}.conv`` + ``{prefix}.bn``."""
        _, shape = self.info(prefix + ".conv.weight")
        w = np.empty(shape, np.float32)
        b = np.empty(shape[0], np.float32)
        _lib.call("va_safetensors_fold_conv_bn", self._h, prefix.encode(), float(eps), w.ctypes.data, b.ctypes.data,
                  w.size, shape[0])
        return w, b

    def has(self, key: str) -> bool:
        dt, rank = C.c_int(), C.c_int()
        shape = (C.c_int64 * 8)()
        return _lib.lib().va_safetensors_tensor_info(self._h, key.encode(), C.byref(dt), shape, C.byref(rank)) == 0


def c2psa_folded(st: SafeTensors, prefix: str, eps: float = YOLO26_BN_EPS):
    """The folded f32 weights of the C2PSA at ``prefix``: (w_cv1, b_cv1,
    [block dicts with w_qkv … b_ffn1], w_cv2, b_cv2); the number of blocks is
    the number of ``{prefix}.m.{i}`` present."""
    mat = lambda w: w.reshape(w.shape[0], -1)
    w_cv1, b_cv1 = st.fold_conv_bn(f"{prefix}.cv1", eps)
    w_cv2, b_cv2 = st.fold_conv_bn(f"{prefix}.cv2", eps)
    blocks = []
    while st.has(f"{prefix}.m.{len(blocks)}.attn.qkv.conv.weight"):
        i, blk = len(blocks), {}
        for name, path in BLOCK_STAGES.items():
            w, b = st.fold_conv_bn(f"{prefix}.m.{i}.{path}", eps)
            blk["w_" + name] = w if name == "pe" else mat(w)
            blk["b_" + name] = b
        blocks.append(blk)
    return mat(w_cv1), b_cv1, blocks, mat(w_cv2), b_cv2


class C2psa:
    """The C2PSA block (c2psa.rs:150-179) as one call of ``va_c2psa_fwd_bf16``:
    bf16 activations, folded bf16 weights, f32 biases on ``device``."""

    def __init__(self, w_cv1, b_cv1, blocks: list, w_cv2, b_cv2, device="cuda"):
        bf = lambda a: torch.as_tensor(np.asarray(a, np.float32)).to(device, torch.bfloat16).contiguous()
        f32 = lambda a: torch.as_tensor(np.asarray(a, np.float32)).to(device).contiguous()
        self.w_cv1, self.b_cv1, self.w_cv2, self.b_cv2 = bf(w_cv1), f32(b_cv1), bf(w_cv2), f32(b_cv2)
        self.C1 = self.w_cv1.shape[0]
        self._blocks = [{k: (bf(v) if k.startswith("w_") else f32(v)) for k, v in b.items()} for b in blocks]
        self._structs = (_lib.PsaBlockWeights * len(blocks))(
            *[_lib.PsaBlockWeights(**{k: v.data_ptr() for k, v in b.items()}) for b in self._blocks])
        self._ws = None

    @classmethod
    def from_safetensors(cls, path: str, prefix: str, eps: float = YOLO26_BN_EPS, device="cuda"):
        with SafeTensors(path) as st:
            return cls(*c2psa_folded(st, prefix, eps), device=device)

    def forward_into(self, x: torch.Tensor, y: torch.Tensor, stream=None):
        B, C1, H, W = x.shape
        need = int(_lib.lib().va_c2psa_workspace_bytes(B, C1, H, W, len(self._blocks)))
        if self._ws is None or self._ws.numel() < need or self._ws.device != x.device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        _lib.call("va_c2psa_fwd_bf16", _p(x), _p(self.w_cv1), _p(self.b_cv1), len(self._blocks),
                  C.byref(self._structs[0]), _p(self.w_cv2), _p(self.b_cv2), _p(y), B, C1, H, W, _p(self._ws),
                  self._ws.numel(), _stream(stream))
        return y

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.forward_into(x, torch.empty_like(x))
