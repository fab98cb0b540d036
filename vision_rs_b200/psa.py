"""Host-side mirror of the reference's PSA operator interface.

The reference registers four graph nodes for the PSA attention
(src/models/yolo/kernels/attention/psa.rs): each is a ``CustomOp`` (``name``,
``infer_output_shape``, ``lower``) wrapping a ``RuntimeOp``
(``n_activation_inputs``, ``param_shapes``, ``pack_args`` + ``grid``/``block``
→ launch, and the training-side ``pack_backward_args``).  The classes here
keep those names, argument meanings and shapes; ``launch`` /
``launch_backward`` hand the same arguments to the C ABI
(``include/visionattn.h``) instead of an ``ArgVisitor``.

Tensors are torch CUDA tensors used only as device buffers; every launch goes
on torch's current stream.  There is no CPU path: a missing library raises.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

from . import _lib

Shape = list  # list[Optional[int]]; None = dynamic (the reference's Option<usize>)


def _stream(stream=None) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _sfx(t: torch.Tensor) -> str:
    if t.dtype == torch.float32:
        return "f32"
    if t.dtype == torch.bfloat16:
        return "bf16"
    raise TypeError(f"unsupported dtype {t.dtype}")


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("visionattn ops take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("visionattn ops take contiguous tensors")
    return t.data_ptr()


# ── psa_pack_qkv (psa.rs:332-428 RuntimeOp, :744-792 CustomOp) ──────────────

class PsaPackQkvRuntimeOp:
    def __init__(self, key_dim: int, num_heads: int):
        self.key_dim, self.num_heads = key_dim, num_heads

    def n_activation_inputs(self) -> int:
        return 1

    def param_shapes(self, input_shapes, output_shape):
        return []

    def pack_args(self, inputs, params, output):
        """Argument tuple in the reference's visitor order (psa.rs:371-377)."""
        (x, _), = inputs
        b, qkv_h, h, w = x.shape
        return (_p(x), _p(output), qkv_h, h, w, b, self.num_heads)

    def launch(self, inputs, params, output, stream=None):
        x = inputs[0][0] if isinstance(inputs[0], tuple) else inputs[0]
        _lib.call(f"va_psa_pack_qkv_{_sfx(x)}", *self.pack_args([(x, None)], params, output), _stream(stream))

    def launch_backward(self, inputs, params, output, grad_output, grad_inputs, grad_params=(), stream=None):
        """d_qkv += scatter(d_packed) (psa.rs:393-417)."""
        x = inputs[0][0] if isinstance(inputs[0], tuple) else inputs[0]
        b, qkv_h, h, w = x.shape
        _lib.call("va_psa_pack_qkv_backward_f32", _p(grad_output), _p(grad_inputs[0]), qkv_h, h, w, b,
                  self.num_heads, _stream(stream))


class PsaPackQkvOp:
    def __init__(self, key_dim: int, num_heads: int):
        self.inner = PsaPackQkvRuntimeOp(key_dim, num_heads)
        self.num_heads = num_heads

    def name(self) -> str:
        return "psa_pack_qkv"

    def infer_output_shape(self, input_shapes: Sequence[Shape]) -> Shape:
        s = input_shapes[0]
        nh = self.num_heads
        n = s[2] * s[3] if s[2] is not None and s[3] is not None else None
        return [s[0], 4, nh, n, s[1] // (nh * 4) if s[1] is not None else None]

    def lower(self):
        return self.name(), self.inner


# ── psa_extract_v_nchw (psa.rs:433-531, :797-828) ───────────────────────────

class PsaExtractVRuntimeOp:
    def __init__(self, key_dim: int, num_heads: int):
        self.key_dim, self.num_heads = key_dim, num_heads

    def n_activation_inputs(self) -> int:
        return 1

    def param_shapes(self, input_shapes, output_shape):
        return []

    def pack_args(self, inputs, params, output):
        """psa.rs:472-478, plus B that grid() reads from the output shape."""
        (x, _), = inputs
        b, qkv_h, h, w = x.shape
        return (_p(x), _p(output), qkv_h, output.shape[1], h, w, self.num_heads, b)

    def launch(self, inputs, params, output, stream=None):
        x = inputs[0][0] if isinstance(inputs[0], tuple) else inputs[0]
        _lib.call(f"va_psa_extract_v_nchw_{_sfx(x)}", *self.pack_args([(x, None)], params, output),
                  _stream(stream))

    def launch_backward(self, inputs, params, output, grad_output, grad_inputs, grad_params=(), stream=None):
        x = inputs[0][0] if isinstance(inputs[0], tuple) else inputs[0]
        b, qkv_h, h, w = x.shape
        _lib.call("va_psa_extract_v_backward_f32", _p(grad_output), _p(grad_inputs[0]), qkv_h, qkv_h // 2, h, w,
                  self.num_heads, b, _stream(stream))


class PsaExtractVOp:
    def __init__(self, key_dim: int, num_heads: int):
        self.inner = PsaExtractVRuntimeOp(key_dim, num_heads)

    def name(self) -> str:
        return "psa_extract_v_nchw"

    def infer_output_shape(self, input_shapes: Sequence[Shape]) -> Shape:
        s = input_shapes[0]
        return [s[0], s[1] // 2 if s[1] is not None else None, s[2], s[3]]

    def lower(self):
        return self.name(), self.inner


# ── psa_merge_attn_nchw (psa.rs:536-633, :836-879) ──────────────────────────

class PsaMergeAttnRuntimeOp:
    def __init__(self, key_dim: int, num_heads: int):
        self.key_dim, self.num_heads = key_dim, num_heads

    def n_activation_inputs(self) -> int:
        return 2

    def param_shapes(self, input_shapes, output_shape):
        return []

    def pack_args(self, inputs, params, output):
        """psa.rs:575-581, plus B from the output shape."""
        (lo, _), (hi, _) = inputs
        b, c, h, w = output.shape
        return (_p(lo), _p(hi), _p(output), c, h, w, self.num_heads, b)

    def launch(self, inputs, params, output, stream=None):
        lo = inputs[0][0] if isinstance(inputs[0], tuple) else inputs[0]
        hi = inputs[1][0] if isinstance(inputs[1], tuple) else inputs[1]
        _lib.call(f"va_psa_merge_attn_nchw_{_sfx(lo)}", *self.pack_args([(lo, None), (hi, None)], params, output),
                  _stream(stream))

    def launch_backward(self, inputs, params, output, grad_output, grad_inputs, grad_params=(), stream=None):
        b, c, h, w = output.shape
        _lib.call("va_psa_merge_attn_backward_f32", _p(grad_output), _p(grad_inputs[0]), _p(grad_inputs[1]),
                  c, h, w, self.num_heads, b, _stream(stream))


class PsaMergeAttnOp:
    def __init__(self, key_dim: int, num_heads: int, h: int, w: int):
        self.inner = PsaMergeAttnRuntimeOp(key_dim, num_heads)
        self.num_heads, self.h, self.w = num_heads, h, w

    def name(self) -> str:
        return "psa_merge_attn_nchw"

    def infer_output_shape(self, input_shapes: Sequence[Shape]) -> Shape:
        lo = input_shapes[0]
        return [lo[0], self.num_heads * 2 * lo[3] if lo[3] is not None else None, self.h, self.w]

    def lower(self):
        return self.name(), self.inner


# ── flash_attention2_forward on the packed buffer (psa.rs:930-1066, :885-921)

class FlashAttn2PsaRuntimeOp:
    """Input: packed ``[4, BH, N, kd]`` (declared shape ``[B,4,nh,N,kd]``);
    output ``[BH, N, kd]``; param: ``[BH*N]`` LSE scratch (psa.rs:958-963)."""

    def __init__(self, key_dim: int, v_section: int, tensor_cores: bool = False):
        self.key_dim, self.v_section, self.tensor_cores = key_dim, v_section, tensor_cores

    @classmethod
    def new_lo(cls, key_dim: int, tensor_cores: bool = False):
        return cls(key_dim, 2, tensor_cores)

    @classmethod
    def new_hi(cls, key_dim: int, tensor_cores: bool = False):
        return cls(key_dim, 3, tensor_cores)

    def n_activation_inputs(self) -> int:
        return 1

    def param_shapes(self, input_shapes, output_shape):
        """psa.rs:958-963: the l scratch [B·nh·N]; the tensor-core variant adds
        its workspace (bytes) as a second parameter."""
        s = input_shapes[0]
        shapes = [[s[0] * s[2] * s[3]]]
        if self.tensor_cores:
            shapes.append([int(_lib.lib().va_flash_attention2_tc_workspace_bytes(s[3], s[0] * s[2], s[4]))])
        return shapes

    def _ptrs(self, packed: torch.Tensor, b: int, nh: int, n: int, kd: int):
        sec = b * nh * n * kd * packed.element_size()
        base = _p(packed)
        return base, base + sec, base + self.v_section * sec

    def pack_args(self, inputs, params, output):
        """psa.rs:967-996: q/k/v are offsets into the packed buffer."""
        (packed, shape), = inputs
        b, _, nh, n, kd = shape
        q, k, v = self._ptrs(packed, b, nh, n, kd)
        scale = 1.0 / math.sqrt(float(kd))
        return (q, k, v, _p(output), _p(params[0]), n, n, scale, float("-inf"), b * nh, kd)

    def launch(self, inputs, params, output, stream=None):
        packed, shape = inputs[0]
        if self.tensor_cores:  # bf16, head dim 32: the tcgen05 attention kernel behind the same node
            ws = params[1]
            _lib.call("va_flash_attention2_forward_tc_bf16", *self.pack_args(inputs, params, output), _p(ws),
                      ws.numel() * ws.element_size(), _stream(stream))
            return
        _lib.call(f"va_flash_attention2_forward_{_sfx(packed)}", *self.pack_args(inputs, params, output),
                  _stream(stream))

    def launch_backward(self, inputs, params, output, grad_output, grad_inputs, grad_params=(), stream=None):
        """psa.rs:1011-1054: dq/dk accumulate into d_packed sections 0/1, dv stored."""
        packed, shape = inputs[0]
        b, _, nh, n, kd = shape
        q, k, v = self._ptrs(packed, b, nh, n, kd)
        dq, dk, dv = self._ptrs(grad_inputs[0], b, nh, n, kd)
        scale = 1.0 / math.sqrt(float(kd))
        _lib.call("va_psa_fa2_backward_f32", q, k, v, _p(output), _p(grad_output), _p(params[0]), dq, dk, dv,
                  n, scale, b * nh, kd, _stream(stream))


class FlashAttn2PsaOp:
    def __init__(self, inner: FlashAttn2PsaRuntimeOp):
        self.inner = inner

    @classmethod
    def new_lo(cls, key_dim: int, tensor_cores: bool = False):
        return cls(FlashAttn2PsaRuntimeOp.new_lo(key_dim, tensor_cores))

    @classmethod
    def new_hi(cls, key_dim: int, tensor_cores: bool = False):
        return cls(FlashAttn2PsaRuntimeOp.new_hi(key_dim, tensor_cores))

    def name(self) -> str:
        return "flash_attention2_forward"

    def infer_output_shape(self, input_shapes: Sequence[Shape]) -> Shape:
        s = input_shapes[0]
        return [s[0], s[2], s[3], s[4]]

    def lower(self):
        return self.name(), self.inner


# ── functional helpers ───────────────────────────────────────────────────────

def flash_attention2_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                             softmax_scale: Optional[float] = None):
    """``[BH,N,D]`` flash attention; returns ``(o, lse)`` (lse f32, natural log)."""
    bh, nq, d = q.shape
    nk = k.shape[1]
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    o = torch.empty(bh, nq, v.shape[2], device=q.device, dtype=q.dtype)
    l = torch.empty(bh, nq, device=q.device, dtype=torch.float32)
    _lib.call(f"va_flash_attention2_forward_{_sfx(q)}", _p(q), _p(k), _p(v), _p(o), _p(l), nq, nk,
              float(softmax_scale), float("-inf"), bh, d, _stream())
    return o, l


def flash_attention2_forward_tc(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                softmax_scale: Optional[float] = None, workspace: Optional[torch.Tensor] = None):
    """The same node on the tensor cores: bf16 ``[BH,N,32]`` self-attention."""
    bh, n, d = q.shape
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    need = int(_lib.lib().va_flash_attention2_tc_workspace_bytes(n, bh, d))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    o = torch.empty(bh, n, v.shape[2], device=q.device, dtype=q.dtype)
    l = torch.empty(bh, n, device=q.device, dtype=torch.float32)
    _lib.call("va_flash_attention2_forward_tc_bf16", _p(q), _p(k), _p(v), _p(o), _p(l), n, k.shape[1],
              float(softmax_scale), float("-inf"), bh, d, _p(workspace), workspace.numel(), _stream())
    return o, l


def fold_bn(w: torch.Tensor, gamma, beta, mean, var, eps: float):
    """Fold eval-mode BN into a bias-free conv on the host (``va_fold_bn_f32``)."""
    w = w.detach().float().contiguous().cpu()
    c_out = w.shape[0]
    k = w.numel() // c_out
    wo = torch.empty_like(w)
    bo = torch.empty(c_out, dtype=torch.float32)
    cp = lambda t: torch.as_tensor(t, dtype=torch.float32).contiguous().cpu()
    g, b, m, v = cp(gamma), cp(beta), cp(mean), cp(var)
    _lib.call("va_fold_bn_f32", w.data_ptr(), g.data_ptr(), b.data_ptr(), m.data_ptr(), v.data_ptr(),
              float(eps), c_out, k, wo.data_ptr(), bo.data_ptr())
    return wo, bo


class PsaAttention:
    """The fused PSA ``Attention`` op (c2psa.rs:61-116) with BN folded.

    ``dtype`` selects the f32 FFMA path or the bf16 tensor-core path.
    Weights: ``w_qkv [nh*4*kd, C]``, ``w_pe [C,1,3,3]``, ``w_proj [C,C]``
    (conv weights with trailing 1×1 dims accepted), biases f32."""

    def __init__(self, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, num_heads: int, key_dim: int = 32,
                 dtype=torch.bfloat16, device="cuda"):
        self.num_heads, self.key_dim, self.dtype = num_heads, key_dim, dtype
        t = lambda a, dt: torch.as_tensor(a).to(device=device, dtype=dt).contiguous()
        self.C = int(torch.as_tensor(w_proj).shape[0])
        self.w_qkv = t(w_qkv, dtype).reshape(-1, self.C)
        self.w_pe = t(w_pe, dtype).reshape(self.C, 1, 3, 3)
        self.w_proj = t(w_proj, dtype).reshape(self.C, self.C)
        self.b_qkv, self.b_pe, self.b_proj = t(b_qkv, torch.float32), t(b_pe, torch.float32), t(b_proj, torch.float32)
        self._ws = None

    def workspace_bytes(self, B: int, H: int, W: int) -> int:
        return int(_lib.lib().va_psa_attention_workspace_bytes(B, self.C, H, W, self.num_heads, self.key_dim,
                                                               0 if self.dtype == torch.float32 else 1))

    def workspace(self, B: int, H: int, W: int, device) -> torch.Tensor:
        need = self.workspace_bytes(B, H, W)
        if self._ws is None or self._ws.numel() < need or self._ws.device != torch.device(device):
            self._ws = torch.empty(need, dtype=torch.uint8, device=device)
        return self._ws

    def forward_into(self, x: torch.Tensor, y: torch.Tensor, stream=None):
        B, C, H, W = x.shape
        ws = self.workspace(B, H, W, x.device)
        _lib.call(f"va_psa_attention_fwd_{_sfx(x)}", _p(x), _p(self.w_qkv), _p(self.b_qkv), _p(self.w_pe),
                  _p(self.b_pe), _p(self.w_proj), _p(self.b_proj), _p(y), B, C, H, W, self.num_heads,
                  self.key_dim, _p(ws), ws.numel(), _stream(stream))
        return y

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != self.dtype:
            raise TypeError(f"input dtype {x.dtype} != op dtype {self.dtype}")
        return self.forward_into(x, torch.empty_like(x))
