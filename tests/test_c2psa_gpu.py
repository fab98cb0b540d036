"""PSABlock and C2PSA forward (va_psa_block_fwd_bf16, va_c2psa_fwd_bf16) on
the GPU through the C ABI.

References: the BN-folded oracle (``psa_block_forward`` /
``c2psa_forward_folded``, pinned to the reference's golden C2PSA fixture on
the CPU) on the same bf16-rounded inputs and weights, and the golden
fixture's own expected output.

Tolerances.  The PSABlock (one bf16 output rounding, the attention output
rounded to bf16 inside) is held to the north star's bf16 rel-L2 bound,
≤ 2e-3.  Its output carries the residual input (|y| up to ≈5, where one bf16
ulp is 2^-5), so max-abs is held to 1e-2 relative to max(1, max |y|), as
below.  The whole C2PSA rounds three activations to bf16 —
the attention op's input and output (its interface is bf16) and the block
output — each worth ≈1.1-1.7e-3 rel-L2 (emulating these roundings on the
CPU gives 2.1e-3 against the exact chain), so it is held to rel-L2 ≤ 4e-3.
Its outputs reach |y| ≈ 5, where one bf16 ulp is 2^-5, so its max-abs bound
is 1e-2 relative to max(1, max |y|).  Against the fixture's expected output,
computed with f32 weights, the bf16 rounding of the weights adds ≈2.7e-3
(also measured on the CPU): ≤ 6e-3."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import BF16_MAX_ABS, BF16_REL_L2, c2psa_checkpoint, folded_c2psa, load_golden, max_abs, rel_l2
from oracle import psa_oracle as po
from vision_rs_b200 import _lib

pytestmark = pytest.mark.gpu

C2PSA_REL_L2 = 4e-3
C2PSA_VS_FIXTURE_REL_L2 = 6e-3


def _bf(a):
    return torch.as_tensor(np.asarray(a, np.float32)).bfloat16().float().numpy()


def _dev_bf16(a):
    return torch.as_tensor(np.asarray(a, np.float32)).to("cuda", torch.bfloat16).contiguous()


def _dev_f32(a):
    return torch.as_tensor(np.asarray(a, np.float32)).cuda().contiguous()


def _round_block(w):
    """bf16-rounded weights (what the op receives), f32 biases."""
    return {k: (_bf(v) if k.startswith("w_") else np.asarray(v, np.float32)) for k, v in w.items()}


def _block_struct(w, keep):
    t = {k: (_dev_bf16(v) if k.startswith("w_") else _dev_f32(v)) for k, v in w.items()}
    keep.append(t)
    return _lib.PsaBlockWeights(**{k: v.data_ptr() for k, v in t.items()})


def _synthetic_block(C, seed):
    rng = np.random.default_rng(seed)
    p = po.psa_synthetic(1, 2, 2, C=C, num_heads=C // 64, seed=seed)
    w = {k: np.asarray(v, np.float64).reshape(v.shape[0], -1) if k in ("w_qkv", "w_proj") else v
         for k, v in p.items() if k != "x"}
    w["w_ffn0"] = rng.standard_normal((2 * C, C)) * 0.02
    w["b_ffn0"] = rng.standard_normal(2 * C) * 0.02
    w["w_ffn1"] = rng.standard_normal((C, 2 * C)) * 0.02
    w["b_ffn1"] = rng.standard_normal(C) * 0.02
    return _round_block(w)


def _run_c2psa(x, w_cv1, b_cv1, blocks, w_cv2, b_cv2):
    B, C1, H, W = x.shape
    keep = []
    arr = (_lib.PsaBlockWeights * len(blocks))(*[_block_struct(b, keep) for b in blocks])
    xd, w1, w2 = _dev_bf16(x), _dev_bf16(w_cv1), _dev_bf16(w_cv2)
    b1, b2 = _dev_f32(b_cv1), _dev_f32(b_cv2)
    y = torch.empty_like(xd)
    need = int(_lib.lib().va_c2psa_workspace_bytes(B, C1, H, W, len(blocks)))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    _lib.call("va_c2psa_fwd_bf16", xd.data_ptr(), w1.data_ptr(), b1.data_ptr(), len(blocks), ctypes.byref(arr[0]),
              w2.data_ptr(), b2.data_ptr(), y.data_ptr(), B, C1, H, W, ws.data_ptr(), need,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def test_c2psa_golden_fixture(cuda):
    """The reference's C2PSA fixture (C2PSA(256, 256, n=1, e=0.5), B=2, 4×4)."""
    g = load_golden("c2psa_fwd.npz")
    w_cv1, b_cv1, blocks, w_cv2, b_cv2 = folded_c2psa(g)
    x = _bf(g["x"])
    w_cv1, w_cv2 = _bf(w_cv1), _bf(w_cv2)
    blocks = [_round_block(b) for b in blocks]
    y = _run_c2psa(x, w_cv1, b_cv1, blocks, w_cv2, b_cv2)
    ref = po.c2psa_forward_folded(x, w_cv1, b_cv1, blocks, w_cv2, b_cv2)
    assert rel_l2(y, ref) < C2PSA_REL_L2 and max_abs(y, ref) < BF16_MAX_ABS * max(1.0, float(np.abs(ref).max()))
    assert rel_l2(y, g["expected_output"]) < C2PSA_VS_FIXTURE_REL_L2


def test_c2psa_from_checkpoint(cuda, tmp_path):
    """The C2PSA op built from a safetensors checkpoint in the reference's key
    layout (read and BN-folded by the library; the fixture's BN eps 1e-5)."""
    from vision_rs_b200 import weights
    f, g = c2psa_checkpoint(tmp_path)
    op = weights.C2psa.from_safetensors(f, "model.10", eps=1e-5)
    y = op(torch.as_tensor(g["x"]).to("cuda", torch.bfloat16)).float().cpu().numpy()
    assert rel_l2(y, g["expected_output"]) < C2PSA_VS_FIXTURE_REL_L2


@pytest.mark.parametrize("C1,B,H,W,n", [(256, 2, 20, 20, 1), (512, 1, 40, 40, 2)])
def test_c2psa_synthetic_vs_oracle(cuda, C1, B, H, W, n):
    """YOLO26n's C2PSA (C1 = 256, one block, 20×20 at 640 input) and a wider
    two-block C2PSA (C1 = 512: 4 heads, as YOLO26 l/x repeat the block)."""
    rng = np.random.default_rng(C1 + n)
    c = C1 // 2
    x = _bf(rng.standard_normal((B, C1, H, W)))
    w_cv1, w_cv2 = _bf(rng.standard_normal((C1, C1)) * 0.05), _bf(rng.standard_normal((C1, C1)) * 0.05)
    b_cv1, b_cv2 = (rng.standard_normal(C1) * 0.02 for _ in range(2))
    blocks = [_synthetic_block(c, 100 + i) for i in range(n)]
    y = _run_c2psa(x, w_cv1, b_cv1, blocks, w_cv2, b_cv2)
    ref = po.c2psa_forward_folded(x, w_cv1, b_cv1, blocks, w_cv2, b_cv2)
    assert rel_l2(y, ref) < C2PSA_REL_L2 and max_abs(y, ref) < BF16_MAX_ABS * max(1.0, float(np.abs(ref).max()))


@pytest.mark.parametrize("C,B,H,W", [(128, 2, 20, 20), (256, 1, 40, 40), (128, 3, 4, 6)])
def test_psa_block_vs_oracle(cuda, C, B, H, W):
    w = _synthetic_block(C, C + H)
    x = _bf(np.random.default_rng(W).standard_normal((B, C, H, W)))
    keep = []
    s = _block_struct(w, keep)
    xd = _dev_bf16(x)
    y = torch.empty_like(xd)
    need = int(_lib.lib().va_psa_block_workspace_bytes(B, C, H, W))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    _lib.call("va_psa_block_fwd_bf16", xd.data_ptr(), ctypes.byref(s), y.data_ptr(), B, C, H, W, ws.data_ptr(), need,
              torch.cuda.current_stream().cuda_stream)
    yh = y.float().cpu().numpy()
    ref = po.psa_block_forward(x, w, C // 64)
    assert rel_l2(yh, ref) < BF16_REL_L2 and max_abs(yh, ref) < BF16_MAX_ABS * max(1.0, float(np.abs(ref).max()))


def test_block_rejects_unaligned_images(cuda):
    w = _synthetic_block(128, 1)
    keep = []
    s = _block_struct(w, keep)
    rc = _lib.lib().va_psa_block_fwd_bf16(None, ctypes.byref(s), None, 1, 128, 3, 3, None, 0, None)
    assert rc != 0
    rc = _lib.lib().va_psa_block_fwd_bf16(1, ctypes.byref(s), 1, 1, 128, 3, 3, None, 0, None)
    assert rc == 1 and b"multiple of 8" in _lib.lib().va_get_last_error_string()
