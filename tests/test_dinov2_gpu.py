"""DINOv2 attention (packed QKV Linear + head-dim-64 flash attention) on the
B200 vs the float64 CPU restatement on the same bf16-rounded inputs.

bf16 mode tolerances: rel-L2 ≤ 2e-3 and max-abs ≤ 1e-2 against the fp32/f64
reference.
"""
import numpy as np
import pytest
import torch

from conftest import BF16_MAX_ABS, BF16_REL_L2, max_abs, rel_l2
from oracle import dinov2_oracle as do

pytestmark = pytest.mark.gpu


def _bf16(a, cuda):
    return torch.as_tensor(a).to(cuda, torch.bfloat16)


def _inputs(S, n, hidden, seed, cuda):
    x, w, b = do.dinov2_synthetic(S=S, n=n, hidden=hidden, seed=seed)
    xt, wt = _bf16(x, cuda), _bf16(w, cuda)
    bt = torch.as_tensor(b).to(cuda)
    # the reference sees exactly the operands the kernels see
    return xt, wt, bt, xt.float().cpu().numpy(), wt.float().cpu().numpy(), b


def _check(got, ref):
    got = got.float().cpu().numpy()
    assert rel_l2(got, ref) <= BF16_REL_L2, rel_l2(got, ref)
    assert max_abs(got, ref) <= BF16_MAX_ABS, max_abs(got, ref)


def test_qkv_linear(cuda):
    from vision_rs_b200 import dinov2
    xt, wt, bt, x, w, b = _inputs(2, 1601, 384, 0, cuda)
    _check(dinov2.qkv_linear(xt, wt, bt), do.qkv_linear(x, w, b))


def test_attention_global_cfg4(cuda):
    from vision_rs_b200 import dinov2
    xt, wt, bt, x, w, b = _inputs(2, 1601, 384, 1, cuda)
    op = dinov2.DinoV2Attention(wt, bt, 6)
    _check(op(xt), do.dinov2_attention(x, w, b, 6))


@pytest.mark.parametrize("S,n,hidden", [(3, 1, 128), (2, 7, 128), (2, 128, 384), (2, 129, 384), (1, 257, 768),
                                        (4, 101, 384), (1, 384, 192)])
def test_attention_shapes(cuda, S, n, hidden):
    from vision_rs_b200 import dinov2
    xt, wt, bt, x, w, b = _inputs(S, n, hidden, 10 + n, cuda)
    op = dinov2.DinoV2Attention(wt, bt, hidden // 64)
    _check(op(xt), do.dinov2_attention(x, w, b, hidden // 64))


def test_windowed_layer_cfg4(cuda):
    """4×4 windows of 10×10 patches over the 40×40 grid, cls in every window."""
    from vision_rs_b200 import dinov2
    B, gh, gw, win = 2, 40, 40, 10
    xt, wt, bt, x, w, b = _inputs(B, 1 + gh * gw, 384, 2, cuda)
    xw = dinov2.window_partition(xt, gh, gw, win)
    xw_ref = do.window_partition(x, gh, gw, win)
    assert np.array_equal(xw.float().cpu().numpy(), xw_ref)  # a gather: bit-exact
    ow = dinov2.DinoV2Attention(wt, bt, 6)(xw)
    ow_ref = do.dinov2_attention(xw_ref, w, b, 6)
    _check(ow, ow_ref)
    o = dinov2.window_unpartition(ow, B, gh, gw, win)
    # compare against un-partitioning the kernel's own window outputs (exact
    # gather; cls = f32 mean rounded to bf16), then end to end against the oracle
    own = do.window_unpartition(ow.float().cpu().numpy(), B, gh, gw, win)
    got = o.float().cpu().numpy()
    assert np.array_equal(got[:, 1:], own[:, 1:])
    assert np.abs(got[:, 0] - own[:, 0]).max() <= 2 ** -7 * np.abs(own[:, 0]).max()
    _check(o, do.window_unpartition(ow_ref, B, gh, gw, win))


def test_global_layer_full_cfg4_batch(cuda):
    """cfg4's global layer at full size (16 images × 1601 tokens): images 0, 7
    and 15 against the oracle, and batch independence (an image's output does
    not depend on its batch neighbours: image 5 alone gives the same bits)."""
    from vision_rs_b200 import dinov2
    xt, wt, bt, x, w, b = _inputs(16, 1601, 384, 5, cuda)
    op = dinov2.DinoV2Attention(wt, bt, 6)
    o = op(xt)
    for i in (0, 7, 15):
        _check(o[i:i + 1], do.dinov2_attention(x[i:i + 1], w, b, 6))
    assert torch.equal(op(xt[5:6].contiguous()), o[5:6])


def test_windowed_layer_full_cfg4_batch(cuda):
    """cfg4's windowed layer at full size (16 images → 256 windows of 1 + 100
    tokens): the windows of images 0 and 15 against the oracle, the whole
    un-partitioned output of image 15, and batch independence."""
    from vision_rs_b200 import dinov2
    B, gh, gw, win = 16, 40, 40, 10
    xt, wt, bt, x, w, b = _inputs(B, 1 + gh * gw, 384, 6, cuda)
    xw = dinov2.window_partition(xt, gh, gw, win)
    op = dinov2.DinoV2Attention(wt, bt, 6)
    ow = op(xw)
    nw = (gh // win) * (gw // win)
    for i in (0, 15):
        xw_ref = do.window_partition(x[i:i + 1], gh, gw, win)
        ow_ref = do.dinov2_attention(xw_ref, w, b, 6)
        _check(ow[i * nw:(i + 1) * nw], ow_ref)
        if i == 15:
            o = dinov2.window_unpartition(ow, B, gh, gw, win)
            _check(o[15:16], do.window_unpartition(ow_ref, 1, gh, gw, win))
    assert torch.equal(op(xw[3 * nw:4 * nw].contiguous()), ow[3 * nw:4 * nw])


def test_deterministic(cuda):
    from vision_rs_b200 import dinov2
    xt, wt, bt, *_ = _inputs(2, 1601, 384, 3, cuda)
    op = dinov2.DinoV2Attention(wt, bt, 6)
    assert torch.equal(op(xt), op(xt))


def test_rejects_bad_hidden(cuda):
    from vision_rs_b200 import _lib, dinov2
    xt, wt, bt, *_ = _inputs(1, 16, 128, 4, cuda)
    with pytest.raises(_lib.VisionAttnError):
        dinov2.DinoV2Attention(wt, bt, 3)(xt)  # 3·64 != 128
