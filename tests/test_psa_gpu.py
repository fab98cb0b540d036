"""PSA attention path on the GPU, through the C ABI, against the CPU oracle
and the reference's golden fixtures.

Tolerances: layout ops are permutations → bit-exact; f32 kernels max-abs
1e-5 (the north star's f32 bound); bf16 paths rel-L2 ≤ 2e-3 and max-abs ≤
1e-2 against the f32 oracle evaluated on the same bf16-rounded inputs."""
import math

import numpy as np
import pytest
import torch

from conftest import BF16_MAX_ABS, BF16_REL_L2, F32_MAX_ABS, load_golden, max_abs, rel_l2
from oracle import psa_oracle as po
from vision_rs_b200 import psa as vp

pytestmark = pytest.mark.gpu
SCALE = 1.0 / math.sqrt(32.0)


def dev(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a)).to("cuda", dtype).contiguous()


def host(t):
    return t.float().cpu().numpy()


def bf16_round(a):
    return torch.as_tensor(np.asarray(a, np.float32)).bfloat16().float().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,W", [(2, 4, 4), (1, 20, 20), (3, 7, 9), (2, 40, 40)])
def test_layout_ops_exact(cuda, dtype, B, H, W):
    nh, kd = 2, 32
    rng = np.random.default_rng(B * 100 + H)
    qkv = bf16_round(rng.standard_normal((B, nh * 4 * kd, H, W)).astype(np.float32))
    x = dev(qkv, dtype)
    pk = vp.PsaPackQkvOp(kd, nh)
    shp = pk.infer_output_shape([list(x.shape)])
    packed = torch.empty(4, B * nh, H * W, kd, device="cuda", dtype=dtype)
    pk.inner.launch([(x, shp)], [], packed)
    ref = po.pack_qkv(qkv, nh)
    assert np.array_equal(host(packed), ref)
    v = torch.empty(B, nh * 2 * kd, H, W, device="cuda", dtype=dtype)
    vp.PsaExtractVOp(kd, nh).inner.launch([x], [], v)
    assert np.array_equal(host(v), po.extract_v_nchw(qkv, nh))
    merged = torch.empty_like(v)
    vp.PsaMergeAttnOp(kd, nh, H, W).inner.launch([packed[2], packed[3]], [], merged)
    assert np.array_equal(host(merged), po.merge_attn_nchw(ref[2], ref[3], nh, H, W))


@pytest.mark.parametrize("B,H,W", [(2, 4, 4), (2, 9, 7)])
def test_layout_backwards_exact(cuda, B, H, W):
    nh, kd = 2, 32
    qkv_h, c = nh * 4 * kd, nh * 2 * kd
    rng = np.random.default_rng(7)
    d_packed = rng.standard_normal((4, B * nh, H * W, kd)).astype(np.float32)
    d0 = rng.standard_normal((B, qkv_h, H, W)).astype(np.float32)
    d_qkv = dev(d0)
    x = torch.zeros(B, qkv_h, H, W, device="cuda")
    vp.PsaPackQkvOp(kd, nh).inner.launch_backward([x], [], None, dev(d_packed), [d_qkv])
    ref = po.pack_qkv_backward(d_packed, B, qkv_h, H, W, nh, d_qkv=d0)
    assert np.array_equal(host(d_qkv), ref)
    d_v = rng.standard_normal((B, c, H, W)).astype(np.float32)
    vp.PsaExtractVOp(kd, nh).inner.launch_backward([x], [], None, dev(d_v), [d_qkv])
    ref = po.extract_v_backward(d_v, qkv_h, nh, d_qkv=ref)
    assert np.array_equal(host(d_qkv), ref)
    dm = rng.standard_normal((B, c, H, W)).astype(np.float32)
    dlo = torch.empty(B * nh, H * W, kd, device="cuda")
    dhi = torch.empty_like(dlo)
    out = torch.empty(B, c, H, W, device="cuda")
    vp.PsaMergeAttnOp(kd, nh, H, W).inner.launch_backward([dlo, dhi], [], out, dev(dm), [dlo, dhi])
    rlo, rhi = po.merge_attn_backward(dm, nh)
    assert np.array_equal(host(dlo), rlo) and np.array_equal(host(dhi), rhi)


def test_fa_forward_golden_fixture(cuda):
    """Direct FA known-answer test: the reference's backward fixture dumps
    Q, K, V_lo, V_hi, O_lo, O_hi, LSE in [4,16,32] (generate_backward.py:202-208)."""
    g = load_golden("c2psa_bwd.npz")
    for half in ("lo", "hi"):
        o, l = vp.flash_attention2_forward(dev(g["attn_q"]), dev(g["attn_k"]), dev(g[f"attn_v_{half}"]), SCALE)
        assert max_abs(host(o), g[f"attn_o_{half}"]) < F32_MAX_ABS
        assert max_abs(host(l), g["attn_l"]) < F32_MAX_ABS


# small problems run the split-row kernel (several threads per query row); (300, 130, 130, 32)
# has enough rows for the row-per-thread kernel
@pytest.mark.parametrize("bh,nq,nk,d", [(2, 400, 400, 32), (4, 37, 129, 32), (1, 1601, 1601, 64),
                                        (3, 100, 100, 64), (2, 1, 5, 16), (5, 70, 333, 16), (300, 130, 130, 32)])
def test_fa_forward_f32_vs_oracle(cuda, bh, nq, nk, d):
    rng = np.random.default_rng(nq + nk)
    q, k, v = (rng.standard_normal((bh, n, d)).astype(np.float32) for n in (nq, nk, nk))
    o, l = vp.flash_attention2_forward(dev(q), dev(k), dev(v), 1 / math.sqrt(d))
    ro, rl = po.flash_attention2_forward(q, k, v, 1 / math.sqrt(d))
    assert max_abs(host(o), ro) < F32_MAX_ABS
    assert max_abs(host(l), rl) < F32_MAX_ABS  # LSE magnitude ~log(N)+|s| ≈ 8: measured ≤ 2.9e-6


def test_fa_forward_bf16_vs_oracle(cuda):
    rng = np.random.default_rng(5)
    q, k, v = (bf16_round(rng.standard_normal((4, 400, 32))) for _ in range(3))
    o, l = vp.flash_attention2_forward(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16), SCALE)
    ro, rl = po.flash_attention2_forward(q, k, v, SCALE)
    assert rel_l2(host(o), ro) < BF16_REL_L2 and max_abs(host(o), ro) < BF16_MAX_ABS


def test_fa_forward_tc_golden_fixture(cuda):
    """The tensor-core node entry on the reference's FA fixture ([4,16,32], lo
    and hi halves; small enough that the entry runs the FFMA kernel), inputs
    rounded to bf16: o within the bf16 bound of the oracle on those inputs and
    of the fixture; l within 1e-3."""
    g = load_golden("c2psa_bwd.npz")
    q, k = bf16_round(g["attn_q"]), bf16_round(g["attn_k"])
    for half in ("lo", "hi"):
        v = bf16_round(g[f"attn_v_{half}"])
        o, l = vp.flash_attention2_forward_tc(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16),
                                              SCALE)
        ro, rl = po.flash_attention2_forward(q, k, v, SCALE)
        assert rel_l2(host(o), ro) < BF16_REL_L2 and max_abs(host(o), ro) < BF16_MAX_ABS
        assert rel_l2(host(o), g[f"attn_o_{half}"]) < 2 * BF16_REL_L2
        assert max_abs(host(l), rl) < 1e-3


# Above 2048 query rows in all the tensor-core kernels run: 100 tokens the short-sequence
# kernel (one key tile), 400 = cfg1/cfg5, 1600 = cfg2, 1601 and 130 ragged last tiles; (4, 100)
# and the fixture (4 × 16) are small enough for the FFMA kernel the entry hands them to.
@pytest.mark.parametrize("bh,n", [(32, 100), (6, 400), (4, 1600), (3, 1601), (24, 130), (128, 400), (4, 100)])
def test_fa_forward_tc_vs_oracle(cuda, bh, n):
    rng = np.random.default_rng(bh * n)
    q, k, v = (bf16_round(rng.standard_normal((bh, n, 32)) * s) for s in (0.8, 0.8, 1.0))
    o, l = vp.flash_attention2_forward_tc(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16),
                                          SCALE)
    idx = [0, bh - 1] if bh > 8 else list(range(bh))
    ro, rl = po.flash_attention2_forward(q[idx], k[idx], v[idx], SCALE)
    oh, lh = host(o)[idx], host(l)[idx]
    assert rel_l2(oh, ro) < BF16_REL_L2 and max_abs(oh, ro) < BF16_MAX_ABS
    assert max_abs(lh, rl) < 1e-3


def test_fa_forward_tc_matches_simt_node(cuda):
    """Both bf16 entries of the node agree on the same inputs (cfg2's per-call
    shape, 128 sequences × 1600 tokens), within the bf16 bound."""
    rng = np.random.default_rng(77)
    q, k, v = (dev(rng.standard_normal((128, 1600, 32)) * 0.7, torch.bfloat16) for _ in range(3))
    o1, l1 = vp.flash_attention2_forward_tc(q, k, v, SCALE)
    o2, l2 = vp.flash_attention2_forward(q, k, v, SCALE)
    assert rel_l2(host(o1), host(o2)) < BF16_REL_L2
    assert max_abs(host(l1), host(l2)) < 1e-3


def test_fa_forward_tc_rejects(cuda):
    """Argument errors return before any launch (4096 query rows: the tensor-core route)."""
    from vision_rs_b200 import _lib
    lib = _lib.lib()
    bh, n = 2, 2048
    x = torch.zeros(bh, n, 32, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(bh, n, device="cuda")
    ws = torch.empty(int(lib.va_flash_attention2_tc_workspace_bytes(n, bh, 32)), dtype=torch.uint8, device="cuda")
    p, l, w = x.data_ptr(), lse.data_ptr(), ws.data_ptr()
    call = lib.va_flash_attention2_forward_tc_bf16
    assert call(p, p, p, p, l, n, n, SCALE, float("-inf"), bh, 16, w, ws.numel(), None) == 1  # head dim
    assert call(p, p, p, p, l, n, n // 2, SCALE, float("-inf"), bh, 32, w, ws.numel(), None) == 1  # cross attention
    assert call(p, p, p, p, None, n, n, SCALE, float("-inf"), bh, 32, w, ws.numel(), None) == 1  # l is required
    assert call(p, p, p, p, l, n, n, SCALE, float("-inf"), bh, 32, w, ws.numel() - 256, None) == 6  # short workspace


def test_reference_node_sequence_bf16_tensor_cores(cuda):
    """The reference graph's two flash_attention2_forward nodes (lo, hi) with
    the tensor-core RuntimeOp variant on a bf16 packed buffer: equal, within
    the bf16 bound, to the oracle's per-half attention."""
    B, nh, N, kd = 4, 2, 400, 32
    rng = np.random.default_rng(3)
    packed = bf16_round(rng.standard_normal((4, B * nh, N, kd)) * 0.8)
    pd = dev(packed, torch.bfloat16)
    shp = [B, 4, nh, N, kd]
    for ctor, sec in ((vp.FlashAttn2PsaOp.new_lo, 2), (vp.FlashAttn2PsaOp.new_hi, 3)):
        op = ctor(kd, tensor_cores=True).inner
        shapes = op.param_shapes([shp], None)
        params = [torch.empty(*shapes[0], device="cuda"), torch.empty(*shapes[1], dtype=torch.uint8, device="cuda")]
        out = torch.empty(B * nh, N, kd, dtype=torch.bfloat16, device="cuda")
        op.launch([(pd, shp)], params, out)
        ro, rl = po.flash_attention2_forward(packed[0], packed[1], packed[sec], SCALE)
        assert rel_l2(host(out), ro) < BF16_REL_L2 and max_abs(host(out), ro) < BF16_MAX_ABS
        assert max_abs(host(params[0]).reshape(B * nh, N), rl) < 1e-3


@pytest.mark.parametrize("bh,n,d", [(4, 16, 32), (2, 400, 32), (3, 77, 16), (2, 130, 64)])
def test_psa_fa2_backward_f32(cuda, bh, n, d):
    """psa_fa2_backward (psa.rs:650-725): dq/dk accumulate, dv stored."""
    rng = np.random.default_rng(n)
    q, k, v, do = (rng.standard_normal((bh, n, d)).astype(np.float32) for _ in range(4))
    o, l = po.flash_attention2_forward(q, k, v, 1 / math.sqrt(d))
    dq0, dk0 = (rng.standard_normal((bh, n, d)).astype(np.float32) for _ in range(2))
    dq, dk, dv = dev(dq0), dev(dk0), torch.empty(bh, n, d, device="cuda")
    from vision_rs_b200 import _lib
    sp = lambda t: t.data_ptr()
    st = torch.cuda.current_stream().cuda_stream
    args = [dev(a) for a in (q, k, v, o, do, l)]
    _lib.call("va_psa_fa2_backward_f32", *map(sp, args), sp(dq), sp(dk), sp(dv), n, 1 / math.sqrt(d), bh, d, st)
    rq, rk, rv = po.psa_fa2_backward(q, k, v, o, do, l, 1 / math.sqrt(d), dq_acc=dq0, dk_acc=dk0)
    # the north star's f32 bound (measured ≤ 7.5e-7 with |dq|, |dk| up to ≈5)
    assert max_abs(host(dq), rq) < F32_MAX_ABS and max_abs(host(dk), rk) < F32_MAX_ABS
    assert max_abs(host(dv), rv) < F32_MAX_ABS
    # split kernels (flash_attn2.rs:129-260) store instead of accumulating
    dq2, dk2, dv2 = (torch.empty(bh, n, d, device="cuda") for _ in range(3))
    _lib.call("va_flash_attention2_backward_dq_f32", *map(sp, args), sp(dq2), n, n, 1 / math.sqrt(d), bh, d, st)
    _lib.call("va_flash_attention2_backward_dkv_f32", *map(sp, args), sp(dk2), sp(dv2), n, n, 1 / math.sqrt(d),
              bh, d, st)
    assert max_abs(host(dq2), rq - dq0) < F32_MAX_ABS and max_abs(host(dk2), rk - dk0) < F32_MAX_ABS
    assert max_abs(host(dv2), rv) < F32_MAX_ABS


def test_dwconv_golden_fixture(cuda):
    g = load_golden("dwconv_depthwise.npz")
    from vision_rs_b200 import _lib
    st = torch.cuda.current_stream().cuda_stream
    x, w, dy = dev(g["x"]), dev(g["conv_w"]), dev(g["dy"])
    y = torch.empty_like(x)
    _lib.call("va_dwconv3x3_bias_f32", x.data_ptr(), w.data_ptr(), None, y.data_ptr(), 2, 128, 4, 4, st)
    assert max_abs(host(y), g["expected_output"]) < 1e-5
    dx, dw = torch.empty_like(x), torch.empty_like(w)
    _lib.call("va_dwconv3x3_backward_f32", x.data_ptr(), w.data_ptr(), dy.data_ptr(), dx.data_ptr(), dw.data_ptr(),
              2, 128, 4, 4, st)
    assert max_abs(host(dx), g["dx_expected"]) < 1e-4
    assert max_abs(host(dw), g["dw_expected"]) < 1e-4


def _op(p, dtype):
    return vp.PsaAttention(p["w_qkv"], p["b_qkv"], p["w_pe"], p["b_pe"], p["w_proj"], p["b_proj"], num_heads=2,
                           key_dim=32, dtype=dtype)


def _oracle(p):
    return po.psa_attention(p["x"], p["w_qkv"], p["b_qkv"], p["w_pe"], p["b_pe"], p["w_proj"], p["b_proj"], 2, 32)


def test_fused_f32_golden_case(cuda):
    g = load_golden("psa_attn_case.npz")
    y = _op(g, torch.float32)(dev(g["x"]))
    assert max_abs(host(y), g["y"]) < F32_MAX_ABS


@pytest.mark.parametrize("B,H,W", [(1, 20, 20), (2, 7, 9), (1, 40, 40)])
def test_fused_f32_vs_oracle(cuda, B, H, W):
    """cfg1 shape (1×128×20×20) and ragged shapes, f32 max-abs 1e-5."""
    p = po.psa_synthetic(B, H, W, seed=B + H)
    y = _op(p, torch.float32)(dev(p["x"]))
    assert max_abs(host(y), _oracle(p)) < F32_MAX_ABS


@pytest.mark.parametrize("B,C,nh,H,W", [(2, 128, 2, 7, 9), (1, 128, 2, 20, 20), (1, 256, 4, 8, 8)])
def test_fused_f32_backward_vs_autograd(cuda, B, C, nh, H, W):
    """va_psa_attention_bwd_f32 (the reference's backward node sequence in f32)
    against f64 autograd's vector-Jacobian product of the same block for an
    upstream gradient dy ~ N(0,1): every gradient block and dx within the f32
    bound, 1e-5 relative to the block's largest magnitude (weight gradients
    are sums over B·H·W tokens, up to ≈30 here)."""
    from vision_rs_b200 import _lib
    p = po.psa_synthetic(B, H, W, C=C, num_heads=nh, seed=5 + H)
    dy = np.random.default_rng(H * W).standard_normal((B, C, H, W)).astype(np.float32)
    prm = {k: p[k] for k in ("w_qkv", "b_qkv", "w_pe", "b_pe", "w_proj", "b_proj")}
    rg, rdx = po.psa_attention_vjp_torch(p["x"], dy, prm, num_heads=nh, key_dim=32)
    d = {k: dev(v) for k, v in prm.items()}
    x, dyd = dev(p["x"]), dev(dy)
    grads = torch.empty(rg.size, device="cuda")
    dx = torch.empty_like(x)
    need = int(_lib.lib().va_psa_attention_bwd_f32_workspace_bytes(B, C, H, W, nh, 32))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("va_psa_attention_bwd_f32", x.data_ptr(), dyd.data_ptr(), d["w_qkv"].data_ptr(), d["b_qkv"].data_ptr(),
              d["w_pe"].data_ptr(), d["b_pe"].data_ptr(), d["w_proj"].data_ptr(), d["b_proj"].data_ptr(),
              dx.data_ptr(), grads.data_ptr(), B, C, H, W, nh, 32, ws.data_ptr(), need, st)
    g = grads.cpu().numpy()
    qkv_h = nh * 128
    sizes = {"w_qkv": qkv_h * C, "w_proj": C * C, "w_pe": C * 9, "b_qkv": qkv_h, "b_proj": C, "b_pe": C}
    off = 0
    for k, n in sizes.items():
        ref = rg[off:off + n]
        assert max_abs(g[off:off + n], ref) <= F32_MAX_ABS * max(1.0, float(np.abs(ref).max())), k
        off += n
    assert max_abs(host(dx), rdx) <= F32_MAX_ABS
    # deterministic: a second call gives the same bits
    g2 = torch.empty_like(grads)
    _lib.call("va_psa_attention_bwd_f32", x.data_ptr(), dyd.data_ptr(), d["w_qkv"].data_ptr(), d["b_qkv"].data_ptr(),
              d["w_pe"].data_ptr(), d["b_pe"].data_ptr(), d["w_proj"].data_ptr(), d["b_proj"].data_ptr(),
              None, g2.data_ptr(), B, C, H, W, nh, 32, ws.data_ptr(), need, st)
    assert torch.equal(grads, g2)


def _bf16_inputs(p):
    q = dict(p)
    for k in ("x", "w_qkv", "w_pe", "w_proj"):
        q[k] = bf16_round(p[k])
    return q


@pytest.mark.parametrize("B,H,W", [(2, 4, 4), (2, 40, 40), (3, 20, 20), (1, 13, 11), (1, 3, 50)])
def test_fused_bf16_vs_oracle(cuda, B, H, W):
    p = _bf16_inputs(po.psa_synthetic(B, H, W, seed=7 + B * H))
    y = _op(p, torch.bfloat16)(dev(p["x"], torch.bfloat16))
    ref = _oracle(p)
    assert rel_l2(host(y), ref) < BF16_REL_L2
    assert max_abs(host(y), ref) < BF16_MAX_ABS


def test_fused_bf16_large_image_matches_f32_path(cuda):
    """A 120×120 map (14400 tokens; its PE plane is larger than the shared-memory
    staging of the fallback PE kernel, so only the register-window PE kernel can
    run it): the bf16 tensor-core op against the f32 op on the same bf16-rounded
    inputs (the f32 path is held to the oracle at 1e-5 above), bf16 bound."""
    p = _bf16_inputs(po.psa_synthetic(1, 120, 120, seed=120))
    y16 = host(_op(p, torch.bfloat16)(dev(p["x"], torch.bfloat16)))
    y32 = host(_op(p, torch.float32)(dev(p["x"])))
    assert rel_l2(y16, y32) < BF16_REL_L2
    assert max_abs(y16, y32) < BF16_MAX_ABS


def test_fused_bf16_full_cfg2_batch(cuda):
    """cfg2 at full size (64×128×40×40): images 0, 31 and 63 against the oracle,
    and a batch-consistency property (an image's output does not depend on its
    batch neighbours)."""
    p = _bf16_inputs(po.psa_synthetic(64, 40, 40, seed=2))
    op = _op(p, torch.bfloat16)
    x = dev(p["x"], torch.bfloat16)
    y = host(op(x))
    for i in (0, 31, 63):
        q = dict(p)
        q["x"] = p["x"][i:i + 1]
        ref = _oracle(q)
        assert rel_l2(y[i:i + 1], ref) < BF16_REL_L2 and max_abs(y[i:i + 1], ref) < BF16_MAX_ABS
    y_single = host(op(x[5:6].contiguous()))
    assert np.array_equal(y_single, y[5:6])


@pytest.mark.parametrize("C,B,H,W", [(256, 2, 20, 20), (384, 2, 40, 40), (256, 3, 13, 11), (64, 2, 9, 7)])
def test_fused_bf16_other_widths_vs_oracle(cuda, C, B, H, W):
    """The tensor-core forward at the other c2psa widths (num_heads = C/64,
    c2psa.rs:158): YOLO26 s/m/l (C = 256, 4 heads) and x (C = 384, 6 heads),
    plus one head and a ragged image, bf16 tolerance against the oracle."""
    nh = C // 64
    p = _bf16_inputs(po.psa_synthetic(B, H, W, C=C, num_heads=nh, seed=C + H))
    op = vp.PsaAttention(p["w_qkv"], p["b_qkv"], p["w_pe"], p["b_pe"], p["w_proj"], p["b_proj"], num_heads=nh,
                         key_dim=32, dtype=torch.bfloat16)
    y = host(op(dev(p["x"], torch.bfloat16)))
    ref = po.psa_attention(p["x"], p["w_qkv"], p["b_qkv"], p["w_pe"], p["b_pe"], p["w_proj"], p["b_proj"], nh, 32)
    assert rel_l2(y, ref) < BF16_REL_L2 and max_abs(y, ref) < BF16_MAX_ABS


def test_reference_node_sequence_matches_fused(cuda):
    """The reference graph's node sequence (c2psa.rs:74-114) run through the
    RuntimeOp mirror equals the fused entry point (f32)."""
    g = load_golden("psa_attn_case.npz")
    B, C, H, W = g["x"].shape
    nh, kd = 2, 32
    from vision_rs_b200 import _lib
    st = torch.cuda.current_stream().cuda_stream
    # keep every device tensor referenced while its raw pointer is in use
    x, wq, bq, wpe, bpe, wpr, bpr = (dev(g[k]) for k in ("x", "w_qkv", "b_qkv", "w_pe", "b_pe", "w_proj", "b_proj"))
    qkv = torch.empty(B, 256, H, W, device="cuda")
    _lib.call("va_conv1x1_bias_f32", x.data_ptr(), wq.data_ptr(), bq.data_ptr(), qkv.data_ptr(), B, C, 256, H * W, st)
    pk = vp.PsaPackQkvOp(kd, nh)
    shp = pk.infer_output_shape([list(qkv.shape)])
    packed = torch.empty(4, B * nh, H * W, kd, device="cuda")
    pk.inner.launch([(qkv, shp)], [], packed)
    lse = torch.empty(*vp.FlashAttn2PsaOp.new_lo(kd).inner.param_shapes([shp], None)[0], device="cuda")
    lo = torch.empty(B * nh, H * W, kd, device="cuda")
    hi = torch.empty_like(lo)
    vp.FlashAttn2PsaOp.new_lo(kd).inner.launch([(packed, shp)], [lse], lo)
    vp.FlashAttn2PsaOp.new_hi(kd).inner.launch([(packed, shp)], [lse], hi)
    merged = torch.empty(B, C, H, W, device="cuda")
    vp.PsaMergeAttnOp(kd, nh, H, W).inner.launch([lo, hi], [], merged)
    v = torch.empty(B, C, H, W, device="cuda")
    vp.PsaExtractVOp(kd, nh).inner.launch([qkv], [], v)
    pe = torch.empty_like(v)
    _lib.call("va_dwconv3x3_bias_f32", v.data_ptr(), wpe.data_ptr(), bpe.data_ptr(), pe.data_ptr(), B, C, H, W, st)
    y = torch.empty_like(v)
    s = (merged + pe).contiguous()
    _lib.call("va_conv1x1_bias_f32", s.data_ptr(), wpr.data_ptr(), bpr.data_ptr(), y.data_ptr(), B, C, C, H * W, st)
    assert max_abs(host(y), g["y"]) < F32_MAX_ABS


@pytest.mark.parametrize("B,H,W", [(1, 4, 4), (2, 20, 20), (2, 40, 40), (1, 13, 11), (3, 16, 16), (1, 8, 25)])
def test_tc_attention_core_vs_oracle(cuda, B, H, W):
    """The tcgen05 attention kernel alone (va_psa_flash_attention_fwd_f16):
    O = softmax(QKᵀ/√32)·V with 64-wide V, f16 operands, against the f64
    oracle on the same f16 values; LSE against the oracle's."""
    from vision_rs_b200 import _lib
    nh, N = 2, H * W
    Np = (N + 7) // 8 * 8
    rng = np.random.default_rng(N + B)
    f16 = lambda a: np.asarray(a, np.float32).astype(np.float16)
    qk = f16(rng.standard_normal((2, B * nh, N, 32)) * 0.6)
    vv = f16(rng.standard_normal((B, 128, N)))
    vpad = np.zeros((B, 128, Np), np.float16)
    vpad[:, :, :N] = vv
    qk_d = torch.as_tensor(qk).cuda()
    v_d = torch.as_tensor(vpad).cuda()
    o_d = torch.zeros(B, 128, Np, dtype=torch.float16, device="cuda")
    l_d = torch.zeros(B * nh, N, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("va_psa_flash_attention_fwd_f16", qk_d.data_ptr(), v_d.data_ptr(), o_d.data_ptr(), l_d.data_ptr(),
              B, nh, H, W, st)
    o = o_d.float().cpu().numpy()[:, :, :N]
    v_t = vv.astype(np.float32).reshape(B, nh, 64, N).transpose(0, 1, 3, 2).reshape(B * nh, N, 64)
    ro, rl = po.flash_attention2_forward(qk[0].astype(np.float32), qk[1].astype(np.float32), v_t, SCALE)
    ro = ro.reshape(B, nh, N, 64).transpose(0, 1, 3, 2).reshape(B, 128, N)
    assert rel_l2(o, ro) < 2e-3 and max_abs(o, ro) < 1e-2
    assert max_abs(l_d.cpu().numpy(), rl) < 2e-3
    status = __import__("ctypes").c_int(-1)
    _lib.call("va_device_status_read", __import__("ctypes").byref(status), st)
    assert status.value == 0


@pytest.mark.parametrize("B,H,W", [(1, 20, 20), (2, 40, 40), (1, 11, 13)])
def test_tc_attention_core_peaked(cuda, B, H, W):
    """Strongly peaked attention (one dominant key per query, at every key
    position mod 128, incl. the ragged last tile): exercises the running-max
    rescale and the row max over every column of a tile."""
    from vision_rs_b200 import _lib
    nh, N = 2, H * W
    Np = (N + 7) // 8 * 8
    rng = np.random.default_rng(11)
    q = rng.standard_normal((B * nh, N, 32)) * 0.1
    k = rng.standard_normal((B * nh, N, 32)) * 0.1
    # queries and a third of the keys point in 2-D directions with norm 10:
    # scores up to 100 (≈25 in scaled log2 units) against ~0 elsewhere, the
    # arg-max key varying with the query
    th = rng.uniform(0, 2 * np.pi, (B * nh, N))
    q[:, :, 0], q[:, :, 1] = 10 * np.cos(th), 10 * np.sin(th)
    hot = rng.permutation(N)[: max(1, N // 3)]
    ph = rng.uniform(0, 2 * np.pi, (B * nh, hot.size))
    k[:, hot, 0], k[:, hot, 1] = 10 * np.cos(ph), 10 * np.sin(ph)
    qk = np.stack([q, k]).astype(np.float16)
    vv = rng.standard_normal((B, 128, N)).astype(np.float16)
    vpad = np.zeros((B, 128, Np), np.float16)
    vpad[:, :, :N] = vv
    qk_d, v_d = torch.as_tensor(qk).cuda(), torch.as_tensor(vpad).cuda()
    o_d = torch.zeros(B, 128, Np, dtype=torch.float16, device="cuda")
    l_d = torch.zeros(B * nh, N, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("va_psa_flash_attention_fwd_f16", qk_d.data_ptr(), v_d.data_ptr(), o_d.data_ptr(), l_d.data_ptr(),
              B, nh, H, W, st)
    o = o_d.float().cpu().numpy()[:, :, :N]
    assert np.isfinite(o).all()
    v_t = vv.astype(np.float32).reshape(B, nh, 64, N).transpose(0, 1, 3, 2).reshape(B * nh, N, 64)
    ro, rl = po.flash_attention2_forward(qk[0].astype(np.float32), qk[1].astype(np.float32), v_t, SCALE)
    ro = ro.reshape(B, nh, N, 64).transpose(0, 1, 3, 2).reshape(B, 128, N)
    assert rel_l2(o, ro) < 2e-3 and max_abs(o, ro) < 1e-2
    assert max_abs(l_d.cpu().numpy(), rl) < 2e-3
