"""The CPU oracle against the reference's own golden fixtures (no GPU).

Pins ``oracle/psa_oracle.py`` before it is trusted as the parity checker:
the reference's ultralytics/PyTorch-generated fixtures for the PSA block
(tests/fixtures/c2psa_yolo26 of the reference crate), the PE-shaped
depthwise conv (tests/fixtures/conv_grouped/depthwise), and
``oracle/conv_oracle.py`` on the YOLO26n stem conv (tests/fixtures/conv_yolo26)
and three eval-mode C3k2 blocks (tests/fixtures/c3k2_yolo26)."""
import numpy as np

from conftest import folded_c2psa, load_golden, max_abs, stage_params
from oracle import conv_oracle as co
from oracle import psa_oracle as po

SCALE = 1.0 / np.sqrt(np.float32(32))


def test_c2psa_eval_forward_matches_reference_fixture():
    g = load_golden("c2psa_fwd.npz")
    y = po.c2psa_forward_eval(g["x"], stage_params(g))
    # reference tolerance 1e-3 (test_c2psa_cuda.rs:673); the oracle is far inside it
    assert max_abs(y, g["expected_output"]) < 1e-5


def test_c2psa_folded_forward_matches_reference_fixture():
    """The BN-folded PSABlock / C2PSA restatement (the form the fused ops take)."""
    g = load_golden("c2psa_fwd.npz")
    w_cv1, b_cv1, blocks, w_cv2, b_cv2 = folded_c2psa(g)
    y = po.c2psa_forward_folded(g["x"], w_cv1, b_cv1, blocks, w_cv2, b_cv2)
    assert max_abs(y, g["expected_output"]) < 1e-5


def test_c2psa_train_backward_matches_reference_fixture():
    g = load_golden("c2psa_bwd.npz")
    y, dx, fa = po.c2psa_backward_train_torch(g["x"], g["dy"], stage_params(g))
    assert max_abs(y, g["expected_output"]) < 1e-4
    assert max_abs(dx, g["dx_expected"]) < 1e-4  # reference tol 5e-3 (test_c2psa_backward_cuda.rs:701)
    for n in ("q", "k", "v_lo", "v_hi", "o_lo", "o_hi", "l"):
        assert max_abs(fa[n], g["attn_" + n]) < 1e-5, n


def test_fa_forward_known_answer():
    g = load_golden("c2psa_bwd.npz")
    for half in ("lo", "hi"):
        o, l = po.flash_attention2_forward(g["attn_q"], g["attn_k"], g[f"attn_v_{half}"], SCALE)
        assert max_abs(o, g[f"attn_o_{half}"]) < 1e-6
        assert max_abs(l, g["attn_l"]) < 1e-6


def test_fa_backward_matches_autograd():
    import torch
    g = load_golden("c2psa_bwd.npz")
    rng = np.random.default_rng(0)
    q, k, v = (torch.tensor(g[f"attn_{n}"], dtype=torch.float64, requires_grad=True) for n in ("q", "k", "v_lo"))
    s = (q @ k.transpose(1, 2)) * float(SCALE)
    o = s.softmax(-1) @ v
    do = torch.tensor(rng.standard_normal(o.shape))
    o.backward(do)
    lse = torch.logsumexp(s, -1).detach().numpy()
    on = o.detach().numpy()
    dq0 = rng.standard_normal(q.shape).astype(np.float32)
    dk0 = rng.standard_normal(k.shape).astype(np.float32)
    dq, dk, dv = po.psa_fa2_backward(g["attn_q"], g["attn_k"], g["attn_v_lo"], on, do.numpy(), lse, SCALE,
                                     dq_acc=dq0, dk_acc=dk0)
    assert max_abs(dq - dq0, q.grad.numpy()) < 1e-5
    assert max_abs(dk - dk0, k.grad.numpy()) < 1e-5
    assert max_abs(dv, v.grad.numpy()) < 1e-6


def test_depthwise_conv_fixture():
    g = load_golden("dwconv_depthwise.npz")
    y = po.dwconv3x3(g["x"], g["conv_w"])
    assert max_abs(y, g["expected_output"]) < 1e-5   # test_conv_grouped_cuda.rs tol 1e-5
    dx, dw = po.dwconv3x3_backward(g["x"], g["conv_w"], g["dy"])
    assert max_abs(dx, g["dx_expected"]) < 1e-4      # test_conv_grouped_backward_cuda.rs tol 1e-4
    assert max_abs(dw, g["dw_expected"]) < 1e-4


def test_layout_ops_roundtrip_and_backward_adjointness():
    rng = np.random.default_rng(1)
    B, nh, kd, H, W = 2, 2, 32, 5, 3
    qkv = rng.standard_normal((B, nh * 4 * kd, H, W)).astype(np.float32)
    packed = po.pack_qkv(qkv, nh)
    assert packed.shape == (4, B * nh, H * W, kd)
    # pack is a permutation: its backward scatters every element back
    back = po.pack_qkv_backward(packed, B, nh * 4 * kd, H, W, nh)
    assert np.array_equal(back, qkv)
    v = po.extract_v_nchw(qkv, nh)
    merged = po.merge_attn_nchw(packed[2], packed[3], nh, H, W)
    assert np.array_equal(v, merged)  # V sections re-merged == extracted V
    dlo, dhi = po.merge_attn_backward(merged, nh)
    assert np.array_equal(dlo, packed[2]) and np.array_equal(dhi, packed[3])
    dq = po.extract_v_backward(v, nh * 4 * kd, nh)
    assert np.array_equal(po.extract_v_nchw(dq, nh), v)


def test_psa_attention_case_consistent():
    g = load_golden("psa_attn_case.npz")
    y = po.psa_attention(g["x"], g["w_qkv"], g["b_qkv"], g["w_pe"], g["b_pe"], g["w_proj"], g["b_proj"], 2, 32)
    assert max_abs(y, g["y"]) < 1e-6


def test_torch_cpu_baseline_matches_oracle():
    import torch
    p = po.psa_synthetic(2, 9, 7, seed=11)
    t = {k: torch.tensor(v) for k, v in p.items()}
    y = po.psa_attention_torch(t["x"], t["w_qkv"], t["b_qkv"], t["w_pe"], t["b_pe"], t["w_proj"], t["b_proj"], 2, 32)
    ref = po.psa_attention(p["x"], p["w_qkv"], p["b_qkv"], p["w_pe"], p["b_pe"], p["w_proj"], p["b_proj"], 2, 32)
    assert max_abs(y.numpy(), ref) < 1e-5


def _conv_prm(g, v):
    stages = {k[len(v) + 1:-len("_conv_w")] for k in g if k.startswith(v + "/") and k.endswith("_conv_w")}
    return {s: tuple(g[f"{v}/{s}_{p}"] for p in ("conv_w", "bn_w", "bn_b", "bn_rm", "bn_rv")) for s in stages}


def test_stem_conv_fixture():
    """Conv(3→16, k3, s2) + training-mode BN + SiLU (conv_yolo26/generate.py)."""
    g = load_golden("conv_c3k2.npz")
    y = co.conv_block_train(g["stem/x"], (g["stem/conv_w"], g["stem/bn_w"], g["stem/bn_b"]), stride=2)
    assert max_abs(y, g["stem/expected_output"]) < 1e-5


def test_c3k2_fixtures():
    """C3k2 without / with shortcut and the C3k inner variant (c3k2.rs:46-127)."""
    g = load_golden("conv_c3k2.npz")
    for v, c3k, sc in (("shallow_sf", False, False), ("shallow_st", False, True), ("deep_st", True, True)):
        y = co.c3k2(g[f"{v}/x"], _conv_prm(g, v), c3k, sc)
        assert max_abs(y, g[f"{v}/expected_output"]) < 1e-5, v


def test_conv2d_matches_torch():
    """The conv restatement against torch's CPU conv2d (f64) for every kernel
    size and stride the GPU op takes."""
    import torch
    for k, s in ((1, 1), (1, 2), (3, 1), (3, 2)):
        x, w, b = co.conv_synthetic(2, 8, 9, 7, 16, k, seed=k + s)
        ref = torch.nn.functional.conv2d(torch.tensor(x), torch.tensor(w), torch.tensor(b), stride=s, padding=k // 2)
        assert max_abs(co.conv2d(x, w, s, b), ref.numpy()) < 1e-12
