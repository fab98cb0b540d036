"""PSA Attention training step (cfg5 shapes) on the B200 against torch-CPU
float64 autograd of the same BN-folded block, on the same bf16 operands.

bf16 mode: rel-L2 ≤ 2e-3 and max-abs ≤ 1e-2 against the f64 reference for
the output y, dx and every gradient block.
"""
import numpy as np
import pytest
import torch

from conftest import BF16_MAX_ABS, BF16_REL_L2, max_abs, rel_l2
from oracle import psa_oracle as po

pytestmark = pytest.mark.gpu

SLICES = {"w_qkv": (0, 32768), "w_proj": (32768, 49152), "w_pe": (49152, 50304), "b_qkv": (50304, 50560),
          "b_proj": (50560, 50688), "b_pe": (50688, 50816)}


def _bf(a, dev):
    return torch.as_tensor(np.asarray(a, np.float32)).to(dev, torch.bfloat16)


def _case(B, H, W, seed, dev):
    s = po.psa_synthetic(B, H, W, seed=seed)
    rng = np.random.default_rng(seed + 1)
    tgt = rng.standard_normal((B, 128, H, W)).astype(np.float32)
    dv = {k: _bf(s[k], dev) for k in ("x", "w_qkv", "w_pe", "w_proj")}
    dv.update({k: torch.as_tensor(s[k]).to(dev) for k in ("b_qkv", "b_pe", "b_proj")})
    dv["target"] = _bf(tgt, dev)
    host = {k: (dv[k].float().cpu().numpy() if dv[k].dtype == torch.bfloat16 else s[k]) for k in dv}
    return dv, host


def _check(got, ref, what):
    assert rel_l2(got, ref) <= BF16_REL_L2, (what, rel_l2(got, ref))
    assert max_abs(got, ref) <= BF16_MAX_ABS * max(1.0, np.abs(ref).max()), (what, max_abs(got, ref))


@pytest.mark.parametrize("a_mn,b_mn,c_bf16", [(0, 0, 0), (1, 0, 0), (0, 1, 0), (1, 1, 1)])
def test_gemm_layouts(cuda, a_mn, b_mn, c_bf16):
    from vision_rs_b200 import _lib
    from vision_rs_b200.psa import _p, _stream
    rng = np.random.default_rng(7)
    Z, M, N, K = 3, 200, 136, 200
    A = rng.standard_normal((Z, M, K)).astype(np.float32)
    Bm = rng.standard_normal((Z, N, K)).astype(np.float32)
    at = torch.as_tensor(A.transpose(0, 2, 1).copy() if a_mn else A).to(cuda, torch.float16)
    bt = torch.as_tensor(Bm.transpose(0, 2, 1).copy() if b_mn else Bm).to(cuda, torch.float16)
    c = torch.zeros(Z, M, N, device=cuda, dtype=torch.bfloat16 if c_bf16 else torch.float32)
    lda = M if a_mn else K
    ldb = N if b_mn else K
    _lib.call("va_gemm_f16", _p(at), a_mn, lda, M * K, 0, _p(bt), b_mn, ldb, N * K, 0, _p(c), c_bf16, N, M * N,
              M, N, K, Z, 0.5, _stream())
    a16 = A.astype(np.float16).astype(np.float64)
    b16 = Bm.astype(np.float16).astype(np.float64)
    ref = 0.5 * np.einsum("zmk,znk->zmn", a16, b16)
    got = c.float().cpu().numpy()
    tol = 1e-2 if c_bf16 else 1e-5
    assert np.abs(got - ref).max() <= tol * np.abs(ref).max()


def test_train_step_cfg5_shard(cuda):
    """One rank's shard at cfg5 shapes (32 × 128×20×20)."""
    from vision_rs_b200 import train
    dv, h = _case(32, 20, 20, 11, cuda)
    step = train.PsaTrainStep(B=32, H=20, W=20, device=cuda)
    y, loss, grads, dx = step.forward_backward(dv["x"], dv["target"], dv, want_dx=True)
    params = {k: h[k] for k in ("w_qkv", "b_qkv", "w_pe", "b_pe", "w_proj", "b_proj")}
    ry, rloss, rg, rdx = po.psa_train_step_torch(h["x"], h["target"], params)
    _check(y.float().cpu().numpy(), ry, "y")
    assert abs(float(loss) - rloss) <= 2e-3 * rloss
    g = grads.cpu().numpy()
    for name, (a, b) in SLICES.items():
        _check(g[a:b], rg[a:b], name)
    _check(dx.float().cpu().numpy(), rdx, "dx")


def test_train_step_deterministic(cuda):
    from vision_rs_b200 import train
    dv, _ = _case(4, 20, 20, 12, cuda)
    step = train.PsaTrainStep(B=4, H=20, W=20, device=cuda)
    g1 = step.forward_backward(dv["x"], dv["target"], dv)[2].clone()
    g2 = step.forward_backward(dv["x"], dv["target"], dv)[2].clone()
    assert torch.equal(g1, g2)


def test_train_step_odd_size(cuda):
    """N = 15×13 (not a multiple of 8: padded rows)."""
    from vision_rs_b200 import train
    dv, h = _case(3, 15, 13, 13, cuda)
    step = train.PsaTrainStep(B=3, H=15, W=13, device=cuda)
    y, loss, grads, dx = step.forward_backward(dv["x"], dv["target"], dv, want_dx=True)
    params = {k: h[k] for k in ("w_qkv", "b_qkv", "w_pe", "b_pe", "w_proj", "b_proj")}
    ry, rloss, rg, rdx = po.psa_train_step_torch(h["x"], h["target"], params)
    _check(y.float().cpu().numpy(), ry, "y")
    g = grads.cpu().numpy()
    for name, (a, b) in SLICES.items():
        _check(g[a:b], rg[a:b], name)
    _check(dx.float().cpu().numpy(), rdx, "dx")


def test_sgd_update(cuda):
    from vision_rs_b200 import train
    dv, h = _case(2, 20, 20, 14, cuda)
    step = train.PsaTrainStep(B=2, H=20, W=20, device=cuda)
    master = step.master_from(dv)
    g = torch.randn(master.numel(), device=cuda)
    before = master.clone()
    step.sgd(master, g, dv, lr=0.1, grad_scale=0.5)
    assert torch.allclose(master, before - 0.05 * g)
    wq = dv["w_qkv"].float().reshape(-1)
    assert torch.equal(dv["w_qkv"].reshape(-1), master[:32768].to(torch.bfloat16))
    assert torch.equal(dv["b_pe"], master[50688:])
    del wq


def test_train_step_long_sequence_fallback(cuda):
    """N = 24×24 = 576 > 512: the attention backward takes the f32 SIMT path."""
    from vision_rs_b200 import train
    dv, h = _case(2, 24, 24, 15, cuda)
    step = train.PsaTrainStep(B=2, H=24, W=24, device=cuda)
    y, loss, grads, dx = step.forward_backward(dv["x"], dv["target"], dv, want_dx=True)
    params = {k: h[k] for k in ("w_qkv", "b_qkv", "w_pe", "b_pe", "w_proj", "b_proj")}
    ry, rloss, rg, rdx = po.psa_train_step_torch(h["x"], h["target"], params)
    g = grads.cpu().numpy()
    for name, (a, b) in SLICES.items():
        _check(g[a:b], rg[a:b], name)
    _check(dx.float().cpu().numpy(), rdx, "dx")


def test_graph_replay_matches_eager(cuda):
    """The CUDA-graph replay of the training step gives bit-identical outputs
    to the eager launches (same kernels, same order)."""
    from vision_rs_b200 import train
    dv, _ = _case(4, 20, 20, 21, cuda)
    eager = train.PsaTrainStep(B=4, H=20, W=20, device=cuda)
    ge = [t.clone() for t in eager.forward_backward(dv["x"], dv["target"], dv)[:3]]
    graphed = train.PsaTrainStep(B=4, H=20, W=20, device=cuda, graph=True)
    for _ in range(3):  # eager set-up + capture, then replays
        got = graphed.forward_backward(dv["x"], dv["target"], dv)[:3]
        torch.cuda.synchronize()
        for a, b in zip(got, ge):
            assert torch.equal(a, b)
    assert graphed.graph_kernels > 0 and graphed.replayed_kernels == 3 * graphed.graph_kernels


@pytest.mark.parametrize("B,H,W,dscale", [(4, 20, 20, 1e-3), (2, 13, 11, 1.0), (32, 20, 20, 2.0 / (32 * 128 * 400))])
def test_attention_backward_any_loss(cuda, B, H, W, dscale):
    """va_psa_attention_bwd_bf16: the fused op's backward for an upstream
    gradient dy (here N(0,1)·dscale, dy_scale = dscale) against f64 autograd
    of the same block, every gradient block and dx at the bf16 bound."""
    from vision_rs_b200 import _lib
    dv, host = _case(B, H, W, 11 + B, "cuda")
    rng = np.random.default_rng(B + H)
    dy_h = torch.as_tensor(rng.standard_normal((B, 128, H, W)).astype(np.float32) * dscale).bfloat16()
    dy = dy_h.cuda()
    grads = torch.empty(50816, device="cuda")
    dx = torch.empty_like(dv["x"])
    need = int(_lib.lib().va_psa_attention_bwd_workspace_bytes(B, H, W))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    _lib.call("va_psa_attention_bwd_bf16", dv["x"].data_ptr(), dy.data_ptr(), float(dscale),
              dv["w_qkv"].data_ptr(), dv["b_qkv"].data_ptr(), dv["w_pe"].data_ptr(), dv["b_pe"].data_ptr(),
              dv["w_proj"].data_ptr(), dv["b_proj"].data_ptr(), dx.data_ptr(), grads.data_ptr(), B, 128, H, W, 2, 32,
              ws.data_ptr(), need, torch.cuda.current_stream().cuda_stream)
    prm = {k: host[k] for k in ("w_qkv", "b_qkv", "w_pe", "b_pe", "w_proj", "b_proj")}
    rg, rdx = po.psa_attention_vjp_torch(host["x"], dy_h.float().numpy(), prm)
    g = grads.cpu().numpy()
    for k, (a, b) in SLICES.items():
        _check(g[a:b], rg[a:b], k)
    _check(dx.float().cpu().numpy(), rdx, "dx")
