"""CPU restatement of the vision-rs PSA attention path.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
library in ``vision_rs_b200``; only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product path never calls into it and has no CPU fallback.

Every function restates the reference's arithmetic (spinorml/vision-rs,
paths relative to the reference crate root) in numpy, computing in float64 and
returning float32 unless noted:

* ``pack_qkv``            — ``src/models/yolo/kernels/attention/psa.rs:58-94``
* ``pack_qkv_backward``   — ``psa.rs:201-233``
* ``extract_v_nchw``      — ``psa.rs:105-142``
* ``extract_v_backward``  — ``psa.rs:244-281``
* ``merge_attn_nchw``     — ``psa.rs:153-189``
* ``merge_attn_backward`` — ``psa.rs:292-327``
* ``flash_attention2_forward`` — ``src/models/yolo/kernels/attention/flash_attn2.rs:54-121``
  (online softmax; the result equals exact softmax attention; LSE = m + ln l)
* ``flash_attention2_backward_dq`` / ``_dkv`` — ``flash_attn2.rs:129-260``
* ``psa_fa2_backward``    — ``psa.rs:650-725`` (dq, dk accumulated; dv stored)
* ``psa_attention``       — the graph in ``src/models/yolo/yolo26/blocks/c2psa.rs:61-116``
  (qkv conv+BN → pack → FA lo/hi → merge; extract_v → pe dw-conv+BN; add;
  proj conv+BN), with BN folded into conv weight + bias as ``graph.optimise()``
  does (``examples/yolo26.rs:3021``).
* ``c2psa_forward_eval``  — ``c2psa.rs:150-179`` + ``psa_block`` ``c2psa.rs:123-137``,
  used to pin this oracle against the reference's golden fixtures
  (``tests/fixtures/c2psa_yolo26/generate.py``).
* ``psa_block_forward`` / ``c2psa_forward_folded`` — the same block and
  C2PSA with BN folded (the form the fused bf16 ops take), checked against
  ``c2psa_forward_eval`` in ``tests/test_oracle_golden.py``.

Parity pin: ``tests/test_oracle_golden.py`` checks these functions against
the reference's committed PyTorch-generated fixtures (copied into
``tests/golden/`` by ``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import numpy as np

F64 = np.float64


def _f64(a):
    return np.asarray(a, dtype=F64)


# ── layout ops (psa.rs) ──────────────────────────────────────────────────────

def pack_qkv(qkv: np.ndarray, num_heads: int) -> np.ndarray:
    """``psa_pack_qkv`` (psa.rs:58-94): NCHW ``[B, qkv_h, H, W]`` → flat
    ``[4, B*nh, N, kd]``; channel ``h*4*kd + s*kd + d`` goes to section ``s``."""
    B, qkv_h, H, W = qkv.shape
    kd = qkv_h // (4 * num_heads)
    x = np.asarray(qkv).reshape(B, num_heads, 4, kd, H * W)
    return np.ascontiguousarray(x.transpose(2, 0, 1, 4, 3)).reshape(4, B * num_heads, H * W, kd)


def pack_qkv_backward(d_packed: np.ndarray, B: int, qkv_h: int, H: int, W: int,
                      num_heads: int, d_qkv: np.ndarray | None = None) -> np.ndarray:
    """``psa_pack_qkv_backward`` (psa.rs:201-233): scatter-add into ``d_qkv``."""
    kd = qkv_h // (4 * num_heads)
    if d_qkv is None:
        d_qkv = np.zeros((B, qkv_h, H, W), np.float32)
    g = np.asarray(d_packed).reshape(4, B, num_heads, H * W, kd).transpose(1, 2, 0, 4, 3)
    out = _f64(d_qkv).reshape(B, num_heads, 4, kd, H * W) + g
    return out.reshape(B, qkv_h, H, W).astype(np.float32)


def extract_v_nchw(qkv: np.ndarray, num_heads: int) -> np.ndarray:
    """``psa_extract_v_nchw`` (psa.rs:105-142): V_lo|V_hi channels of each head
    → NCHW ``[B, c, H, W]`` with ``c = qkv_h/2``, channel ``h*2*kd + d``."""
    B, qkv_h, H, W = qkv.shape
    kd = qkv_h // (4 * num_heads)
    x = np.asarray(qkv).reshape(B, num_heads, 4 * kd, H, W)
    return np.ascontiguousarray(x[:, :, 2 * kd:]).reshape(B, num_heads * 2 * kd, H, W)


def extract_v_backward(d_v: np.ndarray, qkv_h: int, num_heads: int,
                       d_qkv: np.ndarray | None = None) -> np.ndarray:
    """``psa_extract_v_backward`` (psa.rs:244-281): add ``d_v`` into the V
    sections of ``d_qkv``."""
    B, c, H, W = d_v.shape
    kd = qkv_h // (4 * num_heads)
    if d_qkv is None:
        d_qkv = np.zeros((B, qkv_h, H, W), np.float32)
    out = _f64(d_qkv).reshape(B, num_heads, 4 * kd, H, W).copy()
    out[:, :, 2 * kd:] += np.asarray(d_v).reshape(B, num_heads, 2 * kd, H, W)
    return out.reshape(B, qkv_h, H, W).astype(np.float32)


def merge_attn_nchw(lo: np.ndarray, hi: np.ndarray, num_heads: int, H: int, W: int) -> np.ndarray:
    """``psa_merge_attn_nchw`` (psa.rs:153-189): two ``[BH, N, kd]`` halves →
    NCHW ``[B, nh*2*kd, H, W]``; lo → channels ``h*2kd + d``, hi → ``+kd``."""
    BH, N, kd = lo.shape
    B = BH // num_heads
    both = np.concatenate([np.asarray(lo), np.asarray(hi)], axis=2)  # [BH, N, 2kd]
    x = both.reshape(B, num_heads, N, 2 * kd).transpose(0, 1, 3, 2)
    return np.ascontiguousarray(x).reshape(B, num_heads * 2 * kd, H, W)


def merge_attn_backward(d_merged: np.ndarray, num_heads: int):
    """``psa_merge_attn_backward`` (psa.rs:292-327): NCHW grad → (d_lo, d_hi)."""
    B, c, H, W = d_merged.shape
    kd = c // (2 * num_heads)
    x = np.asarray(d_merged).reshape(B, num_heads, 2 * kd, H * W).transpose(0, 1, 3, 2)
    x = x.reshape(B * num_heads, H * W, 2 * kd)
    return np.ascontiguousarray(x[:, :, :kd]), np.ascontiguousarray(x[:, :, kd:])


# ── flash attention (flash_attn2.rs) ─────────────────────────────────────────

def flash_attention2_forward(q, k, v, softmax_scale: float):
    """``flash_attention2_forward`` (flash_attn2.rs:54-121) on ``[BH, N, D]``.

    Returns ``(o [BH,Nq,Dv] f32, l [BH,Nq] f32)`` with ``l = m + ln(sum exp(s-m))``
    (flash_attn2.rs:113-118).  The online recurrence equals exact softmax."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    s = np.einsum("bnd,bmd->bnm", q, k) * softmax_scale
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    o = np.einsum("bnm,bmd->bnd", p / l, v)
    return o.astype(np.float32), (m + np.log(l))[..., 0].astype(np.float32)


def _fa_recompute(q, k, v, o, do, lse, scale):
    q, k, v, o, do, lse = map(_f64, (q, k, v, o, do, lse))
    s = np.einsum("bnd,bmd->bnm", q, k) * scale
    p = np.exp(s - lse[..., None])                      # flash_attn2.rs:167-168
    dmat = (o * do).sum(-1)                             # D = rowsum(O*dO) :155
    dp = np.einsum("bnd,bmd->bnm", do, v)
    ds = p * (dp - dmat[..., None])                     # :171-172
    return q, k, p, ds, do


def flash_attention2_backward_dq(q, k, v, o, do, lse, scale):
    """``flash_attention2_backward_dq`` (flash_attn2.rs:129-187)."""
    q, k, p, ds, _ = _fa_recompute(q, k, v, o, do, lse, scale)
    return (np.einsum("bnm,bmd->bnd", ds, k) * scale).astype(np.float32)


def flash_attention2_backward_dkv(q, k, v, o, do, lse, scale):
    """``flash_attention2_backward_dkv`` (flash_attn2.rs:195-260): (dk, dv)."""
    q, k, p, ds, do = _fa_recompute(q, k, v, o, do, lse, scale)
    dk = np.einsum("bnm,bnd->bmd", ds, q) * scale
    dv = np.einsum("bnm,bnd->bmd", p, do)
    return dk.astype(np.float32), dv.astype(np.float32)


def psa_fa2_backward(q, k, v, o, do, lse, scale, dq_acc=None, dk_acc=None):
    """``psa_fa2_backward`` (psa.rs:650-725): returns ``(dq_acc+dq, dk_acc+dk, dv)``
    — dq and dk are accumulated (atomic_add in the reference, :700, :723),
    dv is stored (:724)."""
    dq = flash_attention2_backward_dq(q, k, v, o, do, lse, scale)
    dk, dv = flash_attention2_backward_dkv(q, k, v, o, do, lse, scale)
    if dq_acc is not None:
        dq = (_f64(dq_acc) + dq).astype(np.float32)
    if dk_acc is not None:
        dk = (_f64(dk_acc) + dk).astype(np.float32)
    return dq, dk, dv


# ── convolutions / BN (teeny-kernels semantics, NCHW) ────────────────────────

def fold_bn(w, gamma, beta, mean, var, eps):
    """Fold eval-mode BatchNorm into the preceding bias-free conv:
    ``w' = w·γ/√(σ²+ε)``, ``b' = β − μ·γ/√(σ²+ε)`` (what ``graph.optimise()``
    does for Conv+BN, examples/yolo26.rs:3021, 3445)."""
    w, gamma, beta, mean, var = map(_f64, (w, gamma, beta, mean, var))
    s = gamma / np.sqrt(var + eps)
    return (w * s.reshape(-1, *([1] * (w.ndim - 1)))), beta - mean * s


def conv1x1(x, w, b=None):
    """1×1 conv, NCHW: ``y[b,o] = Σ_i w[o,i]·x[b,i] (+ bias[o])``."""
    x, w = _f64(x), _f64(w).reshape(w.shape[0], -1)
    y = np.einsum("oi,bihw->bohw", w, x)
    if b is not None:
        y = y + _f64(b)[None, :, None, None]
    return y


def dwconv3x3(x, w, b=None):
    """Depthwise 3×3 conv, stride 1, zero pad 1 (``conv_bn(c,c,3,1,c)``,
    c2psa.rs:66): ``y[b,c,i,j] = Σ w[c,0,di,dj]·x[b,c,i+di-1,j+dj-1]``."""
    x, w = _f64(x), _f64(w).reshape(-1, 3, 3)
    B, C, H, W = x.shape
    xp = np.zeros((B, C, H + 2, W + 2), F64)
    xp[:, :, 1:H + 1, 1:W + 1] = x
    y = np.zeros_like(x)
    for di in range(3):
        for dj in range(3):
            y += w[None, :, di, dj, None, None] * xp[:, :, di:di + H, dj:dj + W]
    if b is not None:
        y = y + _f64(b)[None, :, None, None]
    return y


def dwconv3x3_backward(x, w, dy):
    """(dx, dw) of ``dwconv3x3`` (no bias)."""
    x, w, dy = _f64(x), _f64(w).reshape(-1, 3, 3), _f64(dy)
    B, C, H, W = x.shape
    xp = np.zeros((B, C, H + 2, W + 2), F64)
    xp[:, :, 1:H + 1, 1:W + 1] = x
    dxp = np.zeros_like(xp)
    dw = np.zeros((C, 3, 3), F64)
    for di in range(3):
        for dj in range(3):
            dw[:, di, dj] = (dy * xp[:, :, di:di + H, dj:dj + W]).sum(axis=(0, 2, 3))
            dxp[:, :, di:di + H, dj:dj + W] += w[None, :, di, dj, None, None] * dy
    return dxp[:, :, 1:H + 1, 1:W + 1], dw.reshape(C, 1, 3, 3)


def silu(x):
    return x / (1.0 + np.exp(-x))


# ── PSA attention (c2psa.rs:61-116) ──────────────────────────────────────────

def psa_attention(x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, num_heads: int, key_dim: int,
                  return_parts: bool = False):
    """The YOLO26 PSA ``Attention`` forward with BN already folded.

    Follows the reference graph node by node: qkv = conv1x1(x)+b (c2psa.rs:74);
    packed = pack_qkv (c2psa.rs:77-81); lo/hi = FA(Q,K,V_lo/V_hi) with
    scale ``1/√kd`` (psa.rs:986, c2psa.rs:84-93); merged = merge (c2psa.rs:96-100);
    v = extract_v (c2psa.rs:103-107); pe = dw3x3(v)+b (c2psa.rs:110);
    y = conv1x1(merged + pe) + b (c2psa.rs:111-114)."""
    x = _f64(x)
    B, C, H, W = x.shape
    qkv = conv1x1(x, w_qkv, b_qkv)
    packed = pack_qkv(qkv, num_heads)
    scale = 1.0 / np.sqrt(np.float32(key_dim))
    q, k, vlo, vhi = packed[0], packed[1], packed[2], packed[3]
    o_lo, lse = flash_attention2_forward(q, k, vlo, scale)
    o_hi, _ = flash_attention2_forward(q, k, vhi, scale)
    # Re-evaluate the attention in f64 for the returned output (the f32 casts
    # inside flash_attention2_forward are only for the op-level API).
    s = np.einsum("bnd,bmd->bnm", _f64(q), _f64(k)) * scale
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    lo64 = np.einsum("bnm,bmd->bnd", p, _f64(vlo))
    hi64 = np.einsum("bnm,bmd->bnd", p, _f64(vhi))
    merged = merge_attn_nchw(lo64, hi64, num_heads, H, W)
    v = extract_v_nchw(qkv, num_heads)
    pe = dwconv3x3(v, w_pe, b_pe)
    y = conv1x1(merged + pe, w_proj, b_proj)
    if return_parts:
        return y, dict(qkv=qkv, packed=packed, o_lo=o_lo, o_hi=o_hi, lse=lse,
                       merged=merged, v=v, pe=pe)
    return y


def psa_block_forward(x, w: dict, num_heads: int, key_dim: int = 32):
    """PSABlock with BN folded (``psa_block``, c2psa.rs:123-137):
    b = x + attn(x); out = b + ffn1(SiLU(ffn0(b))), ffn0 = conv1x1 C→2C (+ bias,
    SiLU: ``conv``, conv.rs:31-45), ffn1 = conv1x1 2C→C (+ bias: ``conv_bn``,
    conv.rs:53-69).  ``w`` holds w_qkv … b_proj (as psa_attention takes them)
    and w_ffn0, b_ffn0, w_ffn1, b_ffn1."""
    x = _f64(x)
    b = x + psa_attention(x, w["w_qkv"], w["b_qkv"], w["w_pe"], w["b_pe"], w["w_proj"], w["b_proj"], num_heads,
                          key_dim)
    return b + conv1x1(silu(conv1x1(b, w["w_ffn0"], w["b_ffn0"])), w["w_ffn1"], w["b_ffn1"])


def c2psa_forward_folded(x, w_cv1, b_cv1, blocks: list, w_cv2, b_cv2, key_dim: int = 32):
    """C2PSA with BN folded (c2psa.rs:150-179): h = SiLU(cv1(x)); a, b = split;
    b = PSABlock(b) per entry of ``blocks``; SiLU(cv2(cat(a, b)))."""
    h = silu(conv1x1(_f64(x), w_cv1, b_cv1))
    c = h.shape[1] // 2
    a, b = h[:, :c], h[:, c:]
    for w in blocks:
        b = psa_block_forward(b, w, c // 64, key_dim)
    return silu(conv1x1(np.concatenate([a, b], axis=1), w_cv2, b_cv2))


def c2psa_forward_eval(x, prm: dict, eps: float = 1e-5, num_heads: int = 2, key_dim: int = 32):
    """Eval-mode C2PSA(256,256,n=1,e=0.5) (c2psa.rs:150-179, psa_block :123-137),
    the structure of the reference's golden fixture ``c2psa_yolo26``.
    ``prm`` maps fixture prefixes (``cv1``, ``m0_attn_qkv`` …) to
    ``(conv_w, bn_w, bn_b, bn_rm, bn_rv)``."""
    def cbn(name, t, act):
        w, g, bta, rm, rv = prm[name]
        wf, bf = fold_bn(w, g, bta, rm, rv, eps)
        if w.shape[2] == 3:
            y = dwconv3x3(t, wf, bf)
        else:
            y = conv1x1(t, wf, bf)
        return silu(y) if act else y

    x = _f64(x)
    h = cbn("cv1", x, True)
    c = h.shape[1] // 2
    a, b = h[:, :c], h[:, c:]
    wq, bq = fold_bn(*prm["m0_attn_qkv"], eps)
    wpe, bpe = fold_bn(*prm["m0_attn_pe"], eps)
    wpr, bpr = fold_bn(*prm["m0_attn_proj"], eps)
    b = b + psa_attention(b, wq, bq, wpe, bpe, wpr, bpr, num_heads, key_dim)
    b = b + cbn("m0_ffn1", cbn("m0_ffn0", b, True), False)
    return cbn("cv2", np.concatenate([a, b], axis=1), True)


def c2psa_backward_train_torch(x, dy, prm: dict, eps: float = 1e-5, num_heads: int = 2,
                               key_dim: int = 32):
    """Train-mode (batch-statistics BN) C2PSA forward + autograd backward in
    torch-CPU float64.  Reproduces the reference's backward fixture
    (``tests/fixtures/c2psa_yolo26/generate_backward.py``) so that the
    attention maths above is also pinned through its gradient.  Returns
    ``(y, dx, fa)`` where ``fa`` holds the FA-level q/k/v_lo/v_hi/o_lo/o_hi/l."""
    import torch
    t = lambda a: torch.as_tensor(np.asarray(a, F64))
    xt = t(x).requires_grad_(True)

    def cbn(name, inp, act):
        w, g, bta, _, _ = prm[name]
        w = t(w)
        groups = w.shape[0] if w.shape[1] == 1 and w.shape[2] == 3 else 1
        y = torch.nn.functional.conv2d(inp, w, padding=w.shape[2] // 2, groups=groups)
        y = torch.nn.functional.batch_norm(y, None, None, t(g), t(bta), training=True, eps=eps)
        return torch.nn.functional.silu(y) if act else y

    h = cbn("cv1", xt, True)
    c = h.shape[1] // 2
    a, b = h[:, :c], h[:, c:]
    B, _, H, W = b.shape
    N = H * W
    qkv = cbn("m0_attn_qkv", b, False)
    hd = 2 * key_dim
    qkvh = qkv.view(B, num_heads, 2 * key_dim + hd, N)
    q, k, v = qkvh.split([key_dim, key_dim, hd], dim=2)
    scale = key_dim ** -0.5
    attn = ((q.transpose(-2, -1) @ k) * scale).softmax(dim=-1)
    o = (v @ attn.transpose(-2, -1)).reshape(B, c, H, W)
    pe = cbn("m0_attn_pe", v.reshape(B, c, H, W), False)
    b = b + cbn("m0_attn_proj", o + pe, False)
    b = b + cbn("m0_ffn1", cbn("m0_ffn0", b, True), False)
    y = cbn("cv2", torch.cat([a, b], 1), True)
    y.backward(t(dy))
    # FA-level tensors in [BH, N, 32] layout (generate_backward.py:150-168)
    qf = q.permute(0, 1, 3, 2).reshape(B * num_heads, N, key_dim)
    kf = k.permute(0, 1, 3, 2).reshape(B * num_heads, N, key_dim)
    vf = v.permute(0, 1, 3, 2).reshape(B * num_heads, N, hd)
    s = (qf @ kf.transpose(1, 2)) * scale
    fa = dict(q=qf, k=kf, v_lo=vf[..., :key_dim], v_hi=vf[..., key_dim:],
              l=torch.logsumexp(s, -1))
    pw = s.softmax(-1)
    fa["o_lo"] = pw @ fa["v_lo"]
    fa["o_hi"] = pw @ fa["v_hi"]
    fa = {kk: vv.detach().numpy().astype(np.float32) for kk, vv in fa.items()}
    return y.detach().numpy(), xt.grad.numpy(), fa


# ── seeded synthetic inputs for the benchmark configurations ────────────────

def psa_synthetic(B: int, H: int, W: int, C: int = 128, num_heads: int = 2, key_dim: int = 32,
                  seed: int = 1234, bias_std: float = 0.02):
    """Seeded synthetic PSA inputs with the value distributions of the
    benchmark configurations: activations N(0,1), conv weights N(0,0.02),
    folded-BN biases N(0, ``bias_std``)."""
    rng = np.random.default_rng(seed)
    qkv_h = num_heads * 4 * key_dim
    f = lambda *s, std=1.0: (rng.standard_normal(s) * std).astype(np.float32)
    return dict(
        x=f(B, C, H, W),
        w_qkv=f(qkv_h, C, 1, 1, std=0.02), b_qkv=f(qkv_h, std=bias_std),
        w_pe=f(C, 1, 3, 3, std=0.02), b_pe=f(C, std=bias_std),
        w_proj=f(C, C, 1, 1, std=0.02), b_proj=f(C, std=bias_std),
    )


def psa_attention_torch(x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, num_heads: int, key_dim: int):
    """The same PSA forward as ``psa_attention`` written with torch-CPU f32
    tensor ops — the timed CPU baseline (the reference has no CPU path,
    book/src/appendix/faq-and-roadmap.md:26).  Takes and returns torch
    tensors; uses whatever thread count torch is set to."""
    import torch
    import torch.nn.functional as Fn
    B, C, H, W = x.shape
    N = H * W
    hd = 2 * key_dim
    qkv = Fn.conv2d(x, w_qkv.reshape(-1, C, 1, 1), b_qkv)
    q, k, v = qkv.view(B, num_heads, 2 * key_dim + hd, N).split([key_dim, key_dim, hd], dim=2)
    attn = torch.softmax((q.transpose(-2, -1) @ k) * (key_dim ** -0.5), dim=-1)
    o = (v @ attn.transpose(-2, -1)).reshape(B, C, H, W)
    pe = Fn.conv2d(v.reshape(B, C, H, W), w_pe.reshape(C, 1, 3, 3), b_pe, padding=1, groups=C)
    return Fn.conv2d(o + pe, w_proj.reshape(C, C, 1, 1), b_proj)


# ── training step (data-parallel cfg5) ───────────────────────────────────────

GRAD_ORDER = ("w_qkv", "w_proj", "w_pe", "b_qkv", "b_proj", "b_pe")  # flat gradient buffer layout


def psa_attention_vjp_torch(x, dy, params: dict, num_heads: int = 2, key_dim: int = 32):
    """Vector-Jacobian product of the BN-folded PSA Attention block in
    torch-CPU float64: for an upstream gradient dy = ∂L/∂y, returns
    ``(grads, dx)`` with ``grads`` flat in ``GRAD_ORDER`` — the backward that
    a training graph runs through the attention node (the reference's
    ``psa_fa2_backward``, ``psa_*_backward`` and conv backward kernels,
    psa.rs:201-327, 650-725)."""
    import torch
    t = lambda a: torch.as_tensor(np.asarray(a, F64))
    p = {k: t(v).requires_grad_(True) for k, v in params.items()}
    xt = t(x).requires_grad_(True)
    C = xt.shape[1]
    y = psa_attention_torch(xt, p["w_qkv"], p["b_qkv"], p["w_pe"].reshape(C, 9), p["b_pe"], p["w_proj"],
                            p["b_proj"], num_heads, key_dim)
    y.backward(t(dy))
    grads = np.concatenate([p[k].grad.numpy().reshape(-1) for k in GRAD_ORDER])
    return grads, xt.grad.numpy()


def psa_train_step_torch(x, target, params: dict, num_heads: int = 2, key_dim: int = 32):
    """Forward + autograd backward of the BN-folded PSA Attention block in
    torch-CPU float64 with loss = mean((y − target)²).  ``params`` holds
    w_qkv [256,128], b_qkv [256], w_pe [128,1,3,3] (or [128,9]), b_pe [128],
    w_proj [128,128], b_proj [128].  Returns ``(y, loss, grads, dx)`` with
    ``grads`` the flat float64 vector in ``GRAD_ORDER`` (PyTorch parameter
    layouts) — the layout of the device gradient buffer.  This is the same
    differentiation the reference's backward fixture performs
    (``c2psa_backward_train_torch``), restricted to the attention block."""
    import torch
    t = lambda a: torch.as_tensor(np.asarray(a, F64))
    p = {k: t(v).requires_grad_(True) for k, v in params.items()}
    xt = t(x).requires_grad_(True)
    C = xt.shape[1]
    y = psa_attention_torch(xt, p["w_qkv"], p["b_qkv"], p["w_pe"].reshape(C, 9), p["b_pe"], p["w_proj"],
                            p["b_proj"], num_heads, key_dim)
    loss = ((y - t(target)) ** 2).mean()
    loss.backward()
    grads = np.concatenate([p[k].grad.numpy().reshape(-1) for k in GRAD_ORDER])
    return y.detach().numpy(), float(loss.detach()), grads, xt.grad.numpy()
