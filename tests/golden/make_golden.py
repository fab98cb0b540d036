#!/usr/bin/env python3
"""Copy the reference's own golden fixtures for the PSA attention path into
compact ``.npz`` files under ``tests/golden/``.

The reference (spinorml/vision-rs) commits PyTorch/ultralytics-generated
little-endian f32 fixtures under ``tests/fixtures/`` of its crate:

* ``c2psa_yolo26/``            — eval-mode C2PSA(256,256,n=1,e=0.5), B=2, 4×4
  (generator ``tests/fixtures/c2psa_yolo26/generate.py``; consumed by
  ``tests/test_c2psa_cuda.rs``, tolerance 1e-3 at :673)
* ``c2psa_yolo26/backward/``   — train-mode forward + backward, incl. the
  FA-level Q/K/V_lo/V_hi/O_lo/O_hi/LSE tensors ``[4,16,32]``
  (``generate_backward.py:150-208``; ``tests/test_c2psa_backward_cuda.rs``,
  tolerance 5e-3 at :701)
* ``conv_grouped/depthwise/``  — the PE-shaped depthwise 3×3 conv fwd/bwd
  (``tests/test_conv_grouped_cuda.rs`` tol 1e-5, ``…_backward_cuda.rs`` 1e-4)
* ``conv_yolo26/``             — the YOLO26n stem Conv(3→16, k3, s2), BN in
  training mode, B=2, 16×16 (``generate.py:36-47``; ``tests/test_conv_yolo26.rs``)
* ``c3k2_yolo26/``             — eval-mode C3k2 blocks, B=2, 4×4
  (``generate_all.py``): the top-level C3k2(32,64,c3k=F,sc=F,e=0.25),
  ``shortcut/`` (same, sc=T) and ``deep_st/`` C3k2(128,128,c3k=T,sc=T,e=0.5)
  → ``conv_c3k2.npz`` with keys ``{variant}/{stage}_{conv_w,bn_w,bn_b,bn_rm,bn_rv}``

The GPU box has no copy of the reference, so the tests read these ``.npz``
copies.  Usage (in a checkout that has the reference next to it)::

    python tests/golden/make_golden.py /path/to/vision-rs

Also writes ``psa_attn_case.npz``: the PSA-attention-level input/output of
the same fixture (``b`` after ``cv1`` split → ``attn(b)``), computed by the
oracle after the oracle has reproduced ``expected_output.bin``.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import psa_oracle as po  # noqa: E402

B, C1, H, W = 2, 256, 4, 4
STAGES = ["cv1", "cv2", "m0_attn_qkv", "m0_attn_proj", "m0_attn_pe", "m0_ffn0", "m0_ffn1"]
SHAPES = {"cv1": (256, 256, 1, 1), "cv2": (256, 256, 1, 1), "m0_attn_qkv": (256, 128, 1, 1),
          "m0_attn_proj": (128, 128, 1, 1), "m0_attn_pe": (128, 1, 3, 3),
          "m0_ffn0": (256, 128, 1, 1), "m0_ffn1": (128, 256, 1, 1)}


def rd(d, name, shape=None):
    a = np.fromfile(os.path.join(d, name), dtype="<f4")
    return a.reshape(shape) if shape is not None else a


def load_stages(d):
    out = {}
    for s in STAGES:
        out[f"{s}_conv_w"] = rd(d, f"{s}_conv_w.bin", SHAPES[s])
        for p in ("bn_w", "bn_b", "bn_rm", "bn_rv"):
            out[f"{s}_{p}"] = rd(d, f"{s}_{p}.bin")
    return out


def prm_from(arrs):
    return {s: tuple(arrs[f"{s}_{p}"] for p in ("conv_w", "bn_w", "bn_b", "bn_rm", "bn_rv"))
            for s in STAGES}


# (directory, C_in, C_out, c3k, shortcut, e) of the C3k2 fixtures copied
C3K2_VARIANTS = {"shallow_sf": ("", 32, 64, False, False, 0.25),
                 "shallow_st": ("shortcut", 32, 64, False, True, 0.25),
                 "deep_st": ("deep_st", 128, 128, True, True, 0.5)}


def c3k2_stage_shapes(c_in, c_out, c3k, e):
    c = int(c_out * e)
    sh = {"cv1": (2 * c, c_in, 1, 1), "cv2": (c_out, 3 * c, 1, 1)}
    if c3k:
        h = c // 2
        sh.update({"m0_icv1": (h, c, 1, 1), "m0_icv2": (h, c, 1, 1), "m0_icv3": (c, 2 * h, 1, 1)})
        for m in ("m0_m0_", "m0_m1_"):
            sh.update({m + "cv1": (h, h, 3, 3), m + "cv2": (h, h, 3, 3)})
    else:
        sh.update({"m0_cv1": (c // 2, c, 3, 3), "m0_cv2": (c, c // 2, 3, 3)})
    return sh


def conv_fixtures(fx):
    from oracle import conv_oracle as co
    out, worst = {}, 0.0
    d = os.path.join(fx, "conv_yolo26")
    stem = dict(x=rd(d, "x.bin", (2, 3, 16, 16)), conv_w=rd(d, "conv_weight.bin", (16, 3, 3, 3)),
                bn_w=rd(d, "bn_weight.bin"), bn_b=rd(d, "bn_bias.bin"), bn_rm=rd(d, "bn_running_mean.bin"),
                bn_rv=rd(d, "bn_running_var.bin"), expected_output=rd(d, "expected_output.bin", (2, 16, 8, 8)))
    y = co.conv_block_train(stem["x"], (stem["conv_w"], stem["bn_w"], stem["bn_b"]), stride=2)
    worst = max(worst, float(np.abs(y - stem["expected_output"]).max()))
    out.update({f"stem/{k}": v for k, v in stem.items()})
    for name, (sub, c_in, c_out, c3k, sc, e) in C3K2_VARIANTS.items():
        d = os.path.join(fx, "c3k2_yolo26", sub)
        prm = {}
        for st, shape in c3k2_stage_shapes(c_in, c_out, c3k, e).items():
            prm[st] = (rd(d, f"{st}_conv_w.bin", shape),) + tuple(rd(d, f"{st}_bn_{p}.bin") for p in ("w", "b", "rm", "rv"))
            for p, a in zip(("conv_w", "bn_w", "bn_b", "bn_rm", "bn_rv"), prm[st]):
                out[f"{name}/{st}_{p}"] = a
        x = rd(d, "x.bin", (2, c_in, 4, 4))
        ref = rd(d, "expected_output.bin", (2, c_out, 4, 4))
        out[f"{name}/x"], out[f"{name}/expected_output"] = x, ref
        worst = max(worst, float(np.abs(co.c3k2(x, prm, c3k, sc) - ref).max()))
    assert worst < 1e-5, f"conv oracle does not reproduce the conv/C3k2 fixtures (max-abs {worst})"
    np.savez_compressed(os.path.join(HERE, "conv_c3k2.npz"), **out)
    return worst


def main(ref_root):
    fx = os.path.join(ref_root, "tests", "fixtures")
    # forward (eval)
    d = os.path.join(fx, "c2psa_yolo26")
    fwd = load_stages(d)
    fwd["x"] = rd(d, "x.bin", (B, C1, H, W))
    fwd["expected_output"] = rd(d, "expected_output.bin", (B, C1, H, W))
    np.savez_compressed(os.path.join(HERE, "c2psa_fwd.npz"), **fwd)

    # backward (train)
    d = os.path.join(fx, "c2psa_yolo26", "backward")
    bwd = load_stages(d)
    for n in ("x", "dy", "dx_expected", "expected_output"):
        bwd[n] = rd(d, f"{n}.bin", (B, C1, H, W))
    for n in ("q", "k", "v_lo", "v_hi", "o_lo", "o_hi"):
        bwd[f"attn_{n}"] = rd(d, f"attn_{n}.bin", (4, 16, 32))
    bwd["attn_l"] = rd(d, "attn_l.bin", (4, 16))
    np.savez_compressed(os.path.join(HERE, "c2psa_bwd.npz"), **bwd)

    # depthwise conv (PE shape)
    d = os.path.join(fx, "conv_grouped", "depthwise")
    dw = dict(x=rd(d, "x.bin", (2, 128, 4, 4)), conv_w=rd(d, "conv_w.bin", (128, 1, 3, 3)),
              expected_output=rd(d, "expected_output.bin", (2, 128, 4, 4)),
              dy=rd(d, "dy.bin", (2, 128, 4, 4)), dx_expected=rd(d, "dx_expected.bin", (2, 128, 4, 4)),
              dw_expected=rd(d, "dw_expected.bin", (128, 1, 3, 3)))
    np.savez_compressed(os.path.join(HERE, "dwconv_depthwise.npz"), **dw)

    # attention-level case derived through the pinned oracle
    prm = prm_from(fwd)
    y = po.c2psa_forward_eval(fwd["x"], prm)
    err = float(np.abs(y - fwd["expected_output"]).max())
    assert err < 1e-5, f"oracle does not reproduce expected_output.bin (max-abs {err})"
    eps = 1e-5
    wcv1, bcv1 = po.fold_bn(*prm["cv1"], eps)
    h = po.silu(po.conv1x1(fwd["x"], wcv1, bcv1))
    b_in = h[:, 128:].astype(np.float32)
    wq, bq = po.fold_bn(*prm["m0_attn_qkv"], eps)
    wpe, bpe = po.fold_bn(*prm["m0_attn_pe"], eps)
    wpr, bpr = po.fold_bn(*prm["m0_attn_proj"], eps)
    f32 = lambda a: np.asarray(a, np.float32)
    attn_out = po.psa_attention(b_in, f32(wq), f32(bq), f32(wpe), f32(bpe), f32(wpr), f32(bpr), 2, 32)
    np.savez_compressed(os.path.join(HERE, "psa_attn_case.npz"), x=b_in,
                        w_qkv=f32(wq), b_qkv=f32(bq), w_pe=f32(wpe), b_pe=f32(bpe),
                        w_proj=f32(wpr), b_proj=f32(bpr), y=f32(attn_out))
    print("golden fixtures written; oracle vs expected_output max-abs", err)
    print("conv / C3k2 fixtures: oracle max-abs", conv_fixtures(fx))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the vision-rs checkout>")
    main(sys.argv[1])
