"""Shared fixtures for the visionattn test-suite.

Markers: ``gpu`` — needs a CUDA device (a B200).  Everything else runs on CPU.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


STAGES = ["cv1", "cv2", "m0_attn_qkv", "m0_attn_proj", "m0_attn_pe", "m0_ffn0", "m0_ffn1"]


def stage_params(g):
    return {s: tuple(g[f"{s}_{p}"] for p in ("conv_w", "bn_w", "bn_b", "bn_rm", "bn_rv")) for s in STAGES}


def folded_c2psa(g, eps=1e-5):
    """The golden C2PSA fixture's parameters with BN folded into conv weight +
    bias (1×1 weights as [out][in]): (w_cv1, b_cv1, [block dict], w_cv2, b_cv2)."""
    from oracle import psa_oracle as po
    prm = stage_params(g)
    f = {k: po.fold_bn(*prm[k], eps) for k in prm}
    mat = lambda w: np.asarray(w, np.float64).reshape(w.shape[0], -1)
    blk = {"w_qkv": mat(f["m0_attn_qkv"][0]), "b_qkv": f["m0_attn_qkv"][1],
           "w_pe": np.asarray(f["m0_attn_pe"][0], np.float64), "b_pe": f["m0_attn_pe"][1],
           "w_proj": mat(f["m0_attn_proj"][0]), "b_proj": f["m0_attn_proj"][1],
           "w_ffn0": mat(f["m0_ffn0"][0]), "b_ffn0": f["m0_ffn0"][1],
           "w_ffn1": mat(f["m0_ffn1"][0]), "b_ffn1": f["m0_ffn1"][1]}
    return mat(f["cv1"][0]), f["cv1"][1], [blk], mat(f["cv2"][0]), f["cv2"][1]


FIXTURE_STAGES = {"cv1": "cv1", "cv2": "cv2", "m0_attn_qkv": "m.0.attn.qkv", "m0_attn_pe": "m.0.attn.pe",
                  "m0_attn_proj": "m.0.attn.proj", "m0_ffn0": "m.0.ffn.0", "m0_ffn1": "m.0.ffn.1"}


def c2psa_checkpoint(tmp_path, dtype=None, prefix="model.10"):
    """A safetensors checkpoint with the reference's key layout for a C2PSA
    (``{prefix}.cv1.conv.weight``, ``{prefix}.m.0.attn.qkv.bn.running_var`` …)
    holding the golden C2PSA fixture's parameters; returns (path, fixture)."""
    import torch
    from safetensors.torch import save_file
    dtype = dtype or torch.float32
    g = load_golden("c2psa_fwd.npz")
    prm = stage_params(g)
    t = {}
    for stage, path in FIXTURE_STAGES.items():
        w, *bn = prm[stage]
        t[f"{prefix}.{path}.conv.weight"] = torch.as_tensor(np.asarray(w, np.float32)).to(dtype)
        for name, v in zip(("weight", "bias", "running_mean", "running_var"), bn):
            t[f"{prefix}.{path}.bn.{name}"] = torch.as_tensor(np.asarray(v, np.float32))
    t["model.0.conv.weight"] = torch.zeros(4, 3, 3, 3, dtype=torch.float16)  # an unrelated tensor
    f = os.path.join(str(tmp_path), "yolo26_c2psa.safetensors")
    save_file(t, f, metadata={"format": "pt"})
    return f, g


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


# Tolerances stated by the north star: f32 mode max-abs 1e-5; bf16 mode
# rel-L2 2e-3 and max-abs 1e-2 against the f32 reference.
F32_MAX_ABS = 1e-5
BF16_REL_L2 = 2e-3
BF16_MAX_ABS = 1e-2


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test: no bounded device-side wait may have timed out
    (a timed-out kernel leaves its outputs unwritten rather than faulting)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import ctypes
    import torch
    if not torch.cuda.is_available():
        return
    from vision_rs_b200 import _lib
    st = ctypes.c_int(-1)
    _lib.call("va_device_status_read", ctypes.byref(st), torch.cuda.current_stream().cuda_stream)
    if st.value != 0:
        _lib.call("va_device_status_clear", torch.cuda.current_stream().cuda_stream)
        pytest.fail(f"device status word {st.value}: a bounded wait in a tensor-core kernel gave up")
