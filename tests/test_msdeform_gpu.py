"""MSDeformAttn forward/backward on the GPU through the C ABI against the
CPU restatement (oracle/msdeform_oracle.py).

f32: max-abs ≤ 1e-5 on out and grad_value (the north star's f32 bound);
grad_attn (Σ w·⟨g, v⟩, magnitude up to ~10) and grad_loc (× W_l, up to 80)
inherit the f32 rounding of the pixel coordinate loc·W − 0.5, so they are
held to 1e-5 relative to their largest magnitude.  grad_loc is the
derivative of a piecewise-bilinear function and jumps where a sample crosses
a pixel-cell boundary; samples within 1e-3 of a boundary (where f32 and f64
may pick different cells) are left out of the grad_loc comparison.  bf16 (value, out, grad_out, grad_value in
bf16; loc/attn f32): rel-L2 ≤ 2e-3 and max-abs ≤ 1e-2 against the f32
oracle evaluated on the same bf16-rounded inputs."""
import numpy as np
import pytest
import torch

from conftest import BF16_MAX_ABS, BF16_REL_L2, F32_MAX_ABS, max_abs, rel_l2
from oracle import msdeform_oracle as mo
from vision_rs_b200 import msdeform as ms

pytestmark = pytest.mark.gpu

CASES = [
    dict(B=2, Q=7, nh=3, dh=16, shapes=((9, 11), (5, 4), (2, 3)), P=3, seed=1),
    dict(B=8, Q=300, nh=16, dh=16, shapes=((80, 80), (40, 40), (20, 20)), P=4, seed=2),  # cfg3, full size
    dict(B=1, Q=33, nh=4, dh=32, shapes=((17, 13), (1, 1)), P=5, seed=3),
]


def _dev(p, dtype):
    d = {}
    for k, v in p.items():
        if k in ("value", "grad_out"):
            d[k] = torch.as_tensor(v).to("cuda", dtype).contiguous()
        elif v.dtype.kind == "f":
            d[k] = torch.as_tensor(v).cuda().contiguous()
        else:
            d[k] = torch.as_tensor(v).cuda().contiguous()
    return d


def _off_boundary(p, tol=1e-3):
    """[B,Q,nh,L,P] mask of samples whose pixel coordinates are ≥ tol away
    from an integer (a bilinear cell boundary) in both x and y."""
    sh = p["spatial_shapes"]
    W = sh[:, 1].astype(np.float64)[None, None, None, :, None]
    H = sh[:, 0].astype(np.float64)[None, None, None, :, None]
    x = p["loc"][..., 0].astype(np.float64) * W - 0.5
    y = p["loc"][..., 1].astype(np.float64) * H - 0.5
    fx, fy = x - np.floor(x), y - np.floor(y)
    return (np.minimum(fx, 1 - fx) > tol) & (np.minimum(fy, 1 - fy) > tol)


def _bf16_round(p):
    q = dict(p)
    for k in ("value", "grad_out"):
        q[k] = torch.as_tensor(p[k]).bfloat16().float().numpy()
    return q


@pytest.mark.parametrize("case", CASES)
def test_forward_f32(cuda, case):
    p = mo.msdeform_synthetic(**case)
    d = _dev(p, torch.float32)
    out = ms.msdeform_attn_forward(d["value"], d["spatial_shapes"], d["level_start"], d["loc"], d["attn"])
    ref = mo.msdeform_attn_forward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"])
    assert max_abs(out.cpu().numpy(), ref) < F32_MAX_ABS


@pytest.mark.parametrize("case", CASES)
def test_backward_f32(cuda, case):
    p = mo.msdeform_synthetic(**case)
    d = _dev(p, torch.float32)
    gv, gl, ga = ms.msdeform_attn_backward(d["value"], d["spatial_shapes"], d["level_start"], d["loc"], d["attn"],
                                           d["grad_out"])
    rv, rl, ra = mo.msdeform_attn_backward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"],
                                           p["grad_out"])
    assert max_abs(gv.cpu().numpy(), rv) < F32_MAX_ABS
    assert max_abs(ga.cpu().numpy(), ra) < F32_MAX_ABS * max(1.0, float(np.abs(ra).max()))
    m = _off_boundary(p)
    assert m.mean() > 0.99
    assert max_abs(gl.cpu().numpy()[m], rl[m]) < F32_MAX_ABS * max(1.0, float(np.abs(rl).max()))
    # deterministic: a second run is bit-identical
    gv2, gl2, ga2 = ms.msdeform_attn_backward(d["value"], d["spatial_shapes"], d["level_start"], d["loc"], d["attn"],
                                              d["grad_out"])
    assert torch.equal(gv, gv2) and torch.equal(gl, gl2) and torch.equal(ga, ga2)


@pytest.mark.parametrize("case", CASES[:2])
def test_forward_backward_bf16(cuda, case):
    p = _bf16_round(mo.msdeform_synthetic(**case))
    d = _dev(p, torch.bfloat16)
    out = ms.msdeform_attn_forward(d["value"], d["spatial_shapes"], d["level_start"], d["loc"], d["attn"])
    ref = mo.msdeform_attn_forward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"])
    o = out.float().cpu().numpy()
    assert rel_l2(o, ref) < BF16_REL_L2 and max_abs(o, ref) < BF16_MAX_ABS
    gv, gl, ga = ms.msdeform_attn_backward(d["value"], d["spatial_shapes"], d["level_start"], d["loc"], d["attn"],
                                           d["grad_out"])
    rv, rl, ra = mo.msdeform_attn_backward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"],
                                           p["grad_out"])
    g = gv.float().cpu().numpy()
    assert rel_l2(g, rv) < BF16_REL_L2 and max_abs(g, rv) < BF16_MAX_ABS
    m = _off_boundary(p)
    assert rel_l2(ga.cpu().numpy(), ra) < 1e-5 and rel_l2(gl.cpu().numpy()[m], rl[m]) < 1e-5


def test_out_of_range_and_edge_samples(cuda):
    p = mo.msdeform_synthetic(B=1, Q=16, nh=2, dh=16, shapes=((6, 5), (3, 2)), P=2, seed=9)
    p["loc"][0, :4] = 5.0          # far outside: zero contribution
    p["loc"][0, 4:8] = -0.05       # partly outside: zero-padded corners
    p["loc"][0, 8:12] = 1.0        # right/bottom edge
    d = _dev(p, torch.float32)
    out = ms.msdeform_attn_forward(d["value"], d["spatial_shapes"], d["level_start"], d["loc"], d["attn"])
    ref = mo.msdeform_attn_forward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"])
    assert max_abs(out.cpu().numpy(), ref) < F32_MAX_ABS
    assert np.all(out.cpu().numpy()[0, :4] == 0)
    gv, gl, ga = ms.msdeform_attn_backward(d["value"], d["spatial_shapes"], d["level_start"], d["loc"], d["attn"],
                                           d["grad_out"])
    rv, rl, ra = mo.msdeform_attn_backward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"],
                                           p["grad_out"])
    assert max_abs(gv.cpu().numpy(), rv) < F32_MAX_ABS
    assert max_abs(ga.cpu().numpy(), ra) < F32_MAX_ABS * max(1.0, float(np.abs(ra).max()))
