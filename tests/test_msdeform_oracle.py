"""The MSDeformAttn restatement (numpy, hand-derived backward) against an
independent torch-CPU formulation from grid_sample and its autograd (no GPU).

The reference has no deformable attention, so this operator's parity is
unpinned by the reference; these two independent CPU formulations agreeing
is the check the oracle itself gets."""
import numpy as np
import torch

from conftest import max_abs
from oracle import msdeform_oracle as mo


def _case(**kw):
    return mo.msdeform_synthetic(**kw)


def test_forward_numpy_vs_grid_sample():
    p = _case(B=2, Q=7, nh=3, dh=8, shapes=((9, 11), (5, 4), (2, 3)), P=3, seed=1)
    out = mo.msdeform_attn_forward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"])
    t = {k: torch.tensor(v, dtype=torch.float64) if v.dtype.kind == "f" else torch.tensor(v) for k, v in p.items()}
    ref = mo.msdeform_attn_torch(t["value"], t["spatial_shapes"], t["level_start"], t["loc"], t["attn"])
    assert max_abs(out, ref.numpy()) < 1e-10


def test_backward_numpy_vs_autograd():
    p = _case(B=2, Q=5, nh=2, dh=4, shapes=((6, 7), (3, 3)), P=2, seed=2)
    t = {k: torch.tensor(v, dtype=torch.float64) if v.dtype.kind == "f" else torch.tensor(v) for k, v in p.items()}
    v, l, a = (t[k].clone().requires_grad_(True) for k in ("value", "loc", "attn"))
    out = mo.msdeform_attn_torch(v, t["spatial_shapes"], t["level_start"], l, a)
    out.backward(t["grad_out"])
    gv, gl, ga = mo.msdeform_attn_backward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"],
                                           p["grad_out"])
    assert max_abs(gv, v.grad.numpy()) < 1e-10
    assert max_abs(ga, a.grad.numpy()) < 1e-10
    assert max_abs(gl, l.grad.numpy()) < 1e-9


def test_out_of_range_samples_are_zero_padded():
    p = _case(B=1, Q=3, nh=1, dh=2, shapes=((4, 4),), P=1, seed=3)
    p["loc"][...] = 5.0  # far outside [0,1]
    out = mo.msdeform_attn_forward(p["value"], p["spatial_shapes"], p["level_start"], p["loc"], p["attn"])
    assert np.all(out == 0)
