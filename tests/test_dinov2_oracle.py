"""CPU checks of the DINOv2 attention restatement (oracle/dinov2_oracle.py).

The reference has no DINOv2 code, so the restatement is cross-checked against
an independent formulation: torch's scaled_dot_product_attention in float64.
"""
import numpy as np
import torch

from oracle import dinov2_oracle as do


def _torch64(x, w, b, heads):
    t = lambda a: torch.as_tensor(np.asarray(a, np.float64))
    return do.dinov2_attention_torch(t(x), t(w), t(b), heads).numpy()


def test_restatement_matches_sdpa_small():
    x, w, b = do.dinov2_synthetic(S=3, n=37, hidden=128, seed=1)
    ref = _torch64(x, w, b, 2)
    got = do.dinov2_attention(x, w, b, 2)
    assert np.abs(got - ref).max() < 1e-12


def test_restatement_matches_sdpa_cfg4_global():
    x, w, b = do.dinov2_synthetic(S=1, n=1601, hidden=384, seed=2)
    ref = _torch64(x, w, b, 6)
    got = do.dinov2_attention(x, w, b, 6)
    assert np.abs(got - ref).max() < 1e-12


def test_window_partition_round_trip():
    rng = np.random.default_rng(3)
    B, gh, gw, win, C = 2, 8, 12, 4, 16
    x = rng.standard_normal((B, 1 + gh * gw, C))
    xw = do.window_partition(x, gh, gw, win)
    assert xw.shape == (B * (gh // win) * (gw // win), 1 + win * win, C)
    # token 0 of every window is the cls token; window 1 of image 0 holds patch (0, win)
    assert np.array_equal(xw[:, 0], np.repeat(x[:, 0], (gh // win) * (gw // win), axis=0))
    assert np.array_equal(xw[1, 1], x[0, 1 + win])
    assert np.allclose(do.window_unpartition(xw, B, gh, gw, win), x, rtol=0, atol=1e-15)
