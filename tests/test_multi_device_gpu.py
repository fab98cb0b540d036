"""One process driving two GPUs: the library's one-time kernel set-up
(dynamic shared-memory limits, which CUDA keeps per device) must happen on
every device the process uses, not only on the first.  The fused PSA forward
and the training step run on device 0 and then on device 1 with the same
inputs; both devices must produce the same bits.  Skips with one GPU."""
import numpy as np
import pytest
import torch

from oracle import psa_oracle as po

pytestmark = pytest.mark.gpu


def _params(p, dev):
    bf = lambda a: torch.as_tensor(np.asarray(a, np.float32)).to(dev, torch.bfloat16)
    d = {k: bf(p[k]) for k in ("w_qkv", "w_pe", "w_proj")}
    d.update({k: torch.as_tensor(p[k]).to(dev) for k in ("b_qkv", "b_pe", "b_proj")})
    return d


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_forward_and_training_step_on_two_devices():
    from vision_rs_b200 import psa as vp
    from vision_rs_b200 import train
    p = po.psa_synthetic(2, 40, 40, seed=41)
    tgt = np.random.default_rng(42).standard_normal((2, 128, 20, 20)).astype(np.float32)
    q = po.psa_synthetic(2, 20, 20, seed=43)
    outs = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            op = vp.PsaAttention(p["w_qkv"], p["b_qkv"], p["w_pe"], p["b_pe"], p["w_proj"], p["b_proj"], 2, 32,
                                 dtype=torch.bfloat16, device=dev)
            y = op(torch.as_tensor(p["x"]).to(dev, torch.bfloat16))
            step = train.PsaTrainStep(B=2, H=20, W=20, device=dev)
            x = torch.as_tensor(q["x"]).to(dev, torch.bfloat16)
            t = torch.as_tensor(tgt).to(dev, torch.bfloat16)
            _, loss, grads, _ = step.forward_backward(x, t, _params(q, dev))
            torch.cuda.synchronize(dev)
            outs.append((y.cpu(), loss.cpu(), grads.cpu()))
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
