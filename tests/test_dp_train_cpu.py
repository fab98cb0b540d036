"""Data-parallel training host logic (vision_rs_b200.train.dp_train_step) on
two gloo ranks on CPU: every rank all-reduces its gradient buffer and applies
the mean gradient, so the master weights agree across ranks.  The device
forward/backward is replaced by a rank-dependent stand-in (no GPU here)."""
import datetime
import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from vision_rs_b200 import train

    class Step:
        def __init__(self):
            g = torch.arange(train.GRAD_COUNT, dtype=torch.float32) * 1e-3
            self.grads = g * (rank + 1)
            self.loss = torch.tensor([float(rank)])

        def forward_backward(self, x, t, params):
            return None, self.loss, self.grads, None

        @staticmethod
        def sgd(master, grads, params, lr, grad_scale):
            master.sub_(lr * grad_scale * grads)

    master = torch.ones(train.GRAD_COUNT)
    loss = train.dp_train_step(Step(), None, None, {}, master, lr=0.5)
    q.put((rank, float(loss), master.clone()))
    dist.barrier()
    dist.destroy_process_group()


def test_dp_step_two_ranks_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, loss, m = q.get(timeout=120)
        res[r] = (loss, m)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.arange(50816, dtype=torch.float32) * 1e-3
    expect = 1.0 - 0.5 * (g * 1 + g * 2) / world  # mean of the ranks' gradients
    for r in range(world):
        assert torch.allclose(res[r][1], expect, rtol=1e-6, atol=1e-6)
        assert res[r][0] == float(r)  # the local loss is returned unreduced
