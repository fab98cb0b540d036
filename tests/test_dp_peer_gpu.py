"""Peer-memory gradient all-reduce + SGD (va_psa_dp_allreduce_sgd) on two GPUs,
one process per GPU over NCCL for the set-up.

Parity: three data-parallel training steps through PeerGradComm against the
same steps through NCCL all-reduce + va_psa_sgd_update, from the same weights
and shards: the summed gradients, the f32 master weights and the bf16/f32
parameters are bit-identical (two ranks: both sum g0 + g1 in f32).

Failure detection: rank 0 runs the all-reduce while rank 1 never does; every
bounded device-side wait gives up after about a second, the kernel returns,
and the comm's status word reads 101 (the rank that never published).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port):
    import torch.distributed as dist
    from oracle import psa_oracle as po
    from vision_rs_b200 import train
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        B, H, W = 4, 20, 20
        s = po.psa_synthetic(B, H, W, seed=500 + rank)
        wseed = po.psa_synthetic(1, H, W, seed=78)
        bf = lambda a: torch.as_tensor(np.asarray(a, np.float32)).to(dev, torch.bfloat16)
        x = bf(s["x"])
        t = bf(np.random.default_rng(600 + rank).standard_normal(x.shape))

        def params():
            p = {k: bf(wseed[k]) for k in ("w_qkv", "w_pe", "w_proj")}
            p.update({k: torch.as_tensor(wseed[k]).to(dev) for k in ("b_qkv", "b_pe", "b_proj")})
            return p

        pn, pp = params(), params()
        mn, mp_ = train.PsaTrainStep.master_from(pn), train.PsaTrainStep.master_from(pp)
        step = train.PsaTrainStep(B=B, H=H, W=W, device=dev)
        comm = train.PeerGradComm()
        for _ in range(3):
            train.dp_train_step(step, x, t, pn, mn, lr=0.05)
            gn = step.grads.clone()
            train.dp_train_step(step, x, t, pp, mp_, lr=0.05, comm=comm)
            gp = step.grads.clone()
            torch.cuda.synchronize()
            assert comm.status() == 0
            assert torch.equal(gn, gp)
            assert torch.equal(mn, mp_)
            for k in pn:
                assert torch.equal(pn[k], pp[k]), k
        # the summed gradients agree across ranks
        peer_g = [torch.empty_like(gp) for _ in range(WORLD)]
        dist.all_gather(peer_g, gp)
        assert torch.equal(peer_g[0], peer_g[1])
        comm.close()

        # failure detection: rank 1 never publishes
        comm2 = train.PeerGradComm()
        if rank == 0:
            g = torch.zeros(train.GRAD_COUNT, device=dev)
            m = train.PsaTrainStep.master_from(pp)
            comm2.allreduce_sgd(g, m, pp, lr=0.0)
            torch.cuda.synchronize()
            assert comm2.status() == 101
        comm2.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs two GPUs")
def test_peer_allreduce_sgd_matches_nccl_two_gpus():
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(_free_port(),), nprocs=WORLD, join=True)
