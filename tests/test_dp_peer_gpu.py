"""Peer-memory gradient all-reduce + SGD (va_psa_dp_allreduce_sgd) on every
GPU of the box (2 to 8), one process per GPU over NCCL for the set-up.

Parity: three data-parallel training steps through PeerGradComm against the
same steps through NCCL all-reduce + va_psa_sgd_update, from the same weights
and shards.  The peer kernel sums in rank order, so its sums are
bit-identical on every rank; with two ranks they are also bit-identical to
NCCL's (both compute g0 + g1).  With more ranks NCCL's ring or tree may
associate the sum differently, so there the two paths agree to f32 rounding
and the masters to the same tolerance.

Failure detection (no GPU fault, no trap): ranks 0 .. W-2 run the all-reduce
while rank W-1 does not; their bounded device-side waits give up after the
comm's short time limit, every block returns without updating, and the
status word reads 100 + (W-1).  Then every rank calls again: the failed ranks
return at once (the status is sticky) and update nothing, while the late rank
W-1 finds its peers' step-1 gradients published and completes step 1 (its sum
is checked).  At the next call the failed ranks still publish nothing, so
rank W-1's waits give up in turn: the divergence is detected on every rank
within one step, and the failed ranks' weights never moved.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, world):
    import torch.distributed as dist
    from oracle import psa_oracle as po
    from vision_rs_b200 import train
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
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
        for it in range(3):
            if world > 2:  # NCCL's association may differ: start both paths from the same weights
                pp = {k: v.clone() for k, v in pn.items()}
                mp_ = mn.clone()
            train.dp_train_step(step, x, t, pn, mn, lr=0.05)
            gn = step.grads.clone()
            train.dp_train_step(step, x, t, pp, mp_, lr=0.05, comm=comm)
            gp = step.grads.clone()
            torch.cuda.synchronize()
            assert comm.status() == 0
            if world == 2:
                assert torch.equal(gn, gp)
                assert torch.equal(mn, mp_)
                for k in pn:
                    assert torch.equal(pn[k], pp[k]), k
            else:
                scale = float(gn.abs().max())
                assert float((gn - gp).abs().max()) <= 1e-5 * scale, it
                assert float((mn - mp_).abs().max()) <= 1e-6 * max(1.0, float(mn.abs().max())), it
        # the summed gradients agree bit for bit across ranks
        peer_g = [torch.empty_like(gp) for _ in range(world)]
        dist.all_gather(peer_g, gp)
        for r in range(1, world):
            assert torch.equal(peer_g[0], peer_g[r]), r

        # the whole step replayed from one CUDA graph (DpStepGraph) equals the eager step:
        # from the same weights, two eager steps and two graph steps (the first runs eagerly
        # and captures, the second replays) end in bit-identical weights
        pe, pg = {k: v.clone() for k, v in pp.items()}, {k: v.clone() for k, v in pp.items()}
        me, mg = mp_.clone(), mp_.clone()
        for _ in range(2):
            train.dp_train_step(step, x, t, pe, me, lr=0.05, comm=comm)
        gstep = train.DpStepGraph(train.PsaTrainStep(B=B, H=H, W=W, device=dev, graph=True), comm)
        for _ in range(2):
            gstep(x, t, pg, mg, 0.05)
        torch.cuda.synchronize()
        assert comm.status() == 0 and gstep.graph_kernels > 0
        assert torch.equal(me, mg)
        for k in pe:
            assert torch.equal(pe[k], pg[k]), k
        comm.close()

        # failure detection: the last rank never publishes (short limit: 300 ms per wait)
        comm2 = train.PeerGradComm(timeout_ms=300, check_every=0)
        g = torch.randn(train.GRAD_COUNT, device=dev, generator=torch.Generator(dev).manual_seed(rank))
        all_g = [torch.empty_like(g) for _ in range(world)]
        dist.all_gather(all_g, g)
        before = {k: v.clone() for k, v in pp.items()}
        m = train.PsaTrainStep.master_from(pp)
        m0 = m.clone()
        last = world - 1
        if rank != last:
            comm2.allreduce_sgd(g.clone(), m, pp, lr=0.05)
            torch.cuda.synchronize()
            assert comm2.status() == 100 + last
        dist.barrier()
        # every rank calls again: the failed ranks return at once (sticky status) and update
        # nothing; the late last rank finds its peers' step-1 data published and completes step 1
        g2 = g.clone()
        comm2.allreduce_sgd(g2, m, pp, lr=0.05)
        torch.cuda.synchronize()
        if rank != last:
            assert comm2.status() == 100 + last
        else:
            assert comm2.status() == 0
            ref = all_g[0].clone()
            for r in range(1, world):
                ref = ref + all_g[r]
            assert torch.equal(g2, ref)
            assert not torch.equal(m, m0)
            m0 = m.clone()
            before = {k: v.clone() for k, v in pp.items()}
        dist.barrier()
        # the next step: the failed ranks still publish nothing, so the last rank's waits give up
        comm2.allreduce_sgd(g.clone(), m, pp, lr=0.05)
        torch.cuda.synchronize()
        st = comm2.status()
        if rank != last:
            assert st == 100 + last
        else:
            assert 100 <= st < 100 + last
        assert torch.equal(m, m0)
        for k in pp:
            assert torch.equal(pp[k], before[k]), k
        with pytest.raises(RuntimeError):
            comm2.raise_on_failure()
        comm2.close(check=False)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(WORLD < 2, reason="needs two GPUs or more")
def test_peer_allreduce_sgd_matches_nccl_all_gpus():
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(_free_port(), WORLD), nprocs=WORLD, join=True)
