"""PSA Attention data-parallel training step (cfg5) over the C ABI.

Each rank: ``PsaTrainStep.forward_backward`` (tensor-core forward, backward
into one f32 gradient buffer), then either ``torch.distributed.all_reduce`` of
that buffer (sum) and ``sgd`` with ``grad_scale = 1/world`` on f32 master
weights, or — with a ``PeerGradComm`` — one kernel that sums the ranks'
buffers over NVLink peer memory and applies the same SGD update.  The update
rewrites the bf16 weights the next forward reads.  The
gradient buffer layout is the header's ``VA_PSA_GRAD_*`` offsets:
``[w_qkv 256×128 | w_proj 128×128 | w_pe 128×9 | b_qkv | b_proj | b_pe]``.
"""
from __future__ import annotations

import torch

from . import _lib
from .psa import _p, _stream

GRAD_COUNT = 50816
GRAD_SLICES = {"w_qkv": (0, 32768), "w_proj": (32768, 49152), "w_pe": (49152, 50304), "b_qkv": (50304, 50560),
               "b_proj": (50560, 50688), "b_pe": (50688, 50816)}


class PsaTrainStep:
    """Buffers for one rank's shard of B images of 128×H×W.

    ``graph=True`` replays ``forward_backward`` from a CUDA graph once it has
    run eagerly for a given set of input / parameter tensors: the ≈15 kernel
    launches of a step then cost one graph launch on the host (an eager step
    spends ≈105 µs of host time on ≈160 µs of GPU work at cfg5, which lets
    the host, not the GPU, pace a multi-rank step).  The graph is re-captured
    whenever the tensors' addresses change; it runs on the current stream."""

    def __init__(self, B: int, H: int, W: int, device, C: int = 128, num_heads: int = 2, key_dim: int = 32,
                 graph: bool = False):
        self.B, self.H, self.W, self.C, self.nh, self.kd = B, H, W, C, num_heads, key_dim
        self.use_graph, self._graph, self._graph_key = graph, None, None
        self.graph_kernels = 0     # kernels one replay launches (the library's launch counter skips replays)
        self.replayed_kernels = 0  # kernels launched by replays so far
        need = int(_lib.lib().va_psa_train_workspace_bytes(B, H, W))
        self.ws = torch.empty(need, dtype=torch.uint8, device=device)
        self.grads = torch.empty(GRAD_COUNT, dtype=torch.float32, device=device)
        self.loss = torch.empty(1, dtype=torch.float32, device=device)
        self.y = torch.empty(B, C, H, W, dtype=torch.bfloat16, device=device)
        self.dx = torch.empty(B, C, H, W, dtype=torch.bfloat16, device=device)

    def forward_backward(self, x, target, params: dict, want_dx: bool = False, stream=None):
        """Returns ``(y, loss, grads, dx)`` (device tensors; dx None unless asked)."""
        if self.use_graph and stream is None and not want_dx:
            key = (x.data_ptr(), target.data_ptr()) + tuple(params[k].data_ptr() for k in sorted(params))
            if self._graph is None or self._graph_key != key:
                self._launch(x, target, params, False, None)  # eager first: one-time set-up stays out of the graph
                torch.cuda.current_stream().synchronize()
                g = torch.cuda.CUDAGraph()
                n0 = int(_lib.lib().va_launch_count())
                with torch.cuda.graph(g, capture_error_mode="relaxed"):
                    self._launch(x, target, params, False, None)
                self.graph_kernels = int(_lib.lib().va_launch_count()) - n0
                self._graph, self._graph_key = g, key
            self._graph.replay()
            self.replayed_kernels += self.graph_kernels
        else:
            self._launch(x, target, params, want_dx, stream)
        return self.y, self.loss, self.grads, (self.dx if want_dx else None)

    def _launch(self, x, target, params: dict, want_dx: bool, stream):
        _lib.call("va_psa_train_fwd_bwd_bf16", _p(x), _p(target), _p(params["w_qkv"]), _p(params["b_qkv"]),
                  _p(params["w_pe"]), _p(params["b_pe"]), _p(params["w_proj"]), _p(params["b_proj"]), _p(self.y),
                  _p(self.dx) if want_dx else None, _p(self.grads), _p(self.loss), self.B, self.C, self.H, self.W,
                  self.nh, self.kd, _p(self.ws), self.ws.numel(), _stream(stream))

    @staticmethod
    def master_from(params: dict) -> torch.Tensor:
        """f32 master weights in the gradient layout, from the current parameters."""
        order = ("w_qkv", "w_proj", "w_pe", "b_qkv", "b_proj", "b_pe")
        return torch.cat([params[k].float().reshape(-1) for k in order]).contiguous()

    @staticmethod
    def sgd(master, grads, params: dict, lr: float, grad_scale: float = 1.0, stream=None):
        _lib.call("va_psa_sgd_update", _p(master), _p(grads), float(lr), float(grad_scale), _p(params["w_qkv"]),
                  _p(params["b_qkv"]), _p(params["w_pe"]), _p(params["b_pe"]), _p(params["w_proj"]),
                  _p(params["b_proj"]), _stream(stream))


class PeerGradComm:
    """All-reduce of the gradient buffer over NVLink peer memory, fused with
    the SGD update (``va_psa_dp_allreduce_sgd``): every rank exports one
    device buffer through CUDA IPC, the handles are exchanged once with an
    ``all_gather`` of the process group, and each step is one kernel launch
    per rank with no NCCL call.  One process per GPU, all on one node.  The
    summed gradients are bit-identical on every rank (summed in rank order).
    ``close()`` on every rank (it begins with a barrier) before the process
    group is destroyed.

    ``timeout_ms`` bounds every device-side wait for a peer (0: the library's
    default, 10 s).  A wait that gives up makes the comm's status non-zero;
    from then on its kernel updates nothing, and ``allreduce_sgd`` raises on
    the next status check (every ``check_every`` calls, and in ``close``):
    the weights must then be restored on every rank and the comm recreated."""

    def __init__(self, group=None, timeout_ms: int = 0, check_every: int = 64):
        import ctypes as C
        import torch.distributed as dist
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.check_every, self._calls = check_every, 0
        self._h = C.c_void_p()
        buf = C.create_string_buffer(64)
        _lib.call("va_dp_comm_create", self.rank, self.world, GRAD_COUNT, int(timeout_ms), C.byref(self._h), buf)
        mine = torch.frombuffer(bytearray(buf.raw), dtype=torch.uint8)
        if dist.get_backend(group) == "nccl":
            mine = mine.to(torch.device("cuda", torch.cuda.current_device()))
        parts = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(parts, mine, group=group)
        handles = b"".join(t.cpu().numpy().tobytes() for t in parts)
        _lib.call("va_dp_comm_connect", self._h, C.create_string_buffer(handles, len(handles)))

    def allreduce_sgd(self, grads, master, params: dict, lr: float, stream=None):
        """grads (in place) = Σ over ranks; master -= lr·grads/world; bf16/f32
        parameters rewritten from master."""
        self.count_call()
        self._launch(grads, master, params, lr, stream)

    def count_call(self):
        """One all-reduce issued (eagerly or by a graph replay): every
        ``check_every`` calls the sticky status is read (a host sync)."""
        self._calls += 1
        if self.check_every and self._calls % self.check_every == 0:
            self.raise_on_failure()

    def _launch(self, grads, master, params: dict, lr: float, stream=None):
        _lib.call("va_psa_dp_allreduce_sgd", self._h, _p(grads), _p(master), float(lr), _p(params["w_qkv"]),
                  _p(params["b_qkv"]), _p(params["w_pe"]), _p(params["b_pe"]), _p(params["w_proj"]),
                  _p(params["b_proj"]), _stream(stream))

    def status(self) -> int:
        """0, or 100 + the rank whose flag a device-side wait gave up on (synchronises)."""
        import ctypes as C
        st = C.c_int(0)
        _lib.call("va_dp_comm_status", self._h, C.byref(st))
        return st.value

    def raise_on_failure(self):
        st = self.status()
        if st != 0:
            raise RuntimeError(f"peer all-reduce on rank {self.rank}: a device-side wait for rank {st - 100} gave "
                               f"up (status {st}); restore the weights and recreate the comm on every rank")

    def close(self, check: bool = True):
        """Two-phase teardown: every rank closes its mappings of the peers'
        buffers, then (after a barrier) frees its own.  Raises afterwards if
        the status is non-zero and ``check`` is set."""
        import torch.distributed as dist
        if self._h is None:
            return
        torch.cuda.synchronize()
        st = self.status()
        dist.barrier(group=self.group)      # every rank's last all-reduce has finished
        _lib.call("va_dp_comm_disconnect", self._h)
        dist.barrier(group=self.group)      # no rank maps this rank's buffer any more
        _lib.call("va_dp_comm_destroy", self._h)
        self._h = None
        if check and st != 0:
            raise RuntimeError(f"peer all-reduce on rank {self.rank}: status {st} at close")


def attention_backward(x, dy, params: dict, dy_scale: float = 1.0, want_dx: bool = True, workspace=None,
                       stream=None):
    """Backward of the fused bf16 PSA Attention op for an upstream gradient
    dy = ∂L/∂y (``va_psa_attention_bwd_bf16``): returns ``(grads, dx)`` —
    grads f32 ``[VA_PSA_GRAD_COUNT]`` in the gradient-buffer layout, dx bf16
    or None.  Pass dy_scale ≈ max|dy| so that dy/dy_scale is O(1)."""
    B, C, H, W = x.shape
    need = int(_lib.lib().va_psa_attention_bwd_workspace_bytes(B, H, W))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    grads = torch.empty(GRAD_COUNT, dtype=torch.float32, device=x.device)
    dx = torch.empty_like(x) if want_dx else None
    _lib.call("va_psa_attention_bwd_bf16", _p(x), _p(dy), float(dy_scale), _p(params["w_qkv"]), _p(params["b_qkv"]),
              _p(params["w_pe"]), _p(params["b_pe"]), _p(params["w_proj"]), _p(params["b_proj"]),
              _p(dx) if dx is not None else None, _p(grads), B, C, H, W, 2, 32, _p(workspace), workspace.numel(),
              _stream(stream))
    return grads, dx


class DpStepGraph:
    """The whole data-parallel step with the peer comm — the local forward +
    backward and the all-reduce + SGD kernel — replayed from one CUDA graph
    per rank: one host launch per step instead of two library calls, so a
    rank's host, sharing the machine's cores with the other ranks, cannot
    fall behind its GPU.  The all-reduce kernel keeps its step count on the
    device, so its launch can be replayed.  The first call for a given set of
    tensors (and lr) runs the step eagerly, then captures it."""

    def __init__(self, step: PsaTrainStep, comm: "PeerGradComm"):
        self.step, self.comm = step, comm
        self._graph, self._key = None, None
        self.graph_kernels = 0     # library kernels one replay launches
        self.replayed_kernels = 0  # kernels launched by replays so far

    def __call__(self, x, target, params: dict, master, lr: float):
        key = (x.data_ptr(), target.data_ptr(), master.data_ptr(), float(lr)) + \
            tuple(params[k].data_ptr() for k in sorted(params))
        st = self.step
        if self._graph is None or self._key != key:
            st._launch(x, target, params, False, None)  # eager step: one-time set-up stays out of the graph
            self.comm.allreduce_sgd(st.grads, master, params, lr)
            torch.cuda.current_stream().synchronize()
            g = torch.cuda.CUDAGraph()
            n0 = int(_lib.lib().va_launch_count())
            with torch.cuda.graph(g, capture_error_mode="relaxed"):
                st._launch(x, target, params, False, None)
                self.comm._launch(st.grads, master, params, lr)
            self.graph_kernels = int(_lib.lib().va_launch_count()) - n0
            self._graph, self._key = g, key
            return st.loss
        self.comm.count_call()
        self._graph.replay()
        self.replayed_kernels += self.graph_kernels
        return st.loss


def dp_train_step(step: PsaTrainStep, x, target, params: dict, master, lr: float, group=None,
                  comm: PeerGradComm | None = None):
    """One data-parallel step: local fwd+bwd, all-reduce (sum) of the f32
    gradient buffer, SGD with the mean gradient — through ``comm`` (one fused
    peer-memory kernel) when given, else NCCL all-reduce + ``sgd``.  Returns
    the local loss tensor."""
    import torch.distributed as dist
    _, loss, grads, _ = step.forward_backward(x, target, params)
    if comm is not None:
        comm.allreduce_sgd(grads, master, params, lr)
        return loss
    world = 1
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(grads, op=dist.ReduceOp.SUM, group=group)
        world = dist.get_world_size(group)
    step.sgd(master, grads, params, lr, 1.0 / world)
    return loss
