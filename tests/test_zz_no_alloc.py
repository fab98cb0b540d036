"""The allocation-free PSA Attention entry point (va_psa_attention_fwd_bf16_noalloc).

Some callers cannot give the op a workspace: a graph runtime that plans all
of its device buffers before it runs, or host code that must not enter a
device allocator while it runs.  They call the noalloc entry point, which
uses a scratch area built into the library instead.  This test calls it
through the C ABI twice in a row and checks each result against the
workspace entry point on the same inputs (the kernels are the same, so the
outputs must match bit for bit), plus the size limit.

Named so that pytest collects it last: it must pass both on its own in a
fresh process and after every other test."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import psa_oracle as po
from vision_rs_b200 import _lib

pytestmark = pytest.mark.gpu


def _ptr(t):
    return t.data_ptr()


def _inputs(B, H, W, seed):
    p = po.psa_synthetic(B, H, W, seed=seed)
    bf = lambda a: torch.as_tensor(a).to("cuda", torch.bfloat16).contiguous()
    f32 = lambda a: torch.as_tensor(a).to("cuda", torch.float32).contiguous()
    return dict(x=bf(p["x"]), w_qkv=bf(p["w_qkv"]).reshape(256, 128), b_qkv=f32(p["b_qkv"]),
                w_pe=bf(p["w_pe"]), b_pe=f32(p["b_pe"]), w_proj=bf(p["w_proj"]).reshape(128, 128),
                b_proj=f32(p["b_proj"]))


def _args(t, y):
    B, C, H, W = t["x"].shape
    return (_ptr(t["x"]), _ptr(t["w_qkv"]), _ptr(t["b_qkv"]), _ptr(t["w_pe"]), _ptr(t["b_pe"]), _ptr(t["w_proj"]),
            _ptr(t["b_proj"]), _ptr(y), B, C, H, W, 2, 32)


def test_noalloc_matches_workspace_entry_two_calls_in_a_row(cuda):
    st = torch.cuda.current_stream().cuda_stream
    lib = _lib.lib()
    for call, (B, H, W, seed) in enumerate([(2, 40, 40, 21), (3, 20, 20, 22)]):
        t = _inputs(B, H, W, seed)
        need = int(lib.va_psa_attention_workspace_bytes(B, 128, H, W, 2, 32, 1))
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        y_ref = torch.empty_like(t["x"])
        _lib.call("va_psa_attention_fwd_bf16", *_args(t, y_ref), _ptr(ws), need, st)
        y = torch.full_like(t["x"], float("nan"))
        _lib.call("va_psa_attention_fwd_bf16_noalloc", *_args(t, y), st)
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref), f"call {call}: noalloc output differs from the workspace entry point"
    status = ctypes.c_int(-1)
    _lib.call("va_device_status_read", ctypes.byref(status), st)
    assert status.value == 0


def test_noalloc_rejects_problems_larger_than_its_scratch(cuda):
    st = torch.cuda.current_stream().cuda_stream
    t = _inputs(1, 40, 40, 23)
    y = torch.empty_like(t["x"])
    args = list(_args(t, y))
    args[8] = 64  # B = 64 at 40x40 needs far more than the 16 MiB built-in scratch
    rc = _lib.lib().va_psa_attention_fwd_bf16_noalloc(*args, st)
    assert rc == 6  # VA_ERR_WORKSPACE, before any launch
    assert b"scratch" in _lib.lib().va_get_last_error_string()
