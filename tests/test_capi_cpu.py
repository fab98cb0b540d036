"""The C-ABI library on CPU: it loads, exports every symbol the header
declares, and its host-only functions (shape inference, BN folding, argument
validation that fails before any launch) behave like the reference's
CustomOp methods.  No compute calls: there is no GPU here."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT
from oracle import psa_oracle as po
from vision_rs_b200 import _lib
from vision_rs_b200 import psa as vp

HEADER = os.path.join(ROOT, "include", "visionattn.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(va_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    # the binding table covers exactly the header
    assert sorted(_lib.SIGNATURES) == names


def _shape(fn, inp, *extra, out_len=5):
    a = (C.c_int64 * len(inp))(*inp)
    o = (C.c_int64 * out_len)()
    r = fn(a, len(inp), *extra, o) if extra else fn(a, len(inp), o)
    return r, list(o)[:max(r, 0)]


def test_shape_inference_matches_reference_customops():
    lib = _lib.lib()
    # psa.rs:766-776 (test_c2psa_yolo26.rs:128: [2,4,2,256,32] at B=2, 16x16)
    r, s = _shape(lib.va_psa_pack_qkv_infer_output_shape, [2, 256, 16, 16], 2)
    assert (r, s) == (5, [2, 4, 2, 256, 32])
    r, s = _shape(lib.va_psa_pack_qkv_infer_output_shape, [-1, 256, 16, 16], 2)
    assert s[0] == -1
    r, s = _shape(lib.va_psa_extract_v_infer_output_shape, [2, 256, 16, 16])
    assert s == [2, 128, 16, 16]
    a = (C.c_int64 * 4)(2, 2, 256, 32)
    o = (C.c_int64 * 4)()
    assert lib.va_psa_merge_attn_infer_output_shape(a, 4, 2, 16, 16, o) == 4
    assert list(o) == [2, 128, 16, 16]   # test_c2psa_yolo26.rs:132
    r, s = _shape(lib.va_flash_attention2_infer_output_shape, [2, 4, 2, 256, 32])
    assert s == [2, 2, 256, 32]
    # bad rank
    r, _ = _shape(lib.va_psa_extract_v_infer_output_shape, [2, 256, 16])
    assert r == -1


def test_python_customop_mirror_shapes():
    assert vp.PsaPackQkvOp(32, 2).infer_output_shape([[None, 256, 20, 20]]) == [None, 4, 2, 400, 32]
    assert vp.PsaExtractVOp(32, 2).infer_output_shape([[2, 256, 20, 20]]) == [2, 128, 20, 20]
    assert vp.PsaMergeAttnOp(32, 2, 20, 20).infer_output_shape([[2, 2, 400, 32]]) == [2, 128, 20, 20]
    assert vp.FlashAttn2PsaOp.new_lo(32).infer_output_shape([[2, 4, 2, 400, 32]]) == [2, 2, 400, 32]
    assert vp.FlashAttn2PsaOp.new_hi(32).inner.v_section == 3
    names = [vp.PsaPackQkvOp(32, 2).name(), vp.FlashAttn2PsaOp.new_lo(32).name(),
             vp.PsaMergeAttnOp(32, 2, 4, 4).name(), vp.PsaExtractVOp(32, 2).name()]
    assert names == ["psa_pack_qkv", "flash_attention2_forward", "psa_merge_attn_nchw", "psa_extract_v_nchw"]
    assert vp.FlashAttn2PsaOp.new_lo(32).inner.param_shapes([[2, 4, 2, 400, 32]], None) == [[1600]]


def test_fold_bn_host_function_matches_oracle():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((256, 128, 1, 1)).astype(np.float32)
    g, b, m = (rng.standard_normal(256).astype(np.float32) for _ in range(3))
    v = rng.uniform(0.5, 2, 256).astype(np.float32)
    import torch
    wf, bf = vp.fold_bn(torch.tensor(w), g, b, m, v, 1e-3)
    wo, bo = po.fold_bn(w, g, b, m, v, 1e-3)
    assert np.abs(wf.numpy() - wo).max() < 1e-5
    assert np.abs(bf.numpy() - bo).max() < 1e-5


def test_argument_validation_fails_before_launch():
    lib = _lib.lib()
    # qkv_h not a multiple of 4*num_heads → VA_ERR_SHAPE, message set, nothing launched
    rc = lib.va_psa_pack_qkv_f32(None, None, 250, 4, 4, 2, 2, None)
    assert rc == 1
    assert b"multiple" in lib.va_get_last_error_string()
    rc = lib.va_flash_attention2_forward_f32(None, None, None, None, None, 16, 16, 0.1, float("-inf"), 4, 48, None)
    assert rc == 1 and b"head_dim" in lib.va_get_last_error_string()
    rc = lib.va_psa_attention_fwd_bf16(*([None] * 8), 2, 128, 4, 4, 2, 32, None, 0, None)
    assert rc == 6  # workspace missing
    with pytest.raises(_lib.VisionAttnError):
        _lib.call("va_psa_merge_attn_nchw_f32", None, None, None, 127, 4, 4, 2, 2, None)
    # peer all-reduce set-up: rank/world and the buffer size are checked before any CUDA call
    h, buf = C.c_void_p(), C.create_string_buffer(64)
    assert lib.va_dp_comm_create(0, 9, 50816, 0, C.byref(h), buf) == 1 and b"world" in lib.va_get_last_error_string()
    assert lib.va_dp_comm_create(2, 2, 50816, 0, C.byref(h), buf) == 1
    assert lib.va_dp_comm_create(0, 2, 1000, 0, C.byref(h), buf) == 1 and b"count" in lib.va_get_last_error_string()
    assert lib.va_dp_comm_create(0, 2, 50816, -1, C.byref(h), buf) == 1 and b"timeout" in lib.va_get_last_error_string()
    assert lib.va_psa_dp_allreduce_sgd(None, *([None] * 2), 0.1, *([None] * 6), None) == 1
    assert lib.va_dp_comm_disconnect(None) == 1
    assert lib.va_dp_comm_destroy(None) == 0
    # conv: channel counts, kernel size, stride and alignment are checked before any CUDA call
    conv = lambda x, B, H, W, ci, co, k, s: lib.va_conv_nhwc_bf16(x, 4096, 8192, 12288, B, H, W, ci, co, k, s, 1, None)
    assert conv(1024, 1, 8, 8, 12, 16, 3, 1) == 1 and b"Cin" in lib.va_get_last_error_string()
    assert conv(1024, 1, 8, 8, 16, 20, 3, 1) == 1 and b"Cout" in lib.va_get_last_error_string()
    assert conv(1024, 1, 8, 8, 16, 16, 5, 1) == 1 and b"kernel size" in lib.va_get_last_error_string()
    assert conv(1024, 1, 8, 8, 16, 16, 3, 3) == 1 and b"stride" in lib.va_get_last_error_string()
    assert conv(1024, 1, 0, 8, 16, 16, 3, 1) == 1
    assert conv(None, 1, 8, 8, 16, 16, 3, 1) == 1
    assert conv(1026, 1, 8, 8, 16, 16, 3, 1) == 4 and b"alignment" in lib.va_get_last_error_string()
    # f32 fused backward: null pointers, the width rule and the workspace are checked before any launch
    bwd = lambda x, C, nh, ws, n: lib.va_psa_attention_bwd_f32(x, 64, 128, 192, 256, 320, 384, 448, None, 512, 2,
                                                                C, 4, 4, nh, 32, ws, n, None)
    assert bwd(None, 128, 2, 4096, 1 << 20) == 1 and b"null" in lib.va_get_last_error_string()
    assert bwd(1024, 100, 2, 4096, 1 << 20) == 1 and b"num_heads" in lib.va_get_last_error_string()
    assert bwd(1024, 128, 2, None, 0) == 6 and b"workspace" in lib.va_get_last_error_string()
    need = lib.va_psa_attention_bwd_f32_workspace_bytes(2, 128, 4, 4, 2, 32)
    assert bwd(1024, 128, 2, 4096, need - 1) == 6


def test_workspace_query():
    lib = _lib.lib()
    n32 = lib.va_psa_attention_workspace_bytes(2, 128, 20, 20, 2, 32, 0)
    n16 = lib.va_psa_attention_workspace_bytes(2, 128, 20, 20, 2, 32, 1)
    assert n32 > 0 and n16 > 0 and n16 < n32
    assert lib.va_psa_attention_workspace_bytes(0, 128, 20, 20, 2, 32, 0) == 0
    # the f32 backward holds the forward's intermediates plus its own gradient buffers
    nb = lib.va_psa_attention_bwd_f32_workspace_bytes(2, 128, 20, 20, 2, 32)
    assert nb > n32 and lib.va_psa_attention_bwd_f32_workspace_bytes(2, 128, 0, 20, 2, 32) == 0
