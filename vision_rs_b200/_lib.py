"""ctypes binding of ``libvisionattn.so`` — the C ABI declared in
``include/visionattn.h``.

The library is loaded from this package directory (built in-tree by
``vision_rs_b200.build``).  There is no fallback: if the shared object is
missing or a symbol is absent, loading raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvisionattn.so")

P = C.c_void_p
I = C.c_int
F = C.c_float
I64P = C.POINTER(C.c_int64)
SZ = C.c_size_t
LL = C.c_longlong
S = C.c_void_p  # stream

# name -> (restype, argtypes); mirrors include/visionattn.h
SIGNATURES: dict[str, tuple] = {
    "va_version": (I, []),
    "va_get_last_error_string": (C.c_char_p, []),
    "va_launch_count": (C.c_uint64, []),
    "va_psa_pack_qkv_infer_output_shape": (I, [I64P, I, I, I64P]),
    "va_psa_extract_v_infer_output_shape": (I, [I64P, I, I64P]),
    "va_psa_merge_attn_infer_output_shape": (I, [I64P, I, I, C.c_int64, C.c_int64, I64P]),
    "va_flash_attention2_infer_output_shape": (I, [I64P, I, I64P]),
    "va_psa_pack_qkv_f32": (I, [P, P, I, I, I, I, I, S]),
    "va_psa_pack_qkv_bf16": (I, [P, P, I, I, I, I, I, S]),
    "va_psa_pack_qkv_backward_f32": (I, [P, P, I, I, I, I, I, S]),
    "va_psa_extract_v_nchw_f32": (I, [P, P, I, I, I, I, I, I, S]),
    "va_psa_extract_v_nchw_bf16": (I, [P, P, I, I, I, I, I, I, S]),
    "va_psa_extract_v_backward_f32": (I, [P, P, I, I, I, I, I, I, S]),
    "va_psa_merge_attn_nchw_f32": (I, [P, P, P, I, I, I, I, I, S]),
    "va_psa_merge_attn_nchw_bf16": (I, [P, P, P, I, I, I, I, I, S]),
    "va_psa_merge_attn_backward_f32": (I, [P, P, P, I, I, I, I, I, S]),
    "va_flash_attention2_forward_f32": (I, [P, P, P, P, P, I, I, F, F, I, I, S]),
    "va_flash_attention2_forward_bf16": (I, [P, P, P, P, P, I, I, F, F, I, I, S]),
    "va_flash_attention2_backward_dq_f32": (I, [P, P, P, P, P, P, P, I, I, F, I, I, S]),
    "va_flash_attention2_backward_dkv_f32": (I, [P, P, P, P, P, P, P, P, I, I, F, I, I, S]),
    "va_psa_fa2_backward_f32": (I, [P, P, P, P, P, P, P, P, P, I, F, I, I, S]),
    "va_fold_bn_f32": (I, [P, P, P, P, P, F, I, I, P, P]),
    "va_conv1x1_bias_f32": (I, [P, P, P, P, I, I, I, I, S]),
    "va_dwconv3x3_bias_f32": (I, [P, P, P, P, I, I, I, I, S]),
    "va_dwconv3x3_backward_f32": (I, [P, P, P, P, P, I, I, I, I, S]),
    "va_psa_attention_workspace_bytes": (SZ, [I, I, I, I, I, I, I]),
    "va_psa_attention_fwd_f32": (I, [P, P, P, P, P, P, P, P, I, I, I, I, I, I, P, SZ, S]),
    "va_psa_attention_fwd_bf16": (I, [P, P, P, P, P, P, P, P, I, I, I, I, I, I, P, SZ, S]),
    "va_msdeform_attn_fwd_f32": (I, [P, P, P, P, P, P, I, I, I, I, I, I, I, S]),
    "va_msdeform_attn_fwd_bf16": (I, [P, P, P, P, P, P, I, I, I, I, I, I, I, S]),
    "va_msdeform_attn_bwd_workspace_bytes": (SZ, [I, I, I, I, I]),
    "va_msdeform_attn_bwd_f32": (I, [P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, P, SZ, S]),
    "va_msdeform_attn_bwd_bf16": (I, [P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, P, SZ, S]),
    "va_psa_flash_attention_fwd_f16": (I, [P, P, P, P, I, I, I, I, S]),
    "va_psa_attention_fwd_bf16_noalloc": (I, [P, P, P, P, P, P, P, P, I, I, I, I, I, I, S]),
    "va_dinov2_attention_workspace_bytes": (SZ, [I, I, I]),
    "va_dinov2_attention_fwd_bf16": (I, [P, P, P, P, I, I, I, I, P, SZ, S]),
    "va_dinov2_qkv_linear_bf16": (I, [P, P, P, P, I, I, S]),
    "va_dinov2_flash_attention_fwd_f16": (I, [P, P, P, I, I, I, S]),
    "va_dinov2_window_partition_bf16": (I, [P, P, I, I, I, I, I, S]),
    "va_dinov2_window_unpartition_bf16": (I, [P, P, I, I, I, I, I, S]),
    "va_psa_train_workspace_bytes": (SZ, [I, I, I]),
    "va_psa_train_fwd_bwd_bf16": (I, [P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, P, SZ, S]),
    "va_psa_sgd_update": (I, [P, P, F, F, P, P, P, P, P, P, S]),
    "va_gemm_f16": (I, [P, I, LL, LL, I, P, I, LL, LL, I, P, I, LL, LL, I, I, I, I, F, S]),
    "va_psa_block_workspace_bytes": (SZ, [I, I, I, I]),
    "va_psa_block_fwd_bf16": (I, [P, P, P, I, I, I, I, P, SZ, S]),
    "va_c2psa_workspace_bytes": (SZ, [I, I, I, I, I]),
    "va_c2psa_fwd_bf16": (I, [P, P, P, I, P, P, P, P, I, I, I, I, P, SZ, S]),
    "va_conv_nhwc_bf16": (I, [P, P, P, P, I, I, I, I, I, I, I, I, S]),
    "va_psa_attention_bwd_f32_workspace_bytes": (SZ, [I, I, I, I, I, I]),
    "va_psa_attention_bwd_f32": (I, [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, P, SZ, S]),
    "va_psa_attention_bwd_workspace_bytes": (SZ, [I, I, I]),
    "va_psa_attention_bwd_bf16": (I, [P, P, F, P, P, P, P, P, P, P, P, I, I, I, I, I, I, P, SZ, S]),
    "va_flash_attention2_tc_workspace_bytes": (SZ, [I, I, I]),
    "va_flash_attention2_forward_tc_bf16": (I, [P, P, P, P, P, I, I, F, F, I, I, P, SZ, S]),
    "va_conv_weight_ohwi_bf16": (I, [P, P, I, I, I, S]),
    "va_safetensors_open": (I, [C.c_char_p, C.POINTER(P)]),
    "va_safetensors_close": (None, [P]),
    "va_safetensors_tensor_info": (I, [P, C.c_char_p, C.POINTER(C.c_int), I64P, C.POINTER(C.c_int)]),
    "va_safetensors_read_f32": (I, [P, C.c_char_p, P, SZ]),
    "va_safetensors_fold_conv_bn": (I, [P, C.c_char_p, F, P, P, SZ, I]),
    "va_dp_comm_create": (I, [I, I, I, I, C.POINTER(P), P]),
    "va_dp_comm_connect": (I, [P, P]),
    "va_dp_comm_status": (I, [P, C.POINTER(C.c_int)]),
    "va_dp_comm_disconnect": (I, [P]),
    "va_dp_comm_destroy": (I, [P]),
    "va_psa_dp_allreduce_sgd": (I, [P, P, P, F, P, P, P, P, P, P, S]),
    "va_device_status_read": (I, [C.POINTER(C.c_int), S]),
    "va_device_status_clear": (I, [S]),
}


class VisionAttnError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


_lib = None


def lib() -> C.CDLL:
    """Load (once) and return the library with all signatures bound."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `python -m vision_rs_b200.build`")
        lb = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lb, name)  # AttributeError if the export is missing
            fn.restype = res
            fn.argtypes = args
        _lib = lb
    return _lib


class PsaBlockWeights(C.Structure):
    """``va_psa_block_weights``: device pointers of one PSABlock's folded weights."""
    _fields_ = [(n, P) for n in ("w_qkv", "b_qkv", "w_pe", "b_pe", "w_proj", "b_proj", "w_ffn0", "b_ffn0",
                                 "w_ffn1", "b_ffn1")]


def call(name: str, *args) -> int:
    """Call a status-returning entry point and raise on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        msg = lib().va_get_last_error_string().decode(errors="replace")
        raise VisionAttnError(name, rc, msg)
    return rc
