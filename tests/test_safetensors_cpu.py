"""The safetensors reader and BN folding (va_safetensors_*) on the CPU.

A checkpoint is written with the reference's key layout for the C2PSA
(``model.10.cv1.conv.weight``, ``model.10.m.0.attn.qkv.bn.running_var`` …)
from the golden C2PSA fixture's parameters; the library reads it back,
folds every conv+BN pair, and the C2PSA restatement on those folded weights
must reproduce the fixture's expected output.  Malformed files are refused
with an error, not read out of bounds."""
import os
import struct

import numpy as np
import pytest
import torch

from conftest import c2psa_checkpoint, load_golden, max_abs, stage_params
from oracle import psa_oracle as po
from vision_rs_b200 import _lib, weights


def test_reads_and_folds_reference_layout(tmp_path):
    f, g = c2psa_checkpoint(tmp_path)
    prm = stage_params(g)
    with weights.SafeTensors(f) as st:
        dt, shape = st.info("model.10.cv1.conv.weight")
        assert dt == 0 and shape == tuple(prm["cv1"][0].shape)
        assert np.array_equal(st.read_f32("model.10.m.0.attn.pe.bn.running_var"), prm["m0_attn_pe"][4])
        assert st.info("model.0.conv.weight")[0] == 1  # F16
        w, b = st.fold_conv_bn("model.10.m.0.attn.qkv", eps=1e-5)
        wr, br = po.fold_bn(*prm["m0_attn_qkv"], 1e-5)
        assert max_abs(w, wr) < 1e-6 and max_abs(b, br) < 1e-6
        folded = weights.c2psa_folded(st, "model.10", eps=1e-5)  # the fixture's BN eps
    assert len(folded[2]) == 1
    y = po.c2psa_forward_folded(g["x"], *folded)
    assert max_abs(y, g["expected_output"]) < 1e-5


def test_half_precision_tensors_convert(tmp_path):
    f, g = c2psa_checkpoint(tmp_path, dtype=torch.bfloat16)
    with weights.SafeTensors(f) as st:
        w = st.read_f32("model.10.cv2.conv.weight")
    ref = torch.as_tensor(np.asarray(stage_params(g)["cv2"][0], np.float32)).bfloat16().float().numpy()
    assert np.array_equal(w, ref)
    x = np.array([1.0, -2.5, 65504.0, 6.1e-5, 3e-8, 0.0], np.float16)
    from safetensors.numpy import save_file
    p = os.path.join(tmp_path, "h.safetensors")
    save_file({"h": x}, p)
    with weights.SafeTensors(p) as st:
        assert np.array_equal(st.read_f32("h"), x.astype(np.float32))


def _raw(tmp_path, header: bytes, data: bytes = b"", size=None):
    p = os.path.join(tmp_path, "bad.safetensors")
    with open(p, "wb") as fh:
        fh.write(struct.pack("<Q", len(header) if size is None else size) + header + data)
    return p


@pytest.mark.parametrize("header,data,size", [
    (b'{"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}', b"\0" * 8, None),  # data past the end
    (b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [8, 4]}}', b"\0" * 8, None),   # begin > end
    (b'{"a": {"dtype": "F32", "shape": [2]}}', b"", None),                                 # no offsets
    (b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}', b"\0" * 8, None),   # unterminated
    (b'["not", "an", "object"]', b"", None),
    (b'{}', b"", 1 << 40),                                                                 # header size past the end
])
def test_malformed_files_are_refused(tmp_path, header, data, size):
    with pytest.raises(_lib.VisionAttnError):
        weights.SafeTensors(_raw(tmp_path, header, data, size))


def test_element_count_must_match_bytes(tmp_path):
    p = _raw(tmp_path, b'{"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}', b"\0" * 8)
    with weights.SafeTensors(p) as st:
        with pytest.raises(_lib.VisionAttnError):
            st.read_f32("a")
        with pytest.raises(_lib.VisionAttnError):
            st.info("missing")
