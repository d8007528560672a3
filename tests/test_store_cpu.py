"""Pre-quantized safetensors files: header parsing and validation through the
C ABI (qlm_store_info runs on the host only). Files are written here with the
`safetensors` library in the layout the library stores: codes in the
reference Tensor's layout ("I8" [rows, K] or "U8" [rows, (K+1)/2]), scales
"<name>.qscale" F32 [rows, ceil(K/32)], metadata "qlm.<name>"."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest


@pytest.fixture(scope="module")
def q(qlm_lib):
    import quicklm_b200
    return quicklm_b200


def _write(path, tensors, metadata):
    from safetensors.numpy import save_file
    save_file(tensors, str(path), metadata=metadata)


def _raw(path, header: dict, data: bytes):
    h = json.dumps(header).encode()
    path.write_bytes(struct.pack("<Q", len(h)) + h + data)


def test_info_int8_and_int4(q, coracle, tmp_path):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((37, 100)) * 0.02).astype(np.float32)
    q8, s8 = coracle.quantize(w)
    v4, s4 = coracle.quantize_q4(w)
    from oracle.oracle import pack_q4
    p4 = pack_q4(v4)
    f = tmp_path / "w.safetensors"
    _write(f, {"a": q8, "a.qscale": s8, "b": p4, "b.qscale": s4},
           {"qlm.a": "int8 k=100", "qlm.b": "int4 k=100"})
    assert q.store_info(str(f), "a") == (8, 37, 100)
    assert q.store_info(str(f), "b") == (4, 37, 100)
    with pytest.raises(q.QlmError, match="no quantized weight"):
        q.store_info(str(f), "c")


def test_odd_k_int4(q, tmp_path):
    f = tmp_path / "o.safetensors"
    _write(f, {"w": np.full((3, 4), 0x88, np.uint8), "w.qscale": np.ones((3, 1), np.float32)}, {"qlm.w": "int4 k=7"})
    assert q.store_info(str(f), "w") == (4, 3, 7)


@pytest.mark.parametrize("case", [
    "dtype", "shape", "scale_shape", "no_meta", "bad_meta", "kind", "no_scales",
])
def test_inconsistent_entries_rejected(q, tmp_path, case):
    codes = np.zeros((4, 64), np.int8)
    scales = np.ones((4, 2), np.float32)
    meta = {"qlm.w": "int8 k=64"}
    tensors = {"w": codes, "w.qscale": scales}
    if case == "dtype":
        tensors["w"] = codes.view(np.uint8)
    elif case == "shape":
        tensors["w"] = np.zeros((4, 63), np.int8)
    elif case == "scale_shape":
        tensors["w.qscale"] = np.ones((4, 3), np.float32)
    elif case == "no_meta":
        meta = {}
    elif case == "bad_meta":
        meta = {"qlm.w": "int8"}
    elif case == "kind":
        meta = {"qlm.w": "int3 k=64"}
    elif case == "no_scales":
        del tensors["w.qscale"]
    f = tmp_path / "bad.safetensors"
    _write(f, tensors, meta)
    with pytest.raises(q.QlmError) as e:
        q.store_info(str(f), "w")
    assert e.value.status == 1


def _entry(dtype, shape, a, b):
    return {"dtype": dtype, "shape": shape, "data_offsets": [a, b]}


@pytest.mark.parametrize("case", ["ok", "offsets_out_of_file", "size_mismatch", "truncated_header",
                                  "header_too_long", "not_object", "deep", "fraction", "negative"])
def test_header_bounds(q, tmp_path, case):
    meta = {"qlm.w": "int8 k=32"}
    header = {"__metadata__": meta, "w.qscale": _entry("F32", [2, 1], 0, 8), "w": _entry("I8", [2, 32], 8, 72)}
    data = bytes(72)
    f = tmp_path / "h.safetensors"
    if case == "offsets_out_of_file":
        header["w"] = _entry("I8", [2, 32], 8, 80)
    elif case == "size_mismatch":
        header["w"] = _entry("I8", [2, 32], 8, 40)
    elif case == "fraction":
        header["w"] = {"dtype": "I8", "shape": [2.5, 32], "data_offsets": [8, 72]}
    elif case == "negative":
        header["w"] = _entry("I8", [2, 32], -8, 72)
    if case == "truncated_header":
        h = json.dumps(header).encode()[:-5]
        f.write_bytes(struct.pack("<Q", len(h)) + h + data)
    elif case == "header_too_long":
        h = json.dumps(header).encode()
        f.write_bytes(struct.pack("<Q", len(h) + 1000) + h)
    elif case == "not_object":
        h = b"[1, 2, 3]"
        f.write_bytes(struct.pack("<Q", len(h)) + h)
    elif case == "deep":
        h = ("[" * 40 + "]" * 40).encode()
        h = b'{"x": ' + h + b"}"
        f.write_bytes(struct.pack("<Q", len(h)) + h)
    else:
        _raw(f, header, data)
    if case == "ok":
        assert q.store_info(str(f), "w") == (8, 2, 32)
        return
    with pytest.raises(q.QlmError) as e:
        q.store_info(str(f), "w")
    assert e.value.status == 1


def test_missing_and_tiny_files(q, tmp_path):
    with pytest.raises(q.QlmError, match="cannot open"):
        q.store_info(str(tmp_path / "absent.safetensors"), "w")
    f = tmp_path / "tiny"
    f.write_bytes(b"\x01\x02")
    with pytest.raises(q.QlmError, match="too small"):
        q.store_info(str(f), "w")
