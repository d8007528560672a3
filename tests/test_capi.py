"""CPU-only checks of the C ABI library: it loads without a GPU, exports every
symbol include/qlm_b200.h declares, and rejects bad arguments on the host
before touching a device."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from tests.conftest import ROOT


def header_functions():
    with open(os.path.join(ROOT, "include", "qlm_b200.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qlm_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported(qlm_lib):
    import quicklm_b200 as q
    names = header_functions()
    assert set(names) == set(q.ABI_SYMBOLS), "binding list out of sync with the header"
    for name in names:
        assert hasattr(qlm_lib, name), f"{name} not exported"


def test_abi_version(qlm_lib):
    assert qlm_lib.qlm_abi_version() == 1


def test_null_args_rejected_on_host(qlm_lib):
    import quicklm_b200 as q
    rc = qlm_lib.qlm_linear_int8(None, 1, 16, 16, None, None, 16, 0, None)
    assert rc == 1
    assert b"NULL" in qlm_lib.qlm_last_error()
    out = ctypes.c_void_p()
    w = np.zeros((4, 8), np.float32)
    rc = qlm_lib.qlm_weight_quantize_upload(w.ctypes.data, 7, 8, 4, 8, 0, 4, 0, None, ctypes.byref(out))
    assert rc == 1 and b"dtype" in qlm_lib.qlm_last_error()
    rc = qlm_lib.qlm_weight_quantize_upload(w.ctypes.data, 0, 8, 4, 8, 2, 1, 0, None, ctypes.byref(out))
    assert rc == 1 and b"row range" in qlm_lib.qlm_last_error()
    rc = qlm_lib.qlm_weight_quantize_upload(w.ctypes.data, 0, 4, 4, 8, 0, 4, 0, None, ctypes.byref(out))
    assert rc == 1 and b"stride" in qlm_lib.qlm_last_error()
    i32, f32 = ctypes.c_int(0), ctypes.c_float(0)
    rc = qlm_lib.qlm_argmax_f32(None, 4, 0, None, ctypes.byref(i32), ctypes.byref(f32), 0, None)
    assert rc == 1 and b"NULL" in qlm_lib.qlm_last_error()
    v = np.zeros(4, np.float32)
    rc = qlm_lib.qlm_argmax_f32(v.ctypes.data, 0, 0, None, ctypes.byref(i32), ctypes.byref(f32), 0, None)
    assert rc == 1 and b"n=0" in qlm_lib.qlm_last_error()
    rc = qlm_lib.qlm_argmax_f32(v.ctypes.data, 4, 1 << 24, None, ctypes.byref(i32), ctypes.byref(f32), 0, None)
    assert rc == 1 and b"2^24" in qlm_lib.qlm_last_error()
    with pytest.raises(q.QlmError):
        q._check(1)


def test_more_entry_points_reject_bad_args_on_host(qlm_lib, tmp_path):
    """int4, store and layer-op entry points validate their arguments before any
    device work, so these run without a GPU (no pointer here is dereferenced)."""
    L = qlm_lib
    out = ctypes.c_void_p()
    w = np.zeros((4, 8), np.float32)
    buf = np.zeros(64, np.float32)
    p = buf.ctypes.data
    err = lambda: L.qlm_last_error()
    assert L.qlm_weight_quantize_upload_q4(w.ctypes.data, 7, 8, 4, 8, 0, 4, 0, None, ctypes.byref(out)) == 1
    assert b"dtype" in err()
    assert L.qlm_weight_import_int4(None, None, 4, 8, 0, 4, 0, None, ctypes.byref(out)) == 1 and b"NULL" in err()
    assert L.qlm_weight_import_int8(p, p, 4, 8, 3, 2, 0, None, ctypes.byref(out)) == 1 and b"row range" in err()
    assert L.qlm_weight_export_int4(None, None, None) == 1
    assert L.qlm_weight_bits(None) == -1
    assert L.qlm_store_save(str(tmp_path / "x").encode(), 0, None, None) == 1
    assert L.qlm_store_load(str(tmp_path / "absent").encode(), b"w", 0, -1, 0, None, ctypes.byref(out)) == 1
    assert b"cannot open" in err()
    assert L.qlm_rms_norm(None, p, p, 1, 8, 1e-6, None) == 1 and b"NULL" in err()
    assert L.qlm_rms_norm(p, p, p, 0, 8, 1e-6, None) == 1 and b"positive" in err()
    assert L.qlm_rms_norm_gain(p, p, p, 1, 0, 1e-6, None) == 1
    assert L.qlm_add_rms_norm(p, None, p, p, 1, 8, 1e-6, None) == 1
    assert L.qlm_silu_mul(p, p, 0, None) == 1 and L.qlm_silu(None, 8, None) == 1
    assert L.qlm_rope_neox(p, 1, 2, 8, 7, p, p, None) == 1 and b"RoPE" in err()  # odd rotary_dim
    assert L.qlm_rope_neox(p, 1, 2, 8, 10, p, p, None) == 1                      # rotary_dim > head_dim
    assert L.qlm_conv1d_update_tapmajor(p, p, 3, p, p, 8, 4, None) == 1 and b"ring" in err()  # oldest_tap >= 3
    assert L.qlm_l2norm_heads(p, 0, 8, 1e-6, None) == 1
    assert L.qlm_gdn_gates(p, p, None, p, p, p, 4, None) == 1
    assert L.qlm_gdn_recurrence(p, p, p, p, p, p, p, 2, 2048, None) == 1 and b"1024" in err()
    assert L.qlm_gqa_attend(p, 8, p, p, p, 3, 3, 2, 8, None, None) == 1 and b"shape" in err()  # 3 % 2 heads
    assert L.qlm_gqa_attend(p, 8, p, p, p, 1 << 20, 2, 1, 8, None, None) == 4 and b"too long" in err()


def test_weight_free_null_is_noop(qlm_lib):
    qlm_lib.qlm_weight_free(None)
    assert qlm_lib.qlm_weight_bytes(None) == 0


def test_no_oracle_in_product():
    """The product package never imports or links the checkers."""
    pkg = os.path.join(ROOT, "quicklm_b200")
    for dirpath, _, files in os.walk(pkg):
        for fn in files:
            if fn.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                with open(os.path.join(dirpath, fn), errors="ignore") as f:
                    text = f.read()
                assert "oracle" not in re.sub(r"(#|//).*", "", text).lower().replace("oracle/", ""), fn
