"""Pre-quantized weights: qlm_weight_import_int8/_int4 (device repack of the
reference Tensor's layouts) and the safetensors store (qlm_store_save/load).
A weight loaded from a file must be the same weight: identical exported codes
and scales, bit-identical products, and for files built from QuickLM's own
quantizer output, products bit-identical to QuickLM's matmul."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle.oracle import pack_q4, unpack_q4
from tests.conftest import bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def q(qlm_lib, cuda_device):
    import quicklm_b200
    return quicklm_b200


SHAPES = [(64, 128), (37, 100), (5, 33), (300, 1000), (9, 7)]


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("bits", [8, 4])
def test_save_load_round_trip(q, tmp_path, n, k, bits):
    import torch
    rng = np.random.default_rng(n * 7 + k + bits)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    a = q.Int8Weight.quantize(w, bits=bits)
    b = q.Int8Weight.quantize(w[::-1].copy(), bits=bits)
    f = tmp_path / "m.safetensors"
    q.save(str(f), {"layers.0.mlp.up_proj.weight": a, "lm_head.weight": b})
    assert q.store_info(str(f), "lm_head.weight") == (bits, n, k)
    for name, orig in (("layers.0.mlp.up_proj.weight", a), ("lm_head.weight", b)):
        got = q.Int8Weight.from_file(str(f), name)
        assert got.bits == bits and got.shape == (n, k) and got.nbytes == orig.nbytes
        ex = (lambda h: h.to_int8()) if bits == 8 else (lambda h: h.to_int4())
        (c0, s0), (c1, s1) = ex(orig), ex(got)
        assert np.array_equal(c0, c1) and bits_equal(s0, s1)
        for m in (1, 3, 8):
            x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
            y0 = q.matmul(x, orig, flags=q.SYNC)
            y1 = q.matmul(x, got, flags=q.SYNC)
            assert torch.equal(y0.view(torch.int32), y1.view(torch.int32))
        got.free()
    a.free()
    b.free()


def test_reference_bytes_load_exactly(q, refcpu, tmp_path):
    """A file built from QuickLM's own quantizer output (as a converter would
    write it) gives QuickLM's own products."""
    from safetensors.numpy import save_file
    rng = np.random.default_rng(11)
    n, k = 257, 1000
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((4, k)).astype(np.float32)
    q8, s8 = refcpu.quantize(w)
    p4, s4 = refcpu.quantize_int4(w)
    f = tmp_path / "ref.safetensors"
    save_file({"w8": q8, "w8.qscale": s8, "w4": p4, "w4.qscale": s4}, str(f),
              metadata={"qlm.w8": f"int8 k={k}", "qlm.w4": f"int4 k={k}"})
    w8 = q.Int8Weight.from_file(str(f), "w8")
    w4 = q.Int8Weight.from_file(str(f), "w4")
    y8, _ = refcpu.matmul(x, q8, s8)
    assert bits_equal(q.matmul(x, w8), y8)
    assert bits_equal(q.matmul(x, w4), refcpu.matmul_int4(x, p4, s4, k))
    # a row shard of the same file
    part = q.Int8Weight.from_file(str(f), "w8", row_begin=100, row_end=200)
    assert bits_equal(q.matmul(x, part), y8[:, 100:200])
    # the tensor-core path works on a loaded weight (range exponents computed)
    import torch
    xm = torch.from_numpy(rng.standard_normal((128, k)).astype(np.float32)).cuda()
    yt = q.matmul(xm, w8, flags=q.TENSOR | q.SYNC).cpu().numpy().astype(np.float64)
    ye = refcpu.matmul(xm.cpu().numpy(), q8, s8)[0].astype(np.float64)
    assert np.linalg.norm(yt - ye) / np.linalg.norm(ye) <= 2e-3
    for h in (w8, w4, part):
        h.free()


def test_written_file_is_standard_safetensors(q, tmp_path):
    from safetensors.numpy import load_file
    from safetensors import safe_open
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((40, 300)) * 0.02).astype(np.float32)
    a, b = q.Int8Weight.quantize(w), q.Int8Weight.quantize(w, bits=4)
    f = tmp_path / "std.safetensors"
    q.save(str(f), {"a": a, "b": b})
    t = load_file(str(f))
    qa, sa = a.to_int8()
    pb, sb = b.to_int4()
    assert np.array_equal(t["a"], qa) and bits_equal(t["a.qscale"], sa)
    assert np.array_equal(t["b"], pb) and bits_equal(t["b.qscale"], sb)
    with safe_open(str(f), "np") as fh:
        meta = fh.metadata()
    assert meta["qlm.a"] == "int8 k=300" and meta["qlm.b"] == "int4 k=300"
    a.free()
    b.free()


@pytest.mark.parametrize("bits", [8, 4])
def test_import_from_device_memory(q, coracle, bits):
    """Codes and scales already on the device are repacked in place."""
    import torch
    rng = np.random.default_rng(21 + bits)
    n, k = 96, 520
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if bits == 8:
        codes, s = coracle.quantize(w)
    else:
        v, s = coracle.quantize_q4(w)
        codes = pack_q4(v)
    host = (q.Int8Weight.from_int8(codes, s) if bits == 8 else q.Int8Weight.from_int4(codes, s, k))
    dc = torch.from_numpy(codes.view(np.uint8).copy()).cuda()
    ds = torch.from_numpy(s).cuda()
    h = ctypes.c_void_p()
    fn = q.load().qlm_weight_import_int8 if bits == 8 else q.load().qlm_weight_import_int4
    assert fn(dc.data_ptr(), ds.data_ptr(), n, k, 10, 90, 0, None, ctypes.byref(h)) == 0, q.load().qlm_last_error()
    dev = q.Int8Weight(h.value)
    x = rng.standard_normal((2, k)).astype(np.float32)
    assert bits_equal(q.matmul(x, dev), q.matmul(x, host)[:, 10:90])
    y_ref = coracle.matmul(x, codes if bits == 8 else unpack_q4(codes, k), s)
    assert bits_equal(q.matmul(x, host), y_ref)
    dev.free()
    host.free()


def test_load_errors(q, tmp_path):
    w = q.Int8Weight.quantize(np.ones((8, 64), np.float32))
    f = tmp_path / "e.safetensors"
    q.save(str(f), {"w": w})
    with pytest.raises(q.QlmError, match="no quantized weight"):
        q.Int8Weight.from_file(str(f), "v")
    with pytest.raises(q.QlmError, match="row range"):
        q.Int8Weight.from_file(str(f), "w", row_begin=4, row_end=9)
    with pytest.raises(q.QlmError, match="duplicate"):
        q._check(q.load().qlm_store_save(str(tmp_path / "d").encode(), 2, (ctypes.c_char_p * 2)(b"x", b"x"),
                                         (ctypes.c_void_p * 2)(w.handle.value, w.handle.value)))
    w.free()
