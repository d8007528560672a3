"""Int4 (Q4_0) weights: the quantizer must reproduce QuickLM's
get_tensor_keep_int4 byte for byte (src/io/safetensors.cpp:393-515, 587-656)
and the exact GEMV must reproduce its int4 math::matmul bit for bit
(src/ops/math_ops.cpp:581-794, 837-854). The checkers are the reference's own
CPU code compiled from its sources (oracle/_ref) and the C restatement."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import unpack_q4
from tests.conftest import bits_equal
from tests.golden.cases import SMALL_CASES, make_small_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def q(qlm_lib, cuda_device):
    import quicklm_b200
    return quicklm_b200


def _torch_src(w):
    import torch
    if w.dtype == np.uint16:
        return torch.from_numpy(w.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(w).cuda()


@pytest.mark.parametrize("idx", range(len(SMALL_CASES)))
def test_int4_matches_reference(q, refcpu, coracle, idx):
    import torch
    x, w = make_small_case(SMALL_CASES[idx])
    k = w.shape[1]
    ref_p, ref_s = refcpu.quantize_int4(w)
    for src in (w, _torch_src(w)):  # staged host upload and on-device source
        w4 = q.Int8Weight.quantize(src, bits=4)
        assert w4.bits == 4
        p, s = w4.to_int4()
        assert np.array_equal(p, ref_p)
        assert bits_equal(s, ref_s)
        y_ref = refcpu.matmul_int4(x, ref_p, ref_s, k)
        # the int4 product is the int8 arithmetic on the unpacked values
        assert bits_equal(coracle.matmul(x, unpack_q4(ref_p, k), ref_s), y_ref)
        assert bits_equal(q.matmul(x, w4), y_ref)  # host buffers
        yd = q.matmul(torch.from_numpy(x).cuda(), w4, flags=q.SYNC)
        assert bits_equal(yd.cpu().numpy(), y_ref)
        w4.free()


@pytest.mark.parametrize("m", [1, 2, 5, 8])
def test_int4_row_shards(q, refcpu, m):
    rng = np.random.default_rng(100 + m)
    n, k = 517, 1000
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref_p, ref_s = refcpu.quantize_int4(w)
    y_ref = refcpu.matmul_int4(x, ref_p, ref_s, k)
    for b, e in ((0, 200), (200, 517), (333, 334)):
        w4 = q.Int8Weight.quantize(w, row_begin=b, row_end=e, bits=4)
        p, s = w4.to_int4()
        assert np.array_equal(p, ref_p[b:e]) and bits_equal(s, ref_s[b:e])
        assert bits_equal(q.matmul(x, w4), y_ref[:, b:e])
        w4.free()


# Benchmark-sized projections (the first is a large vocabulary head): the
# quantizer is row-local, so a sample of rows is checked against the reference,
# and the full product against the int8 path fed the unpacked int4 values.
FULL = [(6144, 2048), (9728, 2560), (2560, 9728), (151936, 2560)]


@pytest.mark.slow
@pytest.mark.parametrize("n,k", FULL)
def test_int4_full_size(q, refcpu, n, k):
    import torch
    g = torch.Generator(device="cuda").manual_seed(n ^ k)
    wd = torch.randn((n, k), device="cuda", generator=g) * 0.02
    w4 = q.Int8Weight.quantize(wd, bits=4)
    k_pad = (k + 127) // 128 * 128
    assert w4.nbytes == n * k_pad // 2 + n * (k_pad // 32) * 4
    p, s = w4.to_int4()
    rows = np.unique(np.random.default_rng(n).integers(0, n, 64))
    rp, rs = refcpu.quantize_int4(wd[torch.from_numpy(rows).cuda()].cpu().numpy())
    assert np.array_equal(p[rows], rp) and bits_equal(s[rows], rs)
    del wd
    w8 = q.Int8Weight.from_int8(unpack_q4(p, k), s)
    for m in (1, 4, 8):
        x = torch.randn((m, k), device="cuda", generator=g)
        y4 = q.matmul(x, w4, flags=q.SYNC)
        y8 = q.matmul(x, w8, flags=q.SYNC)
        assert torch.equal(y4.view(torch.int32), y8.view(torch.int32))
    xs = torch.randn((2, k), device="cuda", generator=g)
    ys = refcpu.matmul_int4(xs.cpu().numpy(), p[rows], s[rows], k)
    assert bits_equal(q.matmul(xs, w4, flags=q.SYNC).cpu().numpy()[:, rows], ys)
    w4.free()
    w8.free()


@pytest.mark.parametrize("m", [1, 3, 8])
def test_int4_grouped(q, m):
    import torch
    rng = np.random.default_rng(7 + m)
    k = 1000
    ws = [q.Int8Weight.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), bits=4)
          for n in (300, 45, 1024)]
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    ys = q.matmul_grouped(x, ws, flags=q.SYNC)
    for w, y in zip(ws, ys):
        assert torch.equal(y.view(torch.int32), q.matmul(x, w, flags=q.SYNC).view(torch.int32))
    for w in ws:
        w.free()


def test_int4_rejections(q):
    import torch
    w = np.random.default_rng(1).standard_normal((64, 256)).astype(np.float32)
    w4 = q.Int8Weight.quantize(w, bits=4)
    w8 = q.Int8Weight.quantize(w)
    x = torch.zeros((4, 256), device="cuda")
    with pytest.raises(q.QlmError) as e:
        q.matmul(x, w4, flags=q.TENSOR | q.SYNC)  # the tensor-core path serves int8 only
    assert e.value.status == 4
    with pytest.raises(q.QlmError):
        w4.to_int8()
    with pytest.raises(q.QlmError):
        w8.to_int4()
    with pytest.raises(q.QlmError):
        q.matmul_grouped(x, [w4, w8])              # int8 and int4 in one group
    with pytest.raises(q.QlmError):
        q.Int8Weight.quantize(w, bits=3)
    assert w4.nbytes * 8 < w8.nbytes * 5           # half the codes, the same scales
    w4.free()
    w8.free()
