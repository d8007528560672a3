"""Grouped exact GEMV (qlm_linear_int8_grouped): several weights that share the
activations in one launch. Each output must be bit-identical to the
single-weight exact path (itself pinned bit-for-bit to QuickLM's math::matmul
by test_gpu_exact.py) and to the CPU restatement."""
from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def q(qlm_lib, cuda_device):
    import quicklm_b200
    return quicklm_b200


GROUPS = {
    "gate_up": [(3584, 1024), (3584, 1024)],
    "qkv": [(1024, 1024), (256, 1024), (256, 1024)],
    "ragged": [(130, 1000), (7, 1000), (600, 1000)],
    "eight": [(40 + 13 * i, 384) for i in range(8)],
}


@pytest.mark.parametrize("name", sorted(GROUPS))
@pytest.mark.parametrize("m", [1, 3, 8, 11])
def test_grouped_matches_single(q, name, m):
    import torch
    shapes = GROUPS[name]
    k = shapes[0][1]
    rng = np.random.default_rng(hash((name, m)) % (1 << 32))
    ws = [q.Int8Weight.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32)) for n, _ in shapes]
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    ys = q.matmul_grouped(x, ws, flags=q.SYNC)
    for w, y in zip(ws, ys):
        y1 = q.matmul(x, w, flags=q.SYNC)
        assert bits_equal(y.cpu().numpy(), y1.cpu().numpy())
    for w in ws:
        w.free()


def test_grouped_matches_oracle_and_strided_outputs(q, coracle):
    import torch
    rng = np.random.default_rng(9)
    k = 300
    mats = [(rng.standard_normal((n, k)) * 0.02).astype(np.float32) for n in (50, 33)]
    x = rng.standard_normal((5, k)).astype(np.float32)
    ws = [q.Int8Weight.quantize(w) for w in mats]
    out = torch.full((5, 200), 7.0, device="cuda")
    ys = [out[:, 0:50], out[:, 100:133]]  # row stride 200
    q.matmul_grouped(torch.from_numpy(x).cuda(), ws, ys, flags=q.SYNC)
    host = out.cpu().numpy()
    for w, (c0, n) in zip(mats, ((0, 50), (100, 33))):
        qq, ss = coracle.quantize(w)
        assert bits_equal(host[:, c0:c0 + n], coracle.matmul(x, qq, ss))
    assert np.all(host[:, 50:100] == 7.0) and np.all(host[:, 133:] == 7.0)
    for w in ws:
        w.free()


def test_grouped_rejects_bad_groups(q):
    import torch
    a = q.Int8Weight.quantize(np.zeros((8, 64), np.float32))
    b = q.Int8Weight.quantize(np.zeros((8, 32), np.float32))
    x = torch.zeros((1, 64), device="cuda")
    with pytest.raises(q.QlmError):
        q.matmul_grouped(x, [a, b])          # different k
    with pytest.raises(q.QlmError):
        q.matmul_grouped(x, [a] * 9)         # more than 8 weights
    a.free()
    b.free()
