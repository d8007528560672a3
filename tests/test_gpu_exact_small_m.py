"""The exact product for 9..64 activation rows in one launch (gemm_exact_kernel):
every row of an M-row product must equal the M=1 product of that row (the
GEMV, pinned bit-for-bit to QuickLM's math::matmul by test_gpu_exact.py) and
the CPU restatement of the reference. Shapes cover the three activation-row
buckets (16, 32, 64 staged rows), CTAs that work several passes with a short
last one, ragged K with a scalar tail, K below one block, int4 codes and
matrices of fewer than 4 rows per SM."""
from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import bits_equal

pytestmark = pytest.mark.gpu

SHAPES = [
    (1000, 640, 8),    # one pass per CTA
    (5000, 650, 8),    # two passes at 64 rows (the second 1-2 rows); ragged K
    (20000, 256, 8),   # several passes in every bucket
    (37, 1000, 8),     # fewer than 4 rows per SM
    (3, 256, 8),
    (700, 20, 8),      # K < 32: the tail only
    (5000, 650, 4),
    (2560, 2560, 4),
]
MS = (9, 16, 17, 31, 32, 33, 48, 63, 64)


@pytest.fixture(scope="module")
def q(qlm_lib, cuda_device):
    import quicklm_b200
    return quicklm_b200


@pytest.mark.parametrize("n,k,bits", SHAPES)
def test_rows_match_single_row_products(q, n, k, bits):
    rng = np.random.default_rng(n * 7 + k + bits)
    wf = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((64, k)).astype(np.float32)
    x[5, :7] = 0.0
    w = q.Int8Weight.quantize(wf, bits=bits)
    y64 = q.matmul(x, w)
    rows = range(64) if n * k <= 2_000_000 else (0, 1, 8, 15, 16, 31, 32, 47, 63)
    for i in rows:
        assert bits_equal(q.matmul(x[i], w), y64[i:i + 1]), f"row {i}"
    for mm in MS:
        assert bits_equal(q.matmul(x[:mm], w), y64[:mm]), f"M={mm}"
    w.free()


@pytest.mark.parametrize("n,k", [(37, 1000), (300, 650), (64, 20)])
def test_matches_oracle(q, coracle, n, k):
    rng = np.random.default_rng(n + k)
    wf = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((33, k)).astype(np.float32)
    x[3, 5] = np.inf
    x[7, 9] = np.nan
    w = q.Int8Weight.quantize(wf)
    qq, ss = coracle.quantize(wf)
    for mm in (9, 16, 33):
        assert bits_equal(q.matmul(x[:mm], w), coracle.matmul(x[:mm], qq, ss)), f"M={mm}"
    w.free()


def test_grouped_small_m_matches_single(q):
    import torch
    rng = np.random.default_rng(21)
    k = 1024
    ws = [q.Int8Weight.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32)) for n in (4096, 16, 2048)]
    for mm in (12, 24, 64):
        x = torch.from_numpy(rng.standard_normal((mm, k)).astype(np.float32)).cuda()
        ys = q.matmul_grouped(x, ws, flags=q.SYNC)
        for w, y in zip(ws, ys):
            assert bits_equal(y.cpu().numpy(), q.matmul(x, w, flags=q.SYNC).cpu().numpy())
            assert bits_equal(y[mm - 1:].cpu().numpy(), q.matmul(x[mm - 1], w, flags=q.SYNC).cpu().numpy())
    for w in ws:
        w.free()


def test_forced_kernel_on_tall_matrix_matches_default(qlm_lib, cuda_device, tmp_path):
    """QLM_GEMM_EXACT=2 sends matrices of more than 65536 rows (the vocabulary
    head) to the one-launch kernel as well; its rows must carry the same bits
    as the default path (launches of 8 rows) there. The switch is read once
    per process, so the forced run is a child process."""
    import os
    import subprocess
    import sys
    from tests.conftest import ROOT
    code = (
        "import numpy as np, sys\n"
        "import quicklm_b200 as q\n"
        "rng = np.random.default_rng(5)\n"
        "w = q.Int8Weight.quantize((rng.standard_normal((70001, 160)) * 0.02).astype(np.float32))\n"
        "x = rng.standard_normal((24, 160)).astype(np.float32)\n"
        "np.save(sys.argv[1], q.matmul(x, w))\n"
    )
    outs = []
    for mode in ("1", "2"):
        path = str(tmp_path / f"tall_{mode}.npy")
        env = {**os.environ, "QLM_GEMM_EXACT": mode}
        r = subprocess.run([sys.executable, "-c", code, path], cwd=ROOT, env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(np.load(path))
    assert bits_equal(outs[0], outs[1])
