"""Per-matmul timing inside the library (qlm_prof_*), the counterpart of
QuickLM's QUICKLM_PROF accumulator (src/ops/math_ops.cpp:151-159, 821-823,
896-899; printed by src/main.cpp:706-709). CPU tests cover the switch, the
environment variable and the empty report; GPU tests check that every linear
entry point is counted per (entry, M, N, K) with positive device time, that
calls captured into a CUDA graph and calls made while off are not counted,
and that timing changes no output bit."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

from tests.conftest import ROOT, bits_equal


def test_switch_and_empty_report(qlm_lib):
    import quicklm_b200 as q
    before = q.prof_enable(None)
    try:
        q.prof_enable(True)
        assert q.prof_enable(None) is True
        q.prof_reset()
        assert q.prof_matmul_ms() == (0.0, 0)
        assert q.prof_report() == []
        assert q.prof_enable(False) is True
        assert q.prof_enable(None) is False
    finally:
        q.prof_enable(before)


@pytest.mark.parametrize("var", ["QUICKLM_PROF", "QLM_PROF"])
def test_environment_switch(qlm_lib, var):
    env = {k: v for k, v in os.environ.items() if k not in ("QUICKLM_PROF", "QLM_PROF")}
    code = "import quicklm_b200 as q; print(int(q.prof_enable(None)))"
    off = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    on = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env={**env, var: "1"}, capture_output=True,
                        text=True, timeout=300)
    assert off.returncode == 0 and on.returncode == 0, off.stderr + on.stderr
    assert off.stdout.strip() == "0" and on.stdout.strip() == "1"


@pytest.mark.gpu
def test_linear_calls_timed_per_shape(qlm_lib, cuda_device):
    import torch
    import quicklm_b200 as q
    rng = np.random.default_rng(3)
    k = 512
    w = q.Int8Weight.quantize((rng.standard_normal((640, k)) * 0.02).astype(np.float32))
    w2 = q.Int8Weight.quantize((rng.standard_normal((96, k)) * 0.02).astype(np.float32))
    x1 = torch.from_numpy(rng.standard_normal((1, k)).astype(np.float32)).cuda()
    x16 = rng.standard_normal((16, k)).astype(np.float32)
    ref1 = q.matmul(x1, w, flags=q.SYNC).cpu().numpy()
    ref16 = q.matmul(x16, w)
    before = q.prof_enable(True)
    try:
        q.prof_reset()
        for _ in range(3):
            y1 = q.matmul(x1, w)                      # device buffers, asynchronous
        y16 = q.matmul(x16, w)                        # host buffers (HOST_IO)
        y16b = q.matmul(x16, w)
        q.matmul_grouped(x1, [w, w2], flags=q.SYNC)
        torch.cuda.synchronize()
        ms, calls = q.prof_matmul_ms()
        rows = {(r["entry"], r["M"], r["N"], r["K"]): r for r in q.prof_report()}
        assert calls == 6
        assert rows[("qlm_linear_int8", 1, 640, k)]["calls"] == 3
        assert rows[("qlm_linear_int8", 16, 640, k)]["calls"] == 2
        assert rows[("qlm_linear_int8_grouped", 1, 736, k)]["calls"] == 1
        assert all(r["ms"] > 0 for r in rows.values())
        assert abs(sum(r["ms"] for r in rows.values()) - ms) < 1e-6 * max(ms, 1.0)
        # timing changes nothing in the results
        assert bits_equal(y1.cpu().numpy(), ref1)
        assert bits_equal(y16, ref16) and bits_equal(y16b, ref16)

        # calls captured into a CUDA graph are not timed (nor are their replays)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            q.matmul(x1, w, y1)  # warm the per-device state outside the capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        q.prof_reset()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            q.matmul(x1, w, y1)
        g.replay()
        torch.cuda.synchronize()
        assert q.prof_matmul_ms()[1] == 0
        assert bits_equal(y1.cpu().numpy(), ref1)
        del g

        # switched off: not timed
        q.prof_enable(False)
        q.matmul(x1, w, y1)
        torch.cuda.synchronize()
        assert q.prof_matmul_ms()[1] == 0
    finally:
        q.prof_enable(before)
        q.prof_reset()
        w.free()
        w2.free()
