"""The allocation-free tensor-core entry point (qlm_linear_int8_tc_noalloc).

It serves callers that may not allocate device memory while running (an
engine that gives all device memory to its own pool at start-up, or a decode
loop that cannot take cudaMalloc's device-wide synchronisation): its scratch is
the library's static device array instead of cudaMalloc'd buffers. This test
calls it through the C ABI and checks two calls in a row against the regular
entry point qlm_linear_int8(QLM_LINEAR_TENSOR). Both run the same kernels on
the same inputs, so the outputs must be bit-identical; the second call is
larger than the first, so stale staging left by the first call would show.
It also checks that a call after the first changes the device's free memory
by nothing (cudaMemGetInfo). It sits in its own file, collected last, and
passes both alone in a fresh process and after the other tests.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_matches_regular_entry_point(qlm_lib, cuda_device):
    import torch
    import quicklm_b200 as q

    rng = np.random.default_rng(99)
    n, k = 384, 640
    wf = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w = q.Int8Weight.quantize(wf)
    stream = torch.cuda.current_stream().cuda_stream
    # First call on this device: loads the device code (and the static array).
    x0 = torch.zeros((8, k), device="cuda")
    y0 = torch.empty((8, n), device="cuda")
    assert qlm_lib.qlm_linear_int8_tc_noalloc(x0.data_ptr(), 8, k, k, w.handle, y0.data_ptr(), n, q.SYNC,
                                              stream) == 0, qlm_lib.qlm_last_error()
    for m in (96, 200):  # two calls in a row, growing shapes, different data
        x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
        y_ref = q.matmul(x, w, flags=q.TENSOR | q.SYNC).cpu().numpy()
        y = torch.full((m, n), float("nan"), device="cuda")
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        rc = qlm_lib.qlm_linear_int8_tc_noalloc(x.data_ptr(), m, k, k, w.handle, y.data_ptr(), n, q.SYNC, stream)
        assert rc == 0, qlm_lib.qlm_last_error()
        torch.cuda.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0, f"device free memory changed by {free0 - free1} bytes across the call"
        yh = y.cpu().numpy()
        assert np.array_equal(yh.view(np.uint32), y_ref.view(np.uint32)), \
            f"{int(np.sum(yh.view(np.uint32) != y_ref.view(np.uint32)))} outputs differ from qlm_linear_int8(TENSOR)"
    assert qlm_lib.qlm_device_status(0, 1) == 0, qlm_lib.qlm_last_error()
    w.free()


def test_noalloc_rejects_oversize(qlm_lib, cuda_device):
    import torch
    import quicklm_b200 as q

    k = 4096
    w = q.Int8Weight.quantize(np.zeros((128, k), np.float32))
    m = 2048  # 2048 * 4096 * 2 bytes = 16 MiB of staging > the 8 MiB array
    x = torch.zeros((m, k), device="cuda")
    y = torch.zeros((m, 128), device="cuda")
    rc = qlm_lib.qlm_linear_int8_tc_noalloc(x.data_ptr(), m, k, k, w.handle, y.data_ptr(), 128, 0, None)
    assert rc == 1
    assert b"static scratch" in qlm_lib.qlm_last_error()


def test_noalloc_rejects_int4(qlm_lib, cuda_device):
    import torch
    import quicklm_b200 as q

    w = q.Int8Weight.quantize(np.zeros((64, 256), np.float32), bits=4)
    x = torch.zeros((4, 256), device="cuda")
    y = torch.zeros((4, 64), device="cuda")
    rc = qlm_lib.qlm_linear_int8_tc_noalloc(x.data_ptr(), 4, 256, 256, w.handle, y.data_ptr(), 64, 0, None)
    assert rc == 4
    assert b"int4" in qlm_lib.qlm_last_error()
