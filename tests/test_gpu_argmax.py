"""Device greedy selection (qlm_argmax_f32) against QuickLM's greedy sampling,
DecoderModel::sample(logits, 0, 0) (model/model.cpp:259-272), restated in
oracle.greedy_argmax and pinned to the reference by test_oracle.py. Integer
result: exact match required, and the reported value must be the logit at
that index (bit-identical)."""
from __future__ import annotations

import numpy as np
import pytest

from tests.test_oracle import greedy_cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def q(qlm_lib, cuda_device):
    import quicklm_b200
    return quicklm_b200


def check(q, v):
    import torch
    from oracle.oracle import greedy_argmax
    i, val = q.argmax(torch.from_numpy(np.ascontiguousarray(v, np.float32)).cuda())
    want = greedy_argmax(v)
    assert i == want, (i, want, v[:8])
    if not np.isnan(v[want]):
        assert np.float32(val).view(np.uint32) == np.float32(v[want]).view(np.uint32)


def test_argmax_fuzz(q):
    for v in greedy_cases(seed=1, count=120):
        check(q, v)


@pytest.mark.parametrize("n", [1, 31, 1024, 8193, 151936])
def test_argmax_sizes_and_last_tie(q, n):
    rng = np.random.default_rng(n)
    v = rng.standard_normal(n).astype(np.float32)
    v[-1] = 100.0
    check(q, v)
    v[n // 2] = 100.0  # equal maximum earlier: the lower index wins
    check(q, v)
    v[0] = np.nan      # NaN at index 0: the reference returns 0
    check(q, v)


def test_argmax_of_exact_lm_head_logits(q, refcpu):
    """End to end: the device GEMV's logits are bit-identical to the
    reference's, so the device choice equals the reference's sample() on the
    reference's own logits."""
    import torch
    from oracle.oracle import synth_case
    x, w = synth_case(1, 151936, 256, 44)
    qr, sr = refcpu.quantize(w)
    y_ref, _ = refcpu.matmul(x, qr, sr)
    want = refcpu.greedy_sample(y_ref[0])
    wt = q.Int8Weight.quantize(torch.from_numpy(w).cuda())
    y = q.matmul(torch.from_numpy(x).cuda(), wt, flags=q.SYNC)
    i, val = q.argmax(y)
    assert i == want
    assert np.float32(val).view(np.uint32) == y_ref[0, want].view(np.uint32)
    wt.free()
