"""Host side of the device layer ops: the RoPE cos/sin tables the library
builds on the host (qlm_rope_neox_tables) must be the reference's own
(math::apply_rope_neox computes them with the same float expressions and libm
calls, src/ops/math_ops.cpp:1256-1271). The reference's values are read back
by rotating unit vectors through its apply_rope_neox: with x1 = 1, x2 = 0 the
rotation returns (cos, sin)."""
from __future__ import annotations

import numpy as np
import pytest


@pytest.fixture(scope="module")
def q(qlm_lib):
    import quicklm_b200
    return quicklm_b200


@pytest.mark.parametrize("theta,rotary_dim,head_dim", [(10000.0, 64, 64), (10000000.0, 64, 256), (1e6, 32, 128)])
def test_rope_tables_match_reference(q, refcpu, theta, rotary_dim, head_dim):
    half = rotary_dim // 2
    positions = [0, 1, 2, 17, 1000, 4095, 32767, 65535, 262143]
    c, s = q.rope_neox_tables(0, max(positions) + 1, theta, rotary_dim)
    for pos in positions:
        t = np.zeros((1, head_dim), np.float32)
        t[0, :half] = 1.0
        r = refcpu.rope_neox(t, pos, theta, rotary_dim)
        assert np.array_equal(r[0, :half].view(np.uint32), c[pos].view(np.uint32)), pos
        assert np.array_equal(r[0, half:rotary_dim].view(np.uint32), s[pos].view(np.uint32)), pos
        if rotary_dim < head_dim:  # dims past rotary_dim pass through
            assert np.all(r[0, rotary_dim:] == 0.0)


def test_rope_table_args(q):
    with pytest.raises(q.QlmError):
        q.rope_neox_tables(0, 1, 10000.0, 7)
    with pytest.raises(q.QlmError):
        q.rope_neox_tables(-1, 1, 10000.0, 8)
