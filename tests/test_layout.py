"""The packed P128 weight layout and the permuted activation staging: pure
index arithmetic, restated in Python and checked against the reference lane
structure (element k = 32*b + 8*j + l belongs to lane l, block b, step j —
src/ops/math_ops.cpp:420-426)."""
from __future__ import annotations


def packed_offset(k):
    return (k & ~127) + (k & 7) * 16 + ((k >> 5) & 3) * 4 + ((k >> 3) & 3)


def xperm_offset(k):
    return (k & ~127) + ((k >> 5) & 3) * 32 + (k & 7) * 4 + ((k >> 3) & 3)


def test_packed_is_bijection():
    for kp in (128, 256, 2048):
        assert sorted(packed_offset(k) for k in range(kp)) == list(range(kp))
        assert sorted(xperm_offset(k) for k in range(kp)) == list(range(kp))


def test_lane_slices():
    """Lane l's 16 bytes of chunk c are blocks 4c..4c+3, steps j=0..3, and the
    permuted x float4 (c, bb, l) holds the same four elements in the same order."""
    for k in range(1024):
        c, b, j, l = k // 128, (k // 32) % 4, (k % 32) // 8, k % 8
        assert packed_offset(k) == c * 128 + l * 16 + b * 4 + j
        assert xperm_offset(k) == c * 128 + b * 32 + l * 4 + j
