"""Pins the CPU restatement (oracle/qlm_oracle.c) to QuickLM's own code.

The reference ships no tests or golden vectors for this path, so the pin is
the reference itself, compiled from its sources (oracle/_ref), and the
fixtures generated from it (tests/golden/make_golden.py).
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest

from tests.conftest import GOLDEN, bits_equal
from tests.golden.cases import CFG1, CFG4, make_small_case


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_small_cases_regenerate(small_cases):
    """The stored inputs are exactly what the seeded generator makes."""
    for spec, arr in small_cases:
        x, w = make_small_case(spec)
        assert bits_equal(x, arr["x"]), spec
        assert np.array_equal(w.view(np.uint8), arr["w"].view(np.uint8)), spec


def test_c_oracle_quantize_matches_golden(coracle, small_cases):
    for spec, arr in small_cases:
        q, s = coracle.quantize(arr["w"])
        assert np.array_equal(q, arr["q"]), spec
        assert np.array_equal(s.view(np.uint32), arr["s"].view(np.uint32)), spec


def test_c_oracle_matmul_matches_golden(coracle, small_cases):
    for spec, arr in small_cases:
        y = coracle.matmul(arr["x"], arr["q"], arr["s"])
        assert bits_equal(y, arr["y"]), spec


def _int4_golden():
    return np.load(os.path.join(GOLDEN, "small_cases_int4.npz"))


def test_c_oracle_q4_matches_golden(coracle, small_cases):
    """The int4 restatement against the reference's int4 fixtures: packed bytes,
    scales, and the int4 product as the int8 arithmetic on the unpacked values."""
    from oracle.oracle import pack_q4, unpack_q4
    z = _int4_golden()
    for i, (spec, arr) in enumerate(small_cases):
        v, s = coracle.quantize_q4(arr["w"])
        assert np.array_equal(pack_q4(v), z[f"c{i}_p"]), spec
        assert np.array_equal(s.view(np.uint32), z[f"c{i}_s"].view(np.uint32)), spec
        k = arr["w"].shape[1]
        y = coracle.matmul(arr["x"], unpack_q4(z[f"c{i}_p"], k), z[f"c{i}_s"])
        assert bits_equal(y, z[f"c{i}_y"]), spec


def test_reference_build_matches_golden_q4(refcpu, small_cases):
    z = _int4_golden()
    for i, (spec, arr) in enumerate(small_cases):
        p, s = refcpu.quantize_int4(arr["w"])
        assert np.array_equal(p, z[f"c{i}_p"]) and np.array_equal(s.view(np.uint32), z[f"c{i}_s"].view(np.uint32))
        y = refcpu.matmul_int4(arr["x"], p, s, arr["w"].shape[1])
        assert bits_equal(y, z[f"c{i}_y"]), spec


def test_reference_build_matches_golden(refcpu, small_cases):
    """The prebuilt reference library reproduces the fixtures it generated."""
    for spec, arr in small_cases:
        q, s = refcpu.quantize(arr["w"])
        assert np.array_equal(q, arr["q"]), spec
        y, _ = refcpu.matmul(arr["x"], arr["q"], arr["s"])
        assert bits_equal(y, arr["y"]), spec


def test_cfg1_pinned(coracle, config_hashes):
    """Config 1 end to end through the C restatement equals the reference's bytes."""
    m, n, k, seed = CFG1
    from oracle.oracle import synth_case
    x, w = synth_case(m, n, k, seed)
    h = config_hashes["cfg1"]
    assert sha(w) == h["w"] and sha(x) == h["x"], "seeded generator drifted"
    q, s = coracle.quantize(w)
    assert sha(q) == h["q"] and sha(s) == h["s"]
    y = coracle.matmul(x, q, s)
    assert sha(y) == h["y"]
    assert bits_equal(y, np.load(os.path.join(GOLDEN, "cfg1_y.npy")))


@pytest.mark.parametrize("m,n,k,seed", [c for c in CFG4 if c[1] <= 2560 and c[0] <= 8][:6])
def test_cfg4_small_m_pinned(coracle, config_hashes, m, n, k, seed):
    from oracle.oracle import synth_case
    x, w = synth_case(m, n, k, seed)
    h = config_hashes[f"cfg4_m{m}_n{n}_k{k}"]
    q, s = coracle.quantize(w)
    assert sha(q) == h["q"] and sha(s) == h["s"]
    assert sha(coracle.matmul(x, q, s)) == h["y"]


def test_fuzz_c_oracle_vs_reference(coracle, refcpu):
    """Random shapes and special values: restatement == reference, bit for bit."""
    rng = np.random.default_rng(1234)
    for trial in range(120):
        n = int(rng.integers(1, 12))
        k = int(rng.integers(1, 260))
        m = int(rng.integers(1, 4))
        w = (rng.standard_normal((n, k)) * 10.0 ** rng.integers(-42, 8)).astype(np.float32)
        u = rng.random((n, k))
        w[u < 0.02] = np.nan
        w[(u >= 0.02) & (u < 0.04)] = np.inf
        w[(u >= 0.04) & (u < 0.1)] = 0.0
        if trial % 2:
            w = (w.view(np.uint32) >> 16).astype(np.uint16)
        q1, s1 = refcpu.quantize(w)
        q2, s2 = coracle.quantize(w)
        assert np.array_equal(q1, q2) and np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
        x = (rng.standard_normal((m, k)) * 10.0 ** rng.integers(-30, 20)).astype(np.float32)
        y1, _ = refcpu.matmul(x, q1, s1)
        assert bits_equal(y1, coracle.matmul(x, q1, s1))


def greedy_cases(seed=0, count=200):
    """Fuzzed logit vectors with the values that decide greedy sampling:
    ties, NaN (at index 0 and elsewhere), +-inf, +-0, subnormals."""
    rng = np.random.default_rng(seed)
    specials = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-45, -1e-45, 3.0], np.float32)
    out = []
    for t in range(count):
        n = int(rng.integers(1, 300))
        v = rng.standard_normal(n).astype(np.float32)
        if t % 3 == 0:  # repeated maxima
            v[rng.integers(0, n, size=3)] = v.max() if n else 0
        if t % 4 == 1:
            idx = rng.integers(0, n, size=max(1, n // 5))
            v[idx] = rng.choice(specials, size=idx.size)
        if t % 10 == 2:
            v[0] = np.nan
        if t % 10 == 3:
            v[:] = -np.inf
        if t % 10 == 4:
            v[:] = np.nan
        out.append(v)
    return out


def test_greedy_argmax_matches_reference(refcpu):
    """oracle.greedy_argmax == DecoderModel::sample(logits, 0, 0), compiled
    from the reference (model/model.cpp:259-272)."""
    from oracle.oracle import greedy_argmax
    for v in greedy_cases():
        assert greedy_argmax(v) == refcpu.greedy_sample(v), v


def test_q4_quantizer_matches_reference(coracle, refcpu):
    """int4 (Q4_0-style) quantizer restatement == get_tensor_keep_int4
    (io/safetensors.cpp:393-515), bytes and scales, on fuzzed F32/BF16 rows
    with specials and odd K."""
    from oracle.oracle import pack_q4, unpack_q4
    rng = np.random.default_rng(4)
    for t in range(150):
        n, k = int(rng.integers(1, 12)), int(rng.integers(1, 260))
        w = (rng.standard_normal((n, k)) * (10.0 ** rng.integers(-6, 6))).astype(np.float32)
        if t % 5 == 1:
            idx = rng.integers(0, w.size, size=max(1, w.size // 7))
            w.ravel()[idx] = rng.choice(np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40], np.float32),
                                        size=idx.size)
        src = (w.view(np.uint32) >> 16).astype(np.uint16) if t % 4 == 3 else w
        packed, s_ref = refcpu.quantize_int4(src)
        q, s = coracle.quantize_q4(src)
        assert np.array_equal(pack_q4(q), packed), (n, k, t)
        assert np.array_equal(s.view(np.uint32), s_ref.view(np.uint32)), (n, k, t)
        assert np.array_equal(unpack_q4(packed, k), q)


def test_q4_matmul_is_the_int8_arithmetic(coracle, refcpu):
    """QuickLM's int4 matmul (ops/math_ops.cpp:581-794) performs the int8
    path's exact per-element sequence on value = nibble - 8: the reference's
    int4 output equals its int8 output (and the C restatement's) on the
    unpacked values, bit for bit, ragged K included."""
    from oracle.oracle import unpack_q4
    rng = np.random.default_rng(5)
    for n, k, m in [(9, 64, 1), (17, 100, 3), (33, 2048, 2), (8, 37, 5), (40, 1000, 8)]:
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        x = rng.standard_normal((m, k)).astype(np.float32)
        packed, s = refcpu.quantize_int4(w)
        y4 = refcpu.matmul_int4(x, packed, s, k)
        y8, _ = refcpu.matmul(x, unpack_q4(packed, k), s)
        assert bits_equal(y4, y8)
        assert bits_equal(y4, coracle.matmul(x, unpack_q4(packed, k), s))
