"""Case definitions shared by the golden generator and the tests.

The shapes are the benchmark configurations:
* CFG1 — decode GEMV: x [1, 2048], W [6144, 2048], seed 0.
* CFG2 — prefill GEMM: M in {64, 512, 2048} with W [6144, 2048] and
  [2048, 6144]; seed 1, 2, 3 for M = 64, 512, 2048.
* CFG4 — projection sweep of a ~4B-class model at M in {1, 4, 8, 64, 512}:
  [2560,2560], [512,2560], [9728,2560], [2560,9728] and the [151936,2560]
  lm_head; seed 40 + shape index.
SMALL_CASES are the edge cases, small enough to store in full.
"""
from __future__ import annotations

import numpy as np

CFG1 = (1, 6144, 2048, 0)
CFG2 = [(m, n, k, seed) for seed, m in ((1, 64), (2, 512), (3, 2048)) for (n, k) in ((6144, 2048), (2048, 6144))]
CFG4_SHAPES = [(2560, 2560), (512, 2560), (9728, 2560), (2560, 9728), (151936, 2560)]
CFG4_M = (1, 4, 8, 64, 512)
CFG4 = [(m, n, k, 40 + i) for i, (n, k) in enumerate(CFG4_SHAPES) for m in CFG4_M]

# (m, n, k, seed, source dtype, special values)
SMALL_CASES = [
    (1, 64, 128, 11, "f32", None),
    (3, 37, 100, 12, "f32", None),       # ragged K (tail of 4), N % 8 != 0
    (8, 50, 2048, 13, "f32", None),      # M = 8 (largest single GEMV group)
    (2, 33, 7, 14, "f32", None),         # K < 8: scalar-only quantizer tail
    (1, 9, 45, 15, "bf16", None),        # bf16 source, ragged block with 8-step + scalar tail
    (5, 17, 300, 16, "f32", "specials"), # NaN/Inf/+-0/subnormal in W and x
    (1, 1, 1, 17, "f32", None),          # smallest shape
    (4, 24, 1000, 18, "bf16", None),
    (16, 12, 96, 19, "f32", None),       # M > 8: several launches
    (1, 8, 32, 20, "f32", "zeros"),      # all-zero rows -> scale 1.0
    (9, 130, 384, 21, "f32", "wide"),    # large dynamic range across blocks
]


def make_small_case(spec):
    m, n, k, seed, dtype, special = spec
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if special == "specials":
        u = rng.random((n, k))
        w[u < 0.03] = np.nan
        w[(u >= 0.03) & (u < 0.05)] = np.inf
        w[(u >= 0.05) & (u < 0.06)] = -np.inf
        w[(u >= 0.06) & (u < 0.12)] = 0.0
        w[(u >= 0.12) & (u < 0.15)] = -0.0
        sub = (u >= 0.15) & (u < 0.2)
        w[sub] = (rng.standard_normal(int(sub.sum())) * 1e-40).astype(np.float32)
        w[3, :64] = 1e-39  # a block whose scale is subnormal
        x[0, 5] = np.nan
        x[1, 7] = np.inf
        x[2, :] *= 1e-38
    elif special == "zeros":
        w[:] = 0.0
    elif special == "wide":
        w *= (10.0 ** rng.integers(-30, 30, size=(n, (k + 31) // 32))).repeat(32, axis=1)[:, :k].astype(np.float32)
    if dtype == "bf16":
        w = (w.view(np.uint32) >> 16).astype(np.uint16)
    return x, w


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)
