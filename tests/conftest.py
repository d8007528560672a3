"""Shared fixtures. ``-m gpu`` tests need a CUDA device (a B200); everything
else runs on CPU. The oracle libraries under oracle/ are the checkers: they
are loaded here, never by the product package."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size benchmark shapes")


@pytest.fixture(scope="session")
def coracle():
    from oracle import oracle as o
    if not os.path.exists(o.ORACLE_LIB):
        o.build()
    return o.COracle()


@pytest.fixture(scope="session")
def refcpu():
    """QuickLM's own int8 path compiled from its sources (prebuilt .so)."""
    from oracle import oracle as o
    if not os.path.exists(o.REF_LIB):
        ref_root = o.reference_root()
        if ref_root:
            o.build(ref_root)
    if not os.path.exists(o.REF_LIB):
        pytest.skip("reference build oracle/_ref/libqlm_refcpu.so not available")
    r = o.RefCPU()
    r.init_threads(min(8, os.cpu_count() or 1))
    return r


@pytest.fixture(scope="session")
def small_cases():
    from tests.golden.cases import SMALL_CASES
    z = np.load(os.path.join(GOLDEN, "small_cases.npz"))
    out = []
    for i, spec in enumerate(SMALL_CASES):
        out.append((spec, {n: z[f"c{i}_{n}"] for n in ("x", "w", "q", "s", "y")}))
    return out


@pytest.fixture(scope="session")
def config_hashes():
    with open(os.path.join(GOLDEN, "config_hashes.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="session")
def qlm_lib():
    import quicklm_b200 as q
    from quicklm_b200 import build as b
    if not os.path.exists(q.LIB_PATH):
        b.build()
    return q.load()


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    return 0


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    """Bitwise equality of float32 arrays; NaNs compare equal to NaNs (x86
    and CUDA may produce different NaN payloads)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if a.shape != b.shape:
        return False
    same = a.view(np.uint32) == b.view(np.uint32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(same | nan))
