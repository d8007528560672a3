"""End to end, benchmark configuration 3: greedy decode of a seeded random-init
24-layer hybrid decoder (BF16 checkpoint, int8 weights), 64-token prompt of
random ids, 128 new tokens — QuickLM's own model code with the int8 matmuls on
the B200 (integration/_build/qlm_decode) against QuickLM entirely on the CPU
(oracle/_ref/ref_decode). The exact matmul path makes every logit
bit-identical, so the token streams must be identical."""
from __future__ import annotations

import json
import os
import subprocess

import pytest

from tests.conftest import ROOT

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

REF_BIN = os.path.join(ROOT, "oracle", "_ref", "ref_decode")
GPU_BIN = os.path.join(ROOT, "integration", "_build", "qlm_decode")


def _run(binary, ckpt, n_new, env=None):
    threads = str(len(os.sched_getaffinity(0)))
    out = subprocess.run([binary, ckpt, os.path.join(ckpt, "prompt_ids.txt"), str(n_new), threads],
                         capture_output=True, text=True, timeout=900, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.fixture(scope="module")
def cfg3_checkpoint(tmp_path_factory):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "integration"))
    from make_checkpoint import build
    d = str(tmp_path_factory.mktemp("cfg3"))
    build(d, seed=7, prompt_len=64)
    return d


def test_greedy_tokens_identical_cfg3(cfg3_checkpoint, qlm_lib):
    for b in (REF_BIN, GPU_BIN):
        if not os.path.exists(b):
            pytest.fail(f"{b} missing: build it with __graft_entry__.build() where the reference tree exists")
    ref = _run(REF_BIN, cfg3_checkpoint, 128)
    gpu = _run(GPU_BIN, cfg3_checkpoint, 128)
    print("reference CPU:", {k: ref[k] for k in ref if k != "tokens"})
    print("B200 int8 matmul:", {k: gpu[k] for k in gpu if k != "tokens"})
    assert len(gpu["tokens"]) == 128
    assert gpu["tokens"] == ref["tokens"]
