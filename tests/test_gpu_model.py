"""The device-resident decode step (qlm_model_*) on a small random-init
QuickLM checkpoint of the configuration-3 architecture (gated-delta-net and
gated GQA layers): several sequences decoded in lockstep must give each
sequence exactly the logits and tokens it gets alone (every op is row- or
head-independent), and a single sequence's greedy tokens must equal QuickLM's
own CPU decode of the same checkpoint (oracle/_ref/ref_decode)."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu

REF_BIN = os.path.join(ROOT, "oracle", "_ref", "ref_decode")
SMALL = dict(hidden=256, layers=4, inter=512, vocab=4096, heads=4, kv_heads=2, head_dim=64, lin_heads=4, lin_dim=32)


@pytest.fixture(scope="module")
def small_checkpoint(tmp_path_factory):
    sys.path.insert(0, os.path.join(ROOT, "integration"))
    from make_checkpoint import build
    d = str(tmp_path_factory.mktemp("small_model"))
    build(d, seed=11, prompt_len=9, **SMALL)
    return d


def _decode(m, prompts, n_new):
    """Prefill prompt[:-1], then n_new greedy steps; returns (tokens, logits per step)."""
    B = len(prompts)
    pos = 0
    for i in range(len(prompts[0]) - 1):
        m.decode([p[i] for p in prompts], pos)
        pos += 1
    cur = [p[-1] for p in prompts]
    toks, logs = [], []
    for _ in range(n_new):
        nxt, lg = m.decode(cur, pos, logits=True)
        pos += 1
        toks.append(nxt.copy())
        logs.append(lg.copy())
        cur = list(nxt)
    return np.array(toks).T.reshape(B, n_new), np.stack(logs, 1)


def test_batched_equals_single(qlm_lib, cuda_device, small_checkpoint):
    import quicklm_b200 as q
    rng = np.random.default_rng(5)
    prompts = [list(rng.integers(0, SMALL["vocab"], 7)) for _ in range(3)]
    mb = q.Model(small_checkpoint, max_seq=64, batch=3)
    tb, lb = _decode(mb, prompts, 10)
    mb.free()
    m1 = q.Model(small_checkpoint, max_seq=64, batch=1)
    for b, p in enumerate(prompts):
        m1.reset()
        t1, l1 = _decode(m1, [p], 10)
        assert np.array_equal(t1[0], tb[b]), f"sequence {b}: tokens differ between batched and single decode"
        assert np.array_equal(l1[0].view(np.uint32), lb[b].view(np.uint32)), f"sequence {b}: logits differ"
    m1.free()


def test_single_matches_reference_decode(qlm_lib, cuda_device, small_checkpoint):
    import quicklm_b200 as q
    if not os.path.exists(REF_BIN):
        pytest.fail(f"{REF_BIN} missing: build it with __graft_entry__.build() where the reference tree exists")
    n_new = 24
    out = subprocess.run([REF_BIN, small_checkpoint, os.path.join(small_checkpoint, "prompt_ids.txt"), str(n_new),
                          "4"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    ref = json.loads(out.stdout.strip().splitlines()[-1])["tokens"]
    with open(os.path.join(small_checkpoint, "prompt_ids.txt")) as f:
        prompt = [int(t) for t in f.read().split()]
    m = q.Model(small_checkpoint, max_seq=64)
    toks, _ = _decode(m, [prompt], n_new)
    m.free()
    assert list(toks[0]) == ref


def test_graph_replay_equals_eager(qlm_lib, cuda_device, small_checkpoint):
    """Steps replayed from the captured graph (position and conv ring position
    read from device memory) give exactly the eager steps' logits, also after
    a reset."""
    import quicklm_b200 as q
    rng = np.random.default_rng(9)
    prompts = [list(rng.integers(0, SMALL["vocab"], 6)) for _ in range(2)]
    old = os.environ.get("QLM_MODEL_GRAPH")
    os.environ["QLM_MODEL_GRAPH"] = "0"
    try:
        me = q.Model(small_checkpoint, max_seq=64, batch=2)
    finally:
        if old is None:
            del os.environ["QLM_MODEL_GRAPH"]
        else:
            os.environ["QLM_MODEL_GRAPH"] = old
    mg = q.Model(small_checkpoint, max_seq=64, batch=2)
    for _ in range(2):
        te, le = _decode(me, prompts, 12)
        tg, lg = _decode(mg, prompts, 12)
        assert np.array_equal(te, tg)
        assert np.array_equal(le.view(np.uint32), lg.view(np.uint32))
        me.reset()
        mg.reset()
    me.free()
    mg.free()
