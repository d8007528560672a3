"""Pins the oracle's restatement of the gated-delta-net decode step to the
reference module: Qwen3_5GatedDeltaNet::forward (model/attention.cpp:414-591)
driven through oracle/_ref over several tokens, against the restated step
(reference matmul/conv/sumsq/norm functions + the restated SiLU, gates and
delta-rule recurrence). Bit-equal outputs over the steps pin the restated
recurrence (qlmref_gdn_recurrence), which the device kernel is checked against.
Weights are F32, so the projections take the reference's fp32 matmul path."""
from __future__ import annotations

import numpy as np
import pytest


def _weights(rng, hin, heads, d, ks, hout):
    H = heads * d
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    return {
        "w_qkv": f(3 * H, hin) * 0.1, "w_z": f(H, hin) * 0.1, "w_b": f(heads, hin) * 0.1,
        "w_a": f(heads, hin) * 0.1, "conv_w": f(3 * H, ks) * 0.5, "norm_w": 1.0 + f(d) * 0.1,
        "A_log": f(heads) * 0.5, "dt_bias": f(heads) * 0.5, "w_out": f(hout, H) * 0.1,
    }


@pytest.mark.parametrize("hin,heads,d,ks,hout", [(64, 4, 16, 4, 48), (96, 2, 20, 4, 40), (128, 2, 128, 4, 64)])
def test_restated_step_equals_module(refcpu, hin, heads, d, ks, hout):
    rng = np.random.default_rng(hin + heads + d)
    w = _weights(rng, hin, heads, d, ks, hout)
    x = rng.standard_normal((6, hin)).astype(np.float32)
    y_mod = refcpu.gdn_steps(w, x)
    y_res = refcpu.gdn_steps(w, x, restated=True)
    assert np.isfinite(y_mod).all()
    assert np.array_equal(y_mod.view(np.uint32), y_res.view(np.uint32))


@pytest.mark.parametrize("hin,heads,kv_heads,d,rot", [(64, 4, 2, 32, 16), (96, 2, 1, 20, 8), (128, 4, 1, 256, 64)])
def test_restated_attention_equals_module(refcpu, hin, heads, kv_heads, d, rot):
    """The same pin for the GQA attention decode step (Qwen3_5Attention::forward,
    model/attention.cpp:138-235): the restated per-head attention
    (qlmref_gqa_attend) the device kernel is checked against."""
    rng = np.random.default_rng(hin + heads + d)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    w = {"w_q": f(heads * 2 * d, hin) * 0.2, "w_k": f(kv_heads * d, hin) * 0.2, "w_v": f(kv_heads * d, hin) * 0.2,
         "w_o": f(48, heads * d) * 0.1, "q_norm": f(d) * 0.1, "k_norm": f(d) * 0.1}
    x = f(7, hin)
    y_mod = refcpu.attn_steps(w, x, heads, kv_heads, d, rot, 1e7)
    y_res = refcpu.attn_steps(w, x, heads, kv_heads, d, rot, 1e7, restated=True)
    assert np.isfinite(y_mod).all()
    assert np.array_equal(y_mod.view(np.uint32), y_res.view(np.uint32))
