"""Device layer ops against QuickLM's own functions (oracle/_ref build):
rms_norm, add_rms_norm and the NeoX RoPE rotation bit-identical; silu_mul
within 2 ulp (exp is evaluated differently on the device: a 1-ulp difference
in exp can move 1 + e, the quotient and the product by one rounding each),
with equal NaN/Inf behaviour."""
from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import bits_equal

pytestmark = pytest.mark.gpu

# hidden sizes of the configs (1024, 2560), one with an 8-wide remainder
# (1000 = 31*32 + 8), one with a scalar tail (1003), a tiny one (7), 4096
SIZES = [1024, 2560, 1000, 1003, 7, 4096]


@pytest.fixture(scope="module")
def q(qlm_lib, cuda_device):
    import quicklm_b200
    return quicklm_b200


def _rows(rng, rows, size, special):
    x = rng.standard_normal((rows, size)).astype(np.float32)
    if special == "scaled":
        x *= (10.0 ** rng.integers(-20, 20, size=(rows, 1))).astype(np.float32)
    elif special == "zeros":
        x[:] = 0.0
    elif special == "nan":
        x[0, size // 2] = np.nan
    return x


@pytest.mark.parametrize("size", SIZES)
@pytest.mark.parametrize("rows", [1, 3, 64])
@pytest.mark.parametrize("special", [None, "scaled", "zeros", "nan"])
def test_rms_norm_bit_exact(q, refcpu, size, rows, special):
    import torch
    rng = np.random.default_rng(size * 31 + rows)
    x = _rows(rng, rows, size, special)
    w = (rng.standard_normal(size) * 0.1).astype(np.float32)
    eps = 1e-6
    y_ref = refcpu.rms_norm(x, w, eps)
    xd = torch.from_numpy(x).cuda()
    y = q.rms_norm(xd, torch.from_numpy(w).cuda(), eps)
    assert bits_equal(y.cpu().numpy(), y_ref)
    q.rms_norm(xd, torch.from_numpy(w).cuda(), eps, out=xd)  # in place
    assert bits_equal(xd.cpu().numpy(), y_ref)


@pytest.mark.parametrize("size", SIZES)
@pytest.mark.parametrize("rows", [1, 5])
@pytest.mark.parametrize("special", [None, "scaled", "nan"])
def test_add_rms_norm_bit_exact(q, refcpu, size, rows, special):
    import torch
    rng = np.random.default_rng(size * 7 + rows)
    r = _rows(rng, rows, size, special)
    d = rng.standard_normal((rows, size)).astype(np.float32)
    w = (rng.standard_normal(size) * 0.1).astype(np.float32)
    eps = 1e-6
    r_ref, o_ref = refcpu.add_rms_norm(r, d, w, eps)
    rd = torch.from_numpy(r).cuda()
    o = q.add_rms_norm(rd, torch.from_numpy(d).cuda(), torch.from_numpy(w).cuda(), eps)
    assert bits_equal(rd.cpu().numpy(), r_ref)
    assert bits_equal(o.cpu().numpy(), o_ref)


@pytest.mark.parametrize("size", SIZES)
@pytest.mark.parametrize("rows", [1, 5])
@pytest.mark.parametrize("special", [None, "scaled", "nan"])
def test_add_then_rms_norm_bit_exact(q, refcpu, size, rows, special):
    """elementwise_add then math::rms_norm (the decoder layer's default
    residual step), fused in one launch: the reference's two calls' bits."""
    import torch
    rng = np.random.default_rng(size * 13 + rows)
    r = _rows(rng, rows, size, special)
    d = rng.standard_normal((rows, size)).astype(np.float32)
    w = (rng.standard_normal(size) * 0.1).astype(np.float32)
    eps = 1e-6
    s_ref = r + d  # IEEE single-precision add, as math::elementwise_add
    o_ref = refcpu.rms_norm(s_ref, w, eps)
    rd = torch.from_numpy(r).cuda()
    o = q.add_then_rms_norm(rd, torch.from_numpy(d).cuda(), torch.from_numpy(w).cuda(), eps)
    assert bits_equal(rd.cpu().numpy(), s_ref)
    assert bits_equal(o.cpu().numpy(), o_ref)


def _ulp_diff(a, b):
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)


def test_silu_mul_within_two_ulp(q, refcpu):
    import torch
    rng = np.random.default_rng(3)
    n = 1 << 20
    a = (rng.standard_normal(n) * 4).astype(np.float32)
    a[:8] = [0.0, -0.0, np.inf, -np.inf, np.nan, 88.0, -88.0, -104.0]
    b = rng.standard_normal(n).astype(np.float32)
    ref = refcpu.silu_mul(a, b)
    ad = torch.from_numpy(a).cuda()
    q.silu_mul(ad, torch.from_numpy(b).cuda())
    got = ad.cpu().numpy()
    nan_ref, nan_got = np.isnan(ref), np.isnan(got)
    assert np.array_equal(nan_ref, nan_got)
    ok = ~nan_ref
    assert _ulp_diff(got[ok], ref[ok]).max() <= 2
    # the device and the host agree exactly on the vast majority of inputs
    assert (_ulp_diff(got[ok], ref[ok]) == 0).mean() > 0.99


@pytest.mark.parametrize("theta,heads,head_dim,rotary_dim", [(10000000.0, 16, 256, 64), (10000.0, 4, 64, 64),
                                                               (1e6, 8, 128, 32)])
def test_rope_neox_bit_exact(q, refcpu, theta, heads, head_dim, rotary_dim):
    import torch
    rng = np.random.default_rng(heads * head_dim)
    pos0, n_tok = 1000, 7
    t = rng.standard_normal((n_tok, heads, head_dim)).astype(np.float32)
    ref = np.stack([refcpu.rope_neox(t[i], pos0 + i, theta, rotary_dim) for i in range(n_tok)])
    td = torch.from_numpy(t).cuda()
    q.rope_neox(td, pos0, theta, rotary_dim)
    assert bits_equal(td.cpu().numpy(), ref)


def test_layer_arg_checks(q):
    import torch
    x = torch.zeros((2, 8), device="cuda")
    with pytest.raises(q.QlmError):
        q.rms_norm(x, torch.zeros(3, device="cuda"), 1e-6)  # not whole rows
    with pytest.raises(q.QlmError):
        q.silu_mul(x, torch.zeros(3, device="cuda"))
    with pytest.raises(q.QlmError):
        q.rope_neox(torch.zeros((1, 2, 8), device="cuda"), 0, 1e4, 10)  # rotary_dim > head_dim


def test_silu_within_two_ulp(q, refcpu):
    import torch
    rng = np.random.default_rng(13)
    x = (rng.standard_normal(1 << 18) * 4).astype(np.float32)
    x[:6] = [0.0, -0.0, np.inf, -np.inf, np.nan, -104.0]
    ref = refcpu.silu(x)
    xd = torch.from_numpy(x).cuda()
    got = q.silu(xd).cpu().numpy()
    assert np.array_equal(np.isnan(ref), np.isnan(got))
    ok = ~np.isnan(ref)
    assert _ulp_diff(got[ok], ref[ok]).max() <= 2
    assert (_ulp_diff(got[ok], ref[ok]) == 0).mean() > 0.99


@pytest.mark.parametrize("conv_dim,ks", [(6144, 4), (1000, 4), (37, 2), (512, 5)])
def test_conv1d_tapmajor_bit_exact(q, refcpu, conv_dim, ks):
    """Several steps around the ring, state carried on both sides."""
    import torch
    rng = np.random.default_rng(conv_dim + ks)
    ntaps = ks - 1
    wt = rng.standard_normal((ks, conv_dim)).astype(np.float32)
    st_ref = rng.standard_normal((ntaps, conv_dim)).astype(np.float32)
    st_dev = torch.from_numpy(st_ref.copy()).cuda()
    wt_dev = torch.from_numpy(wt).cuda()
    ring = 0
    for step in range(2 * ks):
        x = rng.standard_normal(conv_dim).astype(np.float32)
        y_ref, st_ref = refcpu.conv1d_update_tapmajor(x, st_ref, ring, wt)
        y = q.conv1d_update_tapmajor(torch.from_numpy(x).cuda(), st_dev, ring, wt_dev)
        assert bits_equal(y.cpu().numpy(), y_ref), step
        assert bits_equal(st_dev.cpu().numpy(), st_ref), step
        ring = (ring + 1) % ntaps


@pytest.mark.parametrize("heads,head_dim", [(16, 128), (32, 128), (3, 7), (5, 1000)])
def test_l2norm_heads_bit_exact(q, refcpu, heads, head_dim):
    import torch
    rng = np.random.default_rng(heads * head_dim)
    x = rng.standard_normal((heads, head_dim)).astype(np.float32)
    x[0] *= 1e-4
    ref = refcpu.l2norm_heads(x, 1e-6)
    xd = torch.from_numpy(x).cuda()
    q.l2norm_heads(xd, head_dim, 1e-6)
    assert bits_equal(xd.cpu().numpy(), ref)


@pytest.mark.parametrize("heads,d", [(16, 128), (3, 20), (2, 7), (1, 256)])
def test_gdn_recurrence_bit_exact(q, refcpu, heads, d):
    """Several tokens with the state carried on both sides, against the
    restated recurrence (itself pinned to Qwen3_5GatedDeltaNet::forward by
    tests/test_gdn_cpu.py)."""
    import torch
    rng = np.random.default_rng(heads * 1000 + d)
    st_ref = (rng.standard_normal((heads, d, d)) * 0.1).astype(np.float32)
    st_dev = torch.from_numpy(st_ref.copy()).cuda()
    for step in range(4):
        qv, kv, vv = (rng.standard_normal((heads, d)).astype(np.float32) for _ in range(3))
        qv /= np.linalg.norm(qv, axis=1, keepdims=True)
        kv /= np.linalg.norm(kv, axis=1, keepdims=True)
        dec = rng.uniform(0.5, 1.0, heads).astype(np.float32)
        beta = rng.uniform(0.0, 1.0, heads).astype(np.float32)
        out_ref, st_ref = refcpu.gdn_recurrence(st_ref, qv, kv, vv, dec, beta)
        t = [torch.from_numpy(a).cuda() for a in (qv, kv, vv, dec, beta)]
        out = q.gdn_recurrence(st_dev, *t)
        assert bits_equal(out.cpu().numpy(), out_ref), step
        assert bits_equal(st_dev.cpu().numpy(), st_ref), step


def test_gdn_gates_within_a_few_ulp(q, refcpu):
    import torch
    rng = np.random.default_rng(17)
    heads = 4096
    a = (rng.standard_normal(heads) * 3).astype(np.float32)
    a[:4] = [25.0, 19.9, -30.0, 0.0]  # both softplus branches
    b = (rng.standard_normal(heads) * 4).astype(np.float32)
    A_log = (rng.standard_normal(heads) * 0.5).astype(np.float32)
    dt = (rng.standard_normal(heads) * 0.5).astype(np.float32)
    dec_ref, beta_ref = refcpu.gdn_gates(a, b, A_log, dt)
    dec, beta = q.gdn_gates(*[torch.from_numpy(x).cuda() for x in (a, b, A_log, dt)])
    dec = dec.cpu().numpy()
    # decay = exp(alpha): a 1-ulp difference in alpha (from exp/log1p last bits)
    # is a relative error of |alpha| ulp in decay, so the bound scales with
    # |alpha| = -ln(decay): 2 ulp x (2 + |alpha|) on the normal range.
    d_ref = dec_ref.astype(np.float64)
    normal = d_ref > 1e-30
    alpha = -np.log(d_ref[normal])
    rel = np.abs(dec[normal] - d_ref[normal]) / d_ref[normal]
    assert (rel <= 2.4e-7 * (2.0 + alpha)).all()
    assert np.all(np.abs(dec[~normal]) <= 1e-29)
    assert _ulp_diff(beta.cpu().numpy(), beta_ref).max() <= 2
    assert (_ulp_diff(dec, dec_ref) == 0).mean() > 0.75


@pytest.mark.parametrize("rows,size", [(16, 128), (3, 20), (5, 1003)])
def test_rms_norm_gain_bit_exact(q, refcpu, rows, size):
    import torch
    rng = np.random.default_rng(rows + size)
    x = rng.standard_normal((rows, size)).astype(np.float32)
    w = (1.0 + rng.standard_normal(size) * 0.1).astype(np.float32)
    ref = refcpu.rms_norm_gain(x, w, 1e-6)
    y = q.rms_norm_gain(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), 1e-6)
    assert bits_equal(y.cpu().numpy(), ref)


@pytest.mark.parametrize("heads,kv_heads,d", [(8, 2, 256), (4, 4, 128), (3, 1, 20)])
@pytest.mark.parametrize("pos", [0, 5, 300, 2047])
def test_gqa_attend(q, refcpu, heads, kv_heads, d, pos):
    """Against the restated per-head attention (pinned to Qwen3_5Attention::forward
    by tests/test_gdn_cpu.py). Scores, the max, the sum order and the V
    accumulation are the reference's; exp is evaluated in double, and where the
    host's expf is off by an ulp the weights move by ~2 ulp, so outputs agree
    within 1e-6 x max|v| (exactly at pos 0, where the single weight is 1)."""
    import torch
    rng = np.random.default_rng(heads * 7 + d + pos)
    T = pos + 3
    qv = rng.standard_normal((heads, 2 * d)).astype(np.float32)  # [query | gate] per head
    kc = rng.standard_normal((T, kv_heads, d)).astype(np.float32)
    vc = rng.standard_normal((T, kv_heads, d)).astype(np.float32)
    ref = refcpu.gqa_attend(qv, kc, vc, pos, kv_heads)
    dev = [torch.from_numpy(a).cuda() for a in (qv, kc, vc)]
    got = q.gqa_attend(*dev, pos, parallel=False).cpu().numpy()
    par = q.gqa_attend(*dev, pos, parallel=True).cpu().numpy()
    assert bits_equal(par, got)  # the two-launch form computes the same values
    if pos == 0:
        assert bits_equal(got, ref)
    else:
        assert np.abs(got - ref).max() <= 1e-6 * np.abs(vc).max()
