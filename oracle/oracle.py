"""TEST INFRASTRUCTURE ONLY — ctypes access to the two CPU parity checkers.

* ``RefCPU``: QuickLM's own int8 path compiled from the reference sources
  (``oracle/_ref/libqlm_refcpu.so``; see ``oracle/ref_shim.cpp``).
* ``COracle``: the plain-C restatement (``oracle/_build/libqlm_oracle.so``;
  see ``oracle/qlm_oracle.c``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm import this module, always as the checker. The product package
``quicklm_b200`` never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libqlm_refcpu.so")
ORACLE_LIB = os.path.join(HERE, "_build", "libqlm_oracle.so")
BLOCK = 32  # Tensor::INT8_BLOCK_SIZE (tensor/tensor.hpp:32)

_P = ctypes.c_void_p
_I = ctypes.c_int


def num_blocks(k: int) -> int:
    return (k + BLOCK - 1) // BLOCK


def reference_root() -> str | None:
    """QuickLM's source tree, if this machine has it: ``$QLM_REFERENCE_SRC``,
    else the ``reference_path`` recorded in the repository's BASELINE.json.
    None when neither names an existing directory (the GPU box: there the
    prebuilt ``oracle/_ref`` files are used)."""
    cand = os.environ.get("QLM_REFERENCE_SRC")
    if not cand:
        meta = os.path.join(os.path.dirname(HERE), "BASELINE.json")
        try:
            import json
            with open(meta) as f:
                cand = json.load(f).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if cand and os.path.isfile(os.path.join(cand, "src", "ops", "math_ops.cpp")):
        return cand
    return None


def build(ref_root: str | None = None) -> None:
    """Compile both checkers with oracle/Makefile (the _ref part only when the
    reference tree is present)."""
    cmd = ["make", "-C", HERE, "--no-print-directory", "all"]
    if ref_root:
        cmd.append(f"REF={ref_root}")
    subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _check_w(w: np.ndarray) -> int:
    if w.dtype == np.float32:
        return 0
    if w.dtype == np.uint16:  # raw bf16 bits
        return 1
    raise TypeError("weights must be float32 or uint16 (bf16 bits)")


class RefCPU:
    """QuickLM's own math::matmul / get_tensor_keep_int8, compiled from source."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference tree exists")
        lib = ctypes.CDLL(path)
        lib.qlmref_last_error.restype = ctypes.c_char_p
        lib.qlmref_init_threads.argtypes = [_I]
        lib.qlmref_quantize.argtypes = [_P, _I, _I, _I, _P, _P]
        lib.qlmref_matmul_int8.argtypes = [_P, _I, _I, _P, _P, _I, _P, _I, _I, ctypes.POINTER(ctypes.c_double)]
        lib.qlmref_matmul_int8_stack.argtypes = [_P, _I, _I, _P, _P, _I, _I, _P, _I,
                                                 ctypes.POINTER(ctypes.c_double)]
        lib.qlmref_greedy_sample.argtypes = [_P, _I, ctypes.POINTER(_I)]
        lib.qlmref_quantize_int4.argtypes = [_P, _I, _I, _I, _P, _P]
        lib.qlmref_matmul_int4.argtypes = [_P, _I, _I, _P, _P, _I, _P, _I]
        _F = ctypes.c_float
        lib.qlmref_rms_norm.argtypes = [_P, _P, _P, _I, _I, _F]
        lib.qlmref_add_rms_norm.argtypes = [_P, _P, _P, _P, _I, _I, _F]
        lib.qlmref_silu_mul.argtypes = [_P, _P, _I]
        lib.qlmref_rope_neox.argtypes = [_P, _I, _I, _I, _F, _I]
        lib.qlmref_silu.argtypes = [_P, _I]
        lib.qlmref_conv1d_update_tapmajor.argtypes = [_P, _P, _I, _P, _P, _I, _I]
        lib.qlmref_l2norm_heads.argtypes = [_P, _I, _I, _F]
        lib.qlmref_gdn_recurrence.argtypes = [_P, _P, _P, _P, _P, _P, _I, _I, _P]
        lib.qlmref_gdn_gates.argtypes = [_P, _P, _P, _P, _P, _P, _I]
        lib.qlmref_rms_norm_gain.argtypes = [_P, _P, _P, _I, _I, _F]
        gdn = [_I, _I, _I, _I, _I] + [_P] * 9 + [_I, _P, _P]
        lib.qlmref_gdn_module_steps.argtypes = gdn
        lib.qlmref_gdn_restated_steps.argtypes = gdn
        lib.qlmref_gqa_attend.argtypes = [_P, _I, _P, _P, _P, _I, _I, _I, _I]
        attn = [_I, _I, _I, _I, _I, _F, _I] + [_P] * 6 + [_I, _P, _P]
        lib.qlmref_attn_module_steps.argtypes = attn
        lib.qlmref_attn_restated_steps.argtypes = attn
        self.lib = lib
        self.threads = 1

    def _rc(self, rc: int) -> None:
        if rc != 0:
            raise RuntimeError(self.lib.qlmref_last_error().decode())

    def quantize_int4(self, w: np.ndarray):
        """get_tensor_keep_int4 on a [n, k] float32 or bf16-bits matrix ->
        (packed uint8 [n, (k+1)//2] (value + 8, low nibble = even column),
        scales float32 [n, ceil(k/32)])."""
        w = np.ascontiguousarray(w)
        dt = _check_w(w)
        n, k = w.shape
        packed = np.empty((n, (k + 1) // 2), np.uint8)
        s = np.empty((n, (k + BLOCK - 1) // BLOCK), np.float32)
        self._rc(self.lib.qlmref_quantize_int4(_ptr(w), dt, n, k, _ptr(packed), _ptr(s)))
        return packed, s

    def matmul_int4(self, x: np.ndarray, packed: np.ndarray, s: np.ndarray, k: int) -> np.ndarray:
        """math::matmul(A=x [m, k], B=int4 [n, k] packed) -> y [m, n]."""
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None, :]
        packed = np.ascontiguousarray(packed, np.uint8)
        s = np.ascontiguousarray(s, np.float32)
        m = x.shape[0]
        n = packed.shape[0]
        y = np.empty((m, n), np.float32)
        self._rc(self.lib.qlmref_matmul_int4(_ptr(x), m, k, _ptr(packed), _ptr(s), n, _ptr(y), n))
        return y

    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        """math::rms_norm over the rows of x [rows, size]."""
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        y = np.empty_like(x)
        self._rc(self.lib.qlmref_rms_norm(_ptr(x), _ptr(w), _ptr(y), x.shape[0], x.shape[1], ctypes.c_float(eps)))
        return y

    def add_rms_norm(self, res: np.ndarray, delta: np.ndarray, w: np.ndarray, eps: float):
        """math::add_rms_norm -> (updated residual, normalised output)."""
        r = np.array(res, np.float32, copy=True, order="C")
        d = np.ascontiguousarray(delta, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(r)
        self._rc(self.lib.qlmref_add_rms_norm(_ptr(r), _ptr(d), _ptr(w), _ptr(out), r.shape[0], r.shape[1],
                                               ctypes.c_float(eps)))
        return r, out

    def silu_mul(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        """math::silu_mul: silu(a) * b (a copy is updated)."""
        a = np.array(a, np.float32, copy=True).ravel()
        b = np.ascontiguousarray(b, np.float32).ravel()
        self._rc(self.lib.qlmref_silu_mul(_ptr(a), _ptr(b), a.size))
        return a

    def silu(self, x: np.ndarray) -> np.ndarray:
        """math::silu (a copy)."""
        x = np.array(x, np.float32, copy=True).ravel()
        self._rc(self.lib.qlmref_silu(_ptr(x), x.size))
        return x

    def conv1d_update_tapmajor(self, inp, state, oldest_tap: int, weight_t):
        """math::causal_conv1d_update_tapmajor -> (output, updated state copy)."""
        inp = np.ascontiguousarray(inp, np.float32)
        st = np.array(state, np.float32, copy=True, order="C")
        wt = np.ascontiguousarray(weight_t, np.float32)
        out = np.empty_like(inp)
        self._rc(self.lib.qlmref_conv1d_update_tapmajor(_ptr(inp), _ptr(st), int(oldest_tap), _ptr(wt), _ptr(out),
                                                        inp.size, wt.shape[0]))
        return out, st

    def l2norm_heads(self, x: np.ndarray, eps: float) -> np.ndarray:
        """The gated-delta-net q/k normalisation on x [heads, head_dim] (a copy)."""
        x = np.array(x, np.float32, copy=True, order="C")
        self._rc(self.lib.qlmref_l2norm_heads(_ptr(x), x.shape[0], x.shape[1], ctypes.c_float(eps)))
        return x

    def gdn_recurrence(self, state, q, k, v, dec, beta):
        """The restated delta-rule recurrence (model/attention.cpp:498-560) ->
        (out [heads, d], updated state copy)."""
        st = np.array(state, np.float32, copy=True, order="C")
        heads, d = st.shape[0], st.shape[1]
        arrs = [np.ascontiguousarray(a, np.float32) for a in (q, k, v, dec, beta)]
        out = np.empty((heads, d), np.float32)
        self._rc(self.lib.qlmref_gdn_recurrence(_ptr(st), *[_ptr(a) for a in arrs], heads, d, _ptr(out)))
        return out, st

    def gdn_gates(self, a_raw, b_raw, A_log, dt_bias):
        """The restated per-head gates (model/attention.cpp:472-482) -> (decay, beta)."""
        arrs = [np.ascontiguousarray(x, np.float32) for x in (a_raw, b_raw, A_log, dt_bias)]
        heads = arrs[0].size
        dec = np.empty(heads, np.float32)
        beta = np.empty(heads, np.float32)
        self._rc(self.lib.qlmref_gdn_gates(*[_ptr(x) for x in arrs], _ptr(dec), _ptr(beta), heads))
        return dec, beta

    def rms_norm_gain(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        """Head-wise RMSNorm with a plain gain (model/attention.cpp:573-577)."""
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        y = np.empty_like(x)
        self._rc(self.lib.qlmref_rms_norm_gain(_ptr(x), _ptr(w), _ptr(y), x.shape[0], x.shape[1], ctypes.c_float(eps)))
        return y

    def gdn_steps(self, w: dict, inputs: np.ndarray, restated: bool = False) -> np.ndarray:
        """Qwen3_5GatedDeltaNet decode steps over inputs [steps, hin] with F32
        weights w (w_qkv, w_z, w_b, w_a, conv_w [3H, ks], norm_w, A_log, dt_bias,
        w_out): the reference module, or (restated=True) this oracle's restatement."""
        keys = ("w_qkv", "w_z", "w_b", "w_a", "conv_w", "norm_w", "A_log", "dt_bias", "w_out")
        a = {k_: np.ascontiguousarray(w[k_], np.float32) for k_ in keys}
        inputs = np.ascontiguousarray(inputs, np.float32)
        heads, hin = a["w_b"].shape
        d = a["norm_w"].size
        ks = a["conv_w"].shape[1]
        hout = a["w_out"].shape[0]
        out = np.empty((inputs.shape[0], hout), np.float32)
        fn = self.lib.qlmref_gdn_restated_steps if restated else self.lib.qlmref_gdn_module_steps
        self._rc(fn(hin, heads, d, ks, hout, *[_ptr(a[k_]) for k_ in keys], inputs.shape[0], _ptr(inputs), _ptr(out)))
        return out

    def gqa_attend(self, q, k_cache, v_cache, pos: int, kv_heads: int) -> np.ndarray:
        """The restated per-head attention (model/attention.cpp:17-81) for one
        token: q [heads, q_stride] (query in the first d), caches [T, kv_heads, d]."""
        q = np.ascontiguousarray(q, np.float32)
        kc = np.ascontiguousarray(k_cache, np.float32)
        vc = np.ascontiguousarray(v_cache, np.float32)
        heads, q_stride = q.shape
        d = kc.shape[-1]
        out = np.empty((heads, d), np.float32)
        self._rc(self.lib.qlmref_gqa_attend(_ptr(q), q_stride, _ptr(kc), _ptr(vc), _ptr(out), int(pos), heads,
                                            int(kv_heads), d))
        return out

    def attn_steps(self, w: dict, inputs: np.ndarray, heads: int, kv_heads: int, d: int, rot: int, theta: float,
                   restated: bool = False) -> np.ndarray:
        """Qwen3_5Attention decode steps (gated q_proj, QK-norm, partial RoPE, no
        biases, F32 weights w_q, w_k, w_v, w_o, q_norm, k_norm) over inputs [steps, hin]."""
        keys = ("w_q", "w_k", "w_v", "w_o", "q_norm", "k_norm")
        a = {k_: np.ascontiguousarray(w[k_], np.float32) for k_ in keys}
        inputs = np.ascontiguousarray(inputs, np.float32)
        hin, hout = inputs.shape[1], a["w_o"].shape[0]
        out = np.empty((inputs.shape[0], hout), np.float32)
        fn = self.lib.qlmref_attn_restated_steps if restated else self.lib.qlmref_attn_module_steps
        self._rc(fn(hin, heads, kv_heads, d, rot, ctypes.c_float(theta), hout, *[_ptr(a[k_]) for k_ in keys],
                    inputs.shape[0], _ptr(inputs), _ptr(out)))
        return out

    def rope_neox(self, t: np.ndarray, pos: int, theta: float, rotary_dim: int) -> np.ndarray:
        """math::apply_rope_neox on one token's t [num_heads, head_dim] (a copy)."""
        t = np.array(t, np.float32, copy=True, order="C")
        self._rc(self.lib.qlmref_rope_neox(_ptr(t), t.shape[0], t.shape[1], int(pos), ctypes.c_float(theta),
                                           int(rotary_dim)))
        return t

    def greedy_sample(self, logits: np.ndarray) -> int:
        """DecoderModel::sample(logits, 0, 0) (model/model.cpp:259-272)."""
        v = np.ascontiguousarray(logits, np.float32).ravel()
        out = _I(0)
        self._rc(self.lib.qlmref_greedy_sample(v.ctypes.data, v.size, ctypes.byref(out)))
        return int(out.value)

    def init_threads(self, n: int) -> None:
        """math::init_thread_pool(n) (ops/math_ops.cpp:161-171)."""
        self._rc(self.lib.qlmref_init_threads(int(n)))
        self.threads = int(n)

    def quantize(self, w: np.ndarray):
        """get_tensor_keep_int8 on a [n, k] float32 or bf16-bits matrix ->
        (q int8 [n, k], scales float32 [n, ceil(k/32)])."""
        w = np.ascontiguousarray(w)
        dt = _check_w(w)
        n, k = w.shape
        q = np.empty((n, k), np.int8)
        s = np.empty((n, num_blocks(k)), np.float32)
        self._rc(self.lib.qlmref_quantize(_ptr(w), dt, n, k, _ptr(q), _ptr(s)))
        return q, s

    def matmul(self, x: np.ndarray, q: np.ndarray, s: np.ndarray, reps: int = 1):
        """math::matmul(A=x [m, k], B=int8 [n, k]) -> (y [m, n], best_ms)."""
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None, :]
        q = np.ascontiguousarray(q, np.int8)
        s = np.ascontiguousarray(s, np.float32)
        m, k = x.shape
        n = q.shape[0]
        y = np.empty((m, n), np.float32)
        best = ctypes.c_double(0.0)
        self._rc(self.lib.qlmref_matmul_int8(_ptr(x), m, k, _ptr(q), _ptr(s), n, _ptr(y), n, int(reps),
                                             ctypes.byref(best)))
        return y, best.value

    def matmul_stack_ms(self, x: np.ndarray, qs, ss, rounds: int = 1) -> float:
        """Wall ms to stream every weight in (qs, ss) through math::matmul once
        per round (rounds in a row)."""
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None, :]
        m, k = x.shape
        n = qs[0].shape[0]
        g = len(qs)
        qp = (ctypes.c_void_p * g)(*[_ptr(a) for a in qs])
        sp = (ctypes.c_void_p * g)(*[_ptr(a) for a in ss])
        y = np.empty((m, n), np.float32)
        tot = ctypes.c_double(0.0)
        self._rc(self.lib.qlmref_matmul_int8_stack(_ptr(x), m, k, qp, sp, g, n, _ptr(y), int(rounds),
                                                   ctypes.byref(tot)))
        return tot.value


class COracle:
    """The plain-C restatement of the same arithmetic (oracle/qlm_oracle.c)."""

    def __init__(self, path: str = ORACLE_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle oracle`")
        lib = ctypes.CDLL(path)
        lib.qlmo_quantize.argtypes = [_P, _I, _I, _I, _P, _P]
        lib.qlmo_quantize_q4.argtypes = [_P, _I, _I, _I, _P, _P]
        lib.qlmo_matmul_int8.argtypes = [_P, _I, _I, _P, _P, _I, _P, _I]
        self.lib = lib

    def quantize(self, w: np.ndarray):
        w = np.ascontiguousarray(w)
        dt = _check_w(w)
        n, k = w.shape
        q = np.empty((n, k), np.int8)
        s = np.empty((n, num_blocks(k)), np.float32)
        self.lib.qlmo_quantize(_ptr(w), dt, n, k, _ptr(q), _ptr(s))
        return q, s

    def quantize_q4(self, w: np.ndarray):
        """int4 quantizer restatement -> (signed values int8 [n, k] in [-8, 7],
        scales [n, ceil(k/32)]); pack_q4 gives the reference's byte layout."""
        w = np.ascontiguousarray(w)
        dt = _check_w(w)
        n, k = w.shape
        q = np.empty((n, k), np.int8)
        s = np.empty((n, (k + BLOCK - 1) // BLOCK), np.float32)
        self.lib.qlmo_quantize_q4(_ptr(w), dt, n, k, _ptr(q), _ptr(s))
        return q, s

    def matmul(self, x: np.ndarray, q: np.ndarray, s: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None, :]
        q = np.ascontiguousarray(q, np.int8)
        s = np.ascontiguousarray(s, np.float32)
        m, k = x.shape
        n = q.shape[0]
        y = np.empty((m, n), np.float32)
        self.lib.qlmo_matmul_int8(_ptr(x), m, k, _ptr(q), _ptr(s), n, _ptr(y), n)
        return y


def synth_weights(n: int, k: int, seed: int, std: float = 0.02) -> np.ndarray:
    """W ~ N(0, std^2) as float64 cast to float32, drawn first from
    default_rng(seed) (the benchmark's synthetic-input convention)."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, k)) * std).astype(np.float32), rng


def synth_case(m: int, n: int, k: int, seed: int):
    """(x [m, k] ~ N(0,1), W [n, k] ~ N(0, 0.02^2)) — W drawn first, then x."""
    w, rng = synth_weights(n, k, seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    return x, w


def greedy_argmax(logits: np.ndarray) -> int:
    """Restatement of QuickLM's greedy sampling (model/model.cpp:259-272): a
    scan from index 0 keeping the first strictly larger value. Equivalently:
    0 if logits[0] is NaN, else the lowest index holding the maximum of the
    non-NaN values (NaN never compares larger; ties keep the lower index;
    +0 and -0 tie)."""
    v = np.asarray(logits, np.float32).ravel()
    if np.isnan(v[0]):
        return 0
    finite = ~np.isnan(v)
    m = v[finite].max()
    return int(np.flatnonzero(finite & (v == m))[0])


def pack_q4(q: np.ndarray) -> np.ndarray:
    """Signed int4 values [n, k] -> the reference's packed bytes [n, (k+1)//2]
    (value + 8, low nibble = even column; a missing odd partner is nibble 8)."""
    q = np.asarray(q, np.int16)
    n, k = q.shape
    u = (q + 8).astype(np.uint8)
    if k % 2:
        u = np.concatenate([u, np.full((n, 1), 8, np.uint8)], axis=1)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def unpack_q4(packed: np.ndarray, k: int) -> np.ndarray:
    """Inverse of pack_q4: signed values int8 [n, k]."""
    p = np.asarray(packed, np.uint8)
    lo = (p & 0x0F).astype(np.int16) - 8
    hi = (p >> 4).astype(np.int16) - 8
    out = np.empty((p.shape[0], 2 * p.shape[1]), np.int16)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out[:, :k].astype(np.int8)
