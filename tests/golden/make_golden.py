"""Generate the committed golden fixtures from QuickLM's OWN int8 path.

Run where the reference tree exists, so that
``oracle/_ref/libqlm_refcpu.so`` (compiled from the reference sources by
``oracle/Makefile``) can be built:

    make -C oracle all REF=<QuickLM source root> && python tests/golden/make_golden.py [--skip-large]

Writes:
* ``small_cases.npz`` — full inputs and outputs of small cases covering the
  edge cases the reference's code has (ragged K, K < 8, N not a multiple of
  8/4, M > 8, all-zero blocks, NaN/Inf/subnormal weights, NaN/Inf
  activations, bf16 sources).
* ``config_hashes.json`` — sha256 of the seeded inputs, of the reference's
  quantized bytes/scales and of its outputs for every benchmark configuration shape
  (cfg1 GEMV, cfg2 prefill, cfg4 projection sweep). Inputs are regenerated
  from the seed at test time; the input hash pins the generator.
* ``cfg1_y.npy`` — the reference's config-1 output vector (6144 floats).
* ``small_cases_int4.npz`` — the same small cases through the reference's int4
  path: get_tensor_keep_int4's packed bytes ((K+1)/2 per row, value + 8, low
  nibble = even column) and scales, and its int4 math::matmul output
  (``--int4-only`` writes just this file).

Synthetic-input convention: numpy ``default_rng(seed)``; W ~ N(0, 0.02^2)
drawn first as float64 and cast to float32, then x ~ N(0, 1) likewise.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import RefCPU, synth_case  # noqa: E402  (test infrastructure)
from tests.golden.cases import CFG1, CFG2, CFG4, SMALL_CASES, make_small_case  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-large", action="store_true", help="skip the lm_head-sized cfg4 shape")
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--int4-only", action="store_true", help="write only small_cases_int4.npz")
    args = ap.parse_args()
    ref = RefCPU()
    ref.init_threads(args.threads)

    arrays4 = {}
    for i, spec in enumerate(SMALL_CASES):
        x, w = make_small_case(spec)
        p4, s4 = ref.quantize_int4(w)
        arrays4[f"c{i}_p"] = p4
        arrays4[f"c{i}_s"] = s4
        arrays4[f"c{i}_y"] = ref.matmul_int4(x, p4, s4, w.shape[1])
    np.savez_compressed(os.path.join(HERE, "small_cases_int4.npz"), **arrays4)
    if args.int4_only:
        return

    arrays = {}
    for i, spec in enumerate(SMALL_CASES):
        x, w = make_small_case(spec)
        q, s = ref.quantize(w)
        y, _ = ref.matmul(x, q, s)
        for name, a in (("x", x), ("w", w), ("q", q), ("s", s), ("y", y)):
            arrays[f"c{i}_{name}"] = a
    np.savez_compressed(os.path.join(HERE, "small_cases.npz"), **arrays)

    hashes = {"convention": "default_rng(seed): W=N(0,0.02^2) first, then x=N(0,1); float64 cast to float32",
              "oracle": "reference math_ops.cpp + safetensors.cpp, -O3 -mavx2 -mfma -ffp-contract=off",
              "cases": {}}

    def record(tag, m, n, k, seed):
        x, w = synth_case(m, n, k, seed)
        q, s = ref.quantize(w)
        y, _ = ref.matmul(x, q, s)
        hashes["cases"][tag] = {"m": m, "n": n, "k": k, "seed": seed, "w": sha(w), "x": sha(x), "q": sha(q),
                                "s": sha(s), "y": sha(y), "y_head": y.ravel()[:8].tolist()}
        print(tag, "done", flush=True)
        return y

    m, n, k, seed = CFG1
    y1 = record("cfg1", m, n, k, seed)
    np.save(os.path.join(HERE, "cfg1_y.npy"), y1)
    for (m, n, k, seed) in CFG2:
        record(f"cfg2_m{m}_n{n}_k{k}", m, n, k, seed)
    for (m, n, k, seed) in CFG4:
        if args.skip_large and n > 100000:
            continue
        record(f"cfg4_m{m}_n{n}_k{k}", m, n, k, seed)
    with open(os.path.join(HERE, "config_hashes.json"), "w") as f:
        json.dump(hashes, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
