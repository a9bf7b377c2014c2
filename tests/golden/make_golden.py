"""Regenerates tests/golden/golden.json from the reference's own sampler.

Run in a tree where oracle/_ref/libref_sampler.so was built from the
reference sources (make -C oracle).  For every case of cases.py (inputs are
deterministic, see synth.py) it stores the reference's sampled ids, the
probability the reference holds for each id (as float32 bit patterns), and
whether rng_float() was called.  It also stores the first rng_float() values
of the reference RNG for a few seeds.
"""
from __future__ import annotations

import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.join(HERE, "..", "..", "oracle")]
import cases  # noqa: E402
import oracle  # noqa: E402


def reference_rng(seed: int, n: int):
    L = oracle.ref_lib()
    L.rng_seed.argtypes = [ctypes.c_uint64]
    L.rng_float.restype = ctypes.c_float
    L.rng_seed(seed)
    return [float(L.rng_float()) for _ in range(n)]


def main():
    if not oracle.has_ref():
        raise SystemExit("oracle/_ref/libref_sampler.so is missing: run make -C oracle")
    out = {"cases": {}, "rng": {}}
    for name, b, u in cases.all_cases() + cases.config_cases(8):
        ids, probs, cons = oracle.ref_sample_batch(b, u)
        out["cases"][name] = {
            "ids": ids.tolist(),
            "prob_bits": probs.view(np.uint32).tolist(),
            "consumed": cons.tolist(),
            "uniforms": u.view(np.uint32).tolist(),
        }
    for seed in (0, 1, 42, 1234567):
        out["rng"][str(seed)] = reference_rng(seed, 8)
    path = os.path.join(HERE, "golden.json")
    with open(path, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(f"wrote {path}: {len(out['cases'])} cases")


if __name__ == "__main__":
    main()
