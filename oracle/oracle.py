"""ctypes access to the sampler oracle (TEST INFRASTRUCTURE ONLY).

Loads oracle/lib/liboracle.so (the C restatement) and, when it was built in a
tree that had the reference sources, oracle/_ref/libref_sampler.so (the
reference's own sampler).  Only tests, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs import this module; the product library never
does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "lib", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_sampler.so")

PATHS = {1: "greedy", 2: "k_guard", 3: "k", 4: "full_guard", 5: "lazy",
         6: "partial", 7: "full"}

RESULT_DTYPE = np.dtype([
    ("token", "<i4"), ("prob", "<f4"), ("consumed", "<i4"), ("path", "<i4"),
    ("n_cand", "<i4"), ("n_final", "<i4"), ("pos", "<i4"), ("r", "<f4"),
    ("new_sum", "<f8"), ("r_margin", "<f8"), ("cut_margin", "<f8"),
    ("max_logit", "<f4"), ("thresh", "<f4")], align=True)
assert RESULT_DTYPE.itemsize == 64

_lib = None
_ref = None


def reference_tree() -> str | None:
    """The reference checkout whose sources oracle/_ref is compiled from:
    $BM_REFERENCE_SRC, else a `reference` directory beside this repository's
    checkout; None when neither holds src/model.c."""
    cands = [os.environ.get("BM_REFERENCE_SRC"),
             os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for c in cands:
        if c and os.path.isfile(os.path.join(c, "src", "model.c")):
            return c
    return None


def build(ref: bool = True) -> None:
    """Compile the oracle (and the reference harness when its sources exist)."""
    cmd = ["make", "-s", "-C", HERE, "oracle"]
    tree = reference_tree() if ref else None
    if tree:
        cmd = ["make", "-s", "-C", HERE, "all", f"REF={tree}"]
    subprocess.run(cmd, check=True)


def _p(a, t):
    return a.ctypes.data_as(ctypes.POINTER(t)) if a is not None else None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build(ref=False)
        L = ctypes.CDLL(ORACLE_SO)
        f = L.bmo_sample_batch
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_int,
                      ctypes.c_int64, ctypes.POINTER(ctypes.c_int32),
                      ctypes.POINTER(ctypes.c_int64)] + \
            [ctypes.POINTER(ctypes.c_float)] * 4 + \
            [ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float),
             ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float),
             ctypes.c_void_p, ctypes.c_int]
        L.bmo_rng_float.restype = ctypes.c_float
        L.bmo_rng_float.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
        L.bmo_rng_seed.argtypes = [ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint64]
        _lib = L
    return _lib


def has_ref() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_SO)
        f = L.bm_ref_sample_row
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int,
                      ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                      ctypes.c_float, ctypes.c_float, ctypes.c_float,
                      ctypes.c_float, ctypes.c_int, ctypes.c_float,
                      ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float),
                      ctypes.c_void_p, ctypes.c_void_p]
        assert L.bm_ref_sizeof_token_prob() == 8
        _ref = L
    return _ref


def sample_batch(b, uniforms, threads: int = 1, with_results: bool = True):
    """Run the oracle on a synth.Batch.  Returns (ids, probs, results)."""
    L = lib()
    B, V = b.logits.shape
    u = np.ascontiguousarray(uniforms, dtype=np.float32)
    assert u.shape == (B,)
    ids = np.empty(B, np.int32)
    probs = np.empty(B, np.float32)
    res = np.zeros(B, RESULT_DTYPE) if with_results else None
    rc = L.bmo_sample_batch(
        _p(b.logits, ctypes.c_float), B, V, V, _p(b.hist, ctypes.c_int32),
        _p(b.hist_off, ctypes.c_int64), _p(b.temp, ctypes.c_float),
        _p(b.penalty, ctypes.c_float), _p(b.min_p, ctypes.c_float),
        _p(b.top_p, ctypes.c_float), _p(b.top_k, ctypes.c_int32),
        _p(u, ctypes.c_float), _p(ids, ctypes.c_int32), _p(probs, ctypes.c_float),
        res.ctypes.data if res is not None else None, threads)
    if rc != 0:
        raise MemoryError("oracle batch failed")
    return ids, probs, res


def ref_sample_batch(b, uniforms):
    """Run the reference's own sampler (oracle/_ref) row by row.
    Returns (ids, probs, consumed)."""
    L = ref_lib()
    B, V = b.logits.shape
    ids = np.empty(B, np.int32)
    probs = np.empty(B, np.float32)
    cons = np.empty(B, np.int32)
    tp = (ctypes.c_byte * (8 * V))()
    vis = (ctypes.c_uint64 * ((V + 63) // 64))()
    c = ctypes.c_int()
    p = ctypes.c_float()
    for r in range(B):
        row = np.array(b.logits[r], dtype=np.float32, copy=True)
        h = np.ascontiguousarray(b.hist[b.hist_off[r]:b.hist_off[r + 1]], np.int32)
        ids[r] = L.bm_ref_sample_row(
            _p(row, ctypes.c_float), V, _p(h, ctypes.c_int32), len(h),
            float(b.penalty[r]), float(b.temp[r]), float(b.min_p[r]),
            float(b.top_p[r]), int(b.top_k[r]), float(uniforms[r]),
            ctypes.byref(c), ctypes.byref(p), ctypes.addressof(tp),
            ctypes.addressof(vis))
        probs[r] = p.value
        cons[r] = c.value
    return ids, probs, cons


def ref_sample_batch_mt(b, uniforms, threads: int):
    """The reference's own sampler over a batch with `threads` pthreads
    (oracle/_ref).  Returns ids."""
    L = ref_lib()
    f = L.bm_ref_sample_batch
    f.restype = ctypes.c_int
    B, V = b.logits.shape
    u = np.ascontiguousarray(uniforms, np.float32)
    out = np.empty(B, np.int32)
    hist = b.hist if b.hist.size else None
    rc = f(_p(b.logits, ctypes.c_float), B, V, ctypes.c_longlong(V),
           _p(hist, ctypes.c_int32) if hist is not None else None,
           _p(b.hist_off, ctypes.c_int64) if hist is not None else None,
           _p(b.temp, ctypes.c_float), _p(b.penalty, ctypes.c_float),
           _p(b.min_p, ctypes.c_float), _p(b.top_p, ctypes.c_float),
           _p(b.top_k, ctypes.c_int32), _p(u, ctypes.c_float),
           _p(out, ctypes.c_int32), threads)
    if rc != 0:
        raise MemoryError("reference batch failed")
    return out
