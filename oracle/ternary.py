"""ctypes access to the ternary lm_head oracle (TEST INFRASTRUCTURE ONLY).

Wraps the C restatement in oracle/lib/liboracle.so (ternary_oracle.c) and,
when present, the reference's own final RMSNorm + BitLinear lm_head compiled
into oracle/_ref/libref_sampler.so (bm_ref_ternary_lmhead in ref_harness.c).
Only tests, __graft_entry__.smoke() and bench.py's CPU legs import this
module; the product library never does.
"""
from __future__ import annotations

import ctypes

import numpy as np

import oracle

_P = ctypes.c_void_p
_done = set()


def _lib():
    L = oracle.lib()
    if "o" not in _done:
        L.bmo_ternary_prep.restype = ctypes.c_int
        L.bmo_ternary_prep.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_float,
                                       _P, _P, _P]
        L.bmo_ternary_unpack.restype = None
        L.bmo_ternary_unpack.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P]
        L.bmo_ternary_logits.restype = None
        L.bmo_ternary_logits.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int,
                                         _P, ctypes.c_int64]
        L.bmo_rms_norm_x86.restype = ctypes.c_float
        L.bmo_rms_norm_x86.argtypes = [_P, ctypes.c_int, _P, _P]
        _done.add("o")
    return L


def _ref():
    L = oracle.ref_lib()
    if "r" not in _done:
        L.bm_ref_ternary_lmhead.restype = ctypes.c_int
        L.bm_ref_ternary_lmhead.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, _P, _P,
                                            ctypes.c_int, ctypes.c_float, _P, ctypes.c_longlong,
                                            _P, _P, ctypes.c_int]
        _done.add("r")
    return L


def _ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


def prep(hidden, norm_f, lmh_norm, w_scale):
    """int8 activations [B x d] and inv_scale [B] (C restatement)."""
    x = np.ascontiguousarray(hidden, np.float32)
    B, d = x.shape
    xq = np.empty((B, d), np.int8)
    inv = np.empty(B, np.float32)
    scratch = np.empty(2 * d, np.float32)
    nf = None if norm_f is None else np.ascontiguousarray(norm_f, np.float32)
    nl = np.ascontiguousarray(lmh_norm, np.float32)
    rc = _lib().bmo_ternary_prep(_ptr(x), B, d, _ptr(nf), _ptr(nl), float(w_scale),
                                 _ptr(scratch), _ptr(xq), _ptr(inv))
    if rc != 0:
        raise ValueError(f"d = {d}: needs a multiple of 32")
    return xq, inv


def unpack(packed, d):
    p = np.ascontiguousarray(packed, np.uint8)
    V = p.shape[0]
    w8 = np.empty((V, d), np.int8)
    _lib().bmo_ternary_unpack(_ptr(p), V, d, _ptr(w8))
    return w8


def logits(xq, inv, packed):
    """fp32 logits [B x V] of the C restatement (exact int32 dot products)."""
    xq = np.ascontiguousarray(xq, np.int8)
    inv = np.ascontiguousarray(inv, np.float32)
    p = np.ascontiguousarray(packed, np.uint8)
    B, d = xq.shape
    V = p.shape[0]
    out = np.empty((B, V), np.float32)
    _lib().bmo_ternary_logits(_ptr(xq), _ptr(inv), B, d, _ptr(p), V, _ptr(out), V)
    return out


def logits_fast(xq, inv, packed):
    """Same values as logits() through a float64 matrix product, for the
    larger checks: every partial sum is an integer below 2^31, so the float64
    arithmetic is exact and the int32 -> float conversion is the reference's."""
    w8 = unpack(packed, xq.shape[1]).astype(np.float64)
    dot = xq.astype(np.float64) @ w8.T
    return dot.astype(np.int32).astype(np.float32) * np.asarray(inv, np.float32)[:, None]


def ref_logits(hidden, norm_f, lmh_norm, packed, w_scale, threads=0, want_prep=False):
    """The reference's own final RMSNorm + BitLinear lm_head (oracle/_ref).
    Returns (logits, kernel_set) or (logits, kernel_set, xq, inv) where
    kernel_set is "avx2" or "scalar"."""
    x = np.ascontiguousarray(hidden, np.float32)
    B, d = x.shape
    p = np.ascontiguousarray(packed, np.uint8)
    V = p.shape[0]
    out = np.empty((B, V), np.float32)
    xq = np.empty((B, d), np.int8) if want_prep else None
    inv = np.empty(B, np.float32) if want_prep else None
    nf = None if norm_f is None else np.ascontiguousarray(norm_f, np.float32)
    nl = np.ascontiguousarray(lmh_norm, np.float32)
    rc = _ref().bm_ref_ternary_lmhead(_ptr(x), B, d, _ptr(nf), _ptr(nl), _ptr(p), V,
                                      float(w_scale), _ptr(out), V, _ptr(xq), _ptr(inv),
                                      int(threads))
    if rc < 0:
        raise MemoryError("reference lm_head failed")
    ks = "avx2" if rc == 1 else "scalar"
    return (out, ks, xq, inv) if want_prep else (out, ks)
