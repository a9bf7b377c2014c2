"""ctypes binding of libbm_sampler.so (include/bm_sampler.h).

The sampling entry points run only on the CUDA path: if the library or a
B200 is missing, every call raises.  There is no Python or CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG, "lib", "libbm_sampler.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "bm_sampler.h")

BM_OK = 0
ERRORS = {-1: "BM_ERR_INVALID_ARG", -2: "BM_ERR_CUDA", -3: "BM_ERR_OOM",
          -4: "BM_ERR_UNSUPPORTED", -5: "BM_ERR_NO_DEVICE", -6: "BM_ERR_DEVICE"}


class BmError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class Knobs(ctypes.Structure):
    """bm_knobs_t (32 bytes)."""
    _fields_ = [("temp", ctypes.c_float), ("penalty", ctypes.c_float),
                ("min_p", ctypes.c_float), ("top_p", ctypes.c_float),
                ("top_k", ctypes.c_int32), ("inv_temp", ctypes.c_float),
                ("log_min_p", ctypes.c_float), ("flags", ctypes.c_int32)]


KNOBS_DTYPE = np.dtype([("temp", "<f4"), ("penalty", "<f4"), ("min_p", "<f4"),
                        ("top_p", "<f4"), ("top_k", "<i4"), ("inv_temp", "<f4"),
                        ("log_min_p", "<f4"), ("flags", "<i4")])
STATS_DTYPE = np.dtype([("path", "<i4"), ("n_cand", "<i4"), ("n_final", "<i4"),
                        ("consumed", "<i4")])
assert ctypes.sizeof(Knobs) == 32 and KNOBS_DTYPE.itemsize == 32

_lib = None
_P = ctypes.c_void_p

HISTORY_MAX = 256
DECODE_ACTIVE, DECODE_STOP_EOS, DECODE_STOP_TOKEN, DECODE_STOP_MAX = 0, 1, 2, 3


class ModelHeadHost(ctypes.Structure):
    """bm_model_head_host_t."""
    _fields_ = [("vocab_size", ctypes.c_int32), ("d_model", ctypes.c_int32),
                ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32),
                ("w_scale", ctypes.c_float), ("norm_f", ctypes.POINTER(ctypes.c_float)),
                ("lm_head_norm", ctypes.POINTER(ctypes.c_float)),
                ("packed", ctypes.POINTER(ctypes.c_uint8))]


class ModelHeadInfo(ctypes.Structure):
    """bm_model_head_info_t."""
    _fields_ = [("vocab_size", ctypes.c_int32), ("d_model", ctypes.c_int32),
                ("n_layers", ctypes.c_int32), ("n_heads", ctypes.c_int32),
                ("w_scale", ctypes.c_float), ("d_norm_f", _P), ("d_lmh_norm", _P),
                ("d_w8", _P), ("d_packed", _P)]


class DecodeViews(ctypes.Structure):
    """bm_decode_views_t: device pointers of a decode state."""
    _fields_ = [("ring", _P), ("ring_off", _P), ("current", _P), ("status", _P),
                ("n_generated", _P), ("n_pushed", _P), ("n_active", _P)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise BmError(-5, f"{LIB_PATH} is not built (run `make -C bitmamba.c_b200`)")
        L = ctypes.CDLL(LIB_PATH)
        L.bm_last_error.restype = ctypes.c_char_p
        L.bm_knobs_init.argtypes = [ctypes.POINTER(Knobs), ctypes.c_float, ctypes.c_float,
                                    ctypes.c_float, ctypes.c_float, ctypes.c_int]
        L.bm_ctx_create.argtypes = [ctypes.c_int, ctypes.POINTER(_P)]
        L.bm_ctx_destroy.argtypes = [_P]
        L.bm_ctx_destroy.restype = None
        L.bm_max_vocab.argtypes = [_P]
        L.bm_ctx_check.argtypes = [_P]
        L.bm_ctx_stream.argtypes = [_P]
        L.bm_ctx_stream.restype = _P
        L.bm_sample_batch.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                      _P, _P, _P, ctypes.c_int64, _P, _P, _P, _P, _P]
        L.bm_sample_batch_noalloc.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                              _P, _P, _P, ctypes.c_int64, _P, _P, _P, _P, _P]
        L.bm_sample_batch_host.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int64, _P, _P, _P, ctypes.c_int64, _P,
                                           _P, _P, _P]
        L.bm_fused_fallback_rows.argtypes = [_P, ctypes.POINTER(ctypes.c_int),
                                             ctypes.POINTER(ctypes.c_int)]
        L.bm_lmhead_logits.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, _P,
                                       ctypes.c_int, _P, ctypes.c_int64, _P]
        L.bm_lmhead_sample_batch.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, _P,
                                             ctypes.c_int, _P, _P, _P, ctypes.c_int64, _P, _P,
                                             _P, _P, _P]
        L.bm_ternary_unpack.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, _P]
        L.bm_ternary_logits.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P,
                                        ctypes.c_float, ctypes.c_int, _P, ctypes.c_int64, _P]
        L.bm_ternary_sample_batch.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P,
                                              ctypes.c_float, ctypes.c_int, _P, _P, _P,
                                              ctypes.c_int64, _P, _P, _P, _P, _P]
        L.bm_ctx_device.argtypes = [_P, ctypes.POINTER(ctypes.c_int)]
        L.bm_decode_create.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int,
                                       ctypes.POINTER(_P)]
        L.bm_decode_destroy.argtypes = [_P]
        L.bm_decode_reset.argtypes = [_P, _P, _P]
        L.bm_decode_step.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int64, _P, ctypes.c_int64,
                                     _P, _P, _P]
        L.bm_decode_ternary_step.argtypes = [_P, _P, ctypes.c_int, _P, _P, _P, ctypes.c_float,
                                             ctypes.c_int, _P, ctypes.c_int64, _P, _P, _P]
        L.bm_decode_views.argtypes = [_P, ctypes.POINTER(DecodeViews)]
        L.bm_decode_active.argtypes = [_P, _P, ctypes.POINTER(ctypes.c_int32)]
        L.bm_decode_read.argtypes = [_P, _P, _P, _P, _P]
        L.bm_model_head_read.argtypes = [ctypes.c_char_p, ctypes.POINTER(ModelHeadHost)]
        L.bm_model_head_host_free.argtypes = [ctypes.POINTER(ModelHeadHost)]
        L.bm_model_head_host_free.restype = None
        L.bm_model_head_load.argtypes = [_P, ctypes.c_char_p, ctypes.POINTER(_P)]
        L.bm_model_head_info.argtypes = [_P, ctypes.POINTER(ModelHeadInfo)]
        L.bm_model_head_free.argtypes = [_P]
        L.bm_model_head_free.restype = None
        L.bm_rng_seed.argtypes = [ctypes.c_uint64]
        L.bm_rng_seed.restype = None
        L.bm_rng_next.restype = ctypes.c_uint64
        L.bm_rng_float.restype = ctypes.c_float
        L.bm_rng_get_state.restype = ctypes.c_uint64
        L.bm_rng_set_state.argtypes = [ctypes.c_uint64]
        L.bm_rng_set_state.restype = None
        L.bm_sample_row.argtypes = [_P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_float,
                                    ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                    ctypes.c_int]
        L.bm_sample_rows.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _P, _P,
                                     _P, ctypes.c_int64, _P]
        _lib = L
    return _lib


def check(rc):
    if rc < 0:
        raise BmError(rc, lib().bm_last_error().decode(errors="replace"))
    return rc


def knobs_array(temp, penalty, min_p, top_p, top_k) -> np.ndarray:
    """Per-row bm_knobs_t array filled by bm_knobs_init (host libm)."""
    L = lib()
    temp, penalty, min_p, top_p, top_k = np.broadcast_arrays(
        np.asarray(temp, np.float32), np.asarray(penalty, np.float32),
        np.asarray(min_p, np.float32), np.asarray(top_p, np.float32),
        np.asarray(top_k, np.int32))
    out = np.zeros(temp.shape[0] if temp.ndim else 1, KNOBS_DTYPE)
    k = Knobs()
    for i in range(out.shape[0]):
        check(L.bm_knobs_init(ctypes.byref(k), float(temp.flat[i]), float(penalty.flat[i]),
                              float(min_p.flat[i]), float(top_p.flat[i]),
                              int(top_k.flat[i])))
        out[i] = (k.temp, k.penalty, k.min_p, k.top_p, k.top_k, k.inv_temp, k.log_min_p,
                  k.flags)
    return out


def _ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


class Context:
    def __init__(self, device: int = 0):
        self._c = _P()
        check(lib().bm_ctx_create(device, ctypes.byref(self._c)))
        self.device = device

    @property
    def handle(self):
        return self._c

    def max_vocab(self) -> int:
        return lib().bm_max_vocab(self._c)

    def close(self):
        if self._c:
            lib().bm_ctx_destroy(self._c)
            self._c = _P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self):
        check(lib().bm_ctx_check(self._c))

    def stream(self) -> int:
        return lib().bm_ctx_stream(self._c) or 0

    def sample_device(self, logits_ptr, B, V, ld, hist_ptr, off_ptr, knobs_ptr, knob_stride,
                      u_ptr, out_id_ptr, out_prob_ptr=None, stats_ptr=None, stream=None):
        """bm_sample_batch on raw device pointers (ints)."""
        c = ctypes.c_void_p
        check(lib().bm_sample_batch(self._c, c(logits_ptr), B, V, ld,
                                    c(hist_ptr) if hist_ptr else None,
                                    c(off_ptr) if off_ptr else None, c(knobs_ptr),
                                    knob_stride, c(u_ptr), c(out_id_ptr),
                                    c(out_prob_ptr) if out_prob_ptr else None,
                                    c(stats_ptr) if stats_ptr else None,
                                    c(stream) if stream else None))

    def lmhead_logits(self, hidden_ptr, B, d_model, norm_w_ptr, w_ptr, V, logits_ptr, ld,
                      stream=None):
        """bm_lmhead_logits on raw device pointers (ints): RMSNorm + bf16 GEMM."""
        c = ctypes.c_void_p
        check(lib().bm_lmhead_logits(self._c, c(hidden_ptr), B, d_model, c(norm_w_ptr),
                                     c(w_ptr), V, c(logits_ptr), ld,
                                     c(stream) if stream else None))

    def lmhead_sample(self, hidden_ptr, B, d_model, norm_w_ptr, w_ptr, V, hist_ptr, off_ptr,
                      knobs_ptr, knob_stride, u_ptr, out_id_ptr, out_prob_ptr=None,
                      stats_ptr=None, stream=None):
        """bm_lmhead_sample_batch on raw device pointers (ints)."""
        c = ctypes.c_void_p
        check(lib().bm_lmhead_sample_batch(self._c, c(hidden_ptr), B, d_model, c(norm_w_ptr),
                                           c(w_ptr), V, c(hist_ptr) if hist_ptr else None,
                                           c(off_ptr) if off_ptr else None, c(knobs_ptr),
                                           knob_stride, c(u_ptr), c(out_id_ptr),
                                           c(out_prob_ptr) if out_prob_ptr else None,
                                           c(stats_ptr) if stats_ptr else None,
                                           c(stream) if stream else None))

    def fused_fallback_rows(self):
        """bm_fused_fallback_rows: (rows sampled from logits, rows whose logits
        took a GEMM of their own) in the last fused call."""
        a, b = ctypes.c_int(0), ctypes.c_int(0)
        check(lib().bm_fused_fallback_rows(self._c, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def ternary_unpack(self, packed_ptr, V, d_model, w8_ptr, stream=None):
        """bm_ternary_unpack on raw device pointers (ints): 2-bit codes -> int8."""
        c = ctypes.c_void_p
        check(lib().bm_ternary_unpack(self._c, c(packed_ptr), V, d_model, c(w8_ptr),
                                      c(stream) if stream else None))

    def ternary_logits(self, hidden_ptr, B, d_model, norm_f_ptr, lmh_norm_ptr, w8_ptr, w_scale,
                       V, logits_ptr, ld, stream=None):
        """bm_ternary_logits on raw device pointers (ints): the reference's final
        RMSNorm + ternary BitLinear lm_head."""
        c = ctypes.c_void_p
        check(lib().bm_ternary_logits(self._c, c(hidden_ptr), B, d_model,
                                      c(norm_f_ptr) if norm_f_ptr else None, c(lmh_norm_ptr),
                                      c(w8_ptr), w_scale, V, c(logits_ptr), ld,
                                      c(stream) if stream else None))

    def ternary_sample(self, hidden_ptr, B, d_model, norm_f_ptr, lmh_norm_ptr, w8_ptr, w_scale,
                       V, hist_ptr, off_ptr, knobs_ptr, knob_stride, u_ptr, out_id_ptr,
                       out_prob_ptr=None, stats_ptr=None, stream=None):
        """bm_ternary_sample_batch on raw device pointers (ints)."""
        c = ctypes.c_void_p
        check(lib().bm_ternary_sample_batch(
            self._c, c(hidden_ptr), B, d_model, c(norm_f_ptr) if norm_f_ptr else None,
            c(lmh_norm_ptr), c(w8_ptr), w_scale, V, c(hist_ptr) if hist_ptr else None,
            c(off_ptr) if off_ptr else None, c(knobs_ptr), knob_stride, c(u_ptr),
            c(out_id_ptr), c(out_prob_ptr) if out_prob_ptr else None,
            c(stats_ptr) if stats_ptr else None, c(stream) if stream else None))

    def sample_host(self, logits, hist, hist_off, knobs, uniform, want_prob=True,
                    want_stats=True):
        """bm_sample_batch_host on numpy arrays.  Returns (ids, probs, stats)."""
        logits = np.ascontiguousarray(logits, np.float32)
        B, V = logits.shape
        knobs = np.ascontiguousarray(knobs, KNOBS_DTYPE)
        stride = 1 if knobs.shape[0] == B and B != 1 else (0 if knobs.shape[0] == 1 else -1)
        if stride < 0:
            raise ValueError("knobs must have 1 or B rows")
        u = np.ascontiguousarray(uniform, np.float32)
        ids = np.empty(B, np.int32)
        probs = np.empty(B, np.float32) if want_prob else None
        stats = np.zeros(B, STATS_DTYPE) if want_stats else None
        if hist is not None:
            hist = np.ascontiguousarray(hist, np.int32)
            hist_off = np.ascontiguousarray(hist_off, np.int64)
            if hist.size == 0:
                hist = np.zeros(1, np.int32)
        check(lib().bm_sample_batch_host(self._c, _ptr(logits), B, V, V, _ptr(hist),
                                         _ptr(hist_off) if hist is not None else None,
                                         _ptr(knobs), stride, _ptr(u), _ptr(ids),
                                         _ptr(probs), _ptr(stats)))
        return ids, probs, stats


def rng_seed(seed: int):
    lib().bm_rng_seed(seed)


def rng_float() -> float:
    return lib().bm_rng_float()


def sample_row(logits, history, penalty, temp, min_p, top_p, top_k) -> int:
    """Reference-convention single row (global RNG, default context)."""
    logits = np.ascontiguousarray(logits, np.float32)
    h = np.ascontiguousarray(history, np.int32)
    return check(lib().bm_sample_row(_ptr(logits), logits.shape[0],
                                     _ptr(h) if h.size else None, int(h.size),
                                     penalty, temp, min_p, top_p, top_k))


def sample_rows(logits, hist, hist_off, knobs) -> np.ndarray:
    logits = np.ascontiguousarray(logits, np.float32)
    B, V = logits.shape
    knobs = np.ascontiguousarray(knobs, KNOBS_DTYPE)
    stride = 0 if knobs.shape[0] == 1 else 1
    ids = np.empty(B, np.int32)
    if hist is not None:
        hist = np.ascontiguousarray(hist, np.int32)
        hist_off = np.ascontiguousarray(hist_off, np.int64)
        if hist.size == 0:
            hist = np.zeros(1, np.int32)
    check(lib().bm_sample_rows(_ptr(logits), B, V, V, _ptr(hist),
                               _ptr(hist_off) if hist is not None else None, _ptr(knobs),
                               stride, _ptr(ids)))
    return ids


def header_symbols() -> list:
    """Function names declared in include/bm_sampler.h."""
    import re
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(bm_[a-z0-9_]+)\s*\(", txt)))


class Decode:
    """A device-resident decode loop state (bm_decode_*): per-row 256-id
    history windows, current tokens and stop status on the GPU."""

    def __init__(self, ctx, B, max_tokens=0, stop_ids=()):
        self._ctx = ctx
        self._d = _P()
        self.B = B
        stop = np.ascontiguousarray(np.asarray(stop_ids, np.int32))
        check(lib().bm_decode_create(ctx._c, B, max_tokens,
                                     stop.ctypes.data_as(_P) if stop.size else None,
                                     int(stop.size), ctypes.byref(self._d)))

    def close(self):
        if self._d:
            lib().bm_decode_destroy(self._d)
            self._d = _P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self, prompts):
        """prompts: one sequence of ids per row."""
        prompts = [np.asarray(p, np.int32) for p in prompts]
        off = np.zeros(len(prompts) + 1, np.int64)
        off[1:] = np.cumsum([len(p) for p in prompts])
        ids = np.ascontiguousarray(np.concatenate(prompts) if off[-1] else np.zeros(1, np.int32),
                                   dtype=np.int32)
        check(lib().bm_decode_reset(self._d, ids.ctypes.data_as(_P), off.ctypes.data_as(_P)))

    def step(self, logits_ptr, V, ld, knobs_ptr, knob_stride, u_ptr, out_id_ptr=None,
             stream=None):
        c = ctypes.c_void_p
        check(lib().bm_decode_step(self._d, c(logits_ptr), V, ld, c(knobs_ptr), knob_stride,
                                   c(u_ptr), c(out_id_ptr) if out_id_ptr else None,
                                   c(stream) if stream else None))

    def ternary_step(self, hidden_ptr, d_model, norm_f_ptr, lmh_norm_ptr, w8_ptr, w_scale, V,
                     knobs_ptr, knob_stride, u_ptr, out_id_ptr=None, stream=None):
        c = ctypes.c_void_p
        check(lib().bm_decode_ternary_step(
            self._d, c(hidden_ptr), d_model, c(norm_f_ptr) if norm_f_ptr else None,
            c(lmh_norm_ptr), c(w8_ptr), w_scale, V, c(knobs_ptr), knob_stride, c(u_ptr),
            c(out_id_ptr) if out_id_ptr else None, c(stream) if stream else None))

    def views(self):
        v = DecodeViews()
        check(lib().bm_decode_views(self._d, ctypes.byref(v)))
        return {k: getattr(v, k) for k, _ in DecodeViews._fields_}

    def read(self):
        """The state on the host: dict of current, status, n_generated [B] and
        ring [B x 256] (synchronises)."""
        B = self.B
        cur, st, ng = (np.empty(B, np.int32) for _ in range(3))
        ring = np.empty((B, HISTORY_MAX), np.int32)
        check(lib().bm_decode_read(self._d, cur.ctypes.data_as(_P), st.ctypes.data_as(_P),
                                   ng.ctypes.data_as(_P), ring.ctypes.data_as(_P)))
        return {"current": cur, "status": st, "n_generated": ng, "ring": ring}

    def active(self, stream=None):
        n = ctypes.c_int32()
        check(lib().bm_decode_active(self._d, ctypes.c_void_p(stream) if stream else None,
                                     ctypes.byref(n)))
        return n.value


def read_model_head(path):
    """bm_model_head_read (host only): the decode tail's tensors of a packed
    model file as numpy arrays."""
    h = ModelHeadHost()
    check(lib().bm_model_head_read(os.fsencode(path), ctypes.byref(h)))
    try:
        d, V = h.d_model, h.vocab_size
        pk = V * ((d + 3) // 4)
        return {"vocab_size": V, "d_model": d, "n_layers": h.n_layers, "n_heads": h.n_heads,
                "w_scale": h.w_scale,
                "norm_f": np.ctypeslib.as_array(h.norm_f, (d,)).copy(),
                "lm_head_norm": np.ctypeslib.as_array(h.lm_head_norm, (d,)).copy(),
                "packed": np.ctypeslib.as_array(h.packed, (pk,)).copy().reshape(V, -1)}
    finally:
        lib().bm_model_head_host_free(ctypes.byref(h))


class ModelHead:
    """bm_model_head_load: the decode tail's tensors on the device."""

    def __init__(self, ctx, path):
        self._h = _P()
        check(lib().bm_model_head_load(ctx._c, os.fsencode(path), ctypes.byref(self._h)))
        i = ModelHeadInfo()
        check(lib().bm_model_head_info(self._h, ctypes.byref(i)))
        self.info = {k: getattr(i, k) for k, _ in ModelHeadInfo._fields_}

    def close(self):
        if self._h:
            lib().bm_model_head_free(self._h)
            self._h = _P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
