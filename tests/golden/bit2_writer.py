"""Writes small model files in the reference's packed format (test
infrastructure): the layout scripts/export-bin.py:110-200 writes and
src/model.c:367-475 / 554-626 reads.

  header   int32 magic 0x42495432, vocab_size, d_model, n_layers, n_heads
  tensors  in order: embed.weight; per layer in_proj.norm.weight,
           in_proj.weight, conv1d.weight, conv1d.bias, dt_bias, A_log, D,
           out_proj.norm.weight, out_proj.weight; then norm_f.weight,
           lm_head.norm.weight, lm_head.weight
  float    int32 0, int32 ndim, ndim x int32 dims, fp32 data
  packed   int32 2, int32 rows, int32 cols, fp32 scale, rows x cols / 4
           bytes of 2-bit codes (w + 1, four per byte, lowest bits first)

The tensors are seeded synthetic values (no checkpoint is involved): float
tensors N(0, 1) scaled, ternary weights from the counter hash.
"""
from __future__ import annotations

import struct

import numpy as np

import synth

MAGIC = 0x42495432
EXPAND = 2      # d_inner = 2 d_model (src/bitmamba.h:48)
CONV = 4        # conv1d width (src/bitmamba.h:49)


def float_tensor(a) -> bytes:
    a = np.ascontiguousarray(a, np.float32)
    return struct.pack("ii", 0, a.ndim) + struct.pack(f"{a.ndim}i", *a.shape) + a.tobytes()


def packed_tensor(codes: np.ndarray, rows: int, cols: int, scale: float) -> bytes:
    return struct.pack("iiif", 2, rows, cols, scale) + \
        np.ascontiguousarray(codes, np.uint8).tobytes()


class Model:
    """The tensors of one synthetic model, kept for the checks."""

    def __init__(self, seed, vocab, d_model, n_layers, n_heads, lm_scale=16.0):
        self.vocab, self.d, self.L, self.H = vocab, d_model, n_layers, n_heads
        di = EXPAND * d_model
        nrm = lambda st, n: (1.0 + 0.02 * synth.normal(seed, st, n)).astype(np.float32)
        g = lambda st, n, s: (s * synth.normal(seed, st, n)).astype(np.float32)
        self.embed = g(1, vocab * d_model, 0.02).reshape(vocab, d_model)
        self.layers = []
        for i in range(n_layers):
            b = 100 * (i + 1)
            self.layers.append(dict(
                in_proj_norm=nrm(b + 1, d_model),
                in_proj=(synth.ternary_codes(seed, b + 2, 2 * di + 3 * n_heads, d_model),
                         2 * di + 3 * n_heads, d_model, 20.0),
                conv1d_w=g(b + 3, di * CONV, 0.1).reshape(di, 1, CONV),
                conv1d_b=g(b + 4, di, 0.1),
                dt_bias=g(b + 5, n_heads, 0.1),
                A_log=g(b + 6, n_heads, 0.1),
                D=g(b + 7, di, 0.1),
                out_proj_norm=nrm(b + 8, di),
                out_proj=(synth.ternary_codes(seed, b + 9, d_model, di), d_model, di, 20.0)))
        self.norm_f = nrm(7001, d_model)
        self.lm_head_norm = nrm(7002, d_model)
        self.lm_codes = synth.ternary_codes(seed, 7003, vocab, d_model)
        self.lm_scale = np.float32(lm_scale)

    def tensors(self):
        """(name, bytes) in the file's order."""
        out = [("embed.weight", float_tensor(self.embed))]
        for i, ly in enumerate(self.layers):
            p = f"layers.{i}."
            out += [(p + "in_proj.norm.weight", float_tensor(ly["in_proj_norm"])),
                    (p + "in_proj.weight", packed_tensor(*ly["in_proj"])),
                    (p + "conv1d.weight", float_tensor(ly["conv1d_w"])),
                    (p + "conv1d.bias", float_tensor(ly["conv1d_b"])),
                    (p + "dt_bias", float_tensor(ly["dt_bias"])),
                    (p + "A_log", float_tensor(ly["A_log"])),
                    (p + "D", float_tensor(ly["D"])),
                    (p + "out_proj.norm.weight", float_tensor(ly["out_proj_norm"])),
                    (p + "out_proj.weight", packed_tensor(*ly["out_proj"]))]
        out += [("norm_f.weight", float_tensor(self.norm_f)),
                ("lm_head.norm.weight", float_tensor(self.lm_head_norm)),
                ("lm_head.weight", packed_tensor(self.lm_codes, self.vocab, self.d,
                                                 float(self.lm_scale)))]
        return out

    def header(self):
        return struct.pack("iiiii", MAGIC, self.vocab, self.d, self.L, self.H)

    def write(self, path, replace=None, header=None, truncate=None):
        """replace: {tensor name: bytes} to plant a malformed tensor."""
        blob = header if header is not None else self.header()
        for name, data in self.tensors():
            blob += (replace or {}).get(name, data)
        if truncate is not None:
            blob = blob[:truncate]
        with open(path, "wb") as f:
            f.write(blob)
        return len(blob)
