"""CPU restatement of the final RMSNorm + bf16 lm_head (TEST INFRASTRUCTURE ONLY).

Checks the CUDA library's bm_lmhead_logits.  Only tests, __graft_entry__ and
bench.py's CPU legs import this module; the product library never does.

rmsnorm_bf16 restates jserv/bitmamba.c src/kernel.c:72-91 (scalar_rms_norm):
four fp32 accumulators over the strided elements i = q, q+4, q+8, ... (each
x*x rounded to fp32, then added), summed left to right, the tail elements
added after, rms = 1 / sqrtf(sum / size + 1e-6f), out = (x * rms) * w, all in
fp32 (numpy float32 arithmetic is IEEE single precision).  The result is then
rounded to bf16 (round to nearest even), the operand the tensor cores read.

The reference's lm_head is a ternary BitLinear (src/model.c:1239-1262); the
bf16 projection has no counterpart there, so lmhead_logits is a plain float64
product of the same bf16 operands (parity unpinned by the reference: the
check is against this exact product, with an fp32-accumulation tolerance).
"""
from __future__ import annotations

import numpy as np


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even (finite x)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return r.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def rmsnorm_bf16(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """bf16 bits of scalar_rms_norm(x[r]) for every row (src/kernel.c:72-91)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    B, D = x.shape
    D4 = (D // 4) * 4
    acc = np.zeros((B, 4), np.float32)
    for i in range(0, D4, 4):
        xi = x[:, i:i + 4]
        acc = acc + xi * xi                      # fp32 multiply, then fp32 add
    s = ((acc[:, 0] + acc[:, 1]) + acc[:, 2]) + acc[:, 3]
    for i in range(D4, D):
        s = s + x[:, i] * x[:, i]
    rms = np.float32(1.0) / np.sqrt(s / np.float32(D) + np.float32(1e-6), dtype=np.float32)
    out = (x * rms[:, None]) * w[None, :]
    return bf16_bits(out)


def lmhead_logits(a_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """float64 product of the bf16 operands: a [B x K] times W [V x K] transposed."""
    a = bf16_to_f32(a_bits).astype(np.float64)
    w = bf16_to_f32(w_bits).astype(np.float64)
    return a @ w.T
