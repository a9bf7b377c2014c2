"""CPU: the ternary lm_head oracle (oracle/ternary_oracle.c) against the
reference's own final RMSNorm + BitLinear lm_head compiled from its sources
(oracle/_ref; src/model.c:1225-1262 through the kernel table of this host).

The restatement follows the AVX2 kernels (src/arch/avx2.c), which the
reference selects on x86-64 hosts with AVX2 and FMA; the comparison is bit for
bit (logits, int8 activations and output scales).  Skipped where the
reference could not be compiled or selects other kernels.
"""
import numpy as np
import pytest

import oracle
import synth
import ternary


def _need_ref():
    if not oracle.has_ref():
        pytest.skip("reference harness not built (no reference sources)")


def test_decode_table():
    """Every byte: four codes, lowest bits first, code c -> min(c, 2) - 1
    (src/quantization.c:27-31)."""
    packed = np.arange(256, dtype=np.uint8).reshape(256, 1)
    packed = np.repeat(packed, 8, axis=1)                     # d = 32
    w8 = ternary.unpack(packed, 32)
    for b in range(256):
        want = [min((b >> (2 * j)) & 3, 2) - 1 for j in range(4)]
        assert list(w8[b, :4]) == want


@pytest.mark.parametrize("B,V,d,final_norm,raw", [
    (3, 1, 32, True, False), (5, 37, 64, False, True), (4, 1000, 256, True, False),
    (2, 513, 2048, True, True), (1, 50257, 2048, True, False)])
def test_restatement_matches_reference(B, V, d, final_norm, raw):
    _need_ref()
    b = synth.make_c6(41 + d, B, V=V, d=d, raw=raw)
    nf = b.norm_f if final_norm else None
    ref, ks, rxq, rinv = ternary.ref_logits(b.hidden, nf, b.lmh_norm, b.packed, b.w_scale,
                                            want_prep=True)
    if ks != "avx2":
        pytest.skip("this host runs the reference's scalar kernels")
    xq, inv = ternary.prep(b.hidden, nf, b.lmh_norm, b.w_scale)
    assert np.array_equal(xq, rxq)
    assert np.array_equal(inv.view(np.uint32), rinv.view(np.uint32))
    got = ternary.logits(xq, inv, b.packed) if V * B <= 50000 else \
        ternary.logits_fast(xq, inv, b.packed)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_extreme_rows_match_reference():
    """A zero row (rms = 1000, every activation 0), a row of one spike (one
    activation at +-127, the rest near 0), large magnitudes, and exact
    half-way products for the round-to-even quantisation."""
    _need_ref()
    d, V = 64, 200
    x = np.zeros((5, d), np.float32)
    x[1, 7] = 3.0
    x[2] = np.linspace(-1e3, 1e3, d, dtype=np.float32)
    x[3] = np.where(np.arange(d) % 2 == 0, 1.0, -1.0).astype(np.float32)
    x[3, :8] = np.float32(0.5)
    x[4] = np.float32(2.0) ** np.arange(-20, -20 + d).clip(-30, 30).astype(np.float32)
    w = np.ones(d, np.float32)
    packed = synth.ternary_codes(5, 9, V, d, raw=True)
    ref, ks, rxq, rinv = ternary.ref_logits(x, w, w, packed, 16.0, want_prep=True)
    if ks != "avx2":
        pytest.skip("this host runs the reference's scalar kernels")
    xq, inv = ternary.prep(x, w, w, 16.0)
    assert np.array_equal(xq, rxq)
    assert np.array_equal(inv.view(np.uint32), rinv.view(np.uint32))
    got = ternary.logits(xq, inv, packed)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_prep_rejects_ragged_width():
    with pytest.raises(ValueError):
        ternary.prep(np.zeros((1, 48), np.float32), None, np.ones(48, np.float32), 1.0)
