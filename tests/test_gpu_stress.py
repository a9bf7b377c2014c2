"""GPU: the sorted full-vocabulary path's rare branches against the oracle.

Rows built to reach: the clamped bucket range (max - min > 40), window lists
beyond 512 entries (block sort) and beyond 2048 (exact passes over global
memory), the exact recount of candidates above the cut (little mass above
it), probability ties at the nucleus cut, min_p thresholds with scaled rows,
and larger batches of the c3 / c4 configurations.  Parity rule of
tests/parity.py.
"""
import numpy as np
import pytest

import parity
import synth

pytestmark = pytest.mark.gpu

V = synth.VOCAB


def _run(ctx, bm, oracle_lib, b, u, label):
    kn = bm.knobs_array(b.temp, b.penalty, b.min_p, b.top_p, b.top_k)
    ids, probs, st = ctx.sample_host(b.logits, b.hist if b.hist.size else None,
                                     b.hist_off if b.hist.size else None, kn, u)
    rids, rprobs, res = oracle_lib.sample_batch(b, u, threads=8)
    rep = parity.compare(ids, probs, rids, rprobs, res)
    assert rep["bad"] == 0 and rep["prob_bad"] == 0, f"{label}: {rep}"
    assert np.array_equal(st["path"], res["path"]), label
    assert np.array_equal(st["n_cand"], res["n_cand"]), label
    # the nucleus size can move by one where the cut lies within 1e-5 of
    # top_p (the parity rule's band; the bucket masses carry up to 4e-6)
    far = (res["cut_margin"] > parity.TOL)
    assert np.array_equal(st["n_final"][far], res["n_final"][far]), label
    return rep


def _batch(logits, temp=1.0, penalty=1.0, min_p=0.0, top_p=0.95, top_k=0):
    B = logits.shape[0]
    full = lambda x, t: np.full(B, x, t)
    return synth.Batch(logits, np.zeros(0, np.int32), np.zeros(B + 1, np.int64),
                       full(temp, np.float32), full(penalty, np.float32),
                       full(min_p, np.float32), full(top_p, np.float32), full(top_k, np.int32))


def test_clamped_range(gpu_ctx, sampler_lib, oracle_lib):
    """max - min beyond 40: the last bucket collects the far tail."""
    B = 16
    z = synth.normal(5, 1, B * V).reshape(B, V).astype(np.float32)
    z[:, 7] += 30.0
    z[:, 11] -= 30.0
    z[::2, 100:5000] -= 60.0
    b = _batch(z, top_p=0.999999)
    u = synth.uniform(5, 2, B).astype(np.float32)
    _run(gpu_ctx, sampler_lib, oracle_lib, b, u, "clamped")


def test_long_window_lists(gpu_ctx, sampler_lib, oracle_lib):
    """Thousands of logits in one bucket at the cut: lists past 512 (block
    sort) and past 2048 (exact passes over global memory)."""
    B = 12
    z = (0.1 * synth.normal(6, 1, B * V)).reshape(B, V).astype(np.float32)
    for r in range(B):
        n = 600 * (r + 1)
        z[r, :n] = np.float32(0.25)                      # one value, n copies
        z[r, n:n + 3000] = np.float32(0.25) + np.float32(1e-4) * (r % 3)
    b = _batch(z, top_p=0.5)
    u = synth.uniform(6, 2, B).astype(np.float32)
    _run(gpu_ctx, sampler_lib, oracle_lib, b, u, "long lists")


def test_cut_near_the_top(gpu_ctx, sampler_lib, oracle_lib):
    """Peaked rows: little mass above the cut, so the cut's position needs the
    exact count (the top-256 heap path decides on it)."""
    B = 32
    z = (3.0 * synth.normal(7, 1, B * V)).reshape(B, V).astype(np.float32)
    z[:, :50] += np.linspace(6.0, 2.0, 50, dtype=np.float32)
    b = _batch(z, temp=0.7, top_p=0.6)
    u = synth.uniform(7, 2, B).astype(np.float32)
    _run(gpu_ctx, sampler_lib, oracle_lib, b, u, "peaked")


def test_ties_at_the_cut(gpu_ctx, sampler_lib, oracle_lib):
    """Quantised logits: many exact probability ties around the nucleus cut
    and the draw (stable order by id decides)."""
    B = 32
    z = np.round(4.0 * synth.normal(8, 1, B * V)).reshape(B, V).astype(np.float32) / 4.0
    b = _batch(z, top_p=0.9)
    u = synth.uniform(8, 2, B).astype(np.float32)
    _run(gpu_ctx, sampler_lib, oracle_lib, b, u, "ties")


def test_min_p_scaled_rows(gpu_ctx, sampler_lib, oracle_lib):
    B = 32
    z = (2.0 * synth.normal(9, 1, B * V)).reshape(B, V).astype(np.float32)
    b = _batch(z, temp=1.3, min_p=0.02, top_p=0.97)
    u = synth.uniform(9, 2, B).astype(np.float32)
    _run(gpu_ctx, sampler_lib, oracle_lib, b, u, "min_p")


def test_few_min_p_candidates(gpu_ctx, sampler_lib, oracle_lib):
    """top_k 0 with a real min_p: about 10 to 200 candidates a row, so the
    rows of up to 64 finish on one warp and the others take the bucket path;
    rows with a tied maximum or quantised values leave the warp undecided."""
    B = 64
    z = (2.0 * synth.normal(10, 1, B * V)).reshape(B, V).astype(np.float32)
    r = np.arange(B)
    temp = np.where(r % 3 == 0, 0.5, np.where(r % 3 == 1, 0.7, 1.0)).astype(np.float32)
    min_p = np.where(r % 2 == 0, 0.05, 0.2).astype(np.float32)
    top_p = np.where(r % 5 == 0, 0.5, 0.9).astype(np.float32)
    for i in range(B):
        if i % 4 == 1:    # the maximum twice
            z[i, 1234] = z[i].max()
        elif i % 4 == 2:  # quantised values: ties among the candidates
            z[i] = np.round(4.0 * z[i]) / 4.0
    b = synth.Batch(z, np.zeros(0, np.int32), np.zeros(B + 1, np.int64), temp,
                    np.ones(B, np.float32), min_p, top_p, np.zeros(B, np.int32))
    u = synth.uniform(10, 2, B).astype(np.float32)
    _run(gpu_ctx, sampler_lib, oracle_lib, b, u, "few min_p candidates")


@pytest.mark.parametrize("name,rows", [("c3", 1024), ("c4", 1024)])
def test_large_batches(gpu_ctx, sampler_lib, oracle_lib, name, rows):
    b = synth.MAKERS[name](303, rows)
    u = synth.uniform(303, 9, rows).astype(np.float32)
    _run(gpu_ctx, sampler_lib, oracle_lib, b, u, name)


@pytest.mark.parametrize("variant", ["plain", "both_penalised", "other_penalised"])
def test_greedy_ties_in_the_ragged_head(gpu_ctx, sampler_lib, oracle_lib, variant):
    """Greedy rows whose maximum is shared by an id in the ragged head slot
    (ids 0-2 of a row whose base is not 16-byte aligned, consumed after the
    interior) and a later id: the lower id wins (src/model.c:144-154), with
    and without those ids penalised."""
    B = 16
    z = synth.normal(12, 1, B * V).reshape(B, V).astype(np.float32)
    hist = []
    for r in range(B):
        z[r, r % 3] = np.float32(9.0)
        z[r, 1000 + 37 * r] = np.float32(9.0)
        if variant == "both_penalised":
            hist.append(np.array([r % 3, 1000 + 37 * r, 5], np.int32))
        elif variant == "other_penalised":
            hist.append(np.array([7, 4000 + r], np.int32))
        else:
            hist.append(np.zeros(0, np.int32))
    off = np.zeros(B + 1, np.int64)
    off[1:] = np.cumsum([len(h) for h in hist])
    full = lambda x, t: np.full(B, x, t)
    b = synth.Batch(z, np.concatenate(hist), off, full(0.0, np.float32),
                    full(1.0 if variant == "plain" else 1.5, np.float32), full(0.0, np.float32),
                    full(0.9, np.float32), full(0, np.int32))
    u = synth.uniform(12, 2, B).astype(np.float32)
    rep = _run(gpu_ctx, sampler_lib, oracle_lib, b, u, "greedy ties " + variant)
    assert rep["exact"] == B
