"""GPU: the sampling configurations at their stated sizes, through the C ABI,
against the oracle (the C restatement of the reference sampler, itself
checked against the compiled reference in tests/test_oracle.py).

  c1  10,000 rows (the configuration's 10,000 single-row steps, each with its
      own logits, history and uniform, sampled as batches: rows are
      independent) plus 2,000 greedy rows with planted exact ties
  c2  100 steps of B = 256 rows
  c3  the benchmark batch: B = 4,096 distinct rows
  c4  B = 1,024 rows with per-row knobs
  c5  one fused B = 8,192 batch (RMSNorm + bf16 lm_head + sampler), its ids
      checked against the oracle on the GPU's own logits

Inputs come from tests/fullsize.py (numpy PCG64, the configurations'
distributions).  Parity rule of tests/parity.py: ids identical except rows
whose draw or nucleus cut lies within 1e-5 of a CDF boundary; probabilities
within 1e-5 relative.
"""
import os

import numpy as np
import pytest

import fullsize
import parity

pytestmark = pytest.mark.gpu

THREADS = max(1, os.cpu_count() or 1)


def _check(ctx, bm, oracle_lib, b, u, label, stats=True):
    kn = bm.knobs_array(b.temp, b.penalty, b.min_p, b.top_p, b.top_k)
    ids, probs, st = ctx.sample_host(b.logits, b.hist if b.hist.size else None,
                                     b.hist_off if b.hist.size else None, kn, u)
    rids, rprobs, res = oracle_lib.sample_batch(b, u, threads=THREADS)
    rep = parity.compare(ids, probs, rids, rprobs, res)
    assert rep["bad"] == 0 and rep["prob_bad"] == 0, f"{label}: {rep}"
    if stats:
        assert np.array_equal(st["path"], res["path"]), label
        assert np.array_equal(st["n_cand"], res["n_cand"]), label
        assert np.array_equal(st["consumed"], res["consumed"]), label
    return rep


def _uniforms(seed, n):
    return np.random.default_rng(seed).random(n, dtype=np.float32)


def test_c1_ten_thousand_rows(gpu_ctx, sampler_lib, oracle_lib):
    exact = 0
    for k in range(10):
        b = fullsize.c1(1000 + k, 1000)
        rep = _check(gpu_ctx, sampler_lib, oracle_lib, b, _uniforms(2000 + k, 1000), f"c1/{k}")
        exact += rep["exact"]
    assert exact >= 9990


def test_c1_greedy_exact_ties(gpu_ctx, sampler_lib, oracle_lib):
    b, want = fullsize.greedy_ties(31, 2000)
    u = np.zeros(b.B, np.float32)
    kn = sampler_lib.knobs_array(b.temp, b.penalty, b.min_p, b.top_p, b.top_k)
    ids, _, st = gpu_ctx.sample_host(b.logits, b.hist, b.hist_off, kn, u)
    rids, _, res = oracle_lib.sample_batch(b, u, threads=THREADS)
    assert np.array_equal(ids, rids)
    assert np.array_equal(ids, want), "the lowest of the tied ids wins"
    assert (st["path"] == 1).all() and (st["consumed"] == 0).all()


def test_c2_hundred_steps(gpu_ctx, sampler_lib, oracle_lib):
    for k in range(10):   # 10 calls of 10 steps x 256 rows
        b = fullsize.c2(3000 + k, 2560)
        _check(gpu_ctx, sampler_lib, oracle_lib, b, _uniforms(4000 + k, 2560), f"c2/{k}")


def test_c3_all_distinct_rows(gpu_ctx, sampler_lib, oracle_lib):
    b = fullsize.c3(5000, 4096)
    rep = _check(gpu_ctx, sampler_lib, oracle_lib, b, _uniforms(5001, 4096), "c3")
    assert rep["exact"] + rep["exempt_mismatch"] == 4096


def test_c4_per_row_knobs(gpu_ctx, sampler_lib, oracle_lib):
    b = fullsize.c4(6000, 1024)
    _check(gpu_ctx, sampler_lib, oracle_lib, b, _uniforms(6001, 1024), "c4")


def test_c5_fused_batch_8192(gpu_ctx, sampler_lib, oracle_lib):
    """The fused call's ids against the oracle run on the logits the same GEMM
    produces (the bf16 projection has no reference counterpart)."""
    import torch
    import synth
    B, V, d = 8192, fullsize.V, 2048
    rng = np.random.default_rng(7000)
    dev = torch.device("cuda", 0)
    hidden = torch.from_numpy(rng.standard_normal((B, d), dtype=np.float32)).to(dev)
    norm_w = torch.from_numpy((1.0 + 0.02 * rng.standard_normal(d)).astype(np.float32)).to(dev)
    W = (0.02 * torch.randn(V, d, generator=torch.Generator(device=dev).manual_seed(7001),
                            device=dev)).to(torch.bfloat16).view(torch.int16).contiguous()
    hist_h = fullsize._zipf_ids(rng, 256 * B, V)
    off_h = np.arange(0, 256 * (B + 1), 256, dtype=np.int64)
    k = synth.DEFAULT_KNOBS
    kn = sampler_lib.knobs_array(k["temp"], k["penalty"], k["min_p"], k["top_p"], k["top_k"])
    u = _uniforms(7002, B)
    hist, off = torch.from_numpy(hist_h).to(dev), torch.from_numpy(off_h).to(dev)
    knd = torch.from_numpy(kn.view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    probs = torch.empty(B, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    gpu_ctx.lmhead_sample(hidden.data_ptr(), B, d, norm_w.data_ptr(), W.data_ptr(), V,
                          hist.data_ptr(), off.data_ptr(), knd.data_ptr(), 0, ud.data_ptr(),
                          ids.data_ptr(), probs.data_ptr(), None, None)
    logits = torch.empty((B, V), dtype=torch.float32, device=dev)
    gpu_ctx.lmhead_logits(hidden.data_ptr(), B, d, norm_w.data_ptr(), W.data_ptr(), V,
                          logits.data_ptr(), V, None)
    torch.cuda.synchronize()
    gpu_ctx.check()
    ids_h, probs_h = ids.cpu().numpy(), probs.cpu().numpy()
    bad = 0
    for s in range(0, B, 1024):
        n = min(1024, B - s)
        lb = logits[s:s + n].cpu().numpy()
        sub = synth.Batch(lb, hist_h[256 * s:256 * (s + n)], off_h[:n + 1],
                          np.full(n, k["temp"]), np.full(n, k["penalty"]),
                          np.full(n, k["min_p"]), np.full(n, k["top_p"]), np.full(n, k["top_k"]))
        rids, rprobs, res = oracle_lib.sample_batch(sub, u[s:s + n], threads=THREADS)
        rep = parity.compare(ids_h[s:s + n], probs_h[s:s + n], rids, rprobs, res)
        bad += rep["bad"] + rep["prob_bad"]
    assert bad == 0
