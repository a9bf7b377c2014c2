"""GPU: the fused lm_head + sampler's per-tile lists (no logits through HBM)
in every branch, through the C ABI, against the sampler oracle run on the
logits the same GEMM produces (bm_lmhead_logits / bm_ternary_logits).

  mixed knobs   greedy rows (argmax over the lists' heads), top_k rows of
                1, 40 and 200 (the top_k path on the lists), top_k = 0 rows
                (the GEMM stores their logits, the full sampler takes them)
  clustered     rows whose largest logits all lie in one 256-column tile, so
                the tile's list cannot hold the cut's buckets: the lists'
                exactness check sends them to a GEMM of their own and the full
                sampler
  ternary       the same through the reference's ternary lm_head (int8)

Parity rule of tests/parity.py.
"""
import numpy as np
import pytest

import parity
import synth

pytestmark = pytest.mark.gpu


def _knobs(rng, B):
    """Per-row knobs: every fourth row greedy, the rest top_k in
    {1, 40, 200, 0} with default-like temperature, penalty and nucleus."""
    temp = rng.uniform(0.5, 1.3, B).astype(np.float32)
    temp[::4] = 0.0
    top_k = np.array([1, 40, 200, 0], np.int32)[np.arange(B) % 4]
    top_p = rng.uniform(0.6, 1.0, B).astype(np.float32)
    min_p = rng.uniform(0.0, 0.1, B).astype(np.float32)
    penalty = rng.uniform(1.0, 1.4, B).astype(np.float32)
    return temp, penalty, min_p, top_p, top_k


def _hist(rng, B, V, H=256):
    hist = rng.integers(-5, V + 5, size=B * H).astype(np.int32)   # some out of range
    off = np.arange(0, H * (B + 1), H, dtype=np.int64)
    return hist, off


def _check_bf16(gpu_ctx, sampler_lib, oracle_lib, hidden, norm_w, W, knobs, hist, off, u):
    import torch
    dev = torch.device("cuda", 0)
    B, d = hidden.shape
    V = W.shape[0]
    kn = sampler_lib.knobs_array(*knobs)
    x = torch.from_numpy(hidden).to(dev)
    w = torch.from_numpy(norm_w).to(dev)
    Wd = torch.from_numpy(W.view(np.int16)).to(dev)
    hd, od = torch.from_numpy(hist).to(dev), torch.from_numpy(off).to(dev)
    knd = torch.from_numpy(kn.view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    ids = torch.full((B,), -7, dtype=torch.int32, device=dev)
    probs = torch.empty(B, dtype=torch.float32, device=dev)
    stats = torch.zeros((B, 4), dtype=torch.int32, device=dev)
    logits = torch.empty((B, V), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    gpu_ctx.lmhead_sample(x.data_ptr(), B, d, w.data_ptr(), Wd.data_ptr(), V, hd.data_ptr(),
                          od.data_ptr(), knd.data_ptr(), 1, ud.data_ptr(), ids.data_ptr(),
                          probs.data_ptr(), stats.data_ptr(), None)
    fallback = gpu_ctx.fused_fallback_rows()
    gpu_ctx.lmhead_logits(x.data_ptr(), B, d, w.data_ptr(), Wd.data_ptr(), V, logits.data_ptr(),
                          V, None)
    torch.cuda.synchronize()
    gpu_ctx.check()
    batch = synth.Batch(logits.cpu().numpy(), hist, off, *knobs)
    rids, rprobs, res = oracle_lib.sample_batch(batch, u, threads=8)
    rep = parity.compare(ids.cpu().numpy(), probs.cpu().numpy(), rids, rprobs, res)
    assert rep["bad"] == 0 and rep["prob_bad"] == 0, rep
    st = stats.cpu().numpy()
    assert np.array_equal(st[:, 0], res["path"])
    assert np.array_equal(st[:, 1], res["n_cand"])
    assert np.array_equal(st[:, 3], res["consumed"])
    return fallback


def _bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >>
            np.uint64(16)).astype(np.uint16)


def test_mixed_knobs(gpu_ctx, sampler_lib, oracle_lib):
    rng = np.random.default_rng(11)
    B, V, d = 256, 50257, 512
    hidden = rng.standard_normal((B, d), dtype=np.float32)
    norm_w = (1.0 + 0.02 * rng.standard_normal(d)).astype(np.float32)
    W = _bf16(0.05 * rng.standard_normal((V, d)).astype(np.float32))
    hist, off = _hist(rng, B, V)
    u = rng.random(B, dtype=np.float32)
    knobs = _knobs(rng, B)
    n_sampled, n_computed = _check_bf16(gpu_ctx, sampler_lib, oracle_lib, hidden, norm_w, W,
                                        knobs, hist, off, u)
    full = int(((knobs[0] >= 0.05) & (knobs[4] == 0)).sum())
    assert n_sampled == full + n_computed      # full-path rows + undecided top_k rows
    # the lists decide nearly every top_k 1 / 40 row; a top_k of 200 can need
    # more of one 128-column list than its 4 entries
    assert n_computed <= int((knobs[4] == 200).sum()) + B // 32, (n_sampled, n_computed)


def test_clustered_tile_falls_back(gpu_ctx, sampler_lib, oracle_lib):
    """Columns 256..455 of W follow the hidden states' common direction, so
    about 200 of each row's largest logits share the second tile: a top_k of
    40 or 200 needs more of that tile than its list holds."""
    rng = np.random.default_rng(12)
    B, V, d = 128, 4099, 256
    base = rng.standard_normal(d).astype(np.float32)
    hidden = (base[None, :] + 0.3 * rng.standard_normal((B, d))).astype(np.float32)
    norm_w = np.ones(d, np.float32)
    Wf = 0.05 * rng.standard_normal((V, d)).astype(np.float32)
    Wf[256:456] += 0.2 * base[None, :] / np.sqrt(d)
    W = _bf16(Wf)
    hist, off = _hist(rng, B, V, H=64)
    temp = np.full(B, 0.7, np.float32)
    top_k = np.where(np.arange(B) % 2 == 0, 40, 200).astype(np.int32)
    knobs = (temp, np.full(B, 1.1, np.float32), np.zeros(B, np.float32),
             np.full(B, 0.95, np.float32), top_k)
    u = rng.random(B, dtype=np.float32)
    n_sampled, n_computed = _check_bf16(gpu_ctx, sampler_lib, oracle_lib, hidden, norm_w, W,
                                        knobs, hist, off, u)
    assert n_computed == n_sampled and n_computed >= B // 2, (n_sampled, n_computed)


@pytest.mark.parametrize("clustered", [False, True])
def test_ternary_lists(gpu_ctx, sampler_lib, oracle_lib, clustered):
    import torch
    import ternary
    rng = np.random.default_rng(13)
    B, V, d = 192, 8197, 256
    b = synth.make_c6(14, B, V=V, d=d)
    packed = b.packed.copy()
    if clustered:
        # hidden states along a common direction, and columns 512..699 with
        # codes equal to its signs: their logits lead every row
        base = rng.standard_normal(d).astype(np.float32)
        b.hidden = (base[None, :] + 0.3 * rng.standard_normal((B, d))).astype(np.float32)
        codes = (np.sign(base) + 1).astype(np.uint8)         # -1/0/+1 -> 0/1/2
        row = (codes[0::4] | (codes[1::4] << 2) | (codes[2::4] << 4) | (codes[3::4] << 6))
        packed[512:700] = row.astype(np.uint8)[None, :]
    dev = torch.device("cuda", 0)
    x, nf, nl = (torch.from_numpy(a).to(dev) for a in (b.hidden, b.norm_f, b.lmh_norm))
    pk = torch.from_numpy(packed).to(dev)
    w8 = torch.empty((V, d), dtype=torch.int8, device=dev)
    gpu_ctx.ternary_unpack(pk.data_ptr(), V, d, w8.data_ptr())
    knobs = _knobs(rng, B)
    kn = sampler_lib.knobs_array(*knobs)
    hist, off = _hist(rng, B, V)
    u = rng.random(B, dtype=np.float32)
    hd, od = torch.from_numpy(hist).to(dev), torch.from_numpy(off).to(dev)
    knd = torch.from_numpy(kn.view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    probs = torch.empty(B, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    gpu_ctx.ternary_sample(x.data_ptr(), B, d, nf.data_ptr(), nl.data_ptr(), w8.data_ptr(),
                           float(b.w_scale), V, hd.data_ptr(), od.data_ptr(), knd.data_ptr(), 1,
                           ud.data_ptr(), ids.data_ptr(), probs.data_ptr())
    torch.cuda.synchronize()
    gpu_ctx.check()
    n_sampled, n_computed = gpu_ctx.fused_fallback_rows()
    full = int(((knobs[0] >= 0.05) & (knobs[4] == 0)).sum())
    assert n_sampled == full + n_computed
    if clustered:
        assert n_computed >= B // 4, (n_sampled, n_computed)   # the top_k 40 / 200 rows
    logits = ternary.logits_fast(*ternary.prep(b.hidden, b.norm_f, b.lmh_norm, b.w_scale), packed)
    rb = synth.Batch(logits, hist, off, *knobs)
    rids, rprobs, res = oracle_lib.sample_batch(rb, u, threads=8)
    rep = parity.compare(ids.cpu().numpy(), probs.cpu().numpy(), rids, rprobs, res)
    assert rep["bad"] == 0 and rep["prob_bad"] == 0, rep
