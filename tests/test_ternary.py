"""GPU: the reference's own logits producer, the final RMSNorm + ternary
BitLinear lm_head (src/model.c:1222-1262), on the tensor cores (int8
tcgen05, exact int32 accumulation), through the C ABI.

The logits are compared BIT FOR BIT with the C restatement
(oracle/ternary_oracle.c), which the CPU tests pin bit for bit against the
reference's compiled AVX2 kernels.  The fused call is checked against the
sampler oracle on the same logits with the sampler parity rule.
"""
import numpy as np
import pytest

import parity
import synth
import ternary

pytestmark = pytest.mark.gpu


def _dev(b):
    import torch
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(b.hidden).to(dev)
    nf = torch.from_numpy(b.norm_f).to(dev)
    nl = torch.from_numpy(b.lmh_norm).to(dev)
    pk = torch.from_numpy(b.packed).to(dev)
    return x, nf, nl, pk


def _unpacked(ctx, pk, V, d):
    import torch
    w8 = torch.empty((V, d), dtype=torch.int8, device=pk.device)
    ctx.ternary_unpack(pk.data_ptr(), V, d, w8.data_ptr(),
                       torch.cuda.current_stream().cuda_stream or None)
    return w8


def gpu_logits(ctx, b, ld, final_norm=True):
    import torch
    x, nf, nl, pk = _dev(b)
    B, d = b.hidden.shape
    V = b.packed.shape[0]
    w8 = _unpacked(ctx, pk, V, d)
    out = torch.full((B, ld), float("nan"), dtype=torch.float32, device=x.device)
    ctx.ternary_logits(x.data_ptr(), B, d, nf.data_ptr() if final_norm else None, nl.data_ptr(),
                       w8.data_ptr(), float(b.w_scale), V, out.data_ptr(), ld,
                       torch.cuda.current_stream().cuda_stream or None)
    torch.cuda.synchronize()
    ctx.check()
    return out.cpu().numpy()


def test_unpack_matches_oracle(gpu_ctx):
    import torch
    V, d = 777, 2048
    packed = synth.ternary_codes(3, 4, V, d, raw=True)       # every code, 3 included
    pk = torch.from_numpy(packed).cuda()
    w8 = _unpacked(gpu_ctx, pk, V, d)
    torch.cuda.synchronize()
    gpu_ctx.check()
    assert np.array_equal(w8.cpu().numpy(), ternary.unpack(packed, d))


@pytest.mark.parametrize("B,V,d,pad,final_norm,raw", [
    (130, 1000, 2048, 3, True, False), (64, 50257, 256, 0, True, False),
    (1, 300, 32, 1, False, True), (257, 513, 512, 4, True, True),
    (8, 50257, 2048, 0, True, False)])
def test_logits_bit_exact(gpu_ctx, B, V, d, pad, final_norm, raw):
    """Tile edges in M (B not a multiple of 128) and N (V not a multiple of
    256), K from one 128-byte stage (d = 32, zero-filled) to 16 stages, row
    pitch, with and without the final norm, every 2-bit code."""
    b = synth.make_c6(13 + d, B, V=V, d=d, raw=raw)
    got = gpu_logits(gpu_ctx, b, V + pad, final_norm)
    xq, inv = ternary.prep(b.hidden, b.norm_f if final_norm else None, b.lmh_norm, b.w_scale)
    ref = ternary.logits_fast(xq, inv, b.packed)
    g = np.ascontiguousarray(got[:, :V])
    bad = np.flatnonzero(g.view(np.uint32).ravel() != ref.view(np.uint32).ravel())
    assert bad.size == 0, (f"{bad.size} logits differ; first at {np.unravel_index(bad[0], g.shape)}:"
                           f" {g.ravel()[bad[0]]!r} vs {ref.ravel()[bad[0]]!r}")
    if pad:
        assert np.isnan(got[:, V:]).all(), "the GEMM wrote past V"


def test_fused_sampler_matches_oracle(gpu_ctx, sampler_lib, oracle_lib):
    import torch
    B, V, d = 96, 50257, 512
    b = synth.make_c6(23, B, V=V, d=d)
    u = synth.uniform(23, 77, B).astype(np.float32)
    kn = sampler_lib.knobs_array(b.temp, b.penalty, b.min_p, b.top_p, b.top_k)
    x, nf, nl, pk = _dev(b)
    dev = x.device
    w8 = _unpacked(gpu_ctx, pk, V, d)
    hist = torch.from_numpy(b.hist).to(dev)
    off = torch.from_numpy(b.hist_off).to(dev)
    knd = torch.from_numpy(kn.view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    probs = torch.empty(B, dtype=torch.float32, device=dev)
    stats = torch.empty((B, 4), dtype=torch.int32, device=dev)
    gpu_ctx.ternary_sample(x.data_ptr(), B, d, nf.data_ptr(), nl.data_ptr(), w8.data_ptr(),
                           float(b.w_scale), V, hist.data_ptr(), off.data_ptr(), knd.data_ptr(),
                           1, ud.data_ptr(), ids.data_ptr(), probs.data_ptr(), stats.data_ptr(),
                           torch.cuda.current_stream().cuda_stream or None)
    torch.cuda.synchronize()
    gpu_ctx.check()
    xq, inv = ternary.prep(b.hidden, b.norm_f, b.lmh_norm, b.w_scale)
    logits = ternary.logits_fast(xq, inv, b.packed)
    batch = synth.Batch(logits, b.hist, b.hist_off, b.temp, b.penalty, b.min_p, b.top_p,
                        b.top_k)
    rids, rprobs, res = oracle_lib.sample_batch(batch, u)
    rep = parity.compare(ids.cpu().numpy(), probs.cpu().numpy(), rids, rprobs, res)
    assert rep["bad"] == 0 and rep["prob_bad"] == 0, rep
    st = stats.cpu().numpy()
    assert np.array_equal(st[:, 0], res["path"])
    assert np.array_equal(st[:, 3], res["consumed"])


def test_ternary_rejects_bad_arguments(gpu_ctx, sampler_lib):
    import torch
    dev = torch.device("cuda", 0)
    x = torch.zeros((4, 48), dtype=torch.float32, device=dev)    # d_model % 32 != 0
    w = torch.ones(48, dtype=torch.float32, device=dev)
    W = torch.zeros((10, 48), dtype=torch.int8, device=dev)
    out = torch.zeros((4, 10), dtype=torch.float32, device=dev)
    with pytest.raises(sampler_lib.BmError):
        gpu_ctx.ternary_logits(x.data_ptr(), 4, 48, None, w.data_ptr(), W.data_ptr(), 1.0, 10,
                               out.data_ptr(), 10)
    x = torch.zeros((4, 64), dtype=torch.float32, device=dev)
    w = torch.ones(64, dtype=torch.float32, device=dev)
    W = torch.zeros((10, 64), dtype=torch.int8, device=dev)
    with pytest.raises(sampler_lib.BmError):                     # ld < V
        gpu_ctx.ternary_logits(x.data_ptr(), 4, 64, None, w.data_ptr(), W.data_ptr(), 1.0, 10,
                               out.data_ptr(), 9)
    pk = torch.zeros((10, 12), dtype=torch.uint8, device=dev)   # d_model 48
    with pytest.raises(sampler_lib.BmError):
        gpu_ctx.ternary_unpack(pk.data_ptr(), 10, 48, W.data_ptr())
