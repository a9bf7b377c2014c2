"""GPU: the final RMSNorm + bf16 lm_head (tcgen05 tensor cores) and the fused
lm_head + sampler call, through the C ABI.

The reference's lm_head is a ternary BitLinear (src/model.c:1239-1262), so the
bf16 projection has no reference counterpart: logits are checked against a
float64 product of the same bf16 operands (oracle/lmhead_oracle.py, whose
RMSNorm restates src/kernel.c:72-91), within 1e-4 absolute (fp32
accumulation over d terms of size ~0.02; typical error ~3e-6).  The fused
call is checked against the sampler oracle run on the GPU's own logits, with
the sampler parity rule (tests/parity.py).
"""
import numpy as np
import pytest

import lmhead_oracle as lo
import parity
import synth

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4


def _dev_inputs(b):
    import torch
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(b.hidden).to(dev)
    w = torch.from_numpy(b.norm_w).to(dev)
    W = torch.from_numpy(b.w_bits.view(np.int16)).to(dev)
    return x, w, W


def gpu_logits(ctx, b, V, ld):
    import torch
    x, w, W = _dev_inputs(b)
    B, d = b.hidden.shape
    out = torch.full((B, ld), float("nan"), dtype=torch.float32, device=x.device)
    ctx.lmhead_logits(x.data_ptr(), B, d, w.data_ptr(), W.data_ptr(), V, out.data_ptr(), ld,
                      torch.cuda.current_stream().cuda_stream or None)
    torch.cuda.synchronize()
    ctx.check()
    return out.cpu().numpy()


@pytest.mark.parametrize("B,V,d,pad", [(130, 1000, 2048, 3), (64, 50257, 256, 0),
                                       (1, 300, 64, 1), (257, 513, 512, 4)])
def test_logits_match_cpu_product(gpu_ctx, B, V, d, pad):
    """Tile edges in M (B not a multiple of 128) and N (V not a multiple of
    256), K from one stage to the full ring (d = 64 .. 2048), row pitch."""
    b = synth.make_c5(11, B, V=V, d=d)
    got = gpu_logits(gpu_ctx, b, V, V + pad)
    ref = lo.lmhead_logits(lo.rmsnorm_bf16(b.hidden, b.norm_w), b.w_bits)
    err = np.abs(got[:, :V].astype(np.float64) - ref)
    assert np.isfinite(got[:, :V]).all()
    assert err.max() <= LOGIT_TOL, f"max |gpu - cpu| = {err.max():.3g}"
    if pad:
        assert np.isnan(got[:, V:]).all(), "the GEMM wrote past V"


def test_fused_sampler_matches_oracle_on_gpu_logits(gpu_ctx, sampler_lib, oracle_lib):
    import torch
    B, V, d = 64, 50257, 256
    b = synth.make_c5(21, B, V=V, d=d)
    u = synth.uniform(21, 77, B).astype(np.float32)
    kn = sampler_lib.knobs_array(b.temp, b.penalty, b.min_p, b.top_p, b.top_k)
    x, w, W = _dev_inputs(b)
    dev = x.device
    hist = torch.from_numpy(b.hist).to(dev)
    off = torch.from_numpy(b.hist_off).to(dev)
    knd = torch.from_numpy(kn.view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    probs = torch.empty(B, dtype=torch.float32, device=dev)
    stats = torch.empty((B, 4), dtype=torch.int32, device=dev)
    gpu_ctx.lmhead_sample(x.data_ptr(), B, d, w.data_ptr(), W.data_ptr(), V, hist.data_ptr(),
                          off.data_ptr(), knd.data_ptr(), 1, ud.data_ptr(), ids.data_ptr(),
                          probs.data_ptr(), stats.data_ptr(),
                          torch.cuda.current_stream().cuda_stream or None)
    torch.cuda.synchronize()
    gpu_ctx.check()
    logits = gpu_logits(gpu_ctx, b, V, V)
    batch = synth.Batch(logits, b.hist, b.hist_off, b.temp, b.penalty, b.min_p, b.top_p,
                        b.top_k)
    rids, rprobs, res = oracle_lib.sample_batch(batch, u)
    rep = parity.compare(ids.cpu().numpy(), probs.cpu().numpy(), rids, rprobs, res)
    assert rep["bad"] == 0 and rep["prob_bad"] == 0, rep
    st = stats.cpu().numpy()
    assert np.array_equal(st[:, 0], res["path"])
    assert np.array_equal(st[:, 3], res["consumed"])


def test_lmhead_rejects_bad_arguments(gpu_ctx, sampler_lib):
    import torch
    dev = torch.device("cuda", 0)
    x = torch.zeros((4, 100), dtype=torch.float32, device=dev)   # d_model % 8 != 0
    w = torch.ones(100, dtype=torch.float32, device=dev)
    W = torch.zeros((10, 100), dtype=torch.int16, device=dev)
    out = torch.zeros((4, 10), dtype=torch.float32, device=dev)
    with pytest.raises(sampler_lib.BmError):
        gpu_ctx.lmhead_logits(x.data_ptr(), 4, 100, w.data_ptr(), W.data_ptr(), 10,
                              out.data_ptr(), 10)
    with pytest.raises(sampler_lib.BmError):   # ld < V
        gpu_ctx.lmhead_logits(x.data_ptr(), 4, 96, w.data_ptr(), W.data_ptr(), 10,
                              out.data_ptr(), 9)
