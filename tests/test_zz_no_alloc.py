"""GPU: bm_sample_batch_noalloc (no context, no allocation, scratch in a
file-scope device array) against bm_sample_batch on the same inputs, two calls
in a row (the second checks that the row schedule returned to zero).

Collected last (file name) and independent of the other tests' state.
"""
import ctypes

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu


def _dev_inputs(sampler_lib, b, u, per_row_knobs):
    import torch
    dev = torch.device("cuda", 0)
    k = sampler_lib.knobs_array(b.temp, b.penalty, b.min_p, b.top_p, b.top_k)
    if not per_row_knobs:
        k = k[:1]
    t = dict(
        logits=torch.from_numpy(b.logits).to(dev),
        knobs=torch.from_numpy(k.view(np.uint8).copy()).to(dev),
        u=torch.from_numpy(u).to(dev),
    )
    if b.hist.size:
        t["hist"] = torch.from_numpy(b.hist).to(dev)
        t["off"] = torch.from_numpy(b.hist_off).to(dev)
    return t


def _outs(B):
    import torch
    dev = torch.device("cuda", 0)
    return (torch.full((B,), -7, dtype=torch.int32, device=dev),
            torch.zeros(B, dtype=torch.float32, device=dev))


def _ptr(t, key):
    return ctypes.c_void_p(t[key].data_ptr()) if key in t else None


@pytest.mark.parametrize("name,rows,per_row", [("c3", 400, False), ("c4", 300, True)])
def test_noalloc_matches_context_path_twice(gpu_ctx, sampler_lib, name, rows, per_row):
    import torch
    torch.cuda.set_device(0)
    b = synth.MAKERS[name](909, rows)
    u = synth.uniform(909, 5, rows).astype(np.float32)
    t = _dev_inputs(sampler_lib, b, u, per_row)
    B, V = b.logits.shape
    stride = 1 if per_row else 0
    ref_id, ref_p = _outs(B)
    torch.cuda.synchronize()
    gpu_ctx.sample_device(t["logits"].data_ptr(), B, V, V,
                          t["hist"].data_ptr() if "hist" in t else 0,
                          t["off"].data_ptr() if "off" in t else 0,
                          t["knobs"].data_ptr(), stride, t["u"].data_ptr(),
                          ref_id.data_ptr(), ref_p.data_ptr(), None, None)
    torch.cuda.synchronize()
    gpu_ctx.check()
    L = sampler_lib.lib()
    for call in range(2):
        ids, probs = _outs(B)
        torch.cuda.synchronize()
        rc = L.bm_sample_batch_noalloc(ctypes.c_void_p(t["logits"].data_ptr()), B, V, V,
                                       _ptr(t, "hist"), _ptr(t, "off"),
                                       ctypes.c_void_p(t["knobs"].data_ptr()), stride,
                                       ctypes.c_void_p(t["u"].data_ptr()),
                                       ctypes.c_void_p(ids.data_ptr()),
                                       ctypes.c_void_p(probs.data_ptr()), None, None)
        assert rc == 0, L.bm_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_id), f"call {call}: ids differ"
        assert torch.equal(probs.view(torch.int32), ref_p.view(torch.int32)), f"call {call}"
        assert int(ids.min()) >= 0


def test_noalloc_rejects_oversized_inputs(gpu_ctx, sampler_lib):
    L = sampler_lib.lib()
    one = ctypes.c_void_p(256)  # never dereferenced: the checks fail first
    big_v = gpu_ctx.max_vocab() + 1
    rc = L.bm_sample_batch_noalloc(one, 1, big_v, big_v, None, None, one, 0, one, one, None,
                                   None, None)
    assert rc == -4 and b"exceeds" in L.bm_last_error()
    rc = L.bm_sample_batch_noalloc(one, (1 << 30) + 1, 8, 8, None, None, one, 0, one, one,
                                   None, None, None)
    assert rc == -1 and b"rows per call" in L.bm_last_error()
