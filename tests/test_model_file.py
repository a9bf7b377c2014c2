"""The packed model file reader (bm_model_head_read / _load) against files in
the reference's format (tests/golden/bit2_writer.py restates the exporter's
layout) and against the reference's own loader compiled from its sources
(oracle/_ref: model_load, src/model.c:477-783): both accept the same files,
both reject the same malformed ones, and the GPU lm_head on the tensors this
reader loads gives the reference's logits bit for bit.
"""
import os
import struct

import numpy as np
import pytest

import bit2_writer as bw
import oracle
import synth

TMP = os.path.join(os.path.dirname(os.path.abspath(__file__)), ".tmp")


def _path(name):
    os.makedirs(TMP, exist_ok=True)
    return os.path.join(TMP, name)


def _ref_accepts(path):
    import ctypes
    L = oracle.ref_lib()
    f = L.bm_ref_model_lmhead
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_longlong, ctypes.c_void_p]
    return f(os.fsencode(path), None, 0, None, 0, None) > 0


def _ref_logits(path, x):
    import ctypes
    L = oracle.ref_lib()
    f = L.bm_ref_model_lmhead
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_longlong, ctypes.c_void_p]
    x = np.ascontiguousarray(x, np.float32)
    B, d = x.shape
    V = f(os.fsencode(path), None, 0, None, 0, None)
    out = np.empty((B, V), np.float32)
    dm = ctypes.c_int()
    assert f(os.fsencode(path), x.ctypes.data, B, out.ctypes.data, V, ctypes.byref(dm)) == V
    return out


def test_read_matches_written(sampler_lib):
    m = bw.Model(3, 300, 64, 2, 4)
    p = _path("ok.bin")
    m.write(p)
    h = sampler_lib.read_model_head(p)
    assert (h["vocab_size"], h["d_model"], h["n_layers"], h["n_heads"]) == (300, 64, 2, 4)
    assert np.float32(h["w_scale"]) == m.lm_scale
    assert np.array_equal(h["norm_f"], m.norm_f)
    assert np.array_equal(h["lm_head_norm"], m.lm_head_norm)
    assert np.array_equal(h["packed"], m.lm_codes)
    if oracle.has_ref():
        assert _ref_accepts(p)


def _malformed(m):
    """(label, write kwargs) of files the reference loader rejects."""
    V, d, L, H = m.vocab, m.d, m.L, m.H
    di = 2 * d
    bad_hdr = struct.pack("iiiii", 0x12345678, V, d, L, H)
    return [
        ("magic", dict(header=bad_hdr)),
        ("vocab 0", dict(header=struct.pack("iiiii", bw.MAGIC, 0, d, L, H))),
        ("n_layers 257", dict(header=struct.pack("iiiii", bw.MAGIC, V, d, 257, H))),
        ("truncated header", dict(truncate=12)),
        ("truncated lm_head", dict(truncate=-7)),
        ("lm_head rows", dict(replace={"lm_head.weight": bw.packed_tensor(
            m.lm_codes[:-1], V - 1, d, 16.0)})),
        ("lm_head float", dict(replace={"lm_head.weight": bw.float_tensor(
            np.zeros((V, d), np.float32))})),
        ("lm_head scale 0", dict(replace={"lm_head.weight": bw.packed_tensor(
            m.lm_codes, V, d, 0.0)})),
        ("lm_head scale nan", dict(replace={"lm_head.weight": bw.packed_tensor(
            m.lm_codes, V, d, float("nan"))})),
        ("norm_f packed", dict(replace={"norm_f.weight": bw.packed_tensor(
            np.zeros((1, d // 4), np.uint8), 1, d, 1.0)})),
        ("norm_f short", dict(replace={"norm_f.weight": bw.float_tensor(
            np.ones(d - 1, np.float32))})),
        ("ndim 5", dict(replace={"lm_head.norm.weight": struct.pack("iiiiiii", 0, 5, 1, 1, 1, 1, d)
                                 + np.ones(d, np.float32).tobytes()})),
        ("in_proj rows", dict(replace={"layers.0.in_proj.weight": bw.packed_tensor(
            np.zeros((2 * di + 3 * H - 1, d // 4), np.uint8), 2 * di + 3 * H - 1, d, 1.0)})),
        ("out_proj float", dict(replace={"layers.1.out_proj.weight": bw.float_tensor(
            np.zeros((d, di), np.float32))})),
        ("D short", dict(replace={"layers.0.D": bw.float_tensor(np.ones(di - 1, np.float32))})),
    ]


@pytest.mark.parametrize("idx", range(15))
def test_malformed_file_rejected(sampler_lib, idx):
    m = bw.Model(4, 200, 32, 2, 4)
    label, kw = _malformed(m)[idx]
    p = _path(f"bad{idx}.bin")
    if kw.get("truncate", 0) < 0:
        n = m.write(p)
        kw = dict(truncate=n + kw["truncate"])
    m.write(p, **kw)
    with pytest.raises(sampler_lib.BmError) as ei:
        sampler_lib.read_model_head(p)
    assert ei.value.code == -1, label
    if oracle.has_ref():
        assert not _ref_accepts(p), f"the reference loader accepts '{label}'"


def test_missing_file(sampler_lib):
    with pytest.raises(sampler_lib.BmError):
        sampler_lib.read_model_head(_path("does-not-exist.bin"))


@pytest.mark.gpu
def test_loaded_head_logits_match_reference(gpu_ctx, sampler_lib):
    """The reader's tensors on the device + the ternary lm_head give the
    reference's logits (its own loader and AVX2 kernels) bit for bit."""
    import torch
    if not oracle.has_ref():
        pytest.skip("reference harness not built")
    m = bw.Model(8, 3000, 256, 1, 8)
    p = _path("gpu.bin")
    m.write(p)
    head = sampler_lib.ModelHead(gpu_ctx, p)
    info = head.info
    B, d, V = 20, 256, 3000
    x = synth.normal(8, 9, B * d).astype(np.float32).reshape(B, d)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty((B, V), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    gpu_ctx.ternary_logits(xd.data_ptr(), B, d, info["d_norm_f"], info["d_lmh_norm"],
                           info["d_w8"], info["w_scale"], V, out.data_ptr(), V)
    torch.cuda.synchronize()
    gpu_ctx.check()
    ref = _ref_logits(p, x)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    head.close()
