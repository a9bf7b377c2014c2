"""CPU: the C ABI library loads, exports its header, validates arguments and
keeps the reference RNG; no kernel is launched here."""
import ctypes

import numpy as np
import pytest

import synth


def test_library_exports_every_header_symbol(sampler_lib):
    L = sampler_lib.lib()
    syms = sampler_lib.header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(L, s), s


def test_abi_version(sampler_lib):
    assert sampler_lib.lib().bm_abi_version() == 1


def test_knobs_init_derived_fields(sampler_lib):
    k = sampler_lib.knobs_array([0.8, 1.0, 0.0], [1.15, 1.0, 1.0], [0.05, 0.0, 1.0],
                                [0.9, 0.95, 1.0], [40, 0, 3])
    assert k["inv_temp"][0] == np.float32(1.0) / np.float32(0.8)
    assert k["log_min_p"][0] == np.float32(np.log(np.float32(0.05)))
    assert k["log_min_p"][1] == 0.0 and k["log_min_p"][2] == 0.0
    assert np.isinf(k["inv_temp"][2])
    assert k["top_k"].tolist() == [40, 0, 3]


def test_rng_matches_reference_stream(sampler_lib):
    L = sampler_lib.lib()
    for seed in (0, 1, 42, 123456789):
        L.bm_rng_seed(seed)
        got = np.array([L.bm_rng_float() for _ in range(64)], np.float32)
        assert np.array_equal(got, synth.rng_uniforms(seed, 64))
    L.bm_rng_set_state(7)
    assert L.bm_rng_get_state() == 7


def test_null_context_is_rejected(sampler_lib):
    L = sampler_lib.lib()
    rc = L.bm_sample_batch(None, None, 1, 10, 10, None, None, None, 0, None, None, None,
                           None, None)
    assert rc == -1
    assert b"ctx" in L.bm_last_error()


def test_no_device_fails_loudly(sampler_lib):
    """Without a usable device the library refuses; there is no fallback."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    c = ctypes.c_void_p()
    assert sampler_lib.lib().bm_ctx_create(0, ctypes.byref(c)) == -5
    with pytest.raises(sampler_lib.BmError):
        sampler_lib.sample_row(np.zeros(10, np.float32), [], 1.0, 0.8, 0.0, 1.0, 0)
