"""GPU: the CUDA sampler through the C ABI against the oracle / golden vectors.

Parity rule (tests/parity.py): ids identical except rows whose draw or nucleus
cut lies within 1e-5 of a CDF boundary; probabilities within 1e-5 relative.
"""
import json
import os

import numpy as np
import pytest

import cases
import parity
import synth

pytestmark = pytest.mark.gpu

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


def knobs_of(bm, b):
    return bm.knobs_array(b.temp, b.penalty, b.min_p, b.top_p, b.top_k)


def run_gpu(ctx, bm, b, u):
    return ctx.sample_host(b.logits, b.hist if b.hist.size else None,
                           b.hist_off if b.hist.size else None, knobs_of(bm, b), u)


def assert_parity(rep, label=""):
    assert rep["bad"] == 0, f"{label}: id mismatches outside the 1e-5 band: {rep}"
    assert rep["prob_bad"] == 0, f"{label}: probability mismatches: {rep}"


@pytest.mark.parametrize("name,rows", [("c1", 64), ("c2", 64), ("c3", 128), ("c4", 128)])
def test_configs_match_oracle(gpu_ctx, sampler_lib, oracle_lib, name, rows):
    b = synth.MAKERS[name](101, rows)
    u = synth.uniform(101, 999, rows).astype(np.float32)
    ids, probs, st = run_gpu(gpu_ctx, sampler_lib, b, u)
    rids, rprobs, res = oracle_lib.sample_batch(b, u, threads=8)
    assert_parity(parity.compare(ids, probs, rids, rprobs, res), name)
    assert np.array_equal(st["path"], res["path"])
    assert np.array_equal(st["n_cand"], res["n_cand"])
    assert np.array_equal(st["consumed"], res["consumed"])


@pytest.mark.parametrize("name", sorted(GOLDEN["cases"]))
def test_cases_match_reference_golden(gpu_ctx, sampler_lib, oracle_lib, name):
    allc = {n: (b, u) for n, b, u in cases.all_cases() + cases.config_cases(8)}
    b, u = allc[name]
    g = GOLDEN["cases"][name]
    ids, probs, st = run_gpu(gpu_ctx, sampler_lib, b, u)
    ref_probs = np.array(g["prob_bits"], np.uint32).view(np.float32)
    _, _, res = oracle_lib.sample_batch(b, u)
    assert_parity(parity.compare(ids, probs, np.array(g["ids"]), ref_probs, res), name)
    assert st["consumed"].tolist() == g["consumed"]


def test_full_size_c3_device_api(gpu_ctx, sampler_lib, oracle_lib):
    """B=4096, V=50257 (the benchmark workload) on device buffers; every
    16th row checked against the oracle, all rows for invariants."""
    import torch
    b = synth.make_c3(202, 256)
    B, V = 4096, synth.VOCAB
    dev = torch.device("cuda", 0)
    logits = torch.from_numpy(np.tile(b.logits, (16, 1))).to(dev)
    u = synth.uniform(202, 3, B).astype(np.float32)
    kn = torch.from_numpy(knobs_of(sampler_lib, b)[:1].view(np.uint8).copy()).to(dev)
    ud = torch.from_numpy(u).to(dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    stats = torch.empty((B, 4), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    gpu_ctx.sample_device(logits.data_ptr(), B, V, V, 0, 0, kn.data_ptr(), 0, ud.data_ptr(),
                          out.data_ptr(), prob.data_ptr(), stats.data_ptr(),
                          torch.cuda.current_stream().cuda_stream or None)
    torch.cuda.synchronize()
    gpu_ctx.check()
    ids = out.cpu().numpy()
    pr = prob.cpu().numpy()
    st = stats.cpu().numpy()
    assert ((ids >= 0) & (ids < V)).all()
    assert (st[:, 3] == 1).all() and (pr > 0).all()
    sel = np.arange(0, B, 16)
    sub = synth.Batch(logits.cpu().numpy()[sel], b.hist, np.zeros(len(sel) + 1, np.int64),
                      b.temp[:1].repeat(len(sel)), b.penalty[:1].repeat(len(sel)),
                      b.min_p[:1].repeat(len(sel)), b.top_p[:1].repeat(len(sel)),
                      b.top_k[:1].repeat(len(sel)))
    rids, rprobs, res = oracle_lib.sample_batch(sub, u[sel], threads=8)
    assert_parity(parity.compare(ids[sel], pr[sel], rids, rprobs, res), "c3 full size")


def test_pitch_and_misaligned_rows(gpu_ctx, sampler_lib, oracle_lib):
    """Row pitch ld > V and row bases at every 4-byte offset inside 16 bytes."""
    import torch
    b = synth.make_c4(303, 16, V=4099)
    u = synth.uniform(303, 1, 16).astype(np.float32)
    rids, rprobs, res = oracle_lib.sample_batch(b, u)
    dev = torch.device("cuda", 0)
    kn = torch.from_numpy(knobs_of(sampler_lib, b).view(np.uint8).copy()).to(dev)
    hist = torch.from_numpy(b.hist).to(dev)
    off = torch.from_numpy(b.hist_off).to(dev)
    ud = torch.from_numpy(u).to(dev)
    for ld in (4099, 4101, 4104):
        for shift in range(4):
            buf = torch.full((16 * ld + shift + 8,), float("nan"), device=dev)
            view = buf[shift:shift + 16 * ld].view(16, ld)
            view[:, :4099] = torch.from_numpy(b.logits).to(dev)
            out = torch.empty(16, dtype=torch.int32, device=dev)
            prob = torch.empty(16, dtype=torch.float32, device=dev)
            torch.cuda.synchronize()
            gpu_ctx.sample_device(view.data_ptr(), 16, 4099, ld, hist.data_ptr(), off.data_ptr(),
                                  kn.data_ptr(), 1, ud.data_ptr(), out.data_ptr(),
                                  prob.data_ptr(), None, None)
            gpu_ctx.check()
            rep = parity.compare(out.cpu().numpy(), prob.cpu().numpy(), rids, rprobs, res)
            assert_parity(rep, f"ld={ld} shift={shift}")


def test_knob_broadcast_equals_per_row(gpu_ctx, sampler_lib):
    b = synth.make_c1(404, 8, V=4099, H=100)
    u = synth.uniform(404, 1, 8).astype(np.float32)
    k = knobs_of(sampler_lib, b)
    a = gpu_ctx.sample_host(b.logits, b.hist, b.hist_off, k[:1], u)
    c = gpu_ctx.sample_host(b.logits, b.hist, b.hist_off, k, u)
    assert np.array_equal(a[0], c[0])


def test_repeatable(gpu_ctx, sampler_lib):
    b = synth.make_c3(505, 32)
    u = synth.uniform(505, 1, 32).astype(np.float32)
    a = run_gpu(gpu_ctx, sampler_lib, b, u)
    c = run_gpu(gpu_ctx, sampler_lib, b, u)
    assert np.array_equal(a[0], c[0]) and np.array_equal(a[1].view(np.uint32), c[1].view(np.uint32))


def test_reference_convention_rng_stream(sampler_lib, oracle_lib):
    """bm_sample_rows / bm_sample_row draw from the global RNG in row order,
    only for rows that draw (greedy and argmax-guard rows do not), exactly as
    repeated model_forward_step calls would (src/main.c:473-500)."""
    b = synth.make_c4(606, 24, V=4099, Hmax=300)
    b.logits[5, :] = np.nan          # fallback/top_k argmax guard: no draw
    b.temp[5] = 1.0
    b.logits[9, :] = -np.inf
    b.temp[9] = 0.7
    b.top_k[9] = 0
    L = sampler_lib.lib()
    seed = 4242
    # expected: walk rows in order, handing out the stream to consumers
    _, _, r0 = oracle_lib.sample_batch(b, np.zeros(b.B, np.float32))
    draws = r0["consumed"].astype(bool)
    stream = synth.rng_uniforms(seed, int(draws.sum()) + 1)
    u = np.zeros(b.B, np.float32)
    u[draws] = stream[:draws.sum()]
    rids, _, _ = oracle_lib.sample_batch(b, u)
    L.bm_rng_seed(seed)
    ids = sampler_lib.sample_rows(b.logits, b.hist, b.hist_off, knobs_of(sampler_lib, b))
    assert np.array_equal(ids, rids)
    assert np.float32(L.bm_rng_float()) == stream[draws.sum()]
    # single-row calls continue the same stream
    L.bm_rng_seed(seed)
    one = [sampler_lib.sample_row(b.logits[r], b.hist[b.hist_off[r]:b.hist_off[r + 1]],
                                  b.penalty[r], b.temp[r], b.min_p[r], b.top_p[r],
                                  b.top_k[r]) for r in range(b.B)]
    assert one == rids.tolist()


def test_invalid_arguments_rejected(gpu_ctx, sampler_lib):
    L = sampler_lib.lib()
    h = gpu_ctx.handle
    assert L.bm_sample_batch(h, None, 4, 10, 10, None, None, None, 0, None, None, None, None,
                             None) == -1
    big = gpu_ctx.max_vocab() + 1
    x = np.zeros(big, np.float32)
    k = sampler_lib.knobs_array(0.8, 1.0, 0.0, 1.0, 0)
    with pytest.raises(sampler_lib.BmError) as e:
        gpu_ctx.sample_host(x[None, :], None, None, k, np.zeros(1, np.float32))
    assert e.value.code == -4


def test_host_calls_small_and_large_match_device_call(gpu_ctx, sampler_lib):
    """bm_sample_batch_host packs calls of at most 16 MB into one pinned
    staging region (one copy each way) and stages larger ones buffer by
    buffer.  Both must return exactly what bm_sample_batch returns on device
    buffers: 1 and 60 rows (small), 90 rows (18 MB: large), then 1 and 3
    rows again after the staging region grew, with per-row knobs and
    histories."""
    import torch
    dev = torch.device("cuda", 0)
    b = synth.make_c4(606, 90)
    u_all = synth.uniform(606, 7, 90).astype(np.float32)
    for n in (1, 60, 90, 1, 3):
        sub = b.rows(np.arange(n))
        u = u_all[:n]
        kn = knobs_of(sampler_lib, sub)
        ids, probs, st = gpu_ctx.sample_host(sub.logits, sub.hist, sub.hist_off, kn, u)
        lg = torch.from_numpy(sub.logits).to(dev)
        hist = torch.from_numpy(sub.hist if sub.hist.size else np.zeros(1, np.int32)).to(dev)
        off = torch.from_numpy(sub.hist_off).to(dev)
        knd = torch.from_numpy(kn.view(np.uint8).copy()).to(dev)
        ud = torch.from_numpy(u).to(dev)
        out = torch.empty(n, dtype=torch.int32, device=dev)
        prob = torch.empty(n, dtype=torch.float32, device=dev)
        std = torch.zeros(n * 4, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        gpu_ctx.sample_device(lg.data_ptr(), n, sub.V, sub.V, hist.data_ptr(), off.data_ptr(),
                              knd.data_ptr(), 1 if n > 1 else 0, ud.data_ptr(),
                              out.data_ptr(), prob.data_ptr(), std.data_ptr(), None)
        gpu_ctx.check()
        assert np.array_equal(ids, out.cpu().numpy()), f"n={n}: ids"
        assert np.array_equal(probs.view(np.uint32), prob.cpu().numpy().view(np.uint32)), \
            f"n={n}: probabilities"
        assert np.array_equal(st.view(np.int32).reshape(-1), std.cpu().numpy()), f"n={n}: stats"
