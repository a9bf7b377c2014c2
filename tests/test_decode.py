"""GPU: the device-resident decode loop state (bm_decode_*) over several
steps against the CPU restatement of the reference's generation loop
(oracle/decode_oracle.py: history_push, stop rules) with the sampler oracle
deciding each step's tokens from the same logits and the same histories.

Rows are planted to stop on EOS, on token 0, on a user stop token and at
max_tokens, with prompts shorter than, equal to and longer than the 256-id
window.  Where a draw lies within the parity rule's band of a CDF boundary
the two may pick neighbouring ids; the oracle then adopts the GPU's id so the
trajectories stay aligned, and the test counts such rows.
"""
import numpy as np
import pytest

import decode_oracle as do
import parity
import synth

pytestmark = pytest.mark.gpu

V = synth.VOCAB


def _step_logits(seed, step, B):
    z = (2.5 * synth.normal(seed, 100 + step, B * V)).astype(np.float32).reshape(B, V)
    return z


def _run(gpu_ctx, sampler_lib, oracle_lib, steps, B, prompts, plants, max_tokens, stop_ids,
         knobs_of, seed):
    import torch
    dev = torch.device("cuda", 0)
    dec = sampler_lib.Decode(gpu_ctx, B, max_tokens=max_tokens, stop_ids=stop_ids)
    dec.reset(prompts)
    ref = do.DecodeState(prompts, max_tokens, stop_ids)
    temp, pen, minp, topp, topk = knobs_of(B)
    kn = sampler_lib.knobs_array(temp, pen, minp, topp, topk)
    knd = torch.from_numpy(kn.view(np.uint8).copy()).to(dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    adopted = 0
    for s in range(steps):
        z = _step_logits(seed, s, B)
        for (r, st, tok) in plants:
            if st == s:
                z[r, tok] = np.float32(z[r].max() + 40.0)
        u = synth.uniform(seed, 500 + s, B).astype(np.float32)
        zd = torch.from_numpy(z).to(dev)
        ud = torch.from_numpy(u).to(dev)
        torch.cuda.synchronize()
        dec.step(zd.data_ptr(), V, V, knd.data_ptr(), 1, ud.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        hist, off = ref.hist_csr()
        b = synth.Batch(z, hist, off, temp, pen, minp, topp, topk)
        rids, rprobs, res = oracle_lib.sample_batch(b, u)
        act = np.array([st == do.ACTIVE for st in ref.status])
        rep = parity.compare(got[act], None, rids[act], None, res[act])
        assert rep["bad"] == 0, (s, rep)
        ids = np.where(act, got, rids)       # near-boundary rows follow the GPU
        adopted += int((got[act] != rids[act]).sum())
        want = ref.apply(ids)
        assert list(got) == want, s
    gpu_ctx.check()
    st = dec.read()
    cur, status, ngen, ring = st["current"], st["status"], st["n_generated"], st["ring"]
    assert list(cur) == ref.current
    assert list(status) == ref.status
    assert list(ngen) == ref.n_gen
    for r in range(B):
        window = sorted(t for t in ring[r] if t != -1)
        assert window == sorted(ref.history[r]), r
    assert dec.active() == sum(1 for st in ref.status if st == do.ACTIVE)
    dec.close()
    return ref, adopted


def _default_knobs(B):
    k = synth.DEFAULT_KNOBS
    return (np.full(B, k["temp"], np.float32), np.full(B, k["penalty"], np.float32),
            np.full(B, k["min_p"], np.float32), np.full(B, k["top_p"], np.float32),
            np.full(B, k["top_k"], np.int32))


def test_decode_steps_match_reference_loop(gpu_ctx, sampler_lib, oracle_lib):
    B, steps = 12, 12
    prompts = [synth.ids_uniform(9, 40 + r, n, V) for r, n in
               enumerate([1, 5, 256, 300, 0, 40, 255, 257, 3, 1000, 17, 64])]
    # (row, step, token): EOS, token 0, a user stop token
    plants = [(2, 3, 50256), (4, 5, 0), (5, 2, 777), (7, 0, 50256)]
    ref, adopted = _run(gpu_ctx, sampler_lib, oracle_lib, steps, B, prompts, plants,
                        max_tokens=10, stop_ids=[777, 888], knobs_of=_default_knobs, seed=31)
    assert ref.status[2] == do.STOP_EOS and ref.status[4] == do.STOP_EOS
    assert ref.status[5] == do.STOP_TOKEN and ref.status[7] == do.STOP_EOS
    assert ref.status[0] == do.STOP_MAX and ref.n_gen[0] == 10
    assert adopted <= 2


def test_decode_penalty_window_full_vocab(gpu_ctx, sampler_lib, oracle_lib):
    """Sorted full-vocabulary knobs with a strong penalty: the window decides
    the penalised ids every step."""
    B, steps = 8, 6
    prompts = [synth.ids_uniform(11, 60 + r, 300, V) for r in range(B)]

    def knobs(B):
        return (np.full(B, 1.0, np.float32), np.full(B, 1.5, np.float32),
                np.full(B, 0.0, np.float32), np.full(B, 0.95, np.float32),
                np.full(B, 0, np.int32))

    _run(gpu_ctx, sampler_lib, oracle_lib, steps, B, prompts, [], max_tokens=0, stop_ids=[],
         knobs_of=knobs, seed=37)


def test_decode_rejects_bad_arguments(gpu_ctx, sampler_lib):
    with pytest.raises(sampler_lib.BmError):
        sampler_lib.Decode(gpu_ctx, 0)
    with pytest.raises(sampler_lib.BmError):
        sampler_lib.Decode(gpu_ctx, 4, max_tokens=-1)


def test_decode_ternary_steps(gpu_ctx, sampler_lib, oracle_lib):
    """bm_decode_ternary_step: the reference's lm_head + sampler + loop state;
    the hidden state is held fixed, so only the growing windows (penalties)
    change the logits the sampler sees from step to step."""
    import torch
    import ternary
    B, d, steps = 8, 256, 5
    b = synth.make_c6(51, B, V=V, d=d)
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(b.hidden).to(dev)
    nf = torch.from_numpy(b.norm_f).to(dev)
    nl = torch.from_numpy(b.lmh_norm).to(dev)
    pk = torch.from_numpy(b.packed).to(dev)
    w8 = torch.empty((V, d), dtype=torch.int8, device=dev)
    gpu_ctx.ternary_unpack(pk.data_ptr(), V, d, w8.data_ptr())
    logits = ternary.logits_fast(*ternary.prep(b.hidden, b.norm_f, b.lmh_norm, b.w_scale),
                                 b.packed)
    prompts = [synth.ids_uniform(5, 70 + r, 30 + 20 * r, V) for r in range(B)]
    dec = sampler_lib.Decode(gpu_ctx, B)
    dec.reset(prompts)
    ref = do.DecodeState(prompts)
    temp, pen, minp, topp, topk = _default_knobs(B)
    pen[:] = 2.0                                  # a strong penalty: the window matters
    kn = sampler_lib.knobs_array(temp, pen, minp, topp, topk)
    knd = torch.from_numpy(kn.view(np.uint8).copy()).to(dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    for s in range(steps):
        u = synth.uniform(53, s, B).astype(np.float32)
        ud = torch.from_numpy(u).to(dev)
        torch.cuda.synchronize()
        dec.ternary_step(x.data_ptr(), d, nf.data_ptr(), nl.data_ptr(), w8.data_ptr(),
                         float(b.w_scale), V, knd.data_ptr(), 1, ud.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        hist, off = ref.hist_csr()
        bb = synth.Batch(logits, hist, off, temp, pen, minp, topp, topk)
        rids, _, res = oracle_lib.sample_batch(bb, u)
        rep = parity.compare(got, None, rids, None, res)
        assert rep["bad"] == 0, (s, rep)
        assert list(got) == ref.apply(got)
    gpu_ctx.check()
    st = dec.read()
    assert list(st["current"]) == ref.current
    assert list(st["n_generated"]) == ref.n_gen
    dec.close()
