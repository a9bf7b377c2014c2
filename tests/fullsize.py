"""Fast generators of the sampler configurations at their stated sizes (test
infrastructure).

numpy's PCG64 generator replaces the counter hash of tests/golden/synth.py
here: synth's inputs are bit-identical on every host (the golden files rely
on that) but cost milliseconds per row, while a full-size parity test needs
tens of thousands of rows.  These arrays are not stored anywhere: the CUDA
sampler and the oracle read the same arrays in the same process, so only
their distributions matter, and they follow the configurations:

  c1  N(0, 2.5^2) logits with 8 ids boosted by +8; 400-id uniform histories;
      the reference CLI's default knobs (0.8, 1.15, 0.05, 0.9, 40)
  c2  3 * Gumbel(0, 1) logits; 1024-id Zipf(1.1) histories; default knobs
  c3  N(0, 1) logits, 25% of rows with one +15 spike, 25% flat N(0, 0.1);
      top_k 0, top_p 0.95, min_p 0, temp 1, penalty 1, no history
  c4  N(0, 2^2) logits with per-row knobs (temp U[0, 1.5] with 10% exactly 0,
      top_k in {0, 1, 40, 200}, top_p U[.5, 1], min_p U[0, .2], penalty
      U[1, 1.5]) and uniform histories of length U[0, 2048]
  greedy_ties  c1 rows sampled greedily (temp 0) with three ids planted at
      one exact maximum after the penalty: one of them is in the history and
      penalised onto the value the other two hold, so the lowest of the three
      ids must win (src/model.c:144-154)
"""
from __future__ import annotations

import numpy as np

import synth

V = synth.VOCAB
_ZIPF = {}


def _zipf_ids(rng, n, V, s=1.1):
    key = (V, s)
    if key not in _ZIPF:
        k = np.arange(1, V + 1, dtype=np.float64)
        _ZIPF[key] = np.cumsum(k ** -s)
    cdf = _ZIPF[key]
    t = rng.random(n) * cdf[-1]
    return np.minimum(np.searchsorted(cdf, t, side="right"), V - 1).astype(np.int32)


def _csr(lists):
    off = np.zeros(len(lists) + 1, np.int64)
    off[1:] = np.cumsum([len(x) for x in lists])
    hist = np.concatenate(lists).astype(np.int32) if off[-1] else np.zeros(0, np.int32)
    return hist, off


def _defaults(B, **kw):
    k = dict(synth.DEFAULT_KNOBS)
    k.update(kw)
    return (np.full(B, k["temp"], np.float32), np.full(B, k["penalty"], np.float32),
            np.full(B, k["min_p"], np.float32), np.full(B, k["top_p"], np.float32),
            np.full(B, k["top_k"], np.int32))


def c1(seed: int, B: int, V: int = V, H: int = 400) -> synth.Batch:
    rng = np.random.default_rng(seed)
    l = (np.float32(2.5) * rng.standard_normal((B, V), dtype=np.float32))
    boost = rng.integers(0, V, size=(B, 8))
    rows = np.arange(B)[:, None]
    l[rows, boost] += np.float32(8.0)
    hist = rng.integers(0, V, size=B * H).astype(np.int32)
    off = np.arange(0, H * (B + 1), H, dtype=np.int64)
    return synth.Batch(l, hist, off, *_defaults(B))


def c2(seed: int, B: int, V: int = V, H: int = 1024) -> synth.Batch:
    rng = np.random.default_rng(seed)
    u = rng.random((B, V), dtype=np.float32)
    u = np.maximum(u, np.float32(1e-30))
    l = (np.float32(-3.0) * np.log(-np.log(u))).astype(np.float32)
    hist = _zipf_ids(rng, B * H, V)
    off = np.arange(0, H * (B + 1), H, dtype=np.int64)
    return synth.Batch(l, hist, off, *_defaults(B))


def c3(seed: int, B: int, V: int = V) -> synth.Batch:
    rng = np.random.default_rng(seed)
    l = rng.standard_normal((B, V), dtype=np.float32)
    kind = np.arange(B) % 4
    l[kind == 1] *= np.float32(0.1)
    sp = np.nonzero(kind == 0)[0]
    ids = rng.integers(0, V, size=sp.size)
    l[sp, ids] += np.float32(15.0)
    off = np.zeros(B + 1, np.int64)
    return synth.Batch(l, np.zeros(0, np.int32), off,
                       *_defaults(B, temp=1.0, penalty=1.0, min_p=0.0, top_p=0.95, top_k=0))


def c4(seed: int, B: int, V: int = V, Hmax: int = 2048) -> synth.Batch:
    rng = np.random.default_rng(seed)
    l = (np.float32(2.0) * rng.standard_normal((B, V), dtype=np.float32))
    u = rng.random((6, B))
    temp = (1.5 * u[0]).astype(np.float32)
    temp[u[1] < 0.1] = 0.0
    top_k = np.array([0, 1, 40, 200], np.int32)[np.minimum((u[2] * 4).astype(int), 3)]
    top_p = (0.5 + 0.5 * u[3]).astype(np.float32)
    min_p = (0.2 * u[4]).astype(np.float32)
    penalty = (1.0 + 0.5 * u[5]).astype(np.float32)
    hl = rng.integers(0, Hmax + 1, size=B)
    hist, off = _csr([rng.integers(0, V, size=int(h)).astype(np.int32) for h in hl])
    return synth.Batch(l, hist, off, temp, penalty, min_p, top_p, top_k)


PROTECTED = (50256, 198, 628, 13)


def greedy_ties(seed: int, B: int, V: int = V, H: int = 400):
    """c1 rows, temp 0, with an exact three-way tie at the maximum after the
    penalty.  Returns (batch, expected ids: the lowest of the three)."""
    b = c1(seed, B, V, H)
    rng = np.random.default_rng(seed + 1)
    pen = np.float32(synth.DEFAULT_KNOBS["penalty"])
    want = np.empty(B, np.int32)
    for r in range(B):
        h = b.hist[b.hist_off[r]:b.hist_off[r + 1]]
        hs = set(int(x) for x in h)
        free = [i for i in rng.choice(V, 16, replace=False)
                if int(i) not in hs and int(i) not in PROTECTED]
        a, c = int(free[0]), int(free[1])
        pid = int(h[0])
        if pid in PROTECTED or pid in (a, c):
            pid = int(free[2])
            b.hist[b.hist_off[r]] = pid      # a history id that is penalised
        top = np.float32(b.logits[r].max()) + np.float32(2.0)
        raw = np.float32(top * pen)           # penalised: raw / pen (IEEE)
        tied = np.float32(raw / pen)
        b.logits[r, pid] = raw
        b.logits[r, a] = tied
        b.logits[r, c] = tied
        want[r] = min(a, c, pid)
    b.temp[:] = 0.0
    return b, want
