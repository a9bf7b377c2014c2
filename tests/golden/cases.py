"""Edge-case catalogue for the sampler (test infrastructure).

Each case is a deterministic function returning (synth.Batch, uniforms).  The
cases cover what the reference's own sampling checks exercise only through a
model file (Makefile:279-299: the histogram top_k path with heap, sort and
CDF walk; the top_k=0 / top_p=1 id-order walk) plus the boundaries of every
branch in src/model.c:135-361 and the penalty block src/model.c:1268-1305.
"""
from __future__ import annotations

import numpy as np

import synth

V = synth.VOCAB


def _batch(rows, knobs, hists=None):
    rows = np.stack([np.asarray(r, np.float32) for r in rows])
    B = rows.shape[0]
    if hists is None:
        hists = [np.zeros(0, np.int32)] * B
    hist, off = synth._csr([np.asarray(h, np.int32) for h in hists])
    k = [dict(synth.DEFAULT_KNOBS, **kk) for kk in knobs]
    return synth.Batch(rows, hist, off,
                       [x["temp"] for x in k], [x["penalty"] for x in k],
                       [x["min_p"] for x in k], [x["top_p"] for x in k],
                       [x["top_k"] for x in k])


def _base(seed, n, scale=2.0, v=V):
    return [(scale * synth.normal(seed, 50 + i, v)).astype(np.float32) for i in range(n)]


def greedy_ties():
    """temp < 0.05: lowest id wins among exact maxima, after the penalty."""
    rows = _base(11, 6)
    rows[0][[10, 500, 40000]] = 50.0
    rows[1][[7, 8]] = 50.0
    rows[1][3] = np.float32(57.5)          # 57.5 / 1.15 = 50.0 after the penalty
    rows[2][:] = -2e9                      # nothing above -1e9: returns 0
    rows[3][:] = np.nan
    rows[3][777] = 1.0
    rows[4][[0, 1]] = [-0.0, 0.0]
    rows[4][2:] = -5.0
    rows[5][[100, 200]] = np.inf
    kn = [dict(temp=0.0)] * 6
    kn[2] = dict(temp=0.049)
    kn[5] = dict(temp=-1.0)
    hists = [[], [3, 3, 3], [], [], [], []]
    return _batch(rows, kn, hists), np.full(6, 0.5, np.float32)


def heap_ties():
    """top_k with many equal logits at the k-th place: the reference's heap
    layout decides membership and the CDF walk order."""
    rows = _base(12, 8, scale=1.0)
    for i, r in enumerate(rows):
        r[np.arange(0, V, 97)[:120]] = 6.0      # 120 equal candidates
        r[np.arange(5, V, 131)[:30]] = 7.0
        if i % 2:
            r[np.arange(9, V, 211)[:60]] = 6.5
    kn = [dict(top_k=40, top_p=1.0, min_p=0.0), dict(top_k=40, top_p=0.9, min_p=0.0),
          dict(top_k=100, top_p=1.0, min_p=0.0), dict(top_k=100, top_p=0.7, min_p=0.0),
          dict(top_k=1, top_p=1.0, min_p=0.0), dict(top_k=256, top_p=0.95, min_p=0.0),
          dict(top_k=150, top_p=1.0, min_p=0.0, temp=0.5),
          dict(top_k=7, top_p=0.5, min_p=0.0, temp=1.3)]
    u = np.array([0.1, 0.5, 0.33, 0.99, 0.5, 0.77, 0.012, 0.61], np.float32)
    return _batch(rows, kn), u


def masked_logits():
    """-1e9 masks (the x86 cvttss2si bucket quirk), -inf entries, min_p=0."""
    rows = _base(13, 6)
    for i, r in enumerate(rows):
        m = np.arange(i, V, 3)
        r[m] = -1e9 if i < 3 else -np.inf
    kn = [dict(top_k=40, min_p=0.0), dict(top_k=40, min_p=0.0, top_p=1.0),
          dict(top_k=0, min_p=0.0, top_p=0.9), dict(top_k=40, min_p=0.0),
          dict(top_k=0, min_p=0.0, top_p=1.0), dict(top_k=0, min_p=0.05, top_p=0.8)]
    return _batch(rows, kn), np.array([0.3, 0.7, 0.5, 0.2, 0.9, 0.4], np.float32)


def nonfinite():
    """+inf and NaN logits: NaN probabilities make the walk return the last
    candidate; all-NaN / all -inf rows take the argmax guards."""
    rows = _base(14, 8)
    rows[0][123] = np.inf
    rows[1][[5, 6000]] = np.inf
    rows[2][:] = np.nan
    rows[3][:] = -np.inf
    rows[4][::2] = np.nan
    rows[5][1000] = np.inf
    rows[6][:] = -3e30
    rows[7][[0, 10]] = [np.nan, 4.0]
    kn = [dict(top_k=40), dict(top_k=0, top_p=0.9, min_p=0.0), dict(top_k=40),
          dict(top_k=0, top_p=0.9), dict(top_k=0, top_p=1.0, min_p=0.0),
          dict(top_k=0, top_p=1.0, min_p=0.0), dict(top_k=0, top_p=0.9, min_p=0.0),
          dict(top_k=40, min_p=0.0)]
    return _batch(rows, kn), np.full(8, 0.25, np.float32)


def knob_boundaries():
    """Branch boundaries of sample_advanced and filter_and_sample."""
    rows = _base(15, 14, scale=3.0)
    kn = [dict(temp=0.05), dict(min_p=1.0), dict(min_p=2.0, top_k=0, top_p=0.5),
          dict(top_k=256), dict(top_k=257, top_p=0.9, min_p=0.0),
          dict(top_k=257, top_p=1.0, min_p=0.0), dict(top_k=5000, top_p=1.0, min_p=0.0),
          dict(top_k=-3, top_p=1.0, min_p=0.0), dict(top_p=0.0),
          dict(top_p=1.0, top_k=0, min_p=0.1), dict(temp=float("nan")),
          dict(temp=float("inf"), top_k=0, top_p=0.9, min_p=0.0),
          dict(min_p=float("nan"), top_k=0, top_p=0.99), dict(top_p=float("nan"))]
    u = np.array([0.5, 0.9, 0.1, 0.999, 0.4, 0.6, 0.2, 0.8, 0.3, 0.7, 0.5, 0.45,
                  0.35, 0.65], np.float32)
    return _batch(rows, kn), u


def uniform_extremes():
    """u = 0 and u = 1.0 (rng_float can return exactly 1.0)."""
    rows = _base(16, 6, scale=2.0)
    kn = [dict(), dict(), dict(top_k=0, top_p=0.9, min_p=0.0),
          dict(top_k=0, top_p=0.9, min_p=0.0), dict(top_k=0, top_p=1.0, min_p=0.0),
          dict(top_k=0, top_p=1.0, min_p=0.0)]
    return _batch(rows, kn), np.array([0.0, 1.0, 0.0, 1.0, 0.0, 1.0], np.float32)


def penalty_history():
    """Out-of-range ids, protected ids, duplicates, penalty <= 0, penalty < 1."""
    rows = _base(17, 6, scale=2.5)
    for r in rows:
        r[[13, 198, 628, 50256, 77, 78]] = [9.0, 9.5, 9.2, 9.9, 9.7, -9.0]
    hist = [-5, 13, 198, 628, 50256, 77, 77, 77, 78, 99999, 50257, 3]
    kn = [dict(top_k=40, min_p=0.0), dict(penalty=0.0, top_k=40, min_p=0.0),
          dict(penalty=-1.5, top_k=40, min_p=0.0), dict(penalty=0.5, top_k=40, min_p=0.0),
          dict(penalty=1.0, top_k=40, min_p=0.0), dict(penalty=3.0, temp=0.0)]
    return _batch(rows, kn, [hist] * 6), np.full(6, 0.6, np.float32)


def flat_ties():
    """Full-vocabulary rows with heavy probability ties (quantised logits):
    the stable sort orders ties by id; top-256 heap order where it applies."""
    rows = []
    for i in range(6):
        z = synth.normal(18, 60 + i, V)
        q = np.round(z * (4 if i < 3 else 40)) / (4 if i < 3 else 40)
        rows.append(q.astype(np.float32))
    rows[2][:] = 0.0                    # every candidate tied
    rows[5][[11, 22, 33]] = 12.0        # tied spikes: the top-256 path with ties
    kn = [dict(top_k=0, top_p=0.9, min_p=0.0), dict(top_k=0, top_p=0.5, min_p=0.0),
          dict(top_k=0, top_p=0.95, min_p=0.0), dict(top_k=1000, top_p=0.95, min_p=0.0),
          dict(top_k=300, top_p=1.0, min_p=0.0), dict(top_k=0, top_p=0.9, min_p=0.0)]
    u = np.array([0.42, 0.77, 0.5, 0.31, 0.88, 0.5], np.float32)
    return _batch(rows, kn), u


def small_vocab():
    """Tiny and ragged vocabularies (row pitch not a multiple of 4)."""
    out = []
    for v in (1, 2, 3, 5, 7, 64, 257):
        rows = _base(19, 4, scale=1.5, v=v)
        kn = [dict(), dict(top_k=0, top_p=0.9, min_p=0.0), dict(temp=0.0),
              dict(top_k=0, top_p=1.0, min_p=0.0)]
        out.append((_batch(rows, kn), np.array([0.2, 0.7, 0.5, 0.9], np.float32)))
    return out


CASES = {
    "greedy_ties": greedy_ties,
    "heap_ties": heap_ties,
    "masked_logits": masked_logits,
    "nonfinite": nonfinite,
    "knob_boundaries": knob_boundaries,
    "uniform_extremes": uniform_extremes,
    "penalty_history": penalty_history,
    "flat_ties": flat_ties,
}


def all_cases():
    """[(name, Batch, uniforms)] for every case, small vocabularies included."""
    out = [(n, *f()) for n, f in CASES.items()]
    for i, (b, u) in enumerate(small_vocab()):
        out.append((f"small_vocab_{b.V}", b, u))
    return out


def config_cases(rows=8):
    """Small slices of the four benchmark configurations."""
    out = []
    for name in ("c1", "c2", "c3", "c4"):
        for seed in (1, 2):
            b = synth.MAKERS[name](seed, rows)
            out.append((f"{name}_s{seed}", b, synth.uniform(seed, 999, rows).astype(np.float32)))
    return out
