"""Deterministic synthetic sampler inputs (test infrastructure).

Every value is built from a SplitMix64 counter hash and IEEE-exact float64
operations (+, -, *, /, sqrt, frexp, ldexp, floor), with log / exp / cos
evaluated by fixed series in that same arithmetic.  The output is therefore
bit-identical on any IEEE-754 host and any numpy version, which lets the
committed golden files store only seeds and expected outputs.

The five workloads mirror the sampler configurations the benchmark names:
  c1  B rows of N(0, 2.5^2) logits with 8 ids boosted by +8; 400-id uniform
      histories; reference default knobs (0.8, 1.15, 0.05, 0.9, 40)
  c2  3*Gumbel(0,1) logits; 1024-id Zipf(1.1) histories; default knobs
  c3  N(0,1) logits, 25% of rows with one +15 spike, 25% flat N(0, 0.1);
      top_k=0, top_p=0.95, min_p=0, temp=1, penalty=1, no history
  c4  N(0, 2^2) logits with per-row knobs (temp U[0,1.5] with 10% exactly
      0, top_k in {0,1,40,200}, top_p U[.5,1], min_p U[0,.2], penalty
      U[1,1.5]) and uniform histories of length U[0,2048]
  c5  the fused lm_head inputs: hidden states N(0,1) [B x d], RMSNorm
      weight 1 + N(0, 0.02), lm_head W [V x d] N(0, 0.02) as bf16, default
      knobs, 256-id Zipf(1.1) histories (make_c5; its logits come from the
      GEMM)
No public dataset is involved; these stand in for real decode logits.
"""
from __future__ import annotations

import numpy as np

LN2 = 0.6931471805599453
TWO_PI = 6.283185307179586
VOCAB = 50257
DEFAULT_KNOBS = dict(temp=0.8, penalty=1.15, min_p=0.05, top_p=0.90, top_k=40)

_U64 = np.uint64


def _mix(x: np.ndarray) -> np.ndarray:
    """SplitMix64 finaliser on a uint64 array (wrapping arithmetic)."""
    with np.errstate(over="ignore"):
        x = x + _U64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> _U64(30))) * _U64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> _U64(27))) * _U64(0x94D049BB133111EB)
        return x ^ (x >> _U64(31))


def hash_stream(seed: int, stream: int, n: int, offset: int = 0) -> np.ndarray:
    base = _mix(np.array([(seed * 0x632BE59BD9B4E019 + stream) & (2**64 - 1)],
                         dtype=np.uint64))[0]
    idx = np.arange(offset, offset + n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix(idx * _U64(0xD1B54A32D192ED03) + base)


def uniform(seed: int, stream: int, n: int, offset: int = 0) -> np.ndarray:
    """float64 uniforms strictly inside (0, 1)."""
    h = hash_stream(seed, stream, n, offset)
    return ((h >> _U64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def det_log(x: np.ndarray) -> np.ndarray:
    m, e = np.frexp(x)
    small = m < 0.7071067811865476
    m = np.where(small, m * 2.0, m)
    e = np.where(small, e - 1, e).astype(np.float64)
    s = (m - 1.0) / (m + 1.0)
    s2 = s * s
    acc = np.zeros_like(s)
    for k in range(23, 0, -2):
        acc = acc * s2 + 1.0 / k
    return e * LN2 + 2.0 * s * acc


def det_exp(y: np.ndarray) -> np.ndarray:
    n = np.floor(y / LN2 + 0.5)
    r = y - n * LN2
    acc = np.ones_like(r)
    for k in range(22, 0, -1):
        acc = acc * r / k + 1.0
    return np.ldexp(acc, n.astype(np.int64))


def det_cos(t: np.ndarray) -> np.ndarray:
    """cos for t in [0, 2*pi): cos(t) = -cos(t - pi)."""
    v = t - 3.141592653589793
    v2 = v * v
    acc = np.ones_like(v)
    for k in range(40, 0, -2):
        acc = 1.0 - acc * v2 / (k * (k - 1))
    return -acc


def normal(seed: int, stream: int, n: int) -> np.ndarray:
    u1 = uniform(seed, stream, n)
    u2 = uniform(seed, stream + 0x5151, n)
    return np.sqrt(-2.0 * det_log(u1)) * det_cos(TWO_PI * u2)


def gumbel(seed: int, stream: int, n: int) -> np.ndarray:
    return -det_log(-det_log(uniform(seed, stream, n)))


def ids_uniform(seed: int, stream: int, n: int, V: int) -> np.ndarray:
    return np.floor(uniform(seed, stream, n) * V).astype(np.int32)


_ZIPF_CACHE: dict = {}


def ids_zipf(seed: int, stream: int, n: int, V: int, s: float = 1.1) -> np.ndarray:
    """Ranks 1..V with P(k) ~ k^-s, returned as ids k-1."""
    key = (V, s)
    if key not in _ZIPF_CACHE:
        k = np.arange(1, V + 1, dtype=np.float64)
        w = det_exp(-s * det_log(k))
        _ZIPF_CACHE[key] = np.cumsum(w)
    cdf = _ZIPF_CACHE[key]
    t = uniform(seed, stream, n) * cdf[-1]
    return np.minimum(np.searchsorted(cdf, t, side="right"), V - 1).astype(np.int32)


class Batch:
    """One batch of sampler inputs in the layout the C ABI takes."""

    def __init__(self, logits, hist, hist_off, temp, penalty, min_p, top_p, top_k):
        self.logits = np.ascontiguousarray(logits, dtype=np.float32)
        self.hist = np.ascontiguousarray(hist, dtype=np.int32)
        self.hist_off = np.ascontiguousarray(hist_off, dtype=np.int64)
        self.temp = np.ascontiguousarray(temp, dtype=np.float32)
        self.penalty = np.ascontiguousarray(penalty, dtype=np.float32)
        self.min_p = np.ascontiguousarray(min_p, dtype=np.float32)
        self.top_p = np.ascontiguousarray(top_p, dtype=np.float32)
        self.top_k = np.ascontiguousarray(top_k, dtype=np.int32)

    @property
    def B(self):
        return self.logits.shape[0]

    @property
    def V(self):
        return self.logits.shape[1]

    def rows(self, sel):
        sel = np.asarray(sel)
        hs = [self.hist[self.hist_off[r]:self.hist_off[r + 1]] for r in sel]
        off = np.zeros(len(sel) + 1, dtype=np.int64)
        off[1:] = np.cumsum([len(h) for h in hs])
        hist = np.concatenate(hs) if hs else np.zeros(0, np.int32)
        return Batch(self.logits[sel], hist, off, self.temp[sel],
                     self.penalty[sel], self.min_p[sel], self.top_p[sel],
                     self.top_k[sel])


def _knobs(B, **kw):
    k = dict(DEFAULT_KNOBS)
    k.update(kw)
    return (np.full(B, k["temp"], np.float32), np.full(B, k["penalty"], np.float32),
            np.full(B, k["min_p"], np.float32), np.full(B, k["top_p"], np.float32),
            np.full(B, k["top_k"], np.int32))


def _csr(lists):
    off = np.zeros(len(lists) + 1, dtype=np.int64)
    off[1:] = np.cumsum([len(x) for x in lists])
    hist = np.concatenate(lists).astype(np.int32) if len(lists) and off[-1] else \
        np.zeros(0, np.int32)
    return hist, off


def make_c1(seed: int, B: int, V: int = VOCAB, H: int = 400) -> Batch:
    rows, hists = [], []
    for r in range(B):
        l = (2.5 * normal(seed, 1000 + r, V)).astype(np.float32)
        boost = ids_uniform(seed, 2000 + r, 8, V)
        l[boost] = (l[boost] + np.float32(8.0)).astype(np.float32)
        rows.append(l)
        hists.append(ids_uniform(seed, 3000 + r, H, V))
    hist, off = _csr(hists)
    return Batch(np.stack(rows), hist, off, *_knobs(B))


def make_c2(seed: int, B: int, V: int = VOCAB, H: int = 1024) -> Batch:
    rows, hists = [], []
    for r in range(B):
        rows.append((3.0 * gumbel(seed, 1000 + r, V)).astype(np.float32))
        hists.append(ids_zipf(seed, 3000 + r, H, V))
    hist, off = _csr(hists)
    return Batch(np.stack(rows), hist, off, *_knobs(B))


def make_c3(seed: int, B: int, V: int = VOCAB) -> Batch:
    rows = []
    for r in range(B):
        z = normal(seed, 1000 + r, V)
        kind = r % 4
        if kind == 1:
            l = (0.1 * z).astype(np.float32)
        else:
            l = z.astype(np.float32)
            if kind == 0:
                i = int(ids_uniform(seed, 2000 + r, 1, V)[0])
                l[i] = np.float32(l[i] + np.float32(15.0))
        rows.append(l)
    hist, off = _csr([np.zeros(0, np.int32)] * B)
    return Batch(np.stack(rows), hist, off,
                 *_knobs(B, temp=1.0, penalty=1.0, min_p=0.0, top_p=0.95, top_k=0))


def make_c4(seed: int, B: int, V: int = VOCAB, Hmax: int = 2048) -> Batch:
    rows, hists = [], []
    u = uniform(seed, 77, 6 * B).reshape(6, B)
    temp = (1.5 * u[0]).astype(np.float32)
    temp[u[1] < 0.1] = 0.0
    top_k = np.array([0, 1, 40, 200], np.int32)[np.floor(u[2] * 4).astype(int)]
    top_p = (0.5 + 0.5 * u[3]).astype(np.float32)
    min_p = (0.2 * u[4]).astype(np.float32)
    penalty = (1.0 + 0.5 * u[5]).astype(np.float32)
    hl = np.floor(uniform(seed, 78, B) * (Hmax + 1)).astype(int)
    for r in range(B):
        rows.append((2.0 * normal(seed, 1000 + r, V)).astype(np.float32))
        hists.append(ids_uniform(seed, 3000 + r, int(hl[r]), V))
    hist, off = _csr(hists)
    return Batch(np.stack(rows), hist, off, temp, penalty, min_p, top_p, top_k)


MAKERS = {"c1": make_c1, "c2": make_c2, "c3": make_c3, "c4": make_c4}


def rng_uniforms(seed: int, n: int) -> np.ndarray:
    """n successive rng_float() values of the reference XorShift64*
    (src/utils.c:117-140) after rng_seed(seed)."""
    s = seed if seed else 0x853C49E6748FEA9B
    out = np.empty(n, np.float32)
    m = 2**64 - 1
    for i in range(n):
        s ^= s >> 12
        s ^= (s << 25) & m
        s ^= s >> 27
        v = (s * 0x2545F4914F6CDD1D) & m
        out[i] = np.float32(float(v >> 11)) * np.float32(1.0 / 9007199254740992.0)
    return out


class LmBatch:
    """Inputs of the fused lm_head + sampler (config c5)."""

    def __init__(self, hidden, norm_w, w_bits, hist, hist_off, knobs):
        self.hidden, self.norm_w, self.w_bits = hidden, norm_w, w_bits
        self.hist, self.hist_off = hist, hist_off
        self.temp, self.penalty, self.min_p, self.top_p, self.top_k = knobs


def make_c5(seed: int, B: int, V: int = VOCAB, d: int = 2048, H: int = 256) -> LmBatch:
    """c5: hidden N(0,1), norm weight 1+N(0,.02), W N(0,.02) rounded to bf16
    (nearest even), default knobs, 256-id Zipf(1.1) histories."""
    hidden = normal(seed, 5001, B * d).astype(np.float32).reshape(B, d)
    norm_w = (1.0 + 0.02 * normal(seed, 5002, d)).astype(np.float32)
    w = (0.02 * normal(seed, 5003, V * d)).astype(np.float32)
    u = w.view(np.uint32).astype(np.uint64)
    w_bits = ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >>
              np.uint64(16)).astype(np.uint16).reshape(V, d)
    hist, off = _csr([ids_zipf(seed, 5100 + r, H, V) for r in range(B)])
    k = DEFAULT_KNOBS
    kn = (np.full(B, k["temp"], np.float32), np.full(B, k["penalty"], np.float32),
          np.full(B, k["min_p"], np.float32), np.full(B, k["top_p"], np.float32),
          np.full(B, k["top_k"], np.int32))
    return LmBatch(hidden, norm_w, w_bits, hist, off, kn)


def ternary_codes(seed: int, stream: int, V: int, d: int, raw: bool = False) -> np.ndarray:
    """2-bit packed ternary weights [V x d/4] from the counter hash: codes 0, 1,
    2 (-1, 0, +1) with probabilities 1/4, 1/2, 1/4 (a hash code 3 becomes 1,
    as the exporter never writes 3); raw=True keeps the 3s (decoded as +1)."""
    n = V * d // 4
    h = hash_stream(seed, stream, (n + 7) // 8)
    p = h.view(np.uint8)[:n].copy()
    if not raw:
        m = p & (p >> np.uint8(1)) & np.uint8(0x55)
        p = p & ~(m << np.uint8(1))
    return p.reshape(V, d // 4)


class TernaryBatch:
    """Inputs of the ternary lm_head + sampler (config c6)."""

    def __init__(self, hidden, norm_f, lmh_norm, packed, w_scale, hist, hist_off, knobs):
        self.hidden = np.ascontiguousarray(hidden, np.float32)
        self.norm_f = np.ascontiguousarray(norm_f, np.float32)
        self.lmh_norm = np.ascontiguousarray(lmh_norm, np.float32)
        self.packed = np.ascontiguousarray(packed, np.uint8)
        self.w_scale = np.float32(w_scale)
        self.hist = np.ascontiguousarray(hist, np.int32)
        self.hist_off = np.ascontiguousarray(hist_off, np.int64)
        self.temp, self.penalty, self.min_p, self.top_p, self.top_k = knobs


def make_c6(seed: int, B: int, V: int = VOCAB, d: int = 2048, H: int = 256,
            raw: bool = False) -> TernaryBatch:
    """c6: the reference's own logits producer: hidden N(0,1) (the last
    layer's output), final-norm and BitLinear-norm weights 1+N(0,.02), ternary
    W (2-bit packed, P(0) = 1/2), weight scale 16 (the exporter's 1 / mean|W|,
    scripts/export-bin.py:172-176, for which the logits have a standard
    deviation near 2 at d = 2048), default knobs, 256-id Zipf(1.1)
    histories."""
    hidden = normal(seed, 6001, B * d).astype(np.float32).reshape(B, d)
    norm_f = (1.0 + 0.02 * normal(seed, 6002, d)).astype(np.float32)
    lmh_norm = (1.0 + 0.02 * normal(seed, 6003, d)).astype(np.float32)
    packed = ternary_codes(seed, 6004, V, d, raw)
    hist, off = _csr([ids_zipf(seed, 6100 + r, H, V) for r in range(B)])
    k = DEFAULT_KNOBS
    kn = (np.full(B, k["temp"], np.float32), np.full(B, k["penalty"], np.float32),
          np.full(B, k["min_p"], np.float32), np.full(B, k["top_p"], np.float32),
          np.full(B, k["top_k"], np.int32))
    return TernaryBatch(hidden, norm_f, lmh_norm, packed, 16.0, hist, off, kn)
