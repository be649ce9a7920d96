"""CPU restatement of the reference's top-k + temperature sampler -- TEST INFRASTRUCTURE ONLY.

Only tests/ (and nothing in the product path) import this module.  It restates, in numpy float32 scalar
arithmetic (every operation rounded on its own, no fused multiply-add), the sampler of batteryphil/VAULT:

  v3_sample_topk   runtime/vault3.c:3204-3230 (declared runtime/vault3.h:221)
  v3_expf          runtime/vault3.c:104-114 (the reference's own exponential)
  v3_argmax        runtime/vault3.c:3198-3202 (greedy: the first maximum)

It is pinned against the reference itself: tests/test_oracle_sample.py calls v3_sample_topk from
oracle/_ref/libvault3.so (built from the reference sources by oracle/Makefile) on the same logits and states.
"""
from __future__ import annotations

import struct

import numpy as np

F = np.float32
GOLDEN = 0x9E3779B97F4A7C15
MASK64 = (1 << 64) - 1


def _u2f(u: int) -> np.float32:
    return F(struct.unpack("<f", struct.pack("<I", u & 0xFFFFFFFF))[0])


def v3_expf(x) -> np.float32:
    """runtime/vault3.c:104-114: k = round(x / ln 2) (half away from zero), two-part ln 2 reduction, degree-7
    polynomial, scale by 2^k (with the subnormal and overflow branches)."""
    x = F(x)
    if x > F(88.72):
        return F(np.inf)
    if x < F(-103.9):
        return F(0.0)
    kf = F(x * F(1.44269504088896341))
    k = int(F(kf + (F(0.5) if kf >= F(0.0) else F(-0.5))))   # C (int): truncation toward zero
    fk = F(k)
    r = F(F(x - F(fk * F(0.693145751953125))) - F(fk * F(1.428606765330187e-06)))
    p = F(F(1.3888889e-3) + F(r * F(1.9841270e-4)))
    for c in (8.3333338e-3, 4.1666668e-2, 1.6666667e-1, 0.5, 1.0, 1.0):
        p = F(F(c) + F(r * p))
    if k > 127:
        return F(F(p * _u2f(254 << 23)) * F(2.0))
    if k < -126:
        return F(F(p * _u2f((k + 126 + 127) << 23)) * _u2f(1 << 23))
    return F(p * _u2f((k + 127) << 23))


def argmax_first(logits: np.ndarray) -> int:
    """runtime/vault3.c:3198-3202 on finite logits (the first maximum); NaN entries are skipped."""
    v = np.asarray(logits, dtype=np.float32)
    ok = ~np.isnan(v)
    if not ok.any():
        return 0
    m = v[ok].max()
    return int(np.flatnonzero(ok & (v == m))[0])


def sample_topk(logits: np.ndarray, k: int, temp: float, rng: int):
    """v3_sample_topk (runtime/vault3.c:3204-3230) on one row of finite logits: returns (token, new rng state).
    The reference's insertion list keeps the k largest values in descending order with equal values in index
    order (a later equal value is placed after, and replaces nothing); that is a stable sort by value."""
    v = np.asarray(logits, dtype=np.float32)
    temp = F(temp)
    if temp <= F(0.0) or k <= 1:
        return argmax_first(v), rng
    k = min(int(k), 64)
    idx_all = np.flatnonzero(~np.isnan(v))
    order = idx_all[np.argsort(-v[idx_all].astype(np.float64), kind="stable")][:k]
    if len(order) == 0:
        return 0, rng
    val = v[order]
    p = []
    s = F(0.0)
    for j in range(len(order)):
        pj = v3_expf(F(F(val[j] - val[0]) / temp))
        p.append(pj)
        s = F(s + pj)
    x = rng if rng else GOLDEN
    x ^= (x << 13) & MASK64
    x ^= x >> 7
    x ^= (x << 17) & MASK64
    r = F(F(F((x >> 40) & 0xFFFFFF) / F(16777216.0)) * s)
    for j in range(len(order)):
        r = F(r - p[j])
        if r <= F(0.0):
            return int(order[j]), x
    return int(order[-1]), x
