"""Shared test helpers: seeded inputs, a double-double reference product and the
correct-bits measure.

Inputs follow the distributions of the reference's accuracy harness
(bench/accuracy.py:311-331 of CharlesCNorton/fp64-emu: randn, wide8/16,
illcond/illcond40, spike), generated here with numpy's seeded PCG64 so the
same arrays can be rebuilt on any machine.

The double-double product accumulates every inner product with the published
error-free transformations (Dekker's two-product with Veltkamp splitting,
Knuth's two-sum), ~106 bits, far below the errors being measured.
"""
import math
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "fp64-emu_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

DISTS = ["randn", "wide8", "wide16", "illcond", "illcond40", "spike"]


def make(dist, M, K, N, seed=0, nt=True):
    """A [M,K] and B ([K,N] if nt else [N,K]) float64 arrays."""
    g = np.random.default_rng(seed)
    A = g.standard_normal((M, K))
    Bt = g.standard_normal((K, N))
    if dist == "randn":
        pass
    elif dist in ("wide8", "wide16"):
        w = 8 if dist == "wide8" else 16
        A *= np.exp2(g.integers(-w, w + 1, A.shape).astype(np.float64))
        Bt *= np.exp2(g.integers(-w, w + 1, Bt.shape).astype(np.float64))
    elif dist in ("illcond", "illcond40"):
        span = 20 if dist == "illcond" else 40
        s = np.exp2(-span * g.random(K))
        A *= s[None, :]
        Bt *= s[:, None]
    elif dist == "spike":
        idx = g.integers(0, K, M)
        A[np.arange(M), idx] *= 2.0 ** 30
    elif dist == "int20":
        A = g.integers(-(1 << 20), (1 << 20) + 1, (M, K)).astype(np.float64)
        Bt = g.integers(-(1 << 20), (1 << 20) + 1, (K, N)).astype(np.float64)
    elif dist == "pm1":
        A = g.integers(-1, 2, (M, K)).astype(np.float64)
        Bt = g.integers(-1, 2, (K, N)).astype(np.float64)
    elif dist == "wide30":
        A *= np.exp2(g.integers(-30, 31, A.shape).astype(np.float64))
        Bt *= np.exp2(g.integers(-30, 31, Bt.shape).astype(np.float64))
    elif dist == "unif":
        A = g.uniform(-1.0, 1.0, (M, K))
        Bt = g.uniform(-1.0, 1.0, (K, N))
    else:
        raise ValueError(dist)
    return (A, Bt) if nt else (A, np.ascontiguousarray(Bt.T))


_SPLIT = float(2 ** 27 + 1)


def _two_prod(a, b):
    p = a * b
    ca, cb = _SPLIT * a, _SPLIT * b
    ah = ca - (ca - a)
    al = a - ah
    bh = cb - (cb - b)
    bl = b - bh
    e = (((ah * bh - p) + ah * bl) + al * bh) + al * bl
    return p, e


def _two_sum(a, b):
    s = a + b
    bb = s - a
    return s, (a - (s - bb)) + (b - bb)


def dd_matmul(A, Bt):
    """A [M,K] @ Bt [K,N] in double-double; returns (hi, lo)."""
    M, K = A.shape
    N = Bt.shape[1]
    hi = np.zeros((M, N))
    lo = np.zeros((M, N))
    with np.errstate(over="ignore", invalid="ignore"):
        for k in range(K):
            p, e = _two_prod(A[:, k:k + 1], Bt[k:k + 1, :])
            hi, s = _two_sum(hi, p)
            lo = lo + (s + e)
            hi, lo = _two_sum(hi, lo)
    return hi, lo


def correct_bits(C, hi, lo):
    """-log2(max|C - hi - lo| / max|hi|): the reference's max-norm measure
    (bench/accuracy.py:301-308); 53.0 for an exact match."""
    err = np.abs((C - hi) - lo).max()
    scale = np.abs(hi).max()
    if err == 0.0:
        return 53.0
    return -math.log2(err / scale)


def per_element_bits(C, hi, lo):
    """Per-element -log2(|C - hi - lo| / |hi|) (capped at 60), for min/median."""
    with np.errstate(divide="ignore", invalid="ignore"):
        rel = np.abs((C - hi) - lo) / np.abs(hi)
        b = -np.log2(rel)
    b[~np.isfinite(b)] = 60.0
    return np.minimum(b, 60.0)


def same_bits(x, y):
    """Bitwise equality of float64 arrays (NaN payloads included)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.ascontiguousarray(y, dtype=np.float64)
    return x.shape == y.shape and np.array_equal(x.view(np.int64), y.view(np.int64))
