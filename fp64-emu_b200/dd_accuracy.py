"""Accuracy of a float64 product against a double-double one (measurement
tooling, not on the product path).  Standalone: it imports torch only, never
the fp64_emu package, so measuring another implementation's product with it
loads none of this repository's libraries.

dd_product(A, Bt) accumulates every inner product of A [R, K] and Bt [K, N]
in double-double: Dekker's two-product (Veltkamp splitting, no fused
multiply-add needed) and Knuth's two-sum per term, renormalised after every
term, so (hi, lo) carries about 106 significant bits.  It runs as elementwise
torch operations on whatever device A lives on, one K step at a time over the
whole [R, N] block.

correct_bits / element_bits are fp64-emu's own measures
(bench/accuracy.py:301-308): -log2(max|C - hi - lo| / max|hi|) over the
block, and -log2(|C - hi - lo| / |hi|) per element.
"""
import math

import torch

_SPLIT = float(2 ** 27 + 1)   # Veltkamp: 53-bit values into two 26-bit halves


def _split(a):
    c = _SPLIT * a
    h = c - (c - a)
    return h, a - h


@torch.no_grad()
def dd_product(A, Bt):
    """(hi, lo) of A [R, K] @ Bt [K, N] in double-double (float64 tensors on
    one device)."""
    if A.dim() != 2 or Bt.dim() != 2 or A.size(1) != Bt.size(0):
        raise ValueError("dd_product takes A [R, K] and Bt [K, N]")
    A = A.to(torch.float64)
    Bt = Bt.to(torch.float64)
    R, K = A.shape
    N = Bt.size(1)
    Ah, Al = _split(A)
    Bh, Bl = _split(Bt)
    hi = torch.zeros(R, N, dtype=torch.float64, device=A.device)
    lo = torch.zeros_like(hi)
    for k in range(K):
        a, ah, al = A[:, k:k + 1], Ah[:, k:k + 1], Al[:, k:k + 1]
        b, bh, bl = Bt[k:k + 1], Bh[k:k + 1], Bl[k:k + 1]
        p = a * b
        e = (((ah * bh - p) + ah * bl) + al * bh) + al * bl   # a*b = p + e exactly
        s = hi + p                                             # two-sum hi + p = s + es
        bb = s - hi
        es = (hi - (s - bb)) + (p - bb)
        lo = lo + (es + e)
        hi = s + lo                                            # renormalise (s, lo)
        bb = hi - s
        lo = (s - (hi - bb)) + (lo - bb)
    return hi, lo


def correct_bits(C, hi, lo):
    """-log2(max|C - hi - lo| / max|hi|); 53.0 when C equals hi + lo rounded."""
    err = float(((C - hi) - lo).abs().max())
    scale = float(hi.abs().max())
    if err == 0.0 or scale == 0.0:
        return 53.0
    return -math.log2(err / scale)


def element_bits(C, hi, lo, cap=60.0):
    """Per-element -log2(|C - hi - lo| / |hi|), capped at `cap` (exact or
    zero elements)."""
    rel = ((C - hi) - lo).abs() / hi.abs()
    b = -torch.log2(rel)
    b = torch.where(torch.isfinite(b), b, torch.full_like(b, cap))
    return torch.clamp(b, max=cap)


def summary(C, hi, lo):
    """Correct bits of C over the block and the per-element minimum / median."""
    eb = element_bits(C, hi, lo).flatten()
    return {"correct_bits": round(correct_bits(C, hi, lo), 2),
            "element_bits_min": round(float(eb.min()), 2),
            "element_bits_median": round(float(eb.median()), 2)}
