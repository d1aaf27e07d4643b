"""dd_accuracy (the double-double measure bench.py reports): the torch
form equals the numpy double-double of the test helpers bit for bit, is exact
on exactly representable sums, and the bit measures read as defined."""
import math
from fractions import Fraction

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from helpers import correct_bits as np_correct_bits, dd_matmul, make  # noqa: E402


@pytest.fixture(scope="module")
def acc():
    import dd_accuracy
    return dd_accuracy


@pytest.mark.parametrize("dist", ["randn", "wide16", "illcond40"])
def test_dd_product_matches_numpy_double_double(acc, dist):
    A, Bt = make(dist, 24, 300, 17, seed=3)
    hi, lo = acc.dd_product(torch.from_numpy(A), torch.from_numpy(Bt))
    h2, l2 = dd_matmul(A, Bt)
    assert np.array_equal(hi.numpy(), h2)
    assert np.array_equal(lo.numpy(), l2)


def test_dd_product_accurate_to_double_double(acc):
    rng = np.random.default_rng(7)
    A = rng.standard_normal((4, 200)) * np.exp2(rng.integers(-20, 21, (4, 200)))
    Bt = rng.standard_normal((200, 3)) * np.exp2(rng.integers(-20, 21, (200, 3)))
    hi, lo = acc.dd_product(torch.from_numpy(A), torch.from_numpy(Bt))
    for i in range(4):
        for j in range(3):
            exact = sum(Fraction(float(A[i, k])) * Fraction(float(Bt[k, j])) for k in range(200))
            got = Fraction(float(hi[i, j])) + Fraction(float(lo[i, j]))
            mag = sum(abs(Fraction(float(A[i, k])) * Fraction(float(Bt[k, j]))) for k in range(200))
            assert abs(got - exact) <= mag * Fraction(1, 2 ** 95)


def test_bit_measures(acc):
    A, Bt = make("randn", 16, 128, 16, seed=1)
    hi, lo = acc.dd_product(torch.from_numpy(A), torch.from_numpy(Bt))
    C = torch.from_numpy(A @ Bt)
    assert acc.correct_bits(C, hi, lo) == pytest.approx(np_correct_bits(C.numpy(), hi.numpy(), lo.numpy()))
    exact = hi + lo
    assert acc.correct_bits(exact, hi, lo) >= 52.0
    s = acc.summary(C, hi, lo)
    assert 40.0 < s["correct_bits"] <= 53.0
    assert s["element_bits_min"] <= s["element_bits_median"] <= 60.0
    # one element off by 2^-20 relative sets the block measure near 20 bits
    C2 = exact.clone()
    C2[0, 0] = C2[0, 0] * (1 + 2.0 ** -20)
    assert acc.correct_bits(C2, hi, lo) == pytest.approx(20 - math.log2(abs(float(exact[0, 0])) / float(exact.abs().max())), abs=0.05)


@pytest.mark.parametrize("kind", ["mm_nt", "mm", "bmm_nt", "bmm"])
def test_bench_accuracy_sample_layouts(kind):
    # bench.py's sample (first rows of the block / of batch member 0) for every
    # operand layout, on CPU tensors: float64 matmul reads about 50 bits
    import os
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    import bench
    g = torch.Generator().manual_seed(2)
    nt = kind.endswith("_nt")
    if kind.startswith("bmm"):
        A = torch.randn(3, 40, 64, dtype=torch.float64, generator=g)
        B = torch.randn((3, 64, 24) if nt else (3, 24, 64), dtype=torch.float64, generator=g)
        C = A @ (B if nt else B.transpose(1, 2))
    else:
        A = torch.randn(40, 64, dtype=torch.float64, generator=g)
        B = torch.randn((64, 24) if nt else (24, 64), dtype=torch.float64, generator=g)
        C = A @ (B if nt else B.t())
    name = "C5" if kind.startswith("bmm") else "C1"   # sample: the first 256 / 128 rows, all columns here
    r = bench.accuracy_sample(kind, A, B, C, name, 1, others={"again": lambda a, b: a @ b})
    assert r["sample"].startswith("C[")
    assert 45.0 < r["value"]["correct_bits"] <= 53.0
    assert r["again"]["correct_bits"] == pytest.approx(r["value"]["correct_bits"], abs=3.0)
