"""CPU checks of the restatement oracle (oracle/f64e_oracle.c) against the
reference's own known-answer tests and accuracy thresholds
(tests/test_fp64_emu.py of CharlesCNorton/fp64-emu), run at the same shapes on
the host.  These pin the oracle before it is trusted as the GPU checker."""
import numpy as np
import pytest

from helpers import correct_bits, dd_matmul, make, per_element_bits


def _int_exact(A, B, nt):
    Ai = A.astype(np.int64)
    Bi = B.astype(np.int64)
    return (Ai @ (Bi if nt else Bi.T)).astype(np.float64)


def test_exact_mode_bitwise_integer_oracle(oracle_mod):
    # reference tests/test_fp64_emu.py:28-36
    g = np.random.default_rng(1)
    A = g.integers(-4096, 4097, (128, 256)).astype(np.float64)
    Bt = g.integers(-4096, 4097, (256, 96)).astype(np.float64)
    C = oracle_mod.emu(A, Bt, nprimes=20, exact=True, b_nt=True)
    assert np.array_equal(C, _int_exact(A, Bt, True))


def test_integer_products_fast_recombine(oracle_mod):
    # reference tests/test_fp64_emu.py:14-23 (>= 45 bits, nprimes=18, default exact)
    g = np.random.default_rng(0)
    A = g.integers(-1000, 1001, (128, 256)).astype(np.float64)
    Bt = g.integers(-1000, 1001, (256, 96)).astype(np.float64)
    ref = _int_exact(A, Bt, True)
    C = oracle_mod.emu(A, Bt, nprimes=18, b_nt=True)
    rel = np.abs(C - ref).max() / np.abs(ref).max()
    assert rel == 0 or -np.log2(rel) >= 45.0


def test_range_rule_adversarial_aligned(oracle_mod):
    # reference tests/test_fp64_emu.py:55-63: all ones, K = 2048 -> exactly K
    K = 2048
    C, d = oracle_mod.emu(np.ones((64, K)), np.ones((K, 48)), exact=True, b_nt=True, details=True)
    assert np.array_equal(C, np.full((64, 48), float(K)))
    assert d["bits_eff"] < 53   # the Cauchy-Schwarz rule narrowed the operands


def test_dyadic_dynamic_range_bitexact(oracle_mod):
    # reference tests/test_fp64_emu.py:66-83: integers under per-k scales 2^-12..2^0
    g = np.random.default_rng(5)
    M, K, N = 64, 512, 48
    ek = g.integers(-12, 1, K)
    Ai = g.integers(-256, 257, (M, K)).astype(np.int64)
    Bi = g.integers(-256, 257, (N, K)).astype(np.int64)
    A = (Ai << (ek + 12)).astype(np.float64) * 2.0 ** -12
    B = (Bi << (ek + 12)).astype(np.float64) * 2.0 ** -12
    w = (4 ** (ek + 12)).astype(np.int64)
    ref = ((Ai * w) @ Bi.T).astype(np.float64) * 2.0 ** -24
    assert np.array_equal(oracle_mod.emu(A, B), ref)


def test_bmm_integer_oracle_bitexact(oracle_mod):
    # reference tests/test_fp64_emu.py:97-104
    g = np.random.default_rng(6)
    A = g.integers(-4096, 4097, (5, 96, 256)).astype(np.float64)
    B = g.integers(-4096, 4097, (5, 64, 256)).astype(np.float64)
    ref = np.stack([_int_exact(A[b], B[b], False) for b in range(5)])
    assert np.array_equal(oracle_mod.emu(A, B), ref)


def test_bmm_single_batch_matches_mm(oracle_mod):
    # reference tests/test_fp64_emu.py:87-93
    g = np.random.default_rng(4)
    A = g.standard_normal((192, 384))
    B = g.standard_normal((160, 384))
    assert np.array_equal(oracle_mod.emu(A[None], B[None])[0], oracle_mod.emu(A, B))


def test_deep_k_integer_bitexact(oracle_mod):
    # reference tests/test_fp64_emu.py:122-131 (K past the single-launch bound)
    g = np.random.default_rng(16)
    K = 200_000
    A = g.integers(-1, 2, (48, K)).astype(np.float64)
    B = g.integers(-1, 2, (32, K)).astype(np.float64)
    assert np.array_equal(oracle_mod.emu(A, B), _int_exact(A, B, False))


@pytest.mark.parametrize("nprimes", [18, 20])
def test_random_fp64_accuracy(oracle_mod, nprimes):
    # reference tests/test_fp64_emu.py:41-50 (>= 45 bits vs native fp64)
    g = np.random.default_rng(2)
    A = g.standard_normal((256, 1024))
    Bt = g.standard_normal((1024, 128))
    ref = A @ Bt
    C = oracle_mod.emu(A, Bt, nprimes=nprimes, b_nt=True)
    rel = np.abs(C - ref).max() / np.abs(ref).max()
    assert -np.log2(rel) >= 45.0


def test_c3_integer_reduced_exact(oracle_mod):
    # C3-style integers U[-2^20, 2^20] at nprimes=13, corr=False stay exact (products < 2^52)
    A, B = make("int20", 64, 512, 48, seed=3, nt=False)
    ref = _int_exact(A, B, False)
    assert np.array_equal(oracle_mod.emu(A, B, nprimes=13, corr=False), ref)
    assert np.array_equal(oracle_mod.emu(A, B), ref)


@pytest.mark.parametrize("dist", ["randn", "wide16", "illcond40", "spike"])
def test_default_accuracy_vs_double_double(oracle_mod, dist):
    # README operating points: default plan reaches >= 52.6 correct bits
    # (reference README.md:200-213); native fp64 is the floor.
    A, Bt = make(dist, 64, 512, 64, seed=7)
    hi, lo = dd_matmul(A, Bt)
    C = oracle_mod.emu(A, Bt, b_nt=True)
    cb = correct_bits(C, hi, lo)
    nb = correct_bits(A @ Bt, hi, lo)
    assert cb >= 52.0 and cb >= nb, (cb, nb)
    pe = per_element_bits(C, hi, lo)
    assert np.median(pe) >= 52.0


def test_corr_improves_and_reduced_is_fp64_competitive(oracle_mod):
    A, Bt = make("randn", 64, 1024, 64, seed=11)
    hi, lo = dd_matmul(A, Bt)
    full = correct_bits(oracle_mod.emu(A, Bt, b_nt=True), hi, lo)
    reduced = correct_bits(oracle_mod.emu(A, Bt, nprimes=13, corr=False, b_nt=True), hi, lo)
    assert full > reduced >= 40.0


def test_exact_false_close_to_exact(oracle_mod):
    A, Bt = make("randn", 32, 300, 40, seed=12)
    hi, lo = dd_matmul(A, Bt)
    assert correct_bits(oracle_mod.emu(A, Bt, exact=False, b_nt=True), hi, lo) >= 50.0


def test_nt_equals_transposed_mm(oracle_mod):
    A, Bt = make("wide8", 40, 200, 30, seed=13)
    assert np.array_equal(oracle_mod.emu(A, Bt, b_nt=True), oracle_mod.emu(A, Bt.T.copy()))


def test_zero_and_empty_shapes(oracle_mod):
    A = np.zeros((5, 7))
    B = np.zeros((3, 7))
    assert np.array_equal(oracle_mod.emu(A, B), np.zeros((5, 3)))
    assert oracle_mod.emu(np.zeros((0, 7)), B).shape == (0, 3)
    assert np.array_equal(oracle_mod.emu(np.zeros((4, 0)), np.zeros((2, 0))), np.zeros((4, 2)))


def test_sizing_matches_reference_rules(oracle_mod):
    # shifts put each row max into [2^(bits-1), 2^bits) (fp64_emu.cu:136-139)
    g = np.random.default_rng(21)
    X = g.standard_normal((16, 700)) * np.exp2(g.integers(-40, 40, (16, 1)))
    sft, lg = oracle_mod.row_stats(X)
    m = np.abs(X).max(axis=1)
    assert np.all(np.abs(m * np.exp2(sft.astype(float))) >= 2.0 ** 52)
    assert np.all(np.abs(m * np.exp2(sft.astype(float))) < 2.0 ** 53)
    # column form over [K, N] equals the row form of the transpose in shift
    sc, _ = oracle_mod.col_stats(X.T.copy())
    assert np.array_equal(sc, sft)


def test_plan_rules():
    from oracle import oracle as O
    assert O.plan_config(4096) == (14, True)
    assert O.plan_config(8192) == (14, True)
    assert O.plan_config(8193) == (15, True)
    assert O.plan_config(131071) == (15, True)
    assert O.plan_config(16384) == (15, True)
    assert abs(O.range_bits(14) - 109.16) < 0.01
