"""The FP64-pipe CRT reconstruction (fp64-emu_b200/csrc/f64e_crt64.cuh) on the
CPU: its host build (tests/native/crt64_check.cpp, the device kernel's
arithmetic on IEEE doubles) against exact integer arithmetic.

For balanced residues r_t of an integer x, the reference's reconstruction
(fp64_emu.cu:854-952 of CharlesCNorton/fp64-emu) yields V, the representative
of x modulo M = prod p_t in the balanced mixed-radix range [L, L + M), then
ldexp(RN(V + c 2^cshift), sh).  Python's int -> float conversion rounds to
nearest even and math.ldexp rounds subnormal results once, so the expected
doubles are exact references.  Cases: uniform residues, V at both ends of
its range and around zero (where the quotient estimate sits on an integer),
values straddling 2^93 (the switch between the two rounding forms) and 2^53,
halfway ties, large corrections, subnormal and overflowing scalings."""
import ctypes
import math
import os
import random
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PRIMES14 = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199]
PRIMES15 = PRIMES14 + [197]
PRIMES13 = PRIMES14[:13]


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    out = tmp_path_factory.mktemp("crt64") / "crt64_check.so"
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-ffp-contract=off",
                    "-I" + os.path.join(ROOT, "fp64-emu_b200", "csrc"),
                    os.path.join(ROOT, "tests", "native", "crt64_check.cpp"), "-o", str(out)], check=True)
    L = ctypes.CDLL(str(out))
    L.crt64_check_size.restype = ctypes.c_int
    L.crt64_check_tables.restype = ctypes.c_int
    L.crt64_check_run.restype = None
    return L


def tables(L, primes):
    buf = ctypes.create_string_buffer(L.crt64_check_size())
    arr = (ctypes.c_int32 * len(primes))(*primes)
    ok = L.crt64_check_tables(arr, len(primes), buf)
    return buf, ok


def low_end(primes):
    L, run = 0, 1
    for p in primes:
        L -= (p // 2) * run
        run *= p
    return L, run


def balanced(x, p):
    r = x % p
    return r - p if r > (p - 1) // 2 else r


def expected(V, c, cshift, sh):
    X = V + c * (1 << cshift)
    return math.ldexp(float(X), sh) if X != 0 else 0.0


SLOW = {"n": 0}   # elements the common path declined, over the module


def run(L, buf, primes, Vs, cs, cshift, shs):
    n = len(Vs)
    res = np.array([[balanced(V, p) for p in primes] for V in Vs], dtype=np.int8)
    corr = np.array(cs, dtype=np.float64)
    sh = np.array(shs, dtype=np.int32)
    out = np.empty(n, dtype=np.float64)
    slow = ctypes.c_int64(0)
    L.crt64_check_run(buf, res.ctypes.data_as(ctypes.c_void_p), corr.ctypes.data_as(ctypes.c_void_p),
                      sh.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(cshift), ctypes.c_int64(n),
                      out.ctypes.data_as(ctypes.c_void_p), ctypes.byref(slow))
    SLOW["n"] += slow.value
    return out


def check(L, primes, Vs, cs, cshift, shs):
    buf, ok = tables(L, primes)
    assert ok
    got = run(L, buf, primes, Vs, cs, cshift, shs)
    want = np.array([expected(V, c, cshift, s) for V, c, s in zip(Vs, cs, shs)], dtype=np.float64)
    bad = np.nonzero(got.view(np.int64) != want.view(np.int64))[0]
    assert bad.size == 0, [(Vs[i], cs[i], shs[i], got[i], want[i]) for i in bad[:5]]


def test_tables_apply_below_2_120(lib):
    assert tables(lib, PRIMES14)[1] == 1 and tables(lib, PRIMES15)[1] == 1
    assert tables(lib, PRIMES14 + [197, 193])[1] == 0            # M > 2^120
    assert tables(lib, [256, 255, 128])[1] == 0                  # not coprime


@pytest.mark.parametrize("primes", [PRIMES14, PRIMES15, PRIMES13, [7, 11, 13]])
def test_uniform_residues(lib, primes):
    rng = random.Random(len(primes))
    Lo, M = low_end(primes)
    Vs = [Lo + rng.randrange(M) for _ in range(20000)]
    cs = [rng.randrange(-(1 << 31), 1 << 31) for _ in Vs]
    shs = [rng.randrange(-200, 60) for _ in Vs]
    check(lib, primes, Vs, cs, 35, shs)


@pytest.mark.parametrize("primes", [PRIMES14, PRIMES15])
def test_range_ends_and_zero(lib, primes):
    # V = L and L + M - 1 put the remainder at the ends of [L, L + M), where
    # the quotient estimate is within 2^-38 of an integer; around zero the
    # value is tiny and every bit counts
    Lo, M = low_end(primes)
    Vs = [Lo + d for d in range(0, 400)] + [Lo + M - 1 - d for d in range(400)] + list(range(-400, 400))
    cs = [0] * len(Vs)
    check(lib, primes, Vs, cs, 30, [0] * len(Vs))
    rng = random.Random(5)
    cs = [rng.randrange(-(1 << 20), 1 << 20) for _ in Vs]
    check(lib, primes, Vs, cs, 12, [-3] * len(Vs))


def test_rounding_form_switch_and_ties(lib):
    # values around 2^53 and 2^93 (where the two rounding forms meet), exact
    # halfway cases at several magnitudes, and sticky bits far below
    primes = PRIMES15
    Lo, M = low_end(primes)
    Vs = []
    for e in (52, 53, 54, 92, 93, 94, 100, 110, 115):
        for s in (1, -1):
            base = s * (1 << e)
            Vs += [base + d for d in (-3, -2, -1, 0, 1, 2, 3)]
            ulp = 1 << max(0, e - 52)
            Vs += [base + ulp // 2, base - ulp // 2, base + ulp // 2 + 1, base + 3 * ulp // 2, base + ulp // 2 - 1]
            Vs += [base + (1 << 39), base + (1 << 40) - 1, base + (1 << 41) + 1]
    Vs = [V for V in Vs if Lo <= V < Lo + M]
    check(lib, primes, Vs, [0] * len(Vs), 30, [0] * len(Vs))
    # the correction moves the same values across the boundaries
    rng = random.Random(9)
    cs = [rng.choice([-1, 1]) * rng.randrange(1 << 33) for _ in Vs]
    for cshift in (1, 20, 38):
        check(lib, primes, Vs, cs, cshift, [0] * len(Vs))


def test_scaling_to_subnormal_and_overflow(lib):
    primes = PRIMES14
    rng = random.Random(11)
    Lo, M = low_end(primes)
    Vs = [Lo + rng.randrange(M) for _ in range(3000)]
    cs = [rng.randrange(-(1 << 31), 1 << 31) for _ in Vs]
    shs = [rng.choice([-1180, -1130, -1100, -1074, -1040, 900, 915, 1000]) for _ in Vs]
    buf, ok = tables(lib, primes)
    got = run(lib, buf, primes, Vs, cs, 35, shs)
    for V, c, s, g in zip(Vs, cs, shs, got):
        X = V + c * (1 << 35)
        x = float(X)
        try:
            w = math.ldexp(x, s)
        except OverflowError:
            w = math.copysign(math.inf, x)
        assert np.float64(g).view(np.int64) == np.float64(w).view(np.int64), (V, c, s, g, w)


def test_large_deep_k_corrections(lib):
    # int64 corrections of deep-K products reach 2^39
    primes = PRIMES15
    rng = random.Random(13)
    Lo, M = low_end(primes)
    Vs = [Lo + rng.randrange(M) for _ in range(5000)]
    cs = [rng.randrange(-(1 << 39), 1 << 39) for _ in Vs]
    check(lib, primes, Vs, cs, 37, [rng.randrange(-100, 100) for _ in Vs])


@pytest.mark.parametrize("primes", [PRIMES14, PRIMES15])
def test_log_uniform_magnitudes(lib, primes):
    # V of every magnitude and sign inside the range, near-halfway low bits,
    # corrections at every shift
    rng = random.Random(17 + len(primes))
    Lo, M = low_end(primes)
    Vs, cs, shs = [], [], []
    for _ in range(40000):
        e = rng.randrange(0, 118)
        V = rng.choice([-1, 1]) * (rng.randrange(1 << e, 1 << (e + 1)) if e else rng.randrange(2))
        if rng.random() < 0.3 and e > 53:
            ulp = 1 << (e - 52)
            V = (V // ulp) * ulp + ulp // 2 + rng.choice([-1, 0, 0, 1])   # near-halfway
        if not Lo <= V < Lo + M:
            continue
        Vs.append(V)
        cs.append(rng.randrange(-(1 << 32), 1 << 32) if rng.random() < 0.5 else 0)
        shs.append(rng.randrange(-300, 300))
    for cshift in (1, 17, 38):
        check(lib, primes, Vs, cs, cshift, shs)


def test_both_paths_were_taken(lib):
    # the cases above reach the exact side path (ties of the quotient
    # estimate at the range ends, zero and non-normal results)
    check(lib, PRIMES14, [0, 1, -1], [0, 0, 0], 30, [0, -1100, 0])
    assert SLOW["n"] > 0
