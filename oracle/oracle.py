"""ctypes wrapper of the CPU restatement oracle (oracle/f64e_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py as the checker.  The product path never imports it.

The modulus table and the plan rule are restated here from the reference's
Python surface (torch-ext/fp64_emu/__init__.py:65-67 and 197-222) so the
oracle picks the same defaults as the reference when nprimes / corr are None.
"""
import ctypes
import math
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liborc.so"

# Pairwise-coprime moduli, largest first (torch-ext/fp64_emu/__init__.py:65-66).
PRIMES = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199,
          197, 193, 191, 181, 179, 173]
MAXP = 20


def range_bits(nprimes):
    """Signed CRT range in bits (torch-ext/fp64_emu/__init__.py:197-202)."""
    r = 0.0
    for p in PRIMES[:nprimes]:
        r += math.log2(p)
    return r - 1.0


def plan_config(K):
    """(nprimes, corr) default rule (torch-ext/fp64_emu/__init__.py:205-212)."""
    need = 2 * 49 + math.ceil(math.log2(max(K, 1))) + 1 - 3.4
    for n in range(1, MAXP + 1):
        if range_bits(n) >= need:
            return n, True
    return MAXP, True


def build():
    """Compile liborc.so with oracle/Makefile if it is missing or stale."""
    src = HERE / "f64e_oracle.c"
    if LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= src.stat().st_mtime:
        return LIB_PATH
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        i64, i32, vp, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_float
        L.orc_emu.argtypes = [vp, vp, vp, i64, i64, i64, i64, i32, vp, i32, i32, i32, i32, i32,
                              vp, vp, vp]
        L.orc_emu.restype = i32
        L.orc_emu_ex.argtypes = [vp, vp, vp, i64, i64, i64, i64, i32, vp, i32, i32, i32, i32, i32,
                                 vp, vp, vp, i64, vp, vp]
        L.orc_emu_ex.restype = i32
        L.orc_row_stats.argtypes = [vp, i64, i64, i32, i32, vp, vp]
        L.orc_col_stats.argtypes = [vp, i64, i64, i64, i32, i32, vp, vp]
        L.orc_log2M.argtypes = [vp, i32]
        L.orc_log2M.restype = f32
        L.orc_pick_bits.argtypes = [vp, i64, vp, i64, f32, i32, vp]
        L.orc_pick_bits.restype = i32
        L.orc_extract.argtypes = [vp, i64, i64, vp, vp, i32, vp, i32, vp, vp, vp]
        L.orc_residue_gemm.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, vp, i32, vp,
                                       vp]
        L.orc_reconstruct.argtypes = [vp, vp, i64, i64, i64, vp, i32, vp, vp, i32, i32, i32, vp]
        L.orc_tables.argtypes = [vp, i32, vp, vp, vp]
        L.orc_set_threads.argtypes = [i32]
        L.orc_max_threads.restype = i32
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n):
    lib().orc_set_threads(int(n))


def max_threads():
    return lib().orc_max_threads()


def emu(A, B, nprimes=None, exact=True, bits=53, corr=None, b_nt=False, contract=True,
        details=False):
    """Emulated product of float64 numpy arrays.

    A: [M,K] or [batch,M,K]; B: [N,K] / [batch,N,K] (b_nt False) or
    [K,N] / [batch,K,N] (b_nt True).  Returns C (and a dict of bits_eff and
    the widened shifts when details=True)."""
    A = np.ascontiguousarray(A, dtype=np.float64)
    B = np.ascontiguousarray(B, dtype=np.float64)
    batched = A.ndim == 3
    A3 = A if batched else A[None]
    B3 = B if batched else B[None]
    batch, M, K = A3.shape
    N = B3.shape[2] if b_nt else B3.shape[1]
    if nprimes is None or corr is None:
        dp, dc = plan_config(K)
        nprimes = dp if nprimes is None else nprimes
        corr = dc if corr is None else corr
    primes = np.array(PRIMES[:nprimes], dtype=np.int32)
    C = np.empty((batch, M, N), dtype=np.float64)
    be = np.zeros(1, dtype=np.int32)
    sA = np.zeros(batch * M, dtype=np.int16)
    sB = np.zeros(batch * N, dtype=np.int16)
    rc = lib().orc_emu(_p(A3), _p(B3), _p(C), batch, M, N, K, int(bool(b_nt)), _p(primes),
                       len(primes), int(bool(exact)), int(bits), int(bool(corr)),
                       int(bool(contract)), _p(be), _p(sA), _p(sB))
    if rc != 0:
        raise RuntimeError("oracle rejected the arguments")
    out = C if batched else C[0]
    if details:
        return out, {"bits_eff": int(be[0]), "sftA": sA, "sftB": sB}
    return out


def row_stats(X, bits=53, contract=True):
    X = np.ascontiguousarray(X, dtype=np.float64)
    rows, cols = X.shape
    sft = np.zeros(rows, dtype=np.int16)
    lg = np.zeros(rows, dtype=np.float32)
    lib().orc_row_stats(_p(X), rows, cols, bits, int(contract), _p(sft), _p(lg))
    return sft, lg


def col_stats(X, bits=53, contract=True):
    """X: [batch, K, N] (or [K, N])."""
    X = np.ascontiguousarray(X, dtype=np.float64)
    X3 = X if X.ndim == 3 else X[None]
    batch, K, N = X3.shape
    sft = np.zeros(batch * N, dtype=np.int16)
    lg = np.zeros(batch * N, dtype=np.float32)
    lib().orc_col_stats(_p(X3), batch, K, N, bits, int(contract), _p(sft), _p(lg))
    return sft, lg


def log2M(nprimes):
    primes = np.array(PRIMES[:nprimes], dtype=np.int32)
    return float(lib().orc_log2M(_p(primes), nprimes))


def pick_bits(lgA, lgB, nprimes, bits=53):
    lgA = np.ascontiguousarray(lgA, dtype=np.float32)
    lgB = np.ascontiguousarray(lgB, dtype=np.float32)
    g = np.zeros(1, dtype=np.int32)
    L = lib()
    be = L.orc_pick_bits(_p(lgA), lgA.size, _p(lgB), lgB.size,
                         ctypes.c_float(L.orc_log2M(_p(np.array(PRIMES[:nprimes], np.int32)),
                                                    nprimes)), bits, _p(g))
    return int(be), int(g[0])


def extract(X, shifts, bits_eff, nprimes, with_corr=True):
    """Residue planes [P, rows, K] plus hi / q planes [rows, K] of row-major X."""
    X = np.ascontiguousarray(X, dtype=np.float64)
    rows, K = X.shape
    shifts = np.ascontiguousarray(shifts, dtype=np.int16)
    primes = np.array(PRIMES[:nprimes], dtype=np.int32)
    planes = np.zeros((nprimes, rows, K), dtype=np.int8)
    hi = np.zeros((rows, K), dtype=np.int8)
    q = np.zeros((rows, K), dtype=np.int8)
    lib().orc_extract(_p(X), rows, K, _p(shifts), None, bits_eff, _p(primes), nprimes,
                      _p(planes), _p(hi) if with_corr else None, _p(q) if with_corr else None)
    return planes, hi, q


def tables(nprimes):
    primes = np.array(PRIMES[:nprimes], dtype=np.int32)
    cfac = np.zeros((nprimes, nprimes), dtype=np.int32)
    minv = np.zeros(nprimes, dtype=np.int32)
    m64 = np.zeros(2, dtype=np.int64)
    lib().orc_tables(_p(primes), nprimes, _p(cfac), _p(minv), _p(m64))
    return cfac, minv, m64


def cpu_count():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def emu_shard(A, B, nprimes=None, exact=True, bits=53, corr=None, b_nt=False, slab_cols=0,
              maxlg_in=None, sizing_only=False):
    """One rank's share of a partitioned product: returns (C or None, local
    maxima float32[2]).  maxlg_in replaces the local maxima in the width
    rule; slab_cols orders the column sums as for that many columns."""
    A = np.ascontiguousarray(A, dtype=np.float64)
    B = np.ascontiguousarray(B, dtype=np.float64)
    A3 = A if A.ndim == 3 else A[None]
    B3 = B if B.ndim == 3 else B[None]
    batch, M, K = A3.shape
    N = B3.shape[2] if b_nt else B3.shape[1]
    if nprimes is None or corr is None:
        dp, dc = plan_config(K)
        nprimes = dp if nprimes is None else nprimes
        corr = dc if corr is None else corr
    primes = np.array(PRIMES[:nprimes], dtype=np.int32)
    C = None if sizing_only else np.empty((batch, M, N), dtype=np.float64)
    mo = np.zeros(2, dtype=np.float32)
    mi = None if maxlg_in is None else np.ascontiguousarray(maxlg_in, dtype=np.float32)
    rc = lib().orc_emu_ex(_p(A3), _p(B3), None if C is None else _p(C), batch, M, N, K,
                          int(bool(b_nt)), _p(primes), len(primes), int(bool(exact)), int(bits),
                          int(bool(corr)), int(bool(contract_default)), None, None, None,
                          int(slab_cols), _p(mo), None if mi is None else _p(mi))
    if rc != 0:
        raise RuntimeError("oracle rejected the arguments")
    if C is not None and A.ndim == 2:
        C = C[0]
    return C, mo


contract_default = True
