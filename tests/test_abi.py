"""CPU checks of the drop-in boundary: libf64e.so loads, exports every symbol
include/f64e.h declares, and rejects invalid arguments the way the reference's
TORCH_CHECKs do (fp64_emu_cuda/fp64_emu.cu:1586-1693) -- all before any device
call.  Also checks that the torch op schemas equal the reference's
(torch-ext/torch_binding.cpp:7-12)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "f64e.h")
LIB = os.path.join(ROOT, "fp64-emu_b200", "fp64_emu", "libf64e.so")


class Problem(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("M", ctypes.c_int64), ("N", ctypes.c_int64),
                ("K", ctypes.c_int64), ("b_layout", ctypes.c_int32), ("nprimes", ctypes.c_int32),
                ("primes", ctypes.POINTER(ctypes.c_int32)), ("exact", ctypes.c_int32),
                ("bits", ctypes.c_int32), ("use_corr", ctypes.c_int32), ("slab_cols", ctypes.c_int64)]


PRIMES = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199,
          197, 193, 191, 181, 179, 173]


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        import subprocess
        import sys
        subprocess.run([sys.executable, os.path.join(ROOT, "fp64-emu_b200", "build.py"), "--lib-only"],
                       check=True)
    L = ctypes.CDLL(LIB)
    L.f64e_workspace_size.argtypes = [ctypes.POINTER(Problem)]
    L.f64e_workspace_size.restype = ctypes.c_size_t
    L.f64e_last_error.restype = ctypes.c_char_p
    L.f64e_maxp.restype = ctypes.c_int64
    return L


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"F64E_API\s+[\w\s\*]+?\b(f64e_\w+)\s*\(", src)))


def test_problem_struct_layout_matches_header():
    # the ctypes mirror above must cover every field of f64e_problem
    src = open(HEADER).read()
    body = src[src.index("typedef struct f64e_problem"):src.index("} f64e_problem;")]
    fields = re.findall(r"^\s+(?:const\s+)?\w+\*?\s+\*?(\w+)(?:,\s*(\w+))?(?:,\s*(\w+))?;", body, re.M)
    names = [n for grp in fields for n in grp if n]
    assert names == [f[0] for f in Problem._fields_]


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("f64e_mm", "f64e_mm_nt", "f64e_bmm", "f64e_bmm_nt", "f64e_mm_timed", "f64e_maxp",
              "f64e_gemm", "f64e_workspace_size", "f64e_last_error", "f64e_status"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for n in declared_symbols():
        assert hasattr(lib, n), n


def test_checking_build_exports_the_same_abi():
    # libf64e_debug.so (F64E_DEBUG_BOUNDS) is a drop-in for libf64e.so
    dbg = os.path.join(ROOT, "fp64-emu_b200", "fp64_emu", "libf64e_debug.so")
    if not os.path.exists(dbg):
        import subprocess
        import sys
        subprocess.run([sys.executable, "-c",
                        "import sys; sys.path.insert(0, %r); import build; build.build_lib(debug=True)"
                        % os.path.join(ROOT, "fp64-emu_b200")], check=True)
    L = ctypes.CDLL(dbg)
    for n in declared_symbols():
        assert hasattr(L, n), n
    L.f64e_workspace_size.argtypes = [ctypes.POINTER(Problem)]
    L.f64e_workspace_size.restype = ctypes.c_size_t
    arr = (ctypes.c_int32 * 14)(*PRIMES[:14])
    p = Problem(1, 300, 200, 100, 0, 14, arr, 1, 53, 1, 0)
    want = ctypes.CDLL(LIB)
    want.f64e_workspace_size.argtypes = [ctypes.POINTER(Problem)]
    want.f64e_workspace_size.restype = ctypes.c_size_t
    assert L.f64e_workspace_size(ctypes.byref(p)) == want.f64e_workspace_size(ctypes.byref(p)) > 0


def test_maxp(lib):
    assert lib.f64e_maxp() == 20


def _problem(**kw):
    pr = kw.pop("primes", PRIMES[:14])
    arr = (ctypes.c_int32 * len(pr))(*pr)
    p = Problem(batch=1, M=64, N=48, K=512, b_layout=1, nprimes=len(pr), primes=arr, exact=1, bits=53,
                use_corr=1, slab_cols=0)
    for k, v in kw.items():
        setattr(p, k, v)
    p._keep = arr
    return p


def test_workspace_size_valid(lib):
    p = _problem()
    n = lib.f64e_workspace_size(ctypes.byref(p))
    G, Kp, ldn = 16, 512, 48
    planes = G * (64 + 48) * Kp
    assert n >= planes + 14 * 64 * ldn + 4 * 64 * ldn
    assert n % 256 == 0


@pytest.mark.parametrize("field,value,msg", [
    ("bits", 15, "bits must be in [16, 53]"),
    ("bits", 54, "bits must be in [16, 53]"),
    ("nprimes", 21, "too many primes"),
    ("K", 131072, "K bound for int32 modular GEMM"),
])
def test_argument_errors(lib, field, value, msg):
    p = _problem()
    if field == "nprimes":
        p = _problem(primes=PRIMES + [167])
    else:
        setattr(p, field, value)
    assert lib.f64e_workspace_size(ctypes.byref(p)) == 0
    assert msg in lib.f64e_last_error().decode()


def test_deep_k_allowed_for_nk_layout_only(lib):
    p = _problem(K=200_000, b_layout=0)
    assert lib.f64e_workspace_size(ctypes.byref(p)) > 0
    p = _problem(K=128 * 65536 + 1, b_layout=0)
    assert lib.f64e_workspace_size(ctypes.byref(p)) == 0
    assert "128 segments" in lib.f64e_last_error().decode()


def test_bad_modulus_rejected(lib):
    p = _problem(primes=[256, 257])
    assert lib.f64e_workspace_size(ctypes.byref(p)) == 0


def test_bmm_batch_bound(lib):
    pr = (ctypes.c_int32 * 14)(*PRIMES[:14])
    fn = lib.f64e_bmm
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4 + [ctypes.c_void_p, ctypes.c_int32,
                                                                  ctypes.c_int32, ctypes.c_int64,
                                                                  ctypes.c_int32, ctypes.c_void_p,
                                                                  ctypes.c_size_t, ctypes.c_void_p]
    rc = fn(None, None, None, 65535 // 16 + 1, 4, 4, 4, pr, 14, 1, 53, 1, None, 0, None)
    assert rc == 1
    assert "z-extent" in lib.f64e_last_error().decode()


def test_empty_problem_is_a_noop(lib):
    fn = lib.f64e_mm_nt
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 3 + [ctypes.c_void_p, ctypes.c_int32,
                                                                  ctypes.c_int32, ctypes.c_int64,
                                                                  ctypes.c_int32, ctypes.c_void_p,
                                                                  ctypes.c_size_t, ctypes.c_void_p]
    pr = (ctypes.c_int32 * 14)(*PRIMES[:14])
    assert fn(None, None, None, 0, 5, 7, pr, 14, 1, 53, 1, None, 0, None) == 0


REF_SCHEMAS = {
    "fp64_emu_maxp": "fp64_emu_maxp() -> int",
    "fp64_emu_mm": "fp64_emu_mm(Tensor(a!) out, Tensor A, Tensor B, Tensor primes_cpu, Tensor inv_cpu, "
                   "Tensor mu_cpu, bool exact, int bits=53, bool use_corr=True) -> ()",
    "fp64_emu_bmm": "fp64_emu_bmm(Tensor(a!) out, Tensor A, Tensor B, Tensor primes_cpu, Tensor inv_cpu, "
                    "Tensor mu_cpu, bool exact, int bits=53, bool use_corr=True) -> ()",
    "fp64_emu_mm_nt": "fp64_emu_mm_nt(Tensor(a!) out, Tensor A, Tensor Bt, Tensor primes_cpu, "
                      "Tensor inv_cpu, Tensor mu_cpu, bool exact, int bits=53, bool use_corr=True) -> ()",
    "fp64_emu_bmm_nt": "fp64_emu_bmm_nt(Tensor(a!) out, Tensor A, Tensor Bt, Tensor primes_cpu, "
                       "Tensor inv_cpu, Tensor mu_cpu, bool exact, int bits=53, bool use_corr=True) -> ()",
    "fp64_emu_mm_timed": "fp64_emu_mm_timed(Tensor(a!) out, Tensor(b!) times, Tensor A, Tensor B, "
                         "Tensor primes_cpu, Tensor inv_cpu, Tensor mu_cpu, bool exact, int bits=53, "
                         "bool use_corr=True) -> ()",
}


def _args(schema):
    return [(a.name, str(a.type), a.default_value if a.has_default_value() else None,
             bool(a.alias_info and a.alias_info.is_write)) for a in schema.arguments]


def test_torch_op_schemas_match_reference():
    import torch
    import fp64_emu
    for name, want in REF_SCHEMAS.items():
        got = getattr(fp64_emu.ops, name).default._schema
        ref = torch._C.parse_schema(want)
        assert got.name == "fp64_emu_b200::" + name
        assert _args(got) == _args(ref), name
        assert [str(r.type) for r in got.returns] == [str(r.type) for r in ref.returns]


def test_python_surface_matches_reference():
    import fp64_emu
    from oracle import oracle as O
    for k in (1, 64, 4096, 8192, 8193, 65536, 131071, 200000):
        assert fp64_emu.plan_config(k) == O.plan_config(k)
    for n in range(1, 21):
        assert fp64_emu.range_bits(n) == O.range_bits(n)
    import math
    for k, b in ((4096, 53), (131071, 53), (512, 32), (8192, 40)):
        need = 2 * b + math.ceil(math.log2(k)) + 1
        assert fp64_emu.plan(k, b) == min(n for n in range(1, 21) if O.range_bits(n) >= need)
    pr, inv, mu = fp64_emu._tables(14)
    assert pr.tolist() == PRIMES[:14] and inv.numel() == 196 and mu.dtype.is_floating_point is False


def test_cpu_tensors_fail_loudly():
    import torch
    import fp64_emu
    A = torch.zeros(4, 8, dtype=torch.float64)
    with pytest.raises((NotImplementedError, RuntimeError)):
        fp64_emu.mm(A, A)
