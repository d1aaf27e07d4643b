"""f64e_mm_nt_noalloc: the entry point for callers that cannot allocate device
memory (code inside another framework's memory arena, plugin hosts and
real-time paths that may not call cudaMalloc / cudaFree).  It runs the
product in the library's fixed device scratch array instead of a caller
workspace.  Called here through the C ABI, like such a caller would, and
checked against f64e_mm_nt (the entry point with a caller workspace) on two
calls in a row: the results must be identical bit for bit, the same standard
as every parity test of this suite.  This file is collected last."""
import ctypes
import os

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "fp64-emu_b200", "fp64_emu", "libf64e.so")
PRIMES = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199]
SCRATCH_BYTES = 64 << 20


class Problem(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("M", ctypes.c_int64), ("N", ctypes.c_int64),
                ("K", ctypes.c_int64), ("b_layout", ctypes.c_int32), ("nprimes", ctypes.c_int32),
                ("primes", ctypes.POINTER(ctypes.c_int32)), ("exact", ctypes.c_int32),
                ("bits", ctypes.c_int32), ("use_corr", ctypes.c_int32), ("slab_cols", ctypes.c_int64)]


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    L = ctypes.CDLL(LIB)
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    L.f64e_mm_nt.argtypes = [vp, vp, vp, i64, i64, i64, vp, i32, i32, i64, i32, vp, ctypes.c_size_t, vp]
    L.f64e_mm_nt.restype = i32
    L.f64e_mm_nt_noalloc.argtypes = [vp, vp, vp, i64, i64, i64, vp, i32, i32, i64, i32, vp]
    L.f64e_mm_nt_noalloc.restype = i32
    L.f64e_workspace_size.argtypes = [ctypes.POINTER(Problem)]
    L.f64e_workspace_size.restype = ctypes.c_size_t
    L.f64e_last_error.restype = ctypes.c_char_p
    return L


def _with_workspace(L, A, Bt, primes, stream):
    M, K = A.shape
    N = Bt.shape[1]
    p = Problem(1, M, N, K, 1, len(PRIMES), primes, 1, 53, 1, 0)
    nb = L.f64e_workspace_size(ctypes.byref(p))
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    out = torch.empty(M, N, dtype=torch.float64, device="cuda")
    rc = L.f64e_mm_nt(out.data_ptr(), A.data_ptr(), Bt.data_ptr(), M, N, K, primes, len(PRIMES), 1, 53, 1,
                      ws.data_ptr(), nb, stream)
    assert rc == 0, L.f64e_last_error()
    return out


def _noalloc(L, A, Bt, primes, stream, M, N, K):
    got = torch.full((M, N), float("nan"), dtype=torch.float64, device="cuda")
    rc = L.f64e_mm_nt_noalloc(got.data_ptr(), A.data_ptr() if A.numel() else None,
                              Bt.data_ptr() if Bt.numel() else None, M, N, K, primes, len(PRIMES), 1, 53, 1, stream)
    assert rc == 0, L.f64e_last_error()
    torch.cuda.synchronize()
    return got


def test_noalloc_matches_workspace_entry_twice(lib):
    primes = (ctypes.c_int32 * len(PRIMES))(*PRIMES)
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(77)
    # two calls in a row, different shapes: the full-K call fills the array
    # first, so the ragged-K call after it runs on the stale bytes the first
    # one left (padding columns up to the next multiple of 16 included)
    for M, K, N in ((513, 1024, 511), (384, 900, 200)):
        A = torch.randn(M, K, dtype=torch.float64, device="cuda", generator=g)
        Bt = torch.randn(K, N, dtype=torch.float64, device="cuda", generator=g) * 2.0 ** 9
        want = _with_workspace(lib, A, Bt, primes, stream)
        got = _noalloc(lib, A, Bt, primes, stream, M, N, K)
        assert torch.equal(got, want)


def test_noalloc_tall_product_takes_the_chunked_path(lib):
    # M >= 2048 with small N and K fits the array and runs the library's
    # chunked pipeline (its own streams) on the shared scratch
    primes = (ctypes.c_int32 * len(PRIMES))(*PRIMES)
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(78)
    M, K, N = 2048, 16, 16
    A = torch.randn(M, K, dtype=torch.float64, device="cuda", generator=g)
    Bt = torch.randn(K, N, dtype=torch.float64, device="cuda", generator=g)
    want = _with_workspace(lib, A, Bt, primes, stream)
    assert torch.equal(_noalloc(lib, A, Bt, primes, stream, M, N, K), want)


def test_noalloc_empty_inner_dimension_gives_zeros(lib):
    primes = (ctypes.c_int32 * len(PRIMES))(*PRIMES)
    stream = torch.cuda.current_stream().cuda_stream
    e = torch.empty(0, dtype=torch.float64, device="cuda")
    got = _noalloc(lib, e, e, primes, stream, 7, 5, 0)
    assert torch.equal(got, torch.zeros(7, 5, dtype=torch.float64, device="cuda"))


def test_noalloc_rejects_problems_beyond_its_scratch(lib):
    primes = (ctypes.c_int32 * len(PRIMES))(*PRIMES)
    p = Problem(1, 4096, 4096, 4096, 1, len(PRIMES), primes, 1, 53, 1, 0)
    assert lib.f64e_workspace_size(ctypes.byref(p)) > SCRATCH_BYTES
    rc = lib.f64e_mm_nt_noalloc(None, None, None, 4096, 4096, 4096, primes, len(PRIMES), 1, 53, 1, None)
    assert rc == 2   # F64E_ERR_WORKSPACE
    assert b"no-alloc" in lib.f64e_last_error()
