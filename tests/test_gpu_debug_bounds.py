"""The checking build, libf64e_debug.so (F64E_DEBUG_BOUNDS), against the
release library, both through the C ABI.

Every extraction read and write, GEMM-epilogue write and reconstruction read
and write of the checking build is tested against the byte range its launcher
gives.  An access outside that range is skipped and its site code recorded in
the workspace status word; nothing traps.  Two properties are tested:

  * no false alarms, and the same bits: on small and odd shapes the checking
    build's products equal the release build's bit for bit, with the status
    word 0.  The shapes are 1x1x1, K = 1, K = 17, odd M/N/K, both B layouts,
    a batch, a chunked product and a deep-K product.
  * a miss is reported: the build's self-test hook moves the end of the output
    range 8 bytes in.  The last four-column group of the last row is then
    reported (site 20) and left unwritten, and everything else matches.
    The skipped writes lie inside the real output buffer, so no access leaves
    the caller's memory."""
import ctypes
import os

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fp64-emu_b200", "fp64_emu")
PRIMES14 = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199]
PRIMES15 = PRIMES14 + [197]
NK, KN = 0, 1
SITE_RECON_STORE = 20


class Problem(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("M", ctypes.c_int64), ("N", ctypes.c_int64),
                ("K", ctypes.c_int64), ("b_layout", ctypes.c_int32), ("nprimes", ctypes.c_int32),
                ("primes", ctypes.POINTER(ctypes.c_int32)), ("exact", ctypes.c_int32),
                ("bits", ctypes.c_int32), ("use_corr", ctypes.c_int32), ("slab_cols", ctypes.c_int64)]


def _load(name):
    L = ctypes.CDLL(os.path.join(PKG, name))
    vp = ctypes.c_void_p
    L.f64e_workspace_size.argtypes = [ctypes.POINTER(Problem)]
    L.f64e_workspace_size.restype = ctypes.c_size_t
    L.f64e_gemm.argtypes = [ctypes.POINTER(Problem), vp, vp, vp, vp, ctypes.c_size_t, vp, ctypes.c_int]
    L.f64e_gemm.restype = ctypes.c_int
    L.f64e_status.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_int32)]
    L.f64e_status.restype = ctypes.c_int
    L.f64e_last_error.restype = ctypes.c_char_p
    return L


@pytest.fixture(scope="module")
def libs():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    if not os.path.exists(os.path.join(PKG, "libf64e_debug.so")):
        pytest.skip("checking build not present (python fp64-emu_b200/build.py)")
    return _load("libf64e.so"), _load("libf64e_debug.so")


def _operands(batch, M, N, K, layout, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    shpA = (batch, M, K) if batch > 1 else (M, K)
    shpB = ((batch, K, N) if layout == KN else (batch, N, K)) if batch > 1 else ((K, N) if layout == KN else (N, K))
    A = torch.randn(shpA, dtype=torch.float64, device="cuda", generator=g)
    B = torch.randn(shpB, dtype=torch.float64, device="cuda", generator=g) * 2.0 ** 7
    return A, B


def _run(L, batch, M, N, K, layout, A, B, primes):
    arr = (ctypes.c_int32 * len(primes))(*primes)
    p = Problem(batch, M, N, K, layout, len(primes), arr, 1, 53, 1, 0)
    nb = L.f64e_workspace_size(ctypes.byref(p))
    assert nb > 0, L.f64e_last_error()
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    out = torch.full((batch * M, N), float("nan"), dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = L.f64e_gemm(ctypes.byref(p), A.data_ptr(), B.data_ptr(), out.data_ptr(), ws.data_ptr(), nb, stream, 15)
    assert rc == 0, L.f64e_last_error()
    st = ctypes.c_int32(-1)
    assert L.f64e_status(ws.data_ptr(), stream, ctypes.byref(st)) == 0, L.f64e_last_error()
    return out, st.value


CASES = [
    # batch, M, N, K, layout, primes
    (1, 1, 1, 1, NK, PRIMES14),
    (1, 7, 5, 1, KN, PRIMES14),
    (1, 33, 17, 17, NK, PRIMES14),
    (1, 129, 65, 257, KN, PRIMES14),
    (3, 40, 24, 100, KN, PRIMES14),
    (3, 40, 24, 100, NK, PRIMES14),
    (1, 2048, 300, 512, KN, PRIMES14),      # chunked pipeline (row chunks, two GEMM streams)
    (1, 64, 48, 140000, NK, PRIMES15),      # deep K: three 65536-deep segments
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b%dx%dx%dx%d_%s" % (c[0], c[1], c[2], c[3], "kn" if c[4] else "nk"))
def test_checking_build_matches_release_without_alarms(libs, case):
    rel, dbg = libs
    batch, M, N, K, layout, primes = case
    A, B = _operands(batch, M, N, K, layout, seed=M + 7 * N + K)
    want, st_rel = _run(rel, batch, M, N, K, layout, A, B, primes)
    got, st_dbg = _run(dbg, batch, M, N, K, layout, A, B, primes)
    assert st_rel == 0 and st_dbg == 0, (st_rel, st_dbg)
    assert torch.equal(got.view(torch.int64), want.view(torch.int64))


def test_checking_build_reports_and_skips_an_out_of_range_write(libs, monkeypatch):
    rel, dbg = libs
    M = N = K = 64
    A, B = _operands(1, M, N, K, NK, seed=3)
    want, _ = _run(rel, 1, M, N, K, NK, A, B, PRIMES14)
    monkeypatch.setenv("F64E_DEBUG_SHRINK_OUT_BYTES", "8")
    got, st = _run(dbg, 1, M, N, K, NK, A, B, PRIMES14)
    assert st == SITE_RECON_STORE
    # the last group of four columns of the last row lay past the shortened
    # range: reported and not written (still the NaN it was filled with)
    assert torch.isnan(got[-1, -4:]).all()
    assert torch.equal(got[:-1].view(torch.int64), want[:-1].view(torch.int64))
    assert torch.equal(got[-1, :-4].view(torch.int64), want[-1, :-4].view(torch.int64))
    monkeypatch.delenv("F64E_DEBUG_SHRINK_OUT_BYTES")
    again, st = _run(dbg, 1, M, N, K, NK, A, B, PRIMES14)
    assert st == 0 and torch.equal(again.view(torch.int64), want.view(torch.int64))
