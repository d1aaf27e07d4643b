"""Caller-level validation: algorithms that use the emulated product as their
GEMM (the reference's application drills and tiled Cholesky, at test sizes).
The drills themselves live in fp64-emu_b200/drills.py; here each runs with
native fp64 GEMMs and with fp64_emu and the application-level figures are
compared:
  * 4-step path counts: exact integers, bit-equal to native fp64;
  * tiled Cholesky with batched trailing updates: residual at native level;
  * CholeskyQR (cond 1e6): Q at least as orthogonal as with native GEMMs;
  * Newton-Schulz polar factor and a Taylor matrix exponential: errors at
    native level."""
import os
import sys

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "fp64-emu_b200"))


@pytest.fixture(scope="module")
def drills():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import drills as d
    return d


def test_path_counts_bitwise_equal(drills):
    Pn = drills.path_counts(drills.native_nt, 1024)
    Pe = drills.path_counts(drills.emu_nt, 1024)
    assert Pn.max().item() > 1e4
    assert torch.equal(Pn, Pe)


def test_tiled_cholesky_batched_updates(drills):
    A = drills.spd_matrix(1536)
    res = {}
    for name, upd in (("native", drills.native_bmm), ("emu", drills.emu_bmm)):
        L, _ = drills.tiled_cholesky(A, 256, upd)
        res[name] = ((A - L @ L.t()).norm() / A.norm()).item()
    assert res["emu"] < 1e-14
    assert res["emu"] <= 4.0 * res["native"] + 1e-16


def test_cholqr_orthogonality(drills):
    rn = drills.cholqr_residual(drills.native_nt, 8192, 256)
    re = drills.cholqr_residual(drills.emu_nt, 8192, 256)
    assert re <= 1.5 * rn


def test_newton_schulz_polar(drills):
    rn = drills.newton_schulz(drills.native_nt, 384, 80)
    re = drills.newton_schulz(drills.emu_nt, 384, 80)
    assert re < 1e-12
    assert re <= 4.0 * rn + 1e-14


def test_expm_taylor(drills):
    en = drills.expm_error(drills.native_nt, 384)
    ee = drills.expm_error(drills.emu_nt, 384)
    assert ee < 1e-13
    assert ee <= 4.0 * en + 1e-15
