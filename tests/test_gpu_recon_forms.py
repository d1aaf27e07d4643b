"""The three exact reconstruction forms must agree bit for bit: the CRT sum on
the FP64 pipe (modulus sets with M < 2^120, the default), the direct CRT sum
on the integer pipe (F64E_RECON_FORM=crt) and the digit-by-digit balanced
Garner form (F64E_RECON_FORM=garner; every modulus set).  Every correction
layout (none, one fused plane, two planes, deep-K int64 sums), several modulus
counts, ragged shapes, batches, non-finite inputs and results that are
subnormal or overflow; the CPU oracle pins one of each."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from helpers import make, same_bits  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def emu():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import fp64_emu
    return fp64_emu


def _forms(fn):
    """The same product under each reconstruction form: (garner, crt, default)."""
    old = os.environ.get("F64E_RECON_FORM")
    out = []
    try:
        for form in ("garner", "crt", None):
            if form is None:
                os.environ.pop("F64E_RECON_FORM", None)
            else:
                os.environ["F64E_RECON_FORM"] = form
            out.append(fn())
    finally:
        if old is None:
            os.environ.pop("F64E_RECON_FORM", None)
        else:
            os.environ["F64E_RECON_FORM"] = old
    torch.cuda.synchronize()
    return out


def _both(fn):
    """(Garner form, default form) of the same product; the direct CRT form
    must give the same bits too."""
    g, c, d = _forms(fn)
    assert torch.equal(g.view(torch.int64), c.view(torch.int64))
    return g, d


CASES = [
    # kind, batch, M, K, N, dist, kwargs
    ("mm_nt", 1, 300, 700, 259, "randn", {}),
    ("mm_nt", 1, 129, 4095, 127, "wide16", {}),
    ("mm", 1, 255, 1000, 999, "illcond40", {}),
    ("mm", 1, 64, 512, 48, "spike", {"nprimes": 13, "corr": False}),     # no correction plane
    ("mm_nt", 1, 96, 700, 80, "wide8", {"bits": 40}),
    ("mm", 1, 50, 300, 70, "randn", {"nprimes": 15}),
    ("mm", 1, 30, 200, 20, "randn", {"nprimes": 8}),
    ("mm", 1, 20, 100, 12, "randn", {"nprimes": 2}),
    ("bmm_nt", 4, 40, 200, 30, "illcond", {}),
    ("mm_nt", 1, 128, 70000, 64, "randn", {}),                          # two correction planes
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[2]}x{c[3]}x{c[4]}-{c[5]}-{c[6]}")
def test_crt_form_equals_garner_form(emu, oracle_mod, case):
    kind, batch, M, K, N, dist, kw = case
    nt = kind.endswith("_nt")
    if batch == 1:
        A, B = make(dist, M, K, N, seed=M + K + N, nt=nt)
    else:
        pairs = [make(dist, M, K, N, seed=50 + b, nt=nt) for b in range(batch)]
        A, B = np.stack([p[0] for p in pairs]), np.stack([p[1] for p in pairs])
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    g, c = _both(lambda: getattr(emu, kind)(Ad, Bd, **kw))
    assert torch.equal(g, c)
    assert same_bits(c.cpu().numpy(), oracle_mod.emu(A, B, b_nt=nt, **kw))


def test_crt_form_deep_k_and_large(emu):
    g0 = torch.Generator(device="cuda").manual_seed(8)
    A = torch.randn(64, 140000, dtype=torch.float64, device="cuda", generator=g0)    # deep K: int64 sums
    B = torch.randn(48, 140000, dtype=torch.float64, device="cuda", generator=g0)
    g, c = _both(lambda: emu.mm(A, B))
    assert torch.equal(g, c)
    A = torch.randn(2048, 1024, dtype=torch.float64, device="cuda", generator=g0) * 2.0 ** 300
    Bt = torch.randn(1024, 2048, dtype=torch.float64, device="cuda", generator=g0) * 2.0 ** -700
    g, c = _both(lambda: emu.mm_nt(A, Bt))
    assert torch.equal(g, c)


def test_crt_form_non_finite(emu):
    A = torch.randn(40, 300, dtype=torch.float64, device="cuda")
    B = torch.randn(30, 300, dtype=torch.float64, device="cuda")
    A[3, 7] = float("inf")
    A[5, 2] = float("nan")
    B[9, 0] = float("-inf")
    g, c = _both(lambda: emu.mm(A, B))
    assert torch.equal(g.isnan(), c.isnan())
    assert torch.equal(torch.nan_to_num(g, nan=0.0), torch.nan_to_num(c, nan=0.0))
    assert np.array_equal(g.cpu().numpy().view(np.uint64), c.cpu().numpy().view(np.uint64))


def test_forms_subnormal_and_overflowing_results(emu):
    # the FP64 form takes its exact side path when a result is not a normal
    # double: every element of these products is subnormal, or overflows
    g0 = torch.Generator(device="cuda").manual_seed(12)
    A = torch.randn(200, 512, dtype=torch.float64, device="cuda", generator=g0) * 2.0 ** -530
    Bt = torch.randn(512, 150, dtype=torch.float64, device="cuda", generator=g0) * 2.0 ** -530
    g, d = _both(lambda: emu.mm_nt(A, Bt))
    assert (d.abs() < 2.0 ** -1022).float().mean() > 0.9
    assert torch.equal(g.view(torch.int64), d.view(torch.int64))
    A = A * 2.0 ** 525 * 2.0 ** 525
    Bt = Bt * 2.0 ** 520 * 2.0 ** 520
    g, d = _both(lambda: emu.mm_nt(A, Bt))
    assert torch.isinf(d).float().mean() > 0.5
    assert torch.equal(g.view(torch.int64), d.view(torch.int64))
