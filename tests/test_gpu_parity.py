"""GPU parity tests: the CUDA path against the CPU oracle (bit for bit), the
reference's own known-answer tests (tests/test_fp64_emu.py of
CharlesCNorton/fp64-emu), and -- when its build is present in oracle/_ref --
the reference's own kernels on the same inputs."""
import math
import os
import sys

import numpy as np
import pytest

from helpers import correct_bits, dd_matmul, make, same_bits

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def emu():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import fp64_emu
    return fp64_emu


@pytest.fixture(scope="module")
def ref():
    ref_dir = os.path.join(ROOT, "oracle", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "fp64_emu_ref.so")):
        pytest.skip("reference build not present (python oracle/build_ref.py)")
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import fp64_emu_ref
    return fp64_emu_ref


def cuda(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _check_status(emu):
    # every product leaves the workspace status word at 0 (no bounded wait ran out)
    A = torch.randn(8, 16, dtype=torch.float64, device="cuda")
    pr = emu._tables(14)[0]
    ws = torch.zeros(emu.ops.fp64_emu_workspace_bytes(A, A, pr, False, True), dtype=torch.uint8, device="cuda")
    out = torch.empty(8, 8, dtype=torch.float64, device="cuda")
    emu.ops.fp64_emu_gemm_ws(out, ws, A, A, pr, False, True, 53, True, 15)
    assert emu.ops.fp64_emu_status(ws) == 0


# ------------------------------------------------ against the CPU oracle --
ORACLE_CASES = [
    # (kind, batch, M, K, N, dist, kwargs)
    ("mm_nt", 1, 128, 4096, 128, "randn", {}),
    ("mm_nt", 1, 129, 4095, 127, "randn", {}),
    ("mm_nt", 1, 17, 23, 29, "wide16", {}),
    ("mm", 1, 300, 1000, 520, "randn", {}),
    ("mm", 1, 255, 1000, 999, "illcond40", {}),
    ("mm", 1, 64, 512, 48, "spike", {"nprimes": 13, "corr": False}),
    ("mm_nt", 1, 64, 300, 50, "randn", {"exact": False}),
    ("mm_nt", 1, 96, 700, 80, "wide8", {"bits": 40}),
    ("mm_nt", 1, 1, 1, 1, "randn", {}),
    ("mm_nt", 1, 33, 1, 20, "randn", {}),               # K = 1
    ("mm", 1, 7, 1, 9, "wide16", {}),
    ("bmm_nt", 2, 3, 1, 5, "randn", {}),
    ("mm", 1, 5, 17, 3, "randn", {"nprimes": 20}),
    ("bmm", 3, 100, 333, 77, "randn", {}),
    ("bmm_nt", 4, 40, 200, 30, "illcond", {}),
    ("mm_nt", 1, 256, 70000, 64, "randn", {}),          # K > 65536: two correction planes
]


@pytest.mark.parametrize("case", ORACLE_CASES, ids=lambda c: f"{c[0]}-{c[1]}x{c[2]}x{c[3]}x{c[4]}-{c[5]}")
def test_bitexact_vs_oracle(emu, oracle_mod, case):
    kind, batch, M, K, N, dist, kw = case
    nt = kind.endswith("_nt")
    if batch == 1:
        A, B = make(dist, M, K, N, seed=M + K + N, nt=nt)
    else:
        pairs = [make(dist, M, K, N, seed=100 + b, nt=nt) for b in range(batch)]
        A = np.stack([p[0] for p in pairs])
        B = np.stack([p[1] for p in pairs])
    C = getattr(emu, kind)(cuda(A), cuda(B), **kw).cpu().numpy()
    W = oracle_mod.emu(A, B, b_nt=nt, **kw)
    assert same_bits(C, W)


# ------------------------------------ the reference's known-answer tests --
def test_integer_products_accurate(emu):
    torch.manual_seed(0)
    A = torch.randint(-1000, 1001, (128, 256), device="cuda").double()
    Bt = torch.randint(-1000, 1001, (256, 96), device="cuda").double()
    ref = (A.long().cpu() @ Bt.long().cpu()).double().cuda()
    C = emu.mm_nt(A, Bt, nprimes=18)
    rel = (C - ref).abs().max().item() / ref.abs().max().item()
    assert (-math.log2(rel) if rel > 0 else 53.0) >= 45.0


def test_exact_mode_bitwise_integer_oracle(emu):
    torch.manual_seed(1)
    A = torch.randint(-4096, 4097, (128, 256), device="cuda").double()
    Bt = torch.randint(-4096, 4097, (256, 96), device="cuda").double()
    ref = (A.long().cpu() @ Bt.long().cpu()).double().cuda()
    assert torch.equal(emu.mm_nt(A, Bt, nprimes=20, exact=True), ref)


@pytest.mark.parametrize("nprimes", [18, 20])
def test_random_fp64_accuracy(emu, nprimes):
    torch.manual_seed(2)
    A = torch.randn(512, 1024, dtype=torch.float64, device="cuda")
    Bt = torch.randn(1024, 512, dtype=torch.float64, device="cuda")
    ref = A @ Bt
    rel = (emu.mm_nt(A, Bt, nprimes=nprimes) - ref).abs().max().item() / ref.abs().max().item()
    assert -math.log2(rel) >= 45.0


def test_range_rule_adversarial_aligned(emu):
    K = 2048
    A = torch.ones(64, K, dtype=torch.float64, device="cuda")
    Bt = torch.ones(K, 48, dtype=torch.float64, device="cuda")
    assert torch.equal(emu.mm_nt(A, Bt, exact=True), torch.full((64, 48), float(K), dtype=torch.float64,
                                                                 device="cuda"))


def test_dyadic_dynamic_range_bitexact(emu):
    torch.manual_seed(5)
    M, K, N = 64, 512, 48
    ek = torch.randint(-12, 1, (K,), device="cuda")
    Ai = torch.randint(-256, 257, (M, K), device="cuda")
    Bi = torch.randint(-256, 257, (N, K), device="cuda")
    A = torch.bitwise_left_shift(Ai, ek + 12).double() * (2.0 ** -12)
    B = torch.bitwise_left_shift(Bi, ek + 12).double() * (2.0 ** -12)
    w = (4 ** (ek + 12)).long().cpu()
    ref = ((Ai.long().cpu() * w) @ Bi.long().cpu().T).double() * (2.0 ** -24)
    assert torch.equal(emu.mm(A, B), ref.cuda())


def test_bmm_single_batch_matches_mm(emu):
    torch.manual_seed(4)
    A = torch.randn(192, 384, dtype=torch.float64, device="cuda")
    B = torch.randn(160, 384, dtype=torch.float64, device="cuda")
    assert torch.equal(emu.bmm(A[None], B[None])[0], emu.mm(A, B))


def test_bmm_integer_oracle_bitexact(emu):
    torch.manual_seed(6)
    A = torch.randint(-4096, 4097, (5, 96, 256), device="cuda").double()
    B = torch.randint(-4096, 4097, (5, 64, 256), device="cuda").double()
    ref = torch.stack([(A[b].long().cpu() @ B[b].long().cpu().T).double() for b in range(5)]).cuda()
    assert torch.equal(emu.bmm(A, B), ref)


def test_bmm_odd_shapes_accuracy(emu):
    torch.manual_seed(8)
    A = torch.randn(3, 100, 333, dtype=torch.float64, device="cuda")
    Bt = torch.randn(3, 333, 77, dtype=torch.float64, device="cuda")
    ref = torch.bmm(A, Bt)
    rel = (emu.bmm_nt(A, Bt) - ref).abs().max().item() / ref.abs().max().item()
    assert -math.log2(rel) >= 45.0


def test_deep_k_integer_bitexact(emu):
    torch.manual_seed(16)
    K = 200_000
    A = torch.randint(-1, 2, (48, K), device="cuda").double()
    B = torch.randint(-1, 2, (32, K), device="cuda").double()
    ref = (A.long().cpu() @ B.long().cpu().T).double().cuda()
    assert torch.equal(emu.mm(A, B), ref)


def test_deep_k_randn_accuracy_and_oracle(emu, oracle_mod):
    torch.manual_seed(17)
    K = 150_000
    A = torch.randn(64, K, dtype=torch.float64, device="cuda")
    B = torch.randn(48, K, dtype=torch.float64, device="cuda")
    C = emu.mm(A, B)
    ref = A @ B.t()
    rel = (C - ref).abs().max().item() / ref.abs().max().item()
    assert -math.log2(rel) >= 40.0
    assert same_bits(C.cpu().numpy(), oracle_mod.emu(A.cpu().numpy(), B.cpu().numpy()))


def test_deep_k_via_mm_nt_routes_through_mm(emu):
    torch.manual_seed(18)
    K = 140_000
    A = torch.randint(-2, 3, (16, K), device="cuda").double()
    Bt = torch.randint(-2, 3, (K, 24), device="cuda").double()
    ref = (A.long().cpu() @ Bt.long().cpu()).double().cuda()
    assert torch.equal(emu.mm_nt(A, Bt), ref)


def test_cuda_graph_capture(emu):
    torch.manual_seed(13)
    A = torch.randn(128, 256, dtype=torch.float64, device="cuda")
    B = torch.randn(96, 256, dtype=torch.float64, device="cuda")
    for _ in range(3):
        emu.mm(A, B)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        C = emu.mm(A, B)
    A.copy_(torch.randn(128, 256, dtype=torch.float64, device="cuda"))
    B.copy_(torch.randn(96, 256, dtype=torch.float64, device="cuda"))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(C, emu.mm(A, B))


def test_torch_compile_traces(emu):
    import shutil
    import torch._inductor.config as icfg
    # The image's default CXX wrapper cannot link OpenMP (missing libgomp.spec),
    # which Inductor's host-code compile needs; point Inductor at the system g++.
    if shutil.which("/usr/bin/g++"):
        icfg.cpp.cxx = (None, "/usr/bin/g++")
    torch.manual_seed(12)
    A = torch.randn(64, 128, dtype=torch.float64, device="cuda")
    B = torch.randn(48, 128, dtype=torch.float64, device="cuda")
    eager = emu.mm(A, B)
    compiled = torch.compile(emu.mm, dynamic=False)
    assert torch.equal(compiled(A, B), eager)


def test_deterministic(emu):
    torch.manual_seed(3)
    A = torch.randn(256, 512, dtype=torch.float64, device="cuda")
    Bt = torch.randn(512, 256, dtype=torch.float64, device="cuda")
    assert torch.equal(emu.mm_nt(A, Bt, nprimes=18), emu.mm_nt(A, Bt, nprimes=18))
    A3 = torch.randn(4, 128, 512, dtype=torch.float64, device="cuda")
    B3 = torch.randn(4, 96, 512, dtype=torch.float64, device="cuda")
    assert torch.equal(emu.bmm(A3, B3), emu.bmm(A3, B3))


def test_nt_and_transposed_mm_agree(emu):
    # the reference pins its engines to identical bits (tests/test_fp64_emu.py:148-161);
    # here the [K, N]-direct extraction must equal the [N, K] form.
    torch.manual_seed(15)
    A = torch.randn(256, 1024, dtype=torch.float64, device="cuda")
    Bt = torch.randn(1024, 200, dtype=torch.float64, device="cuda")
    assert torch.equal(emu.mm_nt(A, Bt), emu.mm(A, Bt.t().contiguous()))


def test_tensor_core_gemm_matches_dp4a_check_kernel(emu):
    torch.manual_seed(19)
    for (M, K, N) in [(300, 1000, 520), (128, 256, 256), (33, 4100, 257)]:
        A = torch.randn(M, K, dtype=torch.float64, device="cuda")
        Bt = torch.randn(K, N, dtype=torch.float64, device="cuda")
        pr = emu._tables(14)[0]
        ws = torch.empty(emu.ops.fp64_emu_workspace_bytes(A, Bt, pr, True, True), dtype=torch.uint8,
                         device="cuda")
        c1 = torch.empty(M, N, dtype=torch.float64, device="cuda")
        c2 = torch.empty_like(c1)
        emu.ops.fp64_emu_gemm_ws(c1, ws, A, Bt, pr, True, True, 53, True, 15)
        emu.ops.fp64_emu_gemm_checked(c2, ws, A, Bt, pr, True, True, 53, True)
        assert torch.equal(c1, c2)


def test_mm_timed(emu):
    torch.manual_seed(20)
    A = torch.randn(512, 1024, dtype=torch.float64, device="cuda")
    B = torch.randn(256, 1024, dtype=torch.float64, device="cuda")
    C, t = emu.mm_timed(A, B)
    assert torch.equal(C, emu.mm(A, B))
    assert len(t) == 4 and all(x >= 0 for x in t) and t[1] > 0


def test_argument_errors(emu):
    A = torch.randn(8, 16, dtype=torch.float64, device="cuda")
    with pytest.raises(RuntimeError, match="bits must be in"):
        emu.mm(A, A, bits=15)
    with pytest.raises(RuntimeError, match="too many primes"):
        emu.ops.fp64_emu_mm(torch.empty(8, 8, dtype=torch.float64, device="cuda"), A, A,
                            torch.arange(2, 23, dtype=torch.int32), torch.zeros(1), torch.zeros(1), True, 53,
                            True)
    with pytest.raises(RuntimeError, match="f64 CUDA"):
        emu.mm(A.float(), A.float())
    with pytest.raises(RuntimeError, match="K bound for int32"):
        emu.ops.fp64_emu_mm_nt(torch.empty(1, 1, dtype=torch.float64, device="cuda"),
                               torch.zeros(1, 131072, dtype=torch.float64, device="cuda"),
                               torch.zeros(131072, 1, dtype=torch.float64, device="cuda"),
                               *emu._tables(14), True, 53, True)


def test_empty_and_zero(emu):
    A = torch.zeros(0, 16, dtype=torch.float64, device="cuda")
    B = torch.randn(5, 16, dtype=torch.float64, device="cuda")
    assert emu.mm(A, B).shape == (0, 5)
    # empty inner dimension: C = 0, as for torch.matmul
    for kind, a, b in (("mm_nt", (4, 0), (0, 3)), ("mm", (4, 0), (3, 0)), ("bmm_nt", (2, 4, 0), (2, 0, 3))):
        C = getattr(emu, kind)(torch.empty(a, dtype=torch.float64, device="cuda"),
                               torch.empty(b, dtype=torch.float64, device="cuda"))
        assert C.shape[-2:] == (4, 3) and not C.any()
    Z = torch.zeros(7, 9, dtype=torch.float64, device="cuda")
    assert torch.equal(emu.mm(Z, torch.zeros(3, 9, dtype=torch.float64, device="cuda")),
                       torch.zeros(7, 3, dtype=torch.float64, device="cuda"))


def test_status_word_clean(emu):
    _check_status(emu)


@pytest.mark.parametrize("dist", ["randn", "wide16", "illcond40", "spike"])
def test_default_accuracy_vs_double_double(emu, dist):
    A, Bt = make(dist, 128, 4096 if dist == "randn" else 512, 128, seed=7)
    hi, lo = dd_matmul(A, Bt)
    C = emu.mm_nt(cuda(A), cuda(Bt)).cpu().numpy()
    assert correct_bits(C, hi, lo) >= 52.5


# -------------------------------------------- against the reference build --
REF_CASES = [
    ("mm_nt", (128, 4096, 128), "randn", {}),
    ("mm_nt", (129, 4095, 127), "wide16", {}),
    ("mm", (256, 1000, 200), "illcond40", {}),
    ("mm", (96, 2048, 64), "spike", {"nprimes": 13, "corr": False}),
    ("mm_nt", (64, 300, 50), "randn", {"exact": False}),
    ("mm_nt", (80, 500, 60), "wide8", {"bits": 44}),
    ("mm", (64, 512, 48), "int20", {"nprimes": 13, "corr": False}),
]


@pytest.mark.parametrize("case", REF_CASES, ids=lambda c: f"{c[0]}-{c[2]}-{c[3]}")
def test_bitexact_vs_reference(emu, ref, case):
    kind, (M, K, N), dist, kw = case
    nt = kind.endswith("_nt")
    A, B = make(dist, M, K, N, seed=11 + M, nt=nt)
    Ad, Bd = cuda(A), cuda(B)
    mine = getattr(emu, kind)(Ad, Bd, **kw)
    theirs = getattr(ref, kind)(Ad, Bd, **kw)
    assert same_bits(mine.cpu().numpy(), theirs.cpu().numpy())


def test_bitexact_vs_reference_batched(emu, ref):
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(4, 128, 512, dtype=torch.float64, device="cuda", generator=g)
    B = torch.randn(4, 96, 512, dtype=torch.float64, device="cuda", generator=g)
    assert torch.equal(emu.bmm(A, B), ref.bmm(A, B))
    Bt = torch.randn(4, 512, 96, dtype=torch.float64, device="cuda", generator=g)
    assert torch.equal(emu.bmm_nt(A, Bt), ref.bmm_nt(A, Bt))


def test_bitexact_vs_reference_deep_k(emu, ref):
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(24, 140_000, dtype=torch.float64, device="cuda", generator=g)
    B = torch.randn(16, 140_000, dtype=torch.float64, device="cuda", generator=g)
    assert torch.equal(emu.mm(A, B), ref.mm(A, B))


def test_bitexact_vs_reference_nonfinite(emu, ref):
    g = torch.Generator(device="cuda").manual_seed(10)
    A = torch.randn(40, 256, dtype=torch.float64, device="cuda", generator=g)
    B = torch.randn(30, 256, dtype=torch.float64, device="cuda", generator=g)
    A[3, 7] = float("inf")
    A[5, 9] = float("nan")
    A[6] *= 1e300
    B[2, 4] = -float("inf")
    mine = emu.mm(A, B).cpu().numpy()
    theirs = ref.mm(A, B).cpu().numpy()
    assert same_bits(mine, theirs)


def test_bounded_wait_runs_out_and_reports(emu):
    # failure detection without a fault: one device thread waits, through the
    # GEMM's bounded wait, on a barrier that nothing arrives at; the wait runs
    # out, its site code lands in the status word, and the context stays usable
    import time
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    t0 = time.perf_counter()
    st = emu.ops.fp64_emu_wait_selftest(ws, 50_000_000)          # 50 ms
    dt = time.perf_counter() - t0
    assert st == 9
    assert 0.04 < dt < 10.0
    assert emu.ops.fp64_emu_status(ws) == 9
    torch.manual_seed(21)
    A = torch.randn(200, 300, dtype=torch.float64, device="cuda")
    B = torch.randn(150, 300, dtype=torch.float64, device="cuda")
    C = emu.mm(A, B)
    torch.cuda.synchronize()
    assert torch.allclose(C, A @ B.t(), rtol=1e-12, atol=1e-12)
    with pytest.raises(RuntimeError):
        emu.ops.fp64_emu_wait_selftest(ws, 0)
