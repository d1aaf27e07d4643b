"""Chunked products: a call that runs extraction, GEMM and reconstruction
together cuts the product into chunks (rows of A and C, or batch members) and
overlaps the chunks' phases on library streams.  Every chunked product must be
bit-identical to the same product run unchunked (F64E_PIPE_CHUNK=0) and to the
CPU oracle.  F64E_PIPE_CHUNK=<n> forces the chunk extent, so ragged and
many-chunk cases run at sizes the oracle finishes in seconds."""
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


class chunk:
    """Set F64E_PIPE_CHUNK (and F64E_PIPE_COLS) for the duration of a block;
    None leaves the library's default policy."""

    def __init__(self, n, cols=None):
        self.vals = {"F64E_PIPE_CHUNK": n, "F64E_PIPE_COLS": cols}

    def __enter__(self):
        self.old = {k: os.environ.get(k) for k in self.vals}
        for k, v in self.vals.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = str(v)

    def __exit__(self, *a):
        for k, v in self.old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _pair(kind, batch, M, K, N, dist, seed):
    nt = kind.endswith("_nt")
    if batch == 1:
        A, B = make(dist, M, K, N, seed=seed, nt=nt)
    else:
        pairs = [make(dist, M, K, N, seed=seed + b, nt=nt) for b in range(batch)]
        A, B = np.stack([p[0] for p in pairs]), np.stack([p[1] for p in pairs])
    return A, B


CASES = [
    # (kind, batch, M, K, N, dist, chunk or (chunk, column block), kwargs)
    ("mm_nt", 1, 1000, 700, 300, "randn", 384, {}),          # 3 chunks, the last ragged
    ("mm_nt", 1, 1000, 700, 300, "randn", (384, 96), {}),    # + column blocks 96, 96, 96, 12 of row chunk 0
    ("mm_nt", 1, 777, 513, 259, "wide16", (256, 64), {}),    # blocks widened to 80 (at most four)
    ("mm", 1, 1030, 900, 520, "illcond40", (512, 256), {}),
    ("mm", 1, 600, 1000, 200, "spike", (300, 48), {"nprimes": 13, "corr": False}),
    ("mm_nt", 1, 777, 513, 259, "wide16", 128, {}),          # 7 chunks of single-CTA GEMMs
    ("mm", 1, 1030, 900, 520, "illcond40", 512, {}),
    ("mm", 1, 600, 1000, 200, "spike", 256, {"nprimes": 13, "corr": False}),
    ("mm_nt", 1, 640, 600, 333, "randn", 256, {"exact": False}),
    ("mm_nt", 1, 520, 300, 90, "wide8", 200, {"bits": 40}),
    ("mm", 1, 300, 200, 100, "randn", 100, {"nprimes": 20}),
    ("bmm_nt", 10, 60, 200, 150, "illcond", 3, {}),          # member chunks 3, 3, 3, 1
    ("bmm", 7, 90, 333, 77, "randn", 2, {}),
    ("mm_nt", 1, 512, 70000, 64, "randn", 256, {}),          # K > 65536: two correction planes
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[1]}x{c[2]}x{c[3]}x{c[4]}-{c[5]}-c{c[6]}")
def test_chunked_matches_unchunked_and_oracle(emu, oracle_mod, case):
    kind, batch, M, K, N, dist, per, kw = case
    per, cols = per if isinstance(per, tuple) else (per, 0)
    A, B = _pair(kind, batch, M, K, N, dist, seed=M + K + N)
    fn = getattr(emu, kind)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    with chunk(0):
        flat = fn(Ad, Bd, **kw)
    with chunk(per, cols):
        chunked = fn(Ad, Bd, **kw)
    torch.cuda.synchronize()
    assert torch.equal(chunked, flat)
    W = oracle_mod.emu(A, B, b_nt=kind.endswith("_nt"), **kw)
    assert same_bits(chunked.cpu().numpy(), W)


@pytest.mark.parametrize("kind,shape", [("mm_nt", (4096, 2048, 1024)), ("mm", (2304, 1024, 2048)),
                                        ("mm_nt", (2048, 512, 4100)), ("bmm_nt", (8, 256, 512, 384))])
def test_default_chunking_matches_unchunked(emu, kind, shape):
    # sizes where the default policy chunks (M >= 2048, or >= 4 members of >= 2048 rows in all)
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    if kind == "bmm_nt":
        b, M, K, N = shape
        A = torch.randn(b, M, K, dtype=torch.float64, device="cuda", generator=g)
        B = torch.randn(b, K, N, dtype=torch.float64, device="cuda", generator=g)
    else:
        M, K, N = shape
        A = torch.randn(M, K, dtype=torch.float64, device="cuda", generator=g)
        B = torch.randn((K, N) if kind == "mm_nt" else (N, K), dtype=torch.float64, device="cuda", generator=g)
    fn = getattr(emu, kind)
    with chunk(None):
        auto = fn(A, B)
    with chunk(0):
        flat = fn(A, B)
    torch.cuda.synchronize()
    assert torch.equal(auto, flat)


def test_gemm_events_count_chunk_launches(emu):
    A = torch.randn(1000, 640, dtype=torch.float64, device="cuda")
    Bt = torch.randn(640, 300, dtype=torch.float64, device="cuda")
    pr = emu._tables(14)[0]
    ws = torch.empty(emu.ops.fp64_emu_workspace_bytes(A, Bt, pr, True, True), dtype=torch.uint8, device="cuda")
    out = torch.empty(1000, 300, dtype=torch.float64, device="cuda")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
    for e in ev:
        e.record()
    with chunk(256, 0):
        emu.ops.fp64_emu_gemm_ws(out, ws, A, Bt, pr, True, True, 53, True, 1, 0)
        n = emu.ops.fp64_emu_gemm_ws_ev(out, ws, A, Bt, pr, True, True, 53, True, 14, 0, [e.cuda_event for e in ev])
    torch.cuda.synchronize()
    assert n == 4
    assert all(ev[2 * i].elapsed_time(ev[2 * i + 1]) > 0 for i in range(4))
    with chunk(256, 128):   # row chunk 0 in three column blocks: 3 + 3 GEMM launches
        n = emu.ops.fp64_emu_gemm_ws_ev(out, ws, A, Bt, pr, True, True, 53, True, 14, 0, [e.cuda_event for e in ev])
    torch.cuda.synchronize()
    assert n == 6
    with chunk(0):
        assert torch.equal(out, emu.mm_nt(A, Bt))
    assert emu.ops.fp64_emu_status(ws) == 0


def test_chunked_product_in_a_cuda_graph(emu):
    A = torch.randn(1100, 500, dtype=torch.float64, device="cuda")
    Bt = torch.randn(500, 260, dtype=torch.float64, device="cuda")
    with chunk(300, 96):
        for _ in range(2):
            emu.mm_nt(A, Bt)                          # eager calls first: they create the library streams
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            got = emu.mm_nt(A, Bt)
        A.copy_(torch.randn(1100, 500, dtype=torch.float64, device="cuda"))
        Bt.copy_(torch.randn(500, 260, dtype=torch.float64, device="cuda"))
        g.replay()
        torch.cuda.synchronize()
        want = emu.mm_nt(A, Bt)
    with chunk(0):
        flat = emu.mm_nt(A, Bt)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(got, flat)


class envset:
    """Set arbitrary environment switches for the duration of a block."""

    def __init__(self, **kv):
        self.kv = kv

    def __enter__(self):
        self.old = {k: os.environ.get(k) for k in self.kv}
        for k, v in self.kv.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = str(v)

    def __exit__(self, *a):
        for k, v in self.old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


@pytest.mark.parametrize("head", [0, 2, 3])
def test_head_depth_same_bits(emu, head):
    # A chunks extracted before the first GEMM (F64E_PIPE_HEAD): 0 = all, n = n chunks;
    # 6144 rows = chunks of 1024, 2048, 2048, 1024 with the half-size ends
    g = torch.Generator(device="cuda").manual_seed(31)
    A = torch.randn(6144, 700, dtype=torch.float64, device="cuda", generator=g)
    Bt = torch.randn(700, 900, dtype=torch.float64, device="cuda", generator=g)
    with envset(F64E_PIPE_HEAD=None):
        want = emu.mm_nt(A, Bt)
    with envset(F64E_PIPE_HEAD=head):
        got = emu.mm_nt(A, Bt)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("ends", [0, 1])
def test_equal_or_half_ends_same_bits(emu, ends):
    g = torch.Generator(device="cuda").manual_seed(32)
    A = torch.randn(8192, 300, dtype=torch.float64, device="cuda", generator=g)   # 4 x 2048 or 1024, 3 x 2048, 1024
    B = torch.randn(500, 300, dtype=torch.float64, device="cuda", generator=g)
    with envset(F64E_PIPE_CHUNK=0):
        want = emu.mm(A, B)
    with envset(F64E_PIPE_ENDS=ends):
        got = emu.mm(A, B)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_single_cta_gemm_same_bits(emu):
    # F64E_GEMM_SINGLE=1: every product on the one-CTA GEMM instead of the CTA pair
    g = torch.Generator(device="cuda").manual_seed(33)
    for (M, K, N) in [(600, 1000, 520), (2304, 512, 700)]:
        A = torch.randn(M, K, dtype=torch.float64, device="cuda", generator=g)
        Bt = torch.randn(K, N, dtype=torch.float64, device="cuda", generator=g)
        with envset(F64E_GEMM_SINGLE=None):
            want = emu.mm_nt(A, Bt)
        with envset(F64E_GEMM_SINGLE=1):
            got = emu.mm_nt(A, Bt)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
