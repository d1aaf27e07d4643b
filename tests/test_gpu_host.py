"""Host-resident products (fp64_emu.mm_nt_host and friends, C ABI
f64e_gemm_host): operands copied in, every finished block of the result copied
back while later blocks compute.  The result must be bit-identical to the
device-resident product for every chunking (row chunks, column blocks of the
first row chunk, member chunks), for page-locked and pageable buffers."""
import os

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def emu():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    import fp64_emu
    return fp64_emu


class env:
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


def _host(t, pinned):
    h = t.cpu()
    return h.pin_memory() if pinned else h


CASES = [
    # kind, shape, chunk, cols
    ("mm_nt", (1500, 700, 900), 512, 0),
    ("mm_nt", (1500, 700, 900), 512, 256),       # column blocks: strided copies of row chunk 0
    ("mm_nt", (2304, 1024, 2048), None, None),   # default policy
    ("mm", (1030, 900, 520), 384, 0),
    ("mm", (300, 200, 100), 0, 0),               # unchunked
    ("bmm_nt", (9, 130, 300, 140), 2, 0),
    ("bmm", (5, 64, 100, 80), 0, 0),
]


@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{'x'.join(map(str, c[1]))}-c{c[2]}-b{c[3]}")
def test_host_product_matches_device_product(emu, case, pinned):
    kind, shape, per, cols = case
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    if kind.startswith("bmm"):
        b, M, K, N = shape
        A = torch.randn(b, M, K, dtype=torch.float64, device="cuda", generator=g)
        B = torch.randn((b, K, N) if kind.endswith("_nt") else (b, N, K), dtype=torch.float64, device="cuda",
                        generator=g)
    else:
        M, K, N = shape
        A = torch.randn(M, K, dtype=torch.float64, device="cuda", generator=g)
        B = torch.randn((K, N) if kind.endswith("_nt") else (N, K), dtype=torch.float64, device="cuda",
                        generator=g)
    with env(F64E_PIPE_CHUNK=per, F64E_PIPE_COLS=cols):
        want = getattr(emu, kind)(A, B).cpu()
        got = getattr(emu, kind + "_host")(_host(A, pinned), _host(B, pinned))
    assert got.device.type == "cpu"
    assert torch.equal(got, want)


def test_host_product_into_given_out(emu):
    A = torch.randn(700, 300, dtype=torch.float64).pin_memory()
    Bt = torch.randn(300, 200, dtype=torch.float64).pin_memory()
    out = torch.full((700, 200), float("nan"), dtype=torch.float64).pin_memory()
    r = emu.mm_nt_host(A, Bt, out=out, nprimes=13, corr=False)
    assert r.data_ptr() == out.data_ptr()
    assert torch.equal(out, emu.mm_nt(A.cuda(), Bt.cuda(), nprimes=13, corr=False).cpu())


def test_host_product_rejects_device_tensors(emu):
    A = torch.randn(8, 8, dtype=torch.float64, device="cuda")
    with pytest.raises((RuntimeError, NotImplementedError)):
        emu.mm_nt_host(A, A)


def test_host_stream_matches_device_products(emu):
    # a stream of products with different operands (and a shape change midway):
    # every result bit-identical to the device call
    g = torch.Generator(device="cuda").manual_seed(5)
    jobs = []
    for i in range(5):
        M, K, N = (600, 300, 200) if i < 3 else (256, 128, 96)
        A = torch.randn(M, K, dtype=torch.float64, device="cuda", generator=g)
        Bt = torch.randn(K, N, dtype=torch.float64, device="cuda", generator=g)
        jobs.append((A, Bt))
    hs = emu.HostStream("mm_nt", depth=2)
    outs = []
    for A, Bt in jobs:
        out = torch.empty(A.size(0), Bt.size(1), dtype=torch.float64).pin_memory()
        hs.submit(A.cpu().pin_memory(), Bt.cpu().pin_memory(), out)
        outs.append(out)
    hs.synchronize()
    for (A, Bt), out in zip(jobs, outs):
        assert torch.equal(out, emu.mm_nt(A, Bt).cpu())


def test_host_stream_batched(emu):
    A = torch.randn(6, 64, 200, dtype=torch.float64)
    B = torch.randn(6, 80, 200, dtype=torch.float64)
    out = torch.empty(6, 64, 80, dtype=torch.float64)
    hs = emu.HostStream("bmm", depth=3)
    hs.submit(A, B, out)
    hs.synchronize()
    assert torch.equal(out, emu.bmm(A.cuda(), B.cuda()).cpu())


def test_host_stream_depth_one_many_small(emu):
    # one slot reused by every product: each one's copies wait for the previous
    # product to read its operands and for its result to leave the device
    g = torch.Generator(device="cuda").manual_seed(9)
    hs = emu.HostStream("mm_nt", depth=1)
    jobs, outs = [], []
    for i in range(12):
        A = torch.randn(96, 300, dtype=torch.float64, device="cuda", generator=g)
        Bt = torch.randn(300, 80, dtype=torch.float64, device="cuda", generator=g)
        out = torch.empty(96, 80, dtype=torch.float64).pin_memory()
        hs.submit(A.cpu().pin_memory(), Bt.cpu().pin_memory(), out)
        jobs.append((A, Bt))
        outs.append(out)
    hs.synchronize()
    for (A, Bt), out in zip(jobs, outs):
        assert torch.equal(out, emu.mm_nt(A, Bt).cpu())


def test_host_stream_rejects_strided_out(emu):
    hs = emu.HostStream("mm_nt")
    A = torch.randn(16, 32, dtype=torch.float64)
    Bt = torch.randn(32, 8, dtype=torch.float64)
    out = torch.empty(8, 16, dtype=torch.float64).t()
    with pytest.raises(RuntimeError):
        hs.submit(A, Bt, out)
