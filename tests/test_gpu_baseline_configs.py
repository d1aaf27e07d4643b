"""Bit-identity at the benchmark configurations themselves (C1-C5), on the
inputs bench.py generates (same seeded device generators):

  * our products against the reference's own kernels (oracle/_ref, built from
    the reference sources) on the whole output, torch.equal;
  * C3 (exact integers, U[-2^20, 2^20], K = 4096) also against the exact
    integer product: every partial sum is an integer below 2^52, so a float64
    GEMM of these operands is exact, and a slice is checked in int64 on the
    CPU as well;
  * the multi-GPU partitions (2-D blocks of C, batch split) emulated on one
    GPU: every rank's block is computed by its own ShardedProduct, the MAX
    all-reduce of the sizing maxima is done here by taking the maximum over
    the blocks, and each block must equal the same block of the
    unpartitioned product bit for bit.  This is the exchange the NCCL path
    performs (fp64_emu.dist.sized_protocol), so the result covers the
    partition arithmetic without a second GPU.

The reference's known-answer tests pin small shapes; these pin the
configurations the throughput figures are quoted on."""
import os
import sys

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


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


def _inputs(name, seed=0):
    import bench
    kind, batch, M, N, K, dist, nprimes, corr = bench.WORKLOADS[name]
    A, B = bench.make_inputs(dist, batch, M, N, K, kind.endswith("_nt"), torch.device("cuda"), seed=seed)
    kw = {k: v for k, v in (("nprimes", nprimes), ("corr", corr)) if v is not None}
    return kind, A, B, kw


def _free():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C3r", "C4", "C5"])
def test_baseline_config_bit_identical_to_reference(emu, ref, name):
    kind, A, B, kw = _inputs(name)
    mine = getattr(emu, kind)(A, B, **kw)
    _free()
    theirs = getattr(ref, kind)(A, B, **kw)
    same = torch.equal(mine.view(torch.int64), theirs.view(torch.int64))
    ndiff = 0 if same else int((mine.view(torch.int64) != theirs.view(torch.int64)).sum())
    del mine, theirs, A, B
    _free()
    assert same, f"{name}: {ndiff} elements differ from the reference"


@pytest.mark.parametrize("name", ["C3", "C3r"])
def test_exact_integer_config_equals_integer_product(emu, name):
    kind, A, B, kw = _inputs(name)
    assert kind == "mm"
    C = emu.mm(A, B, **kw)
    # |a b| <= 2^40 and K = 4096: every partial sum is an integer below 2^52,
    # so the float64 GEMM below is exact in any summation order
    exact = A @ B.t()
    assert torch.equal(C, exact)
    rows = 48
    ai, bi = A[:rows].cpu().long(), B.cpu().long()
    assert torch.equal(C[:rows].cpu().long(), ai @ bi.t())
    del C, exact, A, B
    _free()


def _partitioned_blocks(emu, kind, A, B, kw, world):
    """Every rank's block of the partitioned product, one GPU, with the
    sizing maxima exchanged as the MAX all-reduce would."""
    from fp64_emu.dist import PHASE_COMPUTE, PHASE_SIZING, ShardedProduct, block_range, rank_block
    nt = kind.endswith("_nt")
    batched = A.dim() == 3
    K = A.size(-1)
    parts = []
    for r in range(world):
        if batched:
            b0, b1 = block_range(A.size(0), world, r)
            Al, Bl = A[b0:b1], B[b0:b1]
            slab = A.size(0) * (B.size(2) if nt else B.size(1))
            shape = (b1 - b0, A.size(1), B.size(2) if nt else B.size(1))
            where = (slice(b0, b1),)
        else:
            N = B.size(1) if nt else B.size(0)
            (r0, r1), (c0, c1) = rank_block(r, world, A.size(0), N)
            Al, Bl = A[r0:r1], (B[:, c0:c1] if nt else B[c0:c1])
            slab = N
            shape = (r1 - r0, c1 - c0)
            where = (slice(r0, r1), slice(c0, c1))
        parts.append((Al, Bl, slab, shape, where))
    # sizing of every block; the all-reduce: the maximum over the blocks
    maxima = []
    for Al, Bl, slab, shape, _ in parts:
        sp = ShardedProduct(Al, Bl, nt, slab, K, **kw)
        out = torch.empty(shape, dtype=torch.float64, device="cuda")
        sp._phase(out, PHASE_SIZING)
        maxima.append(sp.maxlg.clone())
        del sp
    g = torch.stack(maxima).max(0).values
    for Al, Bl, slab, shape, where in parts:
        sp = ShardedProduct(Al, Bl, nt, slab, K, **kw)
        out = torch.empty(shape, dtype=torch.float64, device="cuda")
        sp._phase(out, PHASE_SIZING)
        sp.maxlg.copy_(g)
        sp._phase(out, PHASE_COMPUTE)
        yield where, out
        del sp, out


@pytest.mark.parametrize("name,world", [("C2", 2), ("C2", 8), ("C4", 8), ("C5", 8), ("C5", 4)])
def test_partitioned_blocks_bit_identical_on_one_gpu(emu, name, world):
    kind, A, B, kw = _inputs(name)
    full = getattr(emu, kind)(A, B, **kw)
    _free()
    bad = []
    for where, blk in _partitioned_blocks(emu, kind, A, B, kw, world):
        if not torch.equal(blk.view(torch.int64), full[where].view(torch.int64)):
            bad.append(where)
    del full, A, B
    _free()
    assert not bad, f"{name} on {world} ranks: blocks {bad} differ from the unpartitioned product"


def test_block_check_sees_a_changed_maximum(emu):
    # the emulated all-reduce matters: a block sized with only its own maxima
    # differs from the unpartitioned product when the maxima differ by rank
    from fp64_emu.dist import PHASE_COMPUTE, PHASE_SIZING, ShardedProduct
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(512, 4096, dtype=torch.float64, device="cuda", generator=g)
    Bt = torch.randn(4096, 300, dtype=torch.float64, device="cuda", generator=g)
    A[256:] = 1.0        # larger scaled row norms in the second row block only
    full = emu.mm_nt(A, Bt)
    sp = ShardedProduct(A[:256].contiguous(), Bt, True, 300, 4096)
    out = torch.empty(256, 300, dtype=torch.float64, device="cuda")
    sp._phase(out, PHASE_SIZING)
    sp._phase(out, PHASE_COMPUTE)   # no exchange: this block's own maxima
    assert not torch.equal(out, full[:256])
