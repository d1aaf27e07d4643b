"""Partitioned products on several GPUs (NCCL): every rank's block of C must be
bit-identical to the same block of the single-GPU product.  Needs >= 2 GPUs
(skips otherwise).  NVLS stays off (NCCL_NVLS_ENABLE=0): the only collective is
a two-float MAX all-reduce."""
import os
import socket
import sys

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _flatten_second_half(A):
    # flat rows have larger scaled 2-norms than random ones, so the operand
    # maximum lives only on the rank holding them
    if A.dim() == 3:
        A[A.size(0) // 2:] = 1.0
    else:
        A[A.size(0) // 2:] = 1.0


def _worker(rank, world, port, case, outdir):
    for p in (ROOT, os.path.join(ROOT, "fp64-emu_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from fp64_emu.dist import block_range, bmm_nt_sharded, mm_nt_2d, rank_block
        kind, batch, M, K, N = case
        g = torch.Generator(device="cuda").manual_seed(123)
        shpA = (batch, M, K) if batch > 1 else (M, K)
        shpB = (batch, K, N) if batch > 1 else (K, N)
        A = torch.randn(shpA, dtype=torch.float64, device="cuda", generator=g)
        B = torch.randn(shpB, dtype=torch.float64, device="cuda", generator=g) * 2.0 ** 7
        _flatten_second_half(A)   # the ranks' local maxima differ: they must be shared
        if batch > 1:
            b0, b1 = block_range(batch, world, rank)
            C = bmm_nt_sharded(A[b0:b1].contiguous(), B[b0:b1].contiguous(), batch)
        else:
            (r0, r1), (c0, c1) = rank_block(rank, world, M, N)
            C = mm_nt_2d(A[r0:r1].contiguous(), B[:, c0:c1].contiguous(), N)
        torch.save(C.cpu(), os.path.join(outdir, f"block{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [("mm_nt", 1, 700, 1500, 900), ("bmm_nt", 6, 130, 400, 96)])
def test_partitioned_matches_single_gpu(case, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_worker, args=(world, _port(), case, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    import fp64_emu
    from fp64_emu.dist import rank_block
    kind, batch, M, K, N = case
    g = torch.Generator(device="cuda").manual_seed(123)
    shpA = (batch, M, K) if batch > 1 else (M, K)
    shpB = (batch, K, N) if batch > 1 else (K, N)
    A = torch.randn(shpA, dtype=torch.float64, device="cuda", generator=g)
    B = torch.randn(shpB, dtype=torch.float64, device="cuda", generator=g) * 2.0 ** 7
    _flatten_second_half(A)
    full = (fp64_emu.bmm_nt(A, B) if batch > 1 else fp64_emu.mm_nt(A, B)).cpu()
    blocks = [torch.load(tmp_path / f"block{r}.pt") for r in range(world)]
    if batch > 1:
        assert torch.equal(torch.cat(blocks), full)
    else:
        for r in range(world):
            (r0, r1), (c0, c1) = rank_block(r, world, M, N)
            assert torch.equal(blocks[r], full[r0:r1, c0:c1])


def _host_worker(rank, world, port, case, outdir):
    for p in (ROOT, os.path.join(ROOT, "fp64-emu_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from fp64_emu.dist import ShardedHostStream
        kind, M, K, N = case[:4]
        batch = case[4] if len(case) > 4 else 1
        g = torch.Generator().manual_seed(321)
        outs = []
        hs = ShardedHostStream(kind, M, N, K, depth=2, batch=batch)
        for step in range(3):   # three products through the rotating buffers
            A, B = _host_operands(kind, M, K, N, batch, step, g)
            a, b, c = hs.host_shares(A, B)
            hs.submit(a, b, c)
            outs.append(c)
        hs.synchronize()
        torch.save([o.clone() for o in outs], os.path.join(outdir, f"hblock{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _host_operands(kind, M, K, N, batch, step, g):
    """Host operands of one product of the stream test: A's second half of rows
    (of every member) flattened to 1.0, so the ranks' operand maxima differ
    and the MAX all-reduce decides the width."""
    b_kn = kind in ("mm_nt", "bmm_nt")
    shpA = (batch, M, K) if batch > 1 else (M, K)
    shpB = (K, N) if b_kn else (N, K)
    if batch > 1:
        shpB = (batch,) + shpB
    A = torch.randn(shpA, dtype=torch.float64, generator=g)
    B = torch.randn(shpB, dtype=torch.float64, generator=g) * 2.0 ** step
    if batch > 1:
        A[batch // 2:] = 1.0
    else:
        A[M // 2:] = 1.0
    return A, B


@pytest.mark.parametrize("case", [("mm_nt", 700, 1500, 900), ("mm", 520, 640, 333), ("bmm_nt", 200, 300, 150, 6),
                                  ("bmm", 130, 260, 70, 5)])
def test_sharded_host_stream_matches_single_gpu(case, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_host_worker, args=(world, _port(), case, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    import fp64_emu
    from fp64_emu.dist import rank_block
    kind, M, K, N = case[:4]
    batch = case[4] if len(case) > 4 else 1
    g = torch.Generator().manual_seed(321)
    blocks = [torch.load(tmp_path / f"hblock{r}.pt") for r in range(world)]
    for step in range(3):
        A, B = _host_operands(kind, M, K, N, batch, step, g)
        full = getattr(fp64_emu, kind)(A.cuda(), B.cuda()).cpu()
        if batch > 1:
            assert torch.equal(torch.cat([blocks[r][step] for r in range(world)]), full)
            continue
        for r in range(world):
            (r0, r1), (c0, c1) = rank_block(r, world, M, N)
            assert torch.equal(blocks[r][step], full[r0:r1, c0:c1])
