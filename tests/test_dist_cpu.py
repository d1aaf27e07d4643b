"""Multi-rank host logic of the partitioned product, on CPU with gloo ranks.

Each rank takes its block of the 2-D partition (or its batch slice), runs the
sizing phase (here: the CPU oracle), joins the MAX all-reduce of the two
operand maxima through fp64_emu.dist.sized_protocol -- the same function the
GPU path uses -- and computes its block.  The assembled result must be
bit-identical to the single-process product, which is what makes the
partitioned GPU runs match a single-GPU run."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, case, outdir):
    for p in (ROOT, os.path.join(ROOT, "fp64-emu_b200"), os.path.join(ROOT, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from oracle import oracle as O
        from helpers import make
        from fp64_emu import dist as proto_mod
        proto = vars(proto_mod)
        kind, M, K, N, batch, dname = case
        if batch == 1:
            A, Bt = make(dname, M, K, N, seed=3, nt=True)
            (r0, r1), (c0, c1) = proto["rank_block"](rank, world, M, N)
            Al, Bl = A[r0:r1], np.ascontiguousarray(Bt[:, c0:c1])
            slab = N
        else:
            pairs = [make(dname, M, K, N, seed=40 + b, nt=True) for b in range(batch)]
            A = np.stack([p[0] for p in pairs])
            Bt = np.stack([p[1] for p in pairs])
            b0, b1 = proto["block_range"](batch, world, rank)
            Al, Bl = A[b0:b1], Bt[b0:b1]
            slab = batch * N
        maxlg = torch.zeros(2, dtype=torch.float32)

        def sizing():
            _, mo = O.emu_shard(Al, Bl, b_nt=True, slab_cols=slab, sizing_only=True)
            maxlg.copy_(torch.from_numpy(mo))

        proto["sized_protocol"](sizing, maxlg)
        C, _ = O.emu_shard(Al, Bl, b_nt=True, slab_cols=slab, maxlg_in=maxlg.numpy())
        np.save(os.path.join(outdir, f"block{rank}.npy"), C)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,case", [
    (2, ("mm_nt", 64, 300, 48, 1, "wide16")),
    (4, ("mm_nt", 48, 700, 70, 1, "randn")),
    (2, ("bmm_nt", 20, 200, 24, 6, "illcond")),
])
def test_partitioned_blocks_match_single_process(world, case, tmp_path, oracle_mod):
    kind, M, K, N, batch, dname = case
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, case, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    from helpers import make
    from fp64_emu import dist as proto_mod
    proto = vars(proto_mod)
    if batch == 1:
        A, Bt = make(dname, M, K, N, seed=3, nt=True)
        full = oracle_mod.emu(A, Bt, b_nt=True)
        got = np.empty_like(full)
        for r in range(world):
            (r0, r1), (c0, c1) = proto["rank_block"](r, world, M, N)
            got[r0:r1, c0:c1] = np.load(tmp_path / f"block{r}.npy")
    else:
        pairs = [make(dname, M, K, N, seed=40 + b, nt=True) for b in range(batch)]
        A = np.stack([p[0] for p in pairs])
        Bt = np.stack([p[1] for p in pairs])
        full = oracle_mod.emu(A, Bt, b_nt=True)
        got = np.concatenate([np.load(tmp_path / f"block{r}.npy") for r in range(world)])
    assert np.array_equal(got.view(np.int64), full.view(np.int64))


def test_local_sizing_alone_can_differ():
    """Without the all-reduce a rank could pick a different operand width: the
    collective is required, not decorative."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from helpers import make
    from oracle import oracle as O
    A, Bt = make("spike", 64, 300, 48, seed=3, nt=True)
    A[32:] = 1.0   # flat rows: larger scaled 2-norms than the spiky half
    _, m_lo = O.emu_shard(A[:32], Bt, b_nt=True, sizing_only=True)
    _, m_all = O.emu_shard(A, Bt, b_nt=True, sizing_only=True)
    assert m_lo[0] < m_all[0]
    own = O.emu_shard(A[:32], Bt, b_nt=True)[0]
    shared = O.emu_shard(A[:32], Bt, b_nt=True, maxlg_in=m_all)[0]
    full = O.emu(A, Bt, b_nt=True)
    assert np.array_equal(shared, full[:32])
    assert not np.array_equal(own, full[:32])


def test_grid_shapes():
    from fp64_emu import dist as proto_mod
    proto = vars(proto_mod)
    assert [proto["grid_shape"](w) for w in (1, 2, 4, 8)] == [(1, 1), (1, 2), (2, 2), (2, 4)]
    blocks = [proto["rank_block"](r, 8, 8192, 8192) for r in range(8)]
    cover = np.zeros((8, 8), dtype=int)
    for (r0, r1), (c0, c1) in blocks:
        cover[r0 // 1024:r1 // 1024, c0 // 1024:c1 // 1024] += 1
    assert (cover == 1).all()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("shape", [(8192, 8192, 8192), (700, 900, 1500), (5, 3, 17), (1030, 520, 333)])
@pytest.mark.parametrize("b_kn", [True, False])
def test_host_share_ranges_partition_each_block(world, shape, b_kn):
    # the host shares of the ranks of one grid row tile that row's block of A,
    # and those of one grid column tile that column's block of B, exactly once
    from fp64_emu.dist import grid_shape, host_share_ranges, rank_block
    M, N, K = shape
    pr, pc = grid_shape(world)
    for i in range(pr):
        ranks = [i * pc + j for j in range(pc)]
        (r0, r1), _ = rank_block(ranks[0], world, M, N)
        rows = sorted(host_share_ranges(r, world, M, N, K, b_kn)[0] for r in ranks)
        covered = [x for a0, a1 in rows for x in range(a0, a1)]
        assert covered == list(range(r0, r1))
    for j in range(pc):
        ranks = [i * pc + j for i in range(pr)]
        _, (c0, c1) = rank_block(ranks[0], world, M, N)
        ext = K if b_kn else c1 - c0
        parts = sorted(host_share_ranges(r, world, M, N, K, b_kn)[1] for r in ranks)
        covered = [x for b0, b1 in parts for x in range(b0, b1)]
        assert covered == list(range(ext))


def _failing_worker(rank, world, port, outdir):
    # rank 1 leaves between steps (before its next collective); rank 0's next
    # collective -- the MAX all-reduce of the sizing protocol -- must end with
    # an error within the short process-group timeout instead of waiting
    for p in (ROOT, os.path.join(ROOT, "fp64-emu_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import time
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    from fp64_emu import dist as proto_mod
    maxlg = torch.zeros(2, dtype=torch.float32)
    # one good step on both ranks
    proto_mod.sized_protocol(lambda: maxlg.fill_(float(rank)), maxlg)
    assert float(maxlg[0]) == world - 1
    if rank == 1:
        os._exit(3)                  # the rank dies between steps
    t0 = time.perf_counter()
    try:
        proto_mod.sized_protocol(lambda: maxlg.fill_(0.0), maxlg)
        outcome = "no error"
    except Exception as e:  # noqa: BLE001
        outcome = "error " + type(e).__name__
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(f"{outcome} {time.perf_counter() - t0:.1f}")
    os._exit(0)                      # no teardown collective with a dead peer


def test_rank_failure_ends_the_next_collective_with_an_error(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_failing_worker, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(120)
    codes = [p.exitcode for p in ctx.processes]
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    assert codes == [0, 3]
    outcome, secs = (tmp_path / "rank0.txt").read_text().rsplit(" ", 1)
    assert outcome.startswith("error") and float(secs) < 60


def _lonely_worker(rank, world, port, outdir):
    # rank 0 of a world of 2 whose peer never starts: the rendezvous must end
    # with an error within its timeout instead of waiting for good
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import time
    from datetime import timedelta
    t0 = time.perf_counter()
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=timedelta(seconds=3))
        outcome = "joined"
    except Exception as e:  # noqa: BLE001
        outcome = "error " + type(e).__name__
    with open(os.path.join(outdir, "lonely.txt"), "w") as f:
        f.write(f"{outcome} {time.perf_counter() - t0:.1f}")
    os._exit(0)


def test_rank_that_never_joins_ends_the_rendezvous_with_an_error(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_lonely_worker, args=(1, port, str(tmp_path)), nprocs=1, join=False,
                             start_method="spawn")
    ctx.processes[0].join(120)
    if ctx.processes[0].is_alive():
        ctx.processes[0].kill()
    outcome, secs = (tmp_path / "lonely.txt").read_text().rsplit(" ", 1)
    assert outcome.startswith("error") and float(secs) < 60


def _mismatch_worker(rank, world, port, outdir):
    # the ranks disagree on the collective's shape (one of them built a
    # different product): the collective must fail on some rank, not hang
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    t = torch.zeros(2 if rank == 0 else 3, dtype=torch.float32)
    try:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        outcome = "no error"
    except Exception as e:  # noqa: BLE001
        outcome = "error " + type(e).__name__
    with open(os.path.join(outdir, f"mismatch{rank}.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)


def test_mismatched_collective_shapes_end_with_an_error(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_mismatch_worker, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(120)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    outcomes = [(tmp_path / f"mismatch{r}.txt").read_text() for r in range(2)
                if (tmp_path / f"mismatch{r}.txt").exists()]
    assert outcomes and any(o.startswith("error") for o in outcomes)
