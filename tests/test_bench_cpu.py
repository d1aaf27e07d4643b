"""bench.py's host-side pieces on the CPU: the workload table, seeded inputs,
the peak and traffic figures it reads from committed files, and the launch
count it claims per step."""
import json
import os
import sys

import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_workloads_cover_the_baseline_configs():
    assert {"C1", "C2", "C3", "C3r", "C4", "C5"} <= set(bench.WORKLOADS)
    assert bench.WORKLOADS["C2"][:5] == ("mm_nt", 1, 8192, 8192, 8192)
    assert bench.WORKLOADS["C5"][:5] == ("bmm_nt", 64, 1024, 1024, 1024)


@pytest.mark.parametrize("dist", ["randn", "unif", "int20", "wide30"])
@pytest.mark.parametrize("nt", [True, False])
def test_inputs_seeded_and_shaped(dist, nt):
    A, B = bench.make_inputs(dist, 1, 12, 10, 20, nt, "cpu", seed=3)
    A2, B2 = bench.make_inputs(dist, 1, 12, 10, 20, nt, "cpu", seed=3)
    assert A.shape == (12, 20) and B.shape == ((20, 10) if nt else (10, 20))
    assert A.dtype == torch.float64 and torch.equal(A, A2) and torch.equal(B, B2)
    if dist == "int20":
        assert torch.equal(A, A.round()) and A.abs().max() <= 2 ** 20
    Ab, Bb = bench.make_inputs(dist, 3, 4, 5, 6, nt, "cpu")
    assert Ab.shape == (3, 4, 6) and Bb.shape == ((3, 6, 5) if nt else (3, 5, 6))


def test_peaks_and_traffic_from_committed_files():
    sus, burst, src = bench.int8_peak_from_file()
    assert ("measured" in src or "fallback" in src) and 0 < sus <= burst
    t = bench.profiled_traffic_per_step()
    assert t is not None and 5e9 < t < 2e10   # DRAM bytes of the GEMM launches of one C2 step


def test_launch_count_claim():
    # mm_nt: two sizing launches; per chunk extraction of A, GEMM and
    # reconstruction; B extracted once for a single product
    assert bench.our_kernel_launches_per_step("mm_nt", 1, 5, 8192, 8192, 8192) == 2 + 15 + 1
    # mm: one sizing launch; a batch extracts B with every member chunk
    assert bench.our_kernel_launches_per_step("mm", 1, 1, 4096, 4096, 4096) == 1 + 3 + 1
    assert bench.our_kernel_launches_per_step("bmm_nt", 64, 8, 1024, 1024, 1024) == 2 + 24 + 8
    # a small unchunked product extracts both operands in one launch (C1)
    assert bench.our_kernel_launches_per_step("mm_nt", 1, 1, 128, 128, 4096) == 2 + 1 + 1 + 1


@pytest.mark.parametrize("world", [1, 2, 3, 4, 6, 8])
def test_partition_restatement_matches_the_library(world):
    # the reference arm hashes rank 0's block sample without importing the
    # library; its grid and block-0 arithmetic must be the library's
    from fp64_emu.dist import block_range, grid_shape, rank_block
    assert bench.grid_of(world) == grid_shape(world)
    for n in (1, 7, 1024, 8191, 16384):
        for parts in (1, 2, 3, 4, 8):
            if parts <= n:
                assert bench.first_block(n, parts) == block_range(n, parts, 0)[1]
    for name in ("C2", "C4", "C1"):
        kind, batch, M, N = bench.WORKLOADS[name][:4]
        b, R, Nc = bench.sample_region(name, world)
        (r0, r1), (c0, c1) = rank_block(0, world, M, N)
        assert b is None and (r0, c0) == (0, 0) and R == min(256, r1) and Nc == c1
    assert bench.sample_region("C5", world) == (0, 256, 1024)


def test_both_arms_print_the_same_config():
    for name in bench.WORKLOADS:
        c = bench.workload_config(name)
        assert set(c) == {"workload", "l2"} and c["workload"].startswith(name + ":")


def test_reference_arm_imports_nothing_of_this_repository():
    # the reference arm's modules: bench.py itself and dd_accuracy; neither
    # may pull in the fp64_emu package (which loads this repository's .so)
    import subprocess
    code = ("import sys; sys.path[:0] = [%r, %r]; import bench, dd_accuracy; "
            "assert 'fp64_emu' not in sys.modules, sorted(m for m in sys.modules if 'fp64' in m)"
            % (ROOT, os.path.join(ROOT, "fp64-emu_b200")))
    subprocess.run([sys.executable, "-c", code], check=True)


def test_sample_digest_is_of_the_sample_bytes():
    import hashlib
    C1 = torch.randn(128, 128, dtype=torch.float64)
    assert bench.sample_sha256(C1, "C1", 1) == hashlib.sha256(C1.numpy().tobytes()).hexdigest()
    C2 = torch.randn(8192, 64, dtype=torch.float64)   # a narrow stand-in: the sample is 256 rows x all columns
    assert bench.sample_sha256(C2, "C2", 1) == hashlib.sha256(C2[:256].contiguous().numpy().tobytes()).hexdigest()
    C5 = torch.randn(3, 300, 40, dtype=torch.float64)   # batches: member 0's first 256 rows
    assert bench.sample_sha256(C5, "C5", 8) == hashlib.sha256(C5[0, :256].contiguous().numpy().tobytes()).hexdigest()


def _gather_worker(rank, world, port, outdir):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        import bench
        got = bench.gather_ranks({"rank": rank, "ms_per_step": 1.0 + rank, "last_step_gemm_ms": [(0.1 * rank, 0.2)]})
        with open(os.path.join(outdir, f"r{rank}.json"), "w") as f:
            json.dump(got, f)
    finally:
        dist.destroy_process_group()


def test_per_rank_timeline_gather_on_gloo_ranks(tmp_path):
    # the per-rank timeline (--timeline-out) gathers every rank's record in rank order
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_gather_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        got = json.load(open(tmp_path / f"r{r}.json"))
        assert [g["rank"] for g in got] == [0, 1]
        assert [g["ms_per_step"] for g in got] == [1.0, 2.0]
