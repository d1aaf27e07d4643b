"""bench.py's host-side pieces on the CPU: the workload table, seeded inputs,
the peak and traffic figures it reads from committed files, and the launch
count it claims per step."""
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
    assert src in ("measured", "fallback") and 0 < sus <= burst
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
