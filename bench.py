"""Throughput benchmark of the emulated-FP64 product (one JSON line on rank 0).

Default workload: mm_nt, M = N = K = 8192, float64
N(0,1) operands, default plan (14 moduli + 2 correction GEMMs).  A "step" is
one complete product.  With --gpus N > 1 (launched under torchrun) the
product is split into a 2-D grid of C blocks (2 -> 1x2, 4 -> 2x2, 8 -> 2x4):
each rank owns one block, the shared operand slices are distributed once
before timing, and the only collective in a step is the MAX all-reduce of
the two sizing maxima; total work is fixed, so scaling is "strong".

  value   device time (CUDA events, max over ranks) per step with inputs
          resident in HBM, as emulated FP64 TFLOP/s = 2MNK / t
  e2e     the same through the public API with each step's inputs copied
          from pinned host memory and the product copied back inside the
          timed region: fp64_emu.HostStream at N = 1 (copies and products of
          neighbouring steps overlapped), fp64_emu.dist.ShardedHostStream at
          N > 1
  roofline  the modular tensor-core GEMM (the dominant kernel): INT8 ops
          per launch / its average duration over the timed region
  accuracy  the metric's "correct bits vs dd": after timing, the product's
          first 256 rows (rank 0's block) against a double-double product,
          with cuBLAS DGEMM on the same sample (dd_accuracy, which imports
          torch only)
  output_sha256  SHA-256 of the same output sample's float64 bytes (both
          arms print it; equal digests mean bit-identical products); at
          N > 1 rank 0 also recomputes the whole product unpartitioned on one
          GPU after timing and compares every rank's block digest with it
          (blocks_bit_identical)

--impl reference runs the reference's own CUDA kernels (the build in
oracle/_ref, compiled from the reference sources; the reference has no CPU
implementation of this path) through its own Python API on one GPU, with
the same workload and protocol; under torchrun only rank 0 runs it.
"""
import argparse
import hashlib
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "fp64-emu_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "emulated FP64 TFLOP/s (2MNK/t) at n=8192"
UNIT = "TFLOP/s"
PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "residue_gemm_pair_mm_nt_8192.md")

WORKLOADS = {
    # name: (kind, batch, M, N, K, dist, nprimes, corr)
    "C1": ("mm_nt", 1, 128, 128, 4096, "randn", None, None),
    "C2": ("mm_nt", 1, 8192, 8192, 8192, "randn", None, None),
    "C3": ("mm", 1, 4096, 4096, 4096, "int20", None, None),
    "C3r": ("mm", 1, 4096, 4096, 4096, "int20", 13, False),
    "C4": ("mm_nt", 1, 16384, 16384, 16384, "wide30", None, None),
    "C5": ("bmm_nt", 64, 1024, 1024, 1024, "unif", None, None),
    # profiling case: same kernels as C2 at a quarter of the device footprint
    "P4096": ("mm_nt", 1, 4096, 4096, 4096, "randn", None, None),
    # one rank's block of C2 / C4 on eight GPUs (2 x 4 grid; C2blk8t: the 4 x 2
    # grid's block), alone on one GPU: the per-rank timeline of the scaling runs
    "C2blk8": ("mm_nt", 1, 4096, 2048, 8192, "randn", None, None),
    "C2blk8t": ("mm_nt", 1, 2048, 4096, 8192, "randn", None, None),
    "C4blk8": ("mm_nt", 1, 8192, 4096, 16384, "wide30", None, None),
    # deep K: four 65536-deep segments (15 moduli + correction), the reference's
    # segmented path on its side
    "D1": ("mm", 1, 2048, 2048, 262144, "randn", None, None),
}

# Above this depth the double-double accuracy sample (one launch per K step)
# would take minutes; both arms skip it there and say so.
ACCURACY_MAX_K = 65536


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# --------------------------------------------------------------- clocks --
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.path = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.uuid = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.1)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.06)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                if self.uuid and self.uuid.replace("GPU-", "") not in parts[1]:
                    continue
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower().startswith("active")})
        pw = [float(r[4]) for r in rows if r[4].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


# ---------------------------------------------------------------- inputs --
def make_inputs(dist_name, batch, M, N, K, nt, device, seed=0):
    """Seeded synthetic operands on the device (BASELINE configs' value
    distributions; no public dataset exists for this path)."""
    g = torch.Generator(device=device).manual_seed(seed)
    shpA = (batch, M, K) if batch > 1 else (M, K)
    shpB = ((batch, K, N) if nt else (batch, N, K)) if batch > 1 else ((K, N) if nt else (N, K))
    opts = dict(dtype=torch.float64, device=device, generator=g)
    if dist_name == "randn":
        A, B = torch.randn(shpA, **opts), torch.randn(shpB, **opts)
    elif dist_name == "unif":
        A, B = torch.rand(shpA, **opts) * 2 - 1, torch.rand(shpB, **opts) * 2 - 1
    elif dist_name == "int20":
        lim = 1 << 20
        A = torch.randint(-lim, lim + 1, shpA, device=device, generator=g).double()
        B = torch.randint(-lim, lim + 1, shpB, device=device, generator=g).double()
    elif dist_name == "wide30":
        A, B = torch.randn(shpA, **opts), torch.randn(shpB, **opts)
        A *= torch.exp2(torch.randint(-30, 31, shpA, device=device, generator=g).double())
        B *= torch.exp2(torch.randint(-30, 31, shpB, device=device, generator=g).double())
    else:
        raise ValueError(dist_name)
    return A, B


INT8_PEAK_RECORD = os.path.join(ROOT, "profiles", "int8_peak_b200.md")


def int8_peak_from_file():
    """Dense INT8 peak (TOPS): (sustained, burst, source).  The measured
    cuBLAS INT8 GEMM rate on this pool (`bench.py --int8-peak`, committed in
    profiles/int8_peak_b200.md) when that record exists; otherwise twice the
    measured BF16 dense rate of MEASURED_PEAKS.json (B200's INT8 dense rate is
    twice its BF16 one); otherwise the pool's fallback figures."""
    vals = {}
    try:
        with open(INT8_PEAK_RECORD) as f:
            for line in f:
                line = line.strip().strip("`")
                if line.startswith("int8_tops_") and "=" in line:
                    k, v = line.split("=", 1)
                    vals[k.strip()] = float(v.split()[0])
        if "int8_tops_burst" in vals and "int8_tops_sustained" in vals:
            return vals["int8_tops_sustained"], vals["int8_tops_burst"], "measured cuBLAS INT8 GEMM (torch._int_mm)"
    except (OSError, ValueError, IndexError):
        pass
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            mp = json.load(f)
        return 2.0 * float(mp["bf16_tflops_sustained"]), 2.0 * float(mp["bf16_tflops"]), "2 x measured bf16"
    except (OSError, KeyError, ValueError):
        return 2.0 * 1400.0, 2.0 * 1590.0, "2 x fallback bf16"


def bf16_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mp = json.load(f)
        return float(mp["bf16_tflops_sustained"]), float(mp["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1400.0, 1590.0


def profiled_traffic_per_step():
    """DRAM bytes (read + write) of all GEMM launches of one C2 step (the
    chunked pipeline's GEMM chunks) from the committed ncu summary."""
    try:
        with open(PROFILE_SUMMARY) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_step"):
                    return int(float(line.split("=")[1].split()[0]))
    except (OSError, ValueError, IndexError):
        pass
    return None


# ------------------------------------------------ workload / sample helpers --
def grid_of(world):
    """(row blocks, column blocks) of the 2-D partition of C for `world` ranks.
    The same rule as fp64_emu.dist.grid_shape, restated so that the reference
    arm imports nothing of this repository (tests/test_bench_cpu.py checks
    that the two agree)."""
    pr = 1
    while (pr * 2) ** 2 <= world and world % (pr * 2) == 0:
        pr *= 2
    return pr, world // pr


def first_block(n, parts):
    """Length of block 0 when n splits into `parts` nearly equal blocks (as
    fp64_emu.dist.block_range)."""
    base, rem = divmod(n, parts)
    return base + (1 if rem > 0 else 0)


def workload_config(name):
    """The `config` object of both arms: the workload only (same dict in the
    reference arm and ours, whatever the partition)."""
    kind, batch, M, N, K, dist_name, nprimes, corr = WORKLOADS[name]
    plan = "default plan (plan_config(K))" if nprimes is None and corr is None else \
        f"plan nprimes={nprimes} corr={corr}"
    return {"workload": f"{name}: {kind} batch={batch} M={M} N={N} K={K} {dist_name}, {plan}",
            "l2": "operands larger than L2 (no flush)"}


def sample_region(name, world):
    """(batch member or None, rows, columns) of the output sample that both
    arms hash and measure: the first 256 rows of rank 0's block by all of the
    block's columns (of batch member 0 for batches).  Rank 0's block starts at
    row 0 and column 0, so in the full product the sample is C[:rows, :cols]."""
    kind, batch, M, N, K = WORKLOADS[name][:5]
    if batch > 1:
        return 0, min(256, M), N
    pr, pc = grid_of(world)
    return None, min(256, first_block(M, pr)), first_block(N, pc)


def sample_sha256(C, name, world):
    """SHA-256 of the sample's float64 bytes (row-major)."""
    b, R, Nc = sample_region(name, world)
    X = C[b] if b is not None else C
    return hashlib.sha256(X[:R, :Nc].contiguous().cpu().numpy().tobytes()).hexdigest()


# ----------------------------------------------------------- our product --
class Step:
    """One rank's product on the current stream with a preallocated workspace
    (the public entry points allocate the same workspace from torch's caching
    allocator per call): sizing (+ the MAX all-reduce when partitioned), then
    extraction, GEMM and reconstruction in one call, which the library runs as
    a chunked pipeline for large products.  With events, every GEMM launch of
    the step is bracketed by two of them on the stream it runs on."""

    MAX_LAUNCHES = 16

    def __init__(self, kind, A, B, nprimes, corr, slab_cols):
        import fp64_emu
        from fp64_emu.dist import ShardedProduct
        self.nt = kind in ("mm_nt", "bmm_nt")
        K = A.size(-1)
        self.sp = ShardedProduct(A, B, self.nt, slab_cols, K, nprimes=nprimes, corr=corr)
        shape = (A.size(0), A.size(1), B.size(-1) if self.nt else B.size(1)) if A.dim() == 3 else \
            (A.size(0), B.size(-1) if self.nt else B.size(0))
        self.out = torch.empty(shape, dtype=torch.float64, device=A.device)
        self.nprimes, self.corr = self.sp.primes.numel(), self.sp.corr
        self.fp64_emu = fp64_emu

    def new_events(self):
        """Step-start event + two events per possible GEMM launch."""
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(1 + 2 * self.MAX_LAUNCHES)]
        for e in ev:
            e.record()   # creates the underlying CUDA event
        return ev

    def run(self, events=None):
        """Returns the number of GEMM launches of the step."""
        sp, out = self.sp, self.out
        if events is not None:
            events[0].record()
        sp.sizing(out)
        if events is None:
            sp._phase(out, 14)
            return 0
        return self.fp64_emu.ops.fp64_emu_gemm_ws_ev(out, sp.ws, sp.A, sp.B, sp.primes, sp.b_kn, sp.exact, sp.bits,
                                                     sp.corr, 14, sp.slab_cols, [e.cuda_event for e in events[1:]])

    @staticmethod
    def timeline(events, launches, step_ms):
        """(head, gaps, tail) of one step in ms: from the step's start to its
        first GEMM launch, the time between its first GEMM start and last GEMM
        end when no GEMM ran, and from the last GEMM end to the step's end."""
        t0 = events[0]
        iv = [(t0.elapsed_time(events[1 + 2 * i]), t0.elapsed_time(events[2 + 2 * i])) for i in range(launches)]
        if not iv:
            return 0.0, 0.0, step_ms
        first, last = min(a for a, _ in iv), max(b for _, b in iv)
        return first, (last - first) - Step.gemm_ms(events, launches), step_ms - last

    @staticmethod
    def gemm_ms(events, launches):
        """Time during which at least one GEMM launch of the step ran (chunks on
        two streams overlap at their boundaries)."""
        t0 = events[0]
        iv = sorted((t0.elapsed_time(events[1 + 2 * i]), t0.elapsed_time(events[2 + 2 * i])) for i in range(launches))
        busy, end = 0.0, float("-inf")
        for a, b in iv:
            if b > end:
                busy += b - max(a, end)
                end = b
        return busy


def barrier():
    if dist.is_initialized():
        dist.barrier()


def gather_ranks(obj):
    """Every rank's `obj`, in rank order (one all_gather_object, outside
    timing)."""
    if not dist.is_initialized():
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def max_over_ranks(x):
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def our_kernel_launches_per_step(kind, batch, chunks, M=None, N=None, K=None):
    # sizing: A's row statistics with B's column partials in one launch, then
    # the column finalize with the operand maxima (B as [K, N]), or one launch
    # for both operands' row statistics and the maxima; per chunk one
    # extraction of A, one GEMM and one reconstruction; B extracted once
    # (single product) or per chunk (batch).  An unchunked product of at most
    # 4 M operand elements extracts both operands in one launch.
    nt = kind in ("mm_nt", "bmm_nt")
    c = max(1, chunks)
    n = (2 if nt else 1) + 3 * c + (1 if batch == 1 else c)
    if c == 1 and None not in (M, N, K) and (batch * M + batch * N) * K <= (1 << 22):
        n -= 1
    return n


def cpu_baseline_oracle(A_cpu, Bt_cpu, nprimes, corr, rows):
    """The CPU restatement oracle on a bounded sample: `rows` rows of A against
    the whole of Bt (all of B's extraction, a slice of the GEMM)."""
    from oracle import oracle as O
    O.build()
    threads = O.cpu_count()
    O.set_threads(threads)
    a = A_cpu[:rows].numpy()
    b = Bt_cpu.numpy()
    t0 = time.perf_counter()
    O.emu(a, b, nprimes=nprimes, corr=corr, b_nt=True)
    dt = time.perf_counter() - t0
    M, K = a.shape
    N = b.shape[1]
    return {"value": 2.0 * M * N * K / dt / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"oracle/f64e_oracle.c, {M} rows of A x full Bt ({K}x{N}), one product, {dt:.1f} s"}


def cpu_fp64_torch(A_cpu, Bt_cpu, rows):
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    a = A_cpu[:rows]
    a @ Bt_cpu[:, :64]
    t0 = time.perf_counter()
    a @ Bt_cpu
    dt = time.perf_counter() - t0
    return {"value": 2.0 * a.size(0) * Bt_cpu.size(1) * a.size(1) / dt / 1e12, "unit": UNIT, "cores": threads,
            "sample": f"torch.mm float64 on host, {a.size(0)}x{a.size(1)} @ {Bt_cpu.size(0)}x{Bt_cpu.size(1)}"}


def run_ours(args):
    kind, batch, M, N, K, dist_name, nprimes, corr = WORKLOADS[args.workload]
    rank, world = (dist.get_rank(), dist.get_world_size()) if dist.is_initialized() else (0, 1)
    dev = torch.device("cuda", torch.cuda.current_device())
    nt = kind in ("mm_nt", "bmm_nt")
    from fp64_emu import plan_config
    from fp64_emu.dist import block_range, grid_shape, rank_block
    if nprimes is None or corr is None:
        dp, dc = plan_config(K)
        nprimes = dp if nprimes is None else nprimes
        corr = dc if corr is None else corr

    # Full operands are generated from one seed on rank 0 (the shared operand's
    # slices reach the other ranks by one NCCL broadcast, outside timing).
    A, B = make_inputs(dist_name, batch, M, N, K, nt, dev, seed=args.seed) if rank == 0 else (None, None)
    if world > 1:
        if batch > 1:
            shp_a, shp_b = (batch, M, K), ((batch, K, N) if nt else (batch, N, K))
        else:
            shp_a, shp_b = (M, K), ((K, N) if nt else (N, K))
        if rank != 0:
            A = torch.empty(shp_a, dtype=torch.float64, device=dev)
            B = torch.empty(shp_b, dtype=torch.float64, device=dev)
        t0 = time.perf_counter()
        dist.broadcast(A, 0)
        dist.broadcast(B, 0)
        torch.cuda.synchronize()
        bcast_s = time.perf_counter() - t0
    else:
        bcast_s = 0.0
    if batch > 1:
        b0, b1 = block_range(batch, world, rank)
        A_l, B_l = A[b0:b1].contiguous(), B[b0:b1].contiguous()
        slab_cols = batch * N
        work = 2.0 * batch * M * N * K
        part = f"batch split {world}"
    else:
        (r0, r1), (c0, c1) = rank_block(rank, world, M, N)
        A_l = A[r0:r1].contiguous()
        B_l = (B[:, c0:c1] if nt else B[c0:c1]).contiguous()
        slab_cols = N
        work = 2.0 * M * N * K
        pr, pc = grid_shape(world)
        part = f"2-D C blocks {pr}x{pc}"
    A_host_full = A.cpu() if (rank == 0 and world == 1 and not args.no_cpu) else None
    B_host_full = B.cpu() if (rank == 0 and world == 1 and not args.no_cpu) else None
    shs = shares = host_cpus = None
    if world > 1:
        # e2e at N > 1 (fp64_emu.dist.ShardedHostStream): every rank copies in
        # a disjoint share of its blocks and the blocks are completed over
        # NVLink; batches: every rank copies in its own members
        from fp64_emu.dist import ShardedHostStream
        from fp64_emu.host import gpu_local_allocation
        shs = ShardedHostStream(kind, M, N, K, nprimes=nprimes, corr=corr, batch=batch)
        with gpu_local_allocation(dev) as loc:   # page-locked shares on the GPU's NUMA node
            shares = shs.host_shares(A.cpu(), B.cpu())
            host_cpus = loc.cpus
    del A, B
    torch.cuda.empty_cache()

    step = Step(kind, A_l, B_l, nprimes, corr, slab_cols)
    for _ in range(args.warmup):
        step.run()
    torch.cuda.synchronize()

    ev = [step.new_events() for _ in range(args.steps)]
    launches = [0] * args.steps
    torch.cuda.synchronize()
    clocks = ClockSampler(dev)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for i in range(args.steps):
        launches[i] = step.run(ev[i])
    t_stop.record()
    torch.cuda.synchronize()
    barrier()
    ms_local = t_start.elapsed_time(t_stop) / args.steps
    gemm_ms_local = sum(Step.gemm_ms(ev[i], launches[i]) for i in range(args.steps)) / args.steps
    # per-step timeline: each step ends where the next one starts
    ends = [ev[i + 1][0] for i in range(args.steps - 1)] + [t_stop]
    tl = [Step.timeline(ev[i], launches[i], ev[i][0].elapsed_time(ends[i])) for i in range(args.steps)]
    head_local, gaps_local, tail_local = (sum(x[k] for x in tl) / args.steps for k in range(3))
    # this rank's last timed step: its GEMM launches as (start, end) in ms from
    # the step's start, on the rank's own clock
    last = ev[-1]
    chunks_last = [(round(last[0].elapsed_time(last[1 + 2 * i]), 4), round(last[0].elapsed_time(last[2 + 2 * i]), 4))
                   for i in range(launches[-1])]
    per_rank = gather_ranks({"rank": rank, "ms_per_step": round(ms_local, 4), "gemm_busy": round(gemm_ms_local, 4),
                             "head": round(head_local, 4), "gaps": round(gaps_local, 4),
                             "tail": round(tail_local, 4), "last_step_gemm_ms": chunks_last,
                             "block": [int(A_l.shape[-2]), int(B_l.shape[-1] if nt else B_l.shape[-2])]})

    # e2e through the public API with host buffers.
    import fp64_emu
    if shs is None:
        from fp64_emu.host import gpu_local_allocation
        with gpu_local_allocation(dev) as loc:   # page-locked buffers on the GPU's NUMA node
            A_pin = A_l.cpu().pin_memory()
            B_pin = B_l.cpu().pin_memory()
            out_pin = torch.empty(step.out.shape, dtype=torch.float64).pin_memory()
            host_cpus = loc.cpus

    hs = fp64_emu.HostStream(kind, nprimes=nprimes, corr=corr) if world == 1 else None

    def e2e_step():
        if shs is not None:
            shs.submit(*shares)
        else:
            # a stream of host-resident products: the operand copies, the
            # product and the result copy of neighbouring steps overlap
            hs.submit(A_pin, B_pin, out_pin)

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        e2e_step()
    for x in (hs, shs):
        if x is not None:
            x.synchronize()
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    for x in (hs, shs):
        if x is not None:
            x.join()   # the current stream waits for every step's result copy
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms_local = e0.elapsed_time(e1) / e2e_steps
    clk = clocks.stop()

    ms = max_over_ranks(ms_local)
    gemm_ms = max_over_ranks(gemm_ms_local)
    e2e_ms = max_over_ranks(e2e_ms_local)
    # whole job, summed over ranks: the shares copied in, the blocks copied out
    if shs is not None:
        h2d, d2h = batch * (M * K + K * N) * 8, batch * M * N * 8
    else:
        h2d, d2h = (A_l.numel() + B_l.numel()) * 8 * world, step.out.numel() * 8 * world

    # Roofline of the dominant kernel on this rank.
    G = nprimes + (2 if corr else 0)
    Ml, Kl = A_l.shape[-2], A_l.shape[-1]
    Nl = B_l.shape[-1] if nt else B_l.shape[-2]
    bl = A_l.shape[0] if A_l.dim() == 3 else 1
    int8_ops = 2.0 * G * bl * Ml * Nl * Kl
    achieved = int8_ops / (gemm_ms_local * 1e-3) / 1e12
    peak_sus, peak_burst, src = int8_peak_from_file()
    # The burst figure applies while the SM clock holds near its maximum (the
    # GEMM is not power-throttled); the sustained one when the clock sagged.
    held = bool(clk and clk.get("sm_mhz") and clk.get("sm_max_mhz") and clk["sm_mhz"] >= 0.95 * clk["sm_max_mhz"])
    peak = peak_burst if held else peak_sus
    mhz = (clk or {}).get("sm_mhz") or 1965.0
    nominal = 148 * 8192 * 2 * mhz * 1e6 / 1e12   # 8192 INT8 MAC/clk/SM at the sampled clock
    traffic = profiled_traffic_per_step() if (args.workload == "C2" and world == 1) else None

    result = {
        "metric": METRIC if args.workload == "C2" else f"emulated FP64 TFLOP/s (2MNK/t), {args.workload}",
        "value": round(work / (ms * 1e-3) / 1e12, 3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f64",
        "data": "synthetic",
        "config": workload_config(args.workload),
        "partition": part,
        "plan": {"nprimes": nprimes, "corr": corr, "int8_gemms_per_product": G},
        "compute": "s8 x s8 -> s32 tcgen05 residue GEMMs, exact int128 recombine",
        "e2e": {"value": round(work / (e2e_ms * 1e-3) / 1e12, 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "host_buffers": (f"page-locked on the GPU's NUMA node (allocated on {len(host_cpus)} local cores)"
                                 if host_cpus else "page-locked, default placement"),
                "api": ("fp64_emu.HostStream (operand copies, product and result copy of neighbouring steps "
                        "overlap)") if world == 1 else
                       ("fp64_emu.dist.ShardedHostStream (disjoint host shares, "
                        + ("each rank's own batch members" if batch > 1 else "NVLink all-gathers")
                        + ", overlapped stages)")},
        "gpu_launches": sum(our_kernel_launches_per_step(kind, A_l.shape[0] if A_l.dim() == 3 else 1, c, Ml, Nl, Kl)
                            for c in launches),
        "roofline": {"bound": "tensor", "kernel": "residue_gemm_pair_kernel" if Ml > 128 else "residue_gemm_tc_kernel",
                     "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS (int8)",
                     "frac": round(achieved / peak, 4),
                     "peak_note": f"INT8 dense peak of measured: {src}, "
                                  f"{'burst (SM clock held)' if held else 'sustained (SM clock sagged)'}; "
                                  f"for context 2 x measured bf16 dense = {2 * bf16_peaks()[1]:.0f} TOPS burst, "
                                  f"nominal 8192 MAC/clk/SM at the sampled clock = {nominal:.0f} TOPS "
                                  f"(frac of nominal {achieved / nominal:.3f})",
                     "gemm_ms_per_step": round(gemm_ms, 4), "traffic": traffic,
                     "per": "step: achieved over the step's GEMM busy time, traffic summed over its GEMM launches"},
        "phases_ms": {"gemm_busy": round(gemm_ms, 4), "outside_gemm": round(ms - gemm_ms, 4),
                      "head": round(max_over_ranks(head_local), 4), "gaps": round(max_over_ranks(gaps_local), 4),
                      "tail": round(max_over_ranks(tail_local), 4),
                      "rank0": {"head": round(head_local, 4), "gaps": round(gaps_local, 4),
                                "tail": round(tail_local, 4), "gemm_busy": round(gemm_ms_local, 4),
                                "ms_per_step": round(ms_local, 4)},
                      "gemm_launches_per_step": launches[-1] if launches else 0},
        "clocks": clk,
    }
    if world > 1:
        result["operand_broadcast_s"] = round(bcast_s, 3)
        if args.timeline_out and rank == 0:
            with open(args.timeline_out, "w") as f:
                json.dump({"workload": args.workload, "n_gpus": world, "steps": args.steps,
                           "ms_per_step_max": round(ms, 4), "clocks": clk, "per_rank": per_rank}, f, indent=1)
    if rank == 0 and world == 1 and not args.no_cpu and batch == 1 and nt:
        try:
            result["cpu_baseline"] = cpu_baseline_oracle(A_host_full, B_host_full, nprimes, corr,
                                                         rows=args.cpu_rows)
        except Exception as e:  # noqa: BLE001
            result["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        try:
            result["cpu_fp64_torch"] = cpu_fp64_torch(A_host_full, B_host_full, rows=1024)
        except Exception as e:  # noqa: BLE001
            result["cpu_fp64_torch"] = {"value": None, "error": str(e)[:200]}
    if rank == 0 and not args.no_native:
        result["native_dgemm"] = native_dgemm(A_l, B_l, nt, args)
    if rank == 0 and not args.no_accuracy and K > ACCURACY_MAX_K:
        result["accuracy"] = {"skipped": f"K = {K} > {ACCURACY_MAX_K}: one double-double launch per K step"}
    elif rank == 0 and not args.no_accuracy:
        try:
            result["accuracy"] = accuracy_sample(kind, A_l, B_l, step.out, args.workload, world,
                                                 others={"native_dgemm": lambda a, b: a @ b})
        except Exception as e:  # noqa: BLE001
            result["accuracy"] = {"error": str(e)[:200]}
    if rank == 0:
        result["output_sha256"] = {"sample": sample_description(args.workload, world),
                                   "value": sample_sha256(step.out, args.workload, world)}
    if world > 1 and not args.no_block_check:
        # every rank's block against the same block of the unpartitioned
        # product, computed on rank 0's GPU after timing (collective: all ranks)
        ok = check_blocks(args, step.out, rank, world, dev)
        if rank == 0:
            result["blocks_bit_identical"] = ok
    if rank == 0:
        print(json.dumps(result), flush=True)


def sample_description(name, world):
    b, R, Nc = sample_region(name, world)
    return (f"C[{R} rows x {Nc} cols] at row 0, col 0" + (" of batch member 0" if b is not None else "")
            + (f" (rank 0's block of {world})" if world > 1 else "") + ", float64 bytes row-major")


def check_blocks(args, out, rank, world, dev):
    """Digest of every rank's block, gathered; rank 0 recomputes the whole
    product unpartitioned on its GPU (the public fp64_emu API) and compares
    the same blocks.  True when every block is bit-identical."""
    kind, batch, M, N, K, dist_name, nprimes, corr = WORKLOADS[args.workload]
    nt = kind in ("mm_nt", "bmm_nt")
    mine = hashlib.sha256(out.contiguous().cpu().numpy().tobytes()).digest()
    d = torch.tensor(list(mine), dtype=torch.uint8, device=dev)
    allg = torch.empty(world * 32, dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(allg, d)
    if rank != 0:
        return None
    import fp64_emu
    from fp64_emu.dist import block_range, rank_block
    got = bytes(allg.cpu().tolist())
    A, B = make_inputs(dist_name, batch, M, N, K, nt, dev, seed=args.seed)
    kw = {k: v for k, v in (("nprimes", nprimes), ("corr", corr)) if v is not None}
    C = getattr(fp64_emu, kind)(A, B, **kw)
    del A, B
    ok = True
    for r in range(world):
        if batch > 1:
            b0, b1 = block_range(batch, world, r)
            blk = C[b0:b1]
        else:
            (r0, r1), (c0, c1) = rank_block(r, world, M, N)
            blk = C[r0:r1, c0:c1]
        ok = ok and hashlib.sha256(blk.contiguous().cpu().numpy().tobytes()).digest() == got[32 * r:32 * r + 32]
    del C
    torch.cuda.empty_cache()
    return ok


def accuracy_sample(kind, A, B, C, name, world, others=None):
    """Correct bits against the double-double product (dd_accuracy) on the
    output sample of sample_region (the first 256 rows of rank 0's block by
    the block's columns, of batch member 0): A, B and C are rank 0's block
    operands and product (our arm) or the whole ones (reference arm; rank 0's
    block starts at row 0 and column 0).  `others`: name -> callable giving
    another product of the same sample to measure alongside (cuBLAS DGEMM).
    Runs after timing."""
    import dd_accuracy as acc
    nt = kind in ("mm_nt", "bmm_nt")
    batched = A.dim() == 3
    if batched:
        A, B, C = A[0], B[0], C[0]
    _, R, Nc = sample_region(name, world)
    As = A[:R]
    Bt = (B[:, :Nc] if nt else B[:Nc].t()).contiguous()
    C = C[:, :Nc]
    t0 = time.perf_counter()
    hi, lo = acc.dd_product(As, Bt)
    res = {"sample": sample_description(name, world),
           "measure": "-log2(max|C - hi - lo| / max|hi|) against the double-double product (hi, lo); "
                      "element bits: -log2(|C - hi - lo| / |hi|), capped at 60",
           "value": acc.summary(C[:R], hi, lo)}
    for name, fn in (others or {}).items():
        res[name] = acc.summary(fn(As, Bt), hi, lo)
    res["seconds"] = round(time.perf_counter() - t0, 1)
    return res


def native_dgemm(A, B, nt, args):
    """cuBLAS DGEMM on the same per-rank operands, for context."""
    f = (lambda: torch.matmul(A, B)) if nt else (lambda: torch.matmul(A, B.transpose(-1, -2)))
    for _ in range(2):
        f()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(3, min(args.steps, 10))
    s.record()
    for _ in range(n):
        f()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / n
    Ml, Kl = A.shape[-2], A.shape[-1]
    Nl = B.shape[-1] if nt else B.shape[-2]
    bl = A.shape[0] if A.dim() == 3 else 1
    return {"value": round(2.0 * bl * Ml * Nl * Kl / (ms * 1e-3) / 1e12, 3), "unit": UNIT, "ms": round(ms, 4)}


# ------------------------------------------------------------ reference --
def load_reference():
    ref_dir = os.path.join(ROOT, "oracle", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "fp64_emu_ref.so")):
        return None, "reference build oracle/_ref/fp64_emu_ref.so missing (python oracle/build_ref.py)"
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import fp64_emu_ref
    return fp64_emu_ref, None


def run_reference(args):
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    if rank != 0:
        return
    R, why = load_reference()
    kind, batch, M, N, K, dist_name, nprimes, corr = WORKLOADS[args.workload]
    if R is None:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    dev = torch.device("cuda", torch.cuda.current_device())
    nt = kind in ("mm_nt", "bmm_nt")
    A, B = make_inputs(dist_name, batch, M, N, K, nt, dev, seed=args.seed)
    fn = getattr(R, kind)
    kw = {}
    if nprimes is not None:
        kw["nprimes"] = nprimes
    if corr is not None:
        kw["corr"] = corr
    for _ in range(args.warmup + 1):   # the first call runs the reference's dispatch probe
        fn(A, B, **kw)
    torch.cuda.synchronize()
    clocks = ClockSampler(dev)
    clocks.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        fn(A, B, **kw)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    A_pin, B_pin = A.cpu().pin_memory(), B.cpu().pin_memory()
    C0 = fn(A, B, **kw)
    out_pin = torch.empty(C0.shape, dtype=torch.float64).pin_memory()
    A_d, B_d = torch.empty_like(A), torch.empty_like(B)

    def e2e_step():
        A_d.copy_(A_pin, non_blocking=True)
        B_d.copy_(B_pin, non_blocking=True)
        out_pin.copy_(fn(A_d, B_d, **kw), non_blocking=True)

    n2 = max(3, min(args.steps, 20))
    e2e_step()
    torch.cuda.synchronize()
    s.record()
    for _ in range(n2):
        e2e_step()
    e.record()
    torch.cuda.synchronize()
    e2e_ms = s.elapsed_time(e) / n2
    clk = clocks.stop()
    work = 2.0 * batch * M * N * K
    value = round(work / (ms * 1e-3) / 1e12, 3)
    result = {
        "impl": "reference",
        "metric": METRIC if args.workload == "C2" else f"emulated FP64 TFLOP/s (2MNK/t), {args.workload}",
        "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f64", "data": "synthetic",
        "config": workload_config(args.workload),
        "impl_note": ("the reference's own CUDA build (oracle/_ref, compiled from its sources with its JIT recipe) "
                      "through its Python API on one B200, " +
                      (f"FP64EMU_PATH={os.environ['FP64EMU_PATH']}" if os.environ.get("FP64EMU_PATH")
                       else "default dispatch") + ", first-call probe excluded; the reference has no CPU "
                      "implementation of this path, so there is no cpu_baseline in this line"),
        "e2e": {"value": round(work / (e2e_ms * 1e-3) / 1e12, 3), "unit": UNIT,
                "h2d_bytes_per_step": (A.numel() + B.numel()) * 8, "d2h_bytes_per_step": C0.numel() * 8},
        "output_sha256": {"sample": sample_description(args.workload, world),
                          "value": sample_sha256(C0, args.workload, world)},
        "clocks": clk,
    }
    if not args.no_accuracy and K > ACCURACY_MAX_K:
        result["accuracy"] = {"skipped": f"K = {K} > {ACCURACY_MAX_K}: one double-double launch per K step"}
    elif not args.no_accuracy:
        try:
            result["accuracy"] = accuracy_sample(kind, A, B, C0, args.workload, world)
        except Exception as e:  # noqa: BLE001
            result["accuracy"] = {"error": str(e)[:200]}
    print(json.dumps(result), flush=True)


# ------------------------------------------------------------ INT8 peak --
def run_int8_peak(args):
    """Dense INT8 GEMM peak of this B200 through cuBLAS (torch._int_mm, s8 x
    s8 -> s32), n x n x n: the best of 10 back-to-back launches per operand
    layout (burst), then the better layout back to back for about 4 s
    (sustained), with the SM clock sampled throughout.  Prints one JSON line;
    the figures recorded in profiles/int8_peak_b200.md are what bench.py
    divides by."""
    dev = torch.device("cuda", torch.cuda.current_device())
    n = args.peak_n
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
    b_rm = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
    b_cm = b_rm.t().contiguous().t()     # same values, column-major
    ops = 2.0 * n * n * n
    clocks = ClockSampler(dev)
    clocks.start()
    burst = {}
    for name, b in (("b column-major", b_cm), ("b row-major", b_rm)):
        try:
            for _ in range(3):
                torch._int_mm(a, b)
            torch.cuda.synchronize()
            best = float("inf")
            for _ in range(10):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                torch._int_mm(a, b)
                e.record()
                e.synchronize()
                best = min(best, s.elapsed_time(e))
            burst[name] = ops / (best * 1e-3) / 1e12
        except RuntimeError as ex:   # a layout cuBLAS does not take
            burst[name] = None
            log(f"int8 peak: {name}: {ex}")
    clk_burst = clocks.stop()
    layout = max((k for k in burst if burst[k]), key=lambda k: burst[k])
    b = b_cm if layout == "b column-major" else b_rm
    clocks = ClockSampler(dev)
    clocks.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    t0, k = time.perf_counter(), 0
    while time.perf_counter() - t0 < args.peak_seconds:
        for _ in range(20):
            torch._int_mm(a, b)
        k += 20
        if k % 100 == 0:
            torch.cuda.synchronize()
    e.record()
    torch.cuda.synchronize()
    sustained = ops * k / (s.elapsed_time(e) * 1e-3) / 1e12
    clk_sus = clocks.stop()
    print(json.dumps({"int8_peak": {"n": n, "op": "torch._int_mm (cuBLAS), s8 x s8 -> s32",
                                    "burst_tops": {k2: (round(v, 1) if v else None) for k2, v in burst.items()},
                                    "layout": layout, "burst_best_tops": round(burst[layout], 1),
                                    "sustained_tops": round(sustained, 1), "sustained_launches": k,
                                    "clocks_burst": clk_burst, "clocks_sustained": clk_sus,
                                    "gpu": torch.cuda.get_device_name(dev)}}), flush=True)


# ------------------------------------------------------------ PCIe probe --
def run_pcie_probe(args):
    """Host <-> device copy rates of every rank at once (one process per GPU,
    as the end-to-end runs): pinned 1 GiB buffers, one cudaMemcpyAsync per
    copy (torch's copy_), host-to-device alone, device-to-host alone, and both
    directions at once on two streams; CUDA events, the slowest rank's time.
    Run twice: with the buffers allocated after binding the process to its
    GPU's NUMA-local cores (fp64_emu.host.bind_to_gpu_cpus), and without."""
    rank, world = (dist.get_rank(), dist.get_world_size()) if dist.is_initialized() else (0, 1)
    dev = torch.device("cuda", torch.cuda.current_device())
    nbytes = args.probe_mib << 20
    res = {}
    for placement in ("default", "gpu_local"):
        cpus = None
        if placement == "gpu_local":
            from fp64_emu.host import bind_to_gpu_cpus
            cpus = bind_to_gpu_cpus(dev)
        h_in = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        h_out = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        h_in.fill_(1)
        h_out.fill_(2)
        d_in = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        d_out = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        out = {}
        for mode in ("h2d", "d2h", "both"):
            best = float("inf")
            for it in range(4):
                barrier()
                torch.cuda.synchronize()
                e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
                e0.record(s1)
                s2.wait_event(e0)
                if mode in ("h2d", "both"):
                    with torch.cuda.stream(s1):
                        d_in.copy_(h_in, non_blocking=True)
                if mode in ("d2h", "both"):
                    with torch.cuda.stream(s2):
                        h_out.copy_(d_out, non_blocking=True)
                e1.record(s1)
                e2.record(s2)
                torch.cuda.synchronize()
                ms = max(e0.elapsed_time(e1), e0.elapsed_time(e2))
                if it > 0:
                    best = min(best, max_over_ranks(ms))
                else:
                    max_over_ranks(ms)
            moved = nbytes * (2 if mode == "both" else 1)
            out[mode] = {"per_rank_gbs": round(moved / (best * 1e-3) / 1e9, 1),
                         "aggregate_gbs": round(world * moved / (best * 1e-3) / 1e9, 1), "ms": round(best, 3)}
        out["cpus"] = (f"{len(cpus)} cores {min(cpus)}-{max(cpus)}" if cpus else "unchanged")
        res[placement] = out
        del h_in, h_out, d_in, d_out
    if rank == 0:
        print(json.dumps({"pcie_probe": res, "n_gpus": world, "bytes_per_copy": nbytes,
                          "note": "slowest rank's time of each copy pattern, best of 3 after one warm-up"}),
              flush=True)


def run_recon_l2_probe(args):
    """How much an L2-resident reconstruction could save (the bound on fusing
    the reconstruction into the GEMM, or ordering the GEMM's work so that a
    panel's residue planes are read back before they leave L2).  For row
    blocks of C2's shape (rows x 8192, K = 8192, default plan): sizing,
    extraction and the GEMM once, then the reconstruction phase alone,
    (a) right after the GEMM wrote the planes ("after_gemm"), (b) after a
    write of a buffer twice the L2's size ("cold"), (c) straight after another
    reconstruction of the same block ("hot": planes and output in L2).  CUDA
    events around the reconstruction launch only; every output is checked equal
    bit for bit."""
    from fp64_emu.dist import PHASE_EXTRACT, PHASE_GEMM, PHASE_RECON, PHASE_SIZING, ShardedProduct
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    res = []
    for rows in (256, 512, 2048):
        A, B = make_inputs("randn", 1, rows, 8192, 8192, True, dev, seed=args.seed)
        sp = ShardedProduct(A, B, True, 8192, 8192)
        out = torch.empty(rows, 8192, dtype=torch.float64, device=dev)
        sp._phase(out, PHASE_SIZING)
        sp._phase(out, PHASE_EXTRACT | PHASE_GEMM)   # unchunked: every phase sees the whole block
        sp._phase(out, PHASE_RECON)
        ref = out.clone()
        import fp64_emu
        same = torch.equal(fp64_emu.mm_nt(A, B).view(torch.int64), ref.view(torch.int64))
        t = {"after_gemm": [], "cold": [], "hot": []}

        def timed(key):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            sp._phase(out, PHASE_RECON)
            e1.record()
            torch.cuda.synchronize()
            t[key].append(e0.elapsed_time(e1) * 1e3)

        for i in range(args.steps):
            sp._phase(out, PHASE_GEMM)
            timed("after_gemm")
            flush.fill_(i & 255)
            timed("cold")
            timed("hot")
            same = same and torch.equal(out.view(torch.int64), ref.view(torch.int64))
        G = sp.primes.numel() + (2 if sp.corr else 0)
        plane_bytes = rows * 8192 * (sp.primes.numel() + 4)   # residue bytes + one int32 correction
        med = {k: statistics.median(v) for k, v in t.items()}
        res.append({"rows": rows, "elements": rows * 8192, "plane_bytes": plane_bytes,
                    "out_bytes": rows * 8192 * 8, "int8_gemms": G,
                    "us": {k: round(v, 2) for k, v in med.items()},
                    "gbs": {k: round((plane_bytes + rows * 8192 * 8) / (v * 1e-6) / 1e9, 1) for k, v in med.items()},
                    "bit_identical": same})
        del sp, out, ref, A, B
        torch.cuda.empty_cache()
    print(json.dumps({"recon_l2_probe": res, "steps": args.steps,
                      "note": "median reconstruction launch time; L2 126 MB"}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="C2", choices=sorted(WORKLOADS))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-rows", type=int, default=1024)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--no-native", action="store_true", help="skip the cuBLAS DGEMM context number")
    ap.add_argument("--no-accuracy", action="store_true",
                    help="skip the correct-bits measurement after timing (one small launch per K step)")
    ap.add_argument("--no-block-check", action="store_true",
                    help="N > 1: skip the unpartitioned recomputation that checks every rank's block")
    ap.add_argument("--int8-peak", action="store_true",
                    help="measure the dense INT8 GEMM peak (cuBLAS through torch._int_mm) and exit")
    ap.add_argument("--pcie-probe", action="store_true",
                    help="measure every rank's pinned host <-> device copy rates at once and exit")
    ap.add_argument("--probe-mib", type=int, default=1024)
    ap.add_argument("--recon-l2-probe", action="store_true",
                    help="time the reconstruction of C2-shaped row blocks with its planes in L2 and not, and exit")
    ap.add_argument("--timeline-out", default=None,
                    help="N>1: rank 0 writes every rank's per-step phases and its last step's GEMM launch times "
                         "(JSON) to this path")
    ap.add_argument("--peak-n", type=int, default=8192)
    ap.add_argument("--peak-seconds", type=float, default=4.0)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        if args.int8_peak:
            run_int8_peak(args)
        elif args.pcie_probe:
            run_pcie_probe(args)
        elif args.recon_l2_probe:
            run_recon_l2_probe(args)
        elif args.impl == "reference":
            run_reference(args)
        else:
            run_ours(args)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
