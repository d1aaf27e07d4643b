"""Small-n latency: eager fp64_emu.mm against the CUDA-graph replay of the same
call and native cuBLAS DGEMM, for n where launch overhead dominates (the
reference measures the same in bench/smalln.py of fp64-emu).

    python fp64-emu_b200/smalln.py [n ...]

Prints one JSON line: per n the median wall time (µs) of each, and whether the
graph replay's result equals the eager one bit for bit.
"""
import json
import os
import statistics
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def median_us(fn, iters=200, warm=20):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts) * 1e6


def measure(n):
    import fp64_emu
    gen = torch.Generator(device="cuda").manual_seed(n)
    A = torch.randn(n, n, dtype=torch.float64, device="cuda", generator=gen)
    B = torch.randn(n, n, dtype=torch.float64, device="cuda", generator=gen)
    eager = median_us(lambda: fp64_emu.mm(A, B))
    native = median_us(lambda: A @ B.t())
    for _ in range(3):
        fp64_emu.mm(A, B)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        C = fp64_emu.mm(A, B)
    g.replay()
    torch.cuda.synchronize()
    same = bool(torch.equal(C, fp64_emu.mm(A, B)))
    graph = median_us(g.replay)
    return {"n": n, "eager_us": round(eager, 1), "graph_us": round(graph, 1), "native_us": round(native, 1),
            "graph_equal": same}


def main():
    ns = [int(x) for x in sys.argv[1:]] or [64, 128, 256, 512]
    rows = [measure(n) for n in ns]
    print(json.dumps({"device": torch.cuda.get_device_name(0), "smalln": rows}), flush=True)


if __name__ == "__main__":
    main()
