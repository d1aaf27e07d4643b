"""Small-n latency: eager fp64_emu.mm against the CUDA-graph replay of the same
call and native cuBLAS DGEMM, for n where launch overhead dominates (the
reference measures the same in bench/smalln.py of fp64-emu).

    python fp64-emu_b200/smalln.py [--reference] [n ...]

--reference times the reference's own build (oracle/_ref, compiled from its
sources) through its own Python API instead, for comparison.

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


def load(reference):
    if not reference:
        import fp64_emu
        return fp64_emu
    ref = os.path.join(os.path.dirname(HERE), "oracle", "_ref")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import fp64_emu_ref
    return fp64_emu_ref


def measure(n, fp64_emu):
    gen = torch.Generator(device="cuda").manual_seed(n)
    A = torch.randn(n, n, dtype=torch.float64, device="cuda", generator=gen)
    B = torch.randn(n, n, dtype=torch.float64, device="cuda", generator=gen)
    eager = median_us(lambda: fp64_emu.mm(A, B))
    native = median_us(lambda: A @ B.t())
    for _ in range(3):
        fp64_emu.mm(A, B)
    torch.cuda.synchronize()
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            C = fp64_emu.mm(A, B)
        g.replay()
        torch.cuda.synchronize()
        same = bool(torch.equal(C, fp64_emu.mm(A, B)))
        graph = round(median_us(g.replay), 1)
    except Exception as e:  # noqa: BLE001  (a build whose call cannot be captured)
        same, graph = None, f"capture failed: {type(e).__name__}"
    return {"n": n, "eager_us": round(eager, 1), "graph_us": graph, "native_us": round(native, 1),
            "graph_equal": same}


def main():
    args = sys.argv[1:]
    reference = "--reference" in args
    ns = [int(x) for x in args if x != "--reference"] or [64, 128, 256, 512]
    emu = load(reference)
    rows = [measure(n, emu) for n in ns]
    print(json.dumps({"device": torch.cuda.get_device_name(0), "impl": "reference" if reference else "ours",
                      "smalln": rows}), flush=True)


if __name__ == "__main__":
    main()
