"""Caller-level drills: algorithms that use the emulated product as their GEMM,
run once with native fp64 GEMMs (cuBLAS) and once with fp64_emu, reporting
an application-level accuracy figure and wall time for each.  They exercise the
operator the way the reference's application drills and tiled Cholesky do
(bench/apps.py, bench/cholesky.py of fp64-emu); the GPU tests run the same
functions at small sizes with assertions.

    python fp64-emu_b200/drills.py [--small] [--only paths,cholesky,...]

Every function takes `g(A, Bt) -> A @ Bt` (mm_nt convention) or, for the
Cholesky trailing update, `update(X, Y) -> X[b] @ Y[b]^T` (bmm convention).
"""
import argparse
import json
import math
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def native_nt(A, Bt):
    return A @ Bt


def emu_nt(A, Bt):
    import fp64_emu
    return fp64_emu.mm_nt(A, Bt)


def native_bmm(X, Y):
    return torch.bmm(X, Y.transpose(1, 2))


def emu_bmm(X, Y):
    import fp64_emu
    return fp64_emu.bmm(X, Y)


def wall(fn, reps=3, warm=1):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t0)
    ts.sort()
    return ts[len(ts) // 2]


# ------------------------------------------------------------------ drills --
def path_counts(g, n=4096, density=0.05, seed=7):
    """4-step path counts A^4 of a random 0/1 digraph: exact integers far below
    2^53, so native fp64 is exact and the emulated product must equal it bit
    for bit."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    A = (torch.rand(n, n, device="cuda", generator=gen) < density).double()
    A2 = g(A, A)
    return g(A2, A2)


def tiled_cholesky(A, t, update):
    """Right-looking lower Cholesky of A with t x t tiles; the trailing update
    of every step is one batched product over the lower-triangle tile pairs.
    Returns (L, seconds in the batched updates)."""
    W = A.clone()
    n = W.size(0)
    nt = n // t
    upd = 0.0
    for k in range(nt):
        k0 = k * t
        Lkk = torch.linalg.cholesky(W[k0:k0 + t, k0:k0 + t])
        W[k0:k0 + t, k0:k0 + t] = Lkk
        if k + 1 == nt:
            break
        panel = torch.linalg.solve_triangular(Lkk, W[k0 + t:, k0:k0 + t].t(), upper=False).t().contiguous()
        W[k0 + t:, k0:k0 + t] = panel
        rem = nt - k - 1
        tiles = panel.view(rem, t, t)
        ii, jj = torch.tril_indices(rem, rem, device=A.device)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        S = update(tiles[ii].contiguous(), tiles[jj].contiguous())
        # scatter S[p] into tile (ii[p], jj[p]) of the trailing matrix
        trail = W[k0 + t:, k0 + t:].view(rem, t, rem, t).permute(0, 2, 1, 3)
        trail[ii, jj] -= S
        torch.cuda.synchronize()
        upd += time.perf_counter() - t0
    return torch.tril(W), upd


def spd_matrix(n, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    G = torch.randn(n, n, dtype=torch.float64, device="cuda", generator=gen)
    return G @ G.t() / n + 2.0 * torch.eye(n, dtype=torch.float64, device="cuda")


def cholqr_residual(g, m=65536, k=512, cond_decades=6, seed=1):
    """||Q^T Q - I||_F of CholeskyQR with the Gram matrix A^T A from g: the
    Gram product squares the condition number, so GEMM accuracy shows in the
    orthogonality of Q."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    Q1, _ = torch.linalg.qr(torch.randn(m, k, dtype=torch.float64, device="cuda", generator=gen))
    Q2, _ = torch.linalg.qr(torch.randn(k, k, dtype=torch.float64, device="cuda", generator=gen))
    s = torch.logspace(0, -cond_decades, k, dtype=torch.float64, device="cuda")
    A = (Q1 * s) @ Q2.t()
    At = A.t().contiguous()
    G = g(At, A)
    L = torch.linalg.cholesky(G)
    Q = torch.linalg.solve_triangular(L, At, upper=False).t()
    eye = torch.eye(k, dtype=torch.float64, device="cuda")
    return (Q.t() @ Q - eye).norm().item()


def newton_schulz(g, n=3072, iters=50, seed=2):
    """Polar factor by X <- 1.5 X - 0.5 X (X^T X); returns ||X^T X - I||_F."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(n, n, dtype=torch.float64, device="cuda", generator=gen)
    A = A * torch.logspace(0, -2, n, dtype=torch.float64, device="cuda")
    X = A / A.norm()
    for _ in range(iters):
        Y = g(X.t().contiguous(), X)
        X = 1.5 * X - 0.5 * g(X, Y)
    eye = torch.eye(n, dtype=torch.float64, device="cuda")
    return (X.t() @ X - eye).norm().item()


def expm_taylor(g, A, s=6, terms=18):
    """exp(A) by a Taylor series of A / 2^s and s squarings, every product
    through g."""
    eye = torch.eye(A.size(0), dtype=torch.float64, device=A.device)
    As = A * (2.0 ** -s)
    E = eye + As
    T = As
    for k in range(2, terms):
        T = g(T, As) / k
        E = E + T
    for _ in range(s):
        E = g(E, E)
    return E


def expm_error(g, n=2048, seed=3):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(n, n, dtype=torch.float64, device="cuda", generator=gen) / math.sqrt(n)
    ref = torch.matrix_exp(A)
    return ((expm_taylor(g, A) - ref).norm() / ref.norm()).item()


# --------------------------------------------------------------- reporting --
def run(small=False, only=None):
    out = {}
    sz = (lambda big, little: little if small else big)
    if not only or "paths" in only:
        n = sz(4096, 1024)
        Pn, Pe = path_counts(native_nt, n), path_counts(emu_nt, n)
        out["paths"] = {"n": n, "bitwise_equal": bool(torch.equal(Pn, Pe)), "max_count": Pn.max().item(),
                        "native_s": wall(lambda: path_counts(native_nt, n)),
                        "emu_s": wall(lambda: path_counts(emu_nt, n))}
    if not only or "cholesky" in only:
        n, t = sz(16384, 2048), sz(512, 256)
        A = spd_matrix(n)
        res = {"n": n, "tile": t}
        for name, upd in (("native", native_bmm), ("emu", emu_bmm)):
            t0 = time.perf_counter()
            L, u = tiled_cholesky(A, t, upd)
            torch.cuda.synchronize()
            res[name] = {"residual": ((A - L @ L.t()).norm() / A.norm()).item(),
                         "total_s": time.perf_counter() - t0, "update_s": u}
        out["cholesky"] = res
    if not only or "cholqr" in only:
        m, k = sz(65536, 8192), sz(512, 256)
        out["cholqr"] = {"m": m, "k": k, "native": cholqr_residual(native_nt, m, k),
                         "emu": cholqr_residual(emu_nt, m, k)}
    if not only or "polar" in only:
        n, it = sz(3072, 384), sz(50, 80)
        out["polar"] = {"n": n, "iters": it, "native": newton_schulz(native_nt, n, it),
                        "emu": newton_schulz(emu_nt, n, it)}
    if not only or "expm" in only:
        n = sz(2048, 512)
        out["expm"] = {"n": n, "native": expm_error(native_nt, n), "emu": expm_error(emu_nt, n)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--small", action="store_true", help="the test sizes")
    ap.add_argument("--only", default="", help="comma-separated: paths,cholesky,cholqr,polar,expm")
    args = ap.parse_args()
    only = [x for x in args.only.split(",") if x]
    print(json.dumps({"device": torch.cuda.get_device_name(0), **run(args.small, only)}), flush=True)


if __name__ == "__main__":
    main()
