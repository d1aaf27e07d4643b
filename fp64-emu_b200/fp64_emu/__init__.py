"""fp64-emu for B200: emulated FP64 GEMM on INT8 tensor cores (RARE / Ozaki-II CRT).

Drop-in for the reference package of CharlesCNorton/fp64-emu
(torch-ext/fp64_emu/__init__.py): the same functions, defaults, plan rules,
routing and op schemas.  C = A @ B is recovered from products modulo
pairwise-coprime moduli (one tcgen05 INT8 GEMM each, plus two first-order
correction GEMMs) by balanced-Garner reconstruction; exactly representable
inputs reproduce bit for bit, and a runtime Cauchy-Schwarz pass keeps any
modulus count range-safe.
"""
import math
from functools import lru_cache

import torch

from ._ops import ops
from . import _meta  # noqa: F401  (fake kernels for torch.compile)

# Pairwise-coprime moduli to the balanced-residue int8 ceiling of 256, largest
# first (reference: torch-ext/fp64_emu/__init__.py:65-67).
_PRIMES = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199,
           197, 193, 191, 181, 179, 173]
_MAXP = 20

_NT_MAX_K = 131071   # single-launch int32 accumulation bound


def _modinv(a, m):
    a %= m
    for x in range(1, m):
        if (a * x) % m == 1:
            return x
    raise ValueError


@lru_cache(maxsize=None)
def _tables(nprimes):
    """(primes int32, inv int32 [P*P], mu int64): the reference's op arguments
    (torch-ext/fp64_emu/__init__.py:78-90).  Only `primes` is used; inv and mu
    are passed for schema compatibility, as in the reference."""
    primes = _PRIMES[:nprimes]
    P = len(primes)
    inv = [0] * (P * P)
    for a in range(P):
        for b in range(P):
            if a < b:
                inv[a * P + b] = _modinv(primes[a] % primes[b], primes[b])
    mu = [(1 << 62) // p for p in primes]
    return (torch.tensor(primes, dtype=torch.int32),
            torch.tensor(inv, dtype=torch.int32),
            torch.tensor(mu, dtype=torch.int64))


def _defaults(K, nprimes, corr):
    if nprimes is None or corr is None:
        dp, dc = plan_config(K)
        nprimes = dp if nprimes is None else nprimes
        corr = dc if corr is None else corr
    return nprimes, corr


def mm(A: torch.Tensor, B: torch.Tensor, nprimes: int = None,
       exact: bool = True, bits: int = 53, corr: bool = None) -> torch.Tensor:
    """Emulated FP64 C = A @ B, with B given as [N, K].

    nprimes: modulus count, one INT8 GEMM each; default sized by plan_config.
    exact: int128 recombine (correctly rounded) vs fp64 recombine (~52 bits).
    bits: mantissa width kept per operand; 53 keeps the full significand.
    corr: the two cross GEMMs cancelling first-order quantization error.
    """
    assert A.dim() == 2 and B.dim() == 2 and A.size(1) == B.size(1)
    M, K = A.shape
    N = B.size(0)
    nprimes, corr = _defaults(K, nprimes, corr)
    primes, inv, mu = _tables(nprimes)
    out = torch.empty(M, N, dtype=torch.float64, device=A.device)
    Ac = A if A.is_contiguous() else A.contiguous()
    Bc = B if B.is_contiguous() else B.contiguous()
    ops.fp64_emu_mm(out, Ac, Bc, primes, inv, mu, exact, bits, corr)
    return out


def mm_nt(A: torch.Tensor, Bt: torch.Tensor, nprimes: int = None,
          exact: bool = True, bits: int = 53, corr: bool = None) -> torch.Tensor:
    """C = A @ Bt with Bt given as [K, N] (standard matmul layout), consumed
    in place: the extraction transposes tiles on chip, no transpose copy."""
    assert A.dim() == 2 and Bt.dim() == 2 and A.size(1) == Bt.size(0)
    K = A.size(1)
    if K > _NT_MAX_K:   # the in-place layout is single-launch; deep K goes via mm
        return mm(A, Bt.t().contiguous(), nprimes, exact, bits, corr)
    nprimes, corr = _defaults(K, nprimes, corr)
    primes, inv, mu = _tables(nprimes)
    out = torch.empty(A.size(0), Bt.size(1), dtype=torch.float64, device=A.device)
    Ac = A if A.is_contiguous() else A.contiguous()
    Bc = Bt if Bt.is_contiguous() else Bt.contiguous()
    ops.fp64_emu_mm_nt(out, Ac, Bc, primes, inv, mu, exact, bits, corr)
    return out


def bmm(A: torch.Tensor, B: torch.Tensor, nprimes: int = None,
        exact: bool = True, bits: int = 53, corr: bool = None) -> torch.Tensor:
    """Batched emulated FP64 C[b] = A[b] @ B[b], with B given as [batch, N, K].

    One operand width serves the whole batch, sized by its widest member; all
    GEMMs of the batch run in one persistent launch."""
    assert A.dim() == 3 and B.dim() == 3 and A.size(0) == B.size(0) and A.size(2) == B.size(2)
    K = A.size(2)
    nprimes, corr = _defaults(K, nprimes, corr)
    primes, inv, mu = _tables(nprimes)
    out = torch.empty(A.size(0), A.size(1), B.size(1), dtype=torch.float64, device=A.device)
    Ac = A if A.is_contiguous() else A.contiguous()
    Bc = B if B.is_contiguous() else B.contiguous()
    ops.fp64_emu_bmm(out, Ac, Bc, primes, inv, mu, exact, bits, corr)
    return out


def bmm_nt(A: torch.Tensor, Bt: torch.Tensor, nprimes: int = None,
           exact: bool = True, bits: int = 53, corr: bool = None) -> torch.Tensor:
    """C[b] = A[b] @ Bt[b] with Bt given as [batch, K, N] (torch.bmm layout),
    consumed in place."""
    assert A.dim() == 3 and Bt.dim() == 3 and A.size(0) == Bt.size(0) and A.size(2) == Bt.size(1)
    K = A.size(2)
    if K > _NT_MAX_K:
        return bmm(A, Bt.transpose(1, 2).contiguous(), nprimes, exact, bits, corr)
    nprimes, corr = _defaults(K, nprimes, corr)
    primes, inv, mu = _tables(nprimes)
    out = torch.empty(A.size(0), A.size(1), Bt.size(2), dtype=torch.float64, device=A.device)
    Ac = A if A.is_contiguous() else A.contiguous()
    Bc = Bt if Bt.is_contiguous() else Bt.contiguous()
    ops.fp64_emu_bmm_nt(out, Ac, Bc, primes, inv, mu, exact, bits, corr)
    return out


def mm_timed(A: torch.Tensor, B: torch.Tensor, nprimes: int = None, exact: bool = True,
             bits: int = 53, corr: bool = None):
    """Returns (C, phase_ms[4]) = [scale+extract, gemms, marker, reconstruct]."""
    M, K = A.shape
    N = B.size(0)
    nprimes, corr = _defaults(K, nprimes, corr)
    primes, inv, mu = _tables(nprimes)
    out = torch.empty(M, N, dtype=torch.float64, device=A.device)
    times = torch.zeros(4, dtype=torch.float32)
    ops.fp64_emu_mm_timed(out, times, A.contiguous(), B.contiguous(), primes, inv, mu,
                          exact, bits, corr)
    return out, times.tolist()


def _host_product(A, B, b_kn, out, nprimes, exact, bits, corr):
    assert A.dim() == B.dim() and A.dim() in (2, 3)
    K = A.size(-1)
    if A.dim() == 3:
        shape = (A.size(0), A.size(1), B.size(2) if b_kn else B.size(1))
    else:
        shape = (A.size(0), B.size(1) if b_kn else B.size(0))
    nprimes, corr = _defaults(K, nprimes, corr)
    primes = _tables(nprimes)[0]
    if out is None:
        out = torch.empty(shape, dtype=torch.float64, pin_memory=A.is_pinned())
    Ac = A if A.is_contiguous() else A.contiguous()
    Bc = B if B.is_contiguous() else B.contiguous()
    ops.fp64_emu_gemm_host(out, Ac, Bc, primes, b_kn, exact, bits, corr)
    return out


def mm_nt_host(A: torch.Tensor, Bt: torch.Tensor, out: torch.Tensor = None, nprimes: int = None,
               exact: bool = True, bits: int = 53, corr: bool = None) -> torch.Tensor:
    """mm_nt for operands and result in host memory, on the current CUDA
    device: the operands are copied in, and each finished block of C is copied
    back while later blocks are still computing.  Use page-locked tensors
    (pin_memory) for the copies to overlap.  Returns once `out` holds C."""
    return _host_product(A, Bt, True, out, nprimes, exact, bits, corr)


def mm_host(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor = None, nprimes: int = None,
            exact: bool = True, bits: int = 53, corr: bool = None) -> torch.Tensor:
    """mm (B given as [N, K]) for host-resident operands; see mm_nt_host."""
    return _host_product(A, B, False, out, nprimes, exact, bits, corr)


def bmm_nt_host(A: torch.Tensor, Bt: torch.Tensor, out: torch.Tensor = None, nprimes: int = None,
                exact: bool = True, bits: int = 53, corr: bool = None) -> torch.Tensor:
    """bmm_nt for host-resident operands; see mm_nt_host."""
    return _host_product(A, Bt, True, out, nprimes, exact, bits, corr)


def bmm_host(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor = None, nprimes: int = None,
             exact: bool = True, bits: int = 53, corr: bool = None) -> torch.Tensor:
    """bmm for host-resident operands; see mm_nt_host."""
    return _host_product(A, B, False, out, nprimes, exact, bits, corr)


def range_bits(nprimes: int) -> float:
    """Signed CRT range of the first `nprimes` moduli, in bits."""
    r = 0.0
    for p in _PRIMES[:nprimes]:
        r += math.log2(p)
    return r - 1.0


def plan_config(K: int) -> tuple:
    """(nprimes, corr) reaching FP64-equivalent accuracy at depth K; the
    runtime Cauchy-Schwarz pass keeps the choice range-safe."""
    need = 2 * 49 + math.ceil(math.log2(max(K, 1))) + 1 - 3.4
    for n in range(1, _MAXP + 1):
        if range_bits(n) >= need:
            return n, True
    return _MAXP, True


def plan(K: int, bits: int = 53) -> int:
    """Smallest worst-case range-safe nprimes at depth K and width bits: the
    exact product needs 2*bits + ceil(log2 K) + 1 bits."""
    need = 2 * bits + math.ceil(math.log2(max(K, 1))) + 1
    for n in range(1, _MAXP + 1):
        if range_bits(n) >= need:
            return n
    raise ValueError(f"K={K} at bits={bits} needs more range than {_MAXP} primes give")


from .host import HostStream  # noqa: E402  (uses _defaults and _tables above)

__all__ = ["mm", "mm_nt", "bmm", "bmm_nt", "mm_timed", "plan", "plan_config", "range_bits",
           "mm_host", "mm_nt_host", "bmm_host", "bmm_nt_host", "HostStream"]
