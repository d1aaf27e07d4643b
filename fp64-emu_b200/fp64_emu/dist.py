"""Partitioned multi-GPU products: one process per GPU, torch.distributed over
NCCL for the plumbing.

The product shards with no data-path collective:
  * mm / mm_nt: C is split into a pr x pc grid of blocks (2-D: 2 -> 1x2,
    4 -> 2x2, 8 -> 2x4); rank (i, j) holds A's row block i and B's column
    block j, so each rank extracts only its own share of both operands;
  * bmm / bmm_nt: the batch is split.
The only collective on the timed path is one MAX all-reduce of two floats
(the operand maxima of the log2 norms) between the sizing and compute phases,
which makes every rank use the single-GPU operand width; with the column-slab
rule pinned to the full column count, every block is bit-identical to the
corresponding block of a single-GPU run.  Distributing the operands (a
broadcast or scatter of the shared operand) happens once, outside the
steady-state loop.
"""
import torch
import torch.distributed as dist

from . import _tables, plan_config
from ._ops import ops

PHASE_SIZING, PHASE_EXTRACT, PHASE_GEMM, PHASE_RECON = 1, 2, 4, 8
PHASE_COMPUTE = PHASE_EXTRACT | PHASE_GEMM | PHASE_RECON


def grid_shape(world):
    """(row blocks, column blocks) of the 2-D partition for `world` ranks: as
    square as the rank count allows, with the extra factor on the columns
    (2 -> 1x2, 4 -> 2x2, 8 -> 2x4).  Each rank extracts its rows of A and its
    columns of B; the rows of A are extracted chunk by chunk behind the GEMM,
    while B's columns are extracted before it starts, so B is the operand to
    split further."""
    pr = 1
    while (pr * 2) ** 2 <= world and world % (pr * 2) == 0:
        pr *= 2
    return pr, world // pr


def block_range(n, parts, i):
    """[start, stop) of block i when n splits into `parts` nearly equal blocks."""
    base, rem = divmod(n, parts)
    start = i * base + min(i, rem)
    return start, start + base + (1 if i < rem else 0)


def rank_block(rank, world, M, N):
    """(row range, column range) of C owned by `rank` in the 2-D partition."""
    pr, pc = grid_shape(world)
    i, j = divmod(rank, pc)
    return block_range(M, pr, i), block_range(N, pc, j)


def sized_protocol(sizing, maxlg, group=None):
    """Run this rank's sizing (which fills `maxlg`, the two operand maxima of
    the log2 norms), then MAX-all-reduce them over the group so every rank
    derives the single-GPU operand width.  Every rank calls this in the same
    order; it is the only collective of a partitioned product."""
    sizing()
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(maxlg, op=dist.ReduceOp.MAX, group=group)
    return maxlg


class ShardedProduct:
    """One rank's share of a partitioned emulated-FP64 product.

    A_local: [M_i, K] (or [b_i, M, K]); B_local: [K, N_j] / [N_j, K] (or the
    batched forms); slab_cols: the full column count of B over all ranks
    (batch * N for batched products) so the per-column norm sums are ordered
    as in a single-GPU run.  Call run() on every rank in the same order."""

    def __init__(self, A_local, B_local, b_kn, slab_cols, K, nprimes=None, exact=True, bits=53, corr=None,
                 group=None):
        nprimes, corr = _defaults(K, nprimes, corr)
        self.A, self.B = A_local.contiguous(), B_local.contiguous()
        self.b_kn, self.exact, self.bits, self.corr = b_kn, exact, bits, corr
        self.slab_cols = int(slab_cols) if b_kn else 0
        self.primes = _tables(nprimes)[0]
        self.group = group
        nbytes = ops.fp64_emu_workspace_bytes(self.A, self.B, self.primes, b_kn, corr, self.slab_cols)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=self.A.device)
        self.maxlg = self.ws[:8].view(torch.float32)

    def _phase(self, out, phases):
        ops.fp64_emu_gemm_ws(out, self.ws, self.A, self.B, self.primes, self.b_kn, self.exact, self.bits,
                             self.corr, phases, self.slab_cols)

    def sizing(self, out):
        sized_protocol(lambda: self._phase(out, PHASE_SIZING), self.maxlg, self.group)

    def run(self, out):
        self.sizing(out)
        self._phase(out, PHASE_COMPUTE)
        return out


def _defaults(K, nprimes, corr):
    if nprimes is None or corr is None:
        dp, dc = plan_config(K)
        nprimes = dp if nprimes is None else nprimes
        corr = dc if corr is None else corr
    return nprimes, corr


def mm_nt_2d(A_rows, Bt_cols, n_total, group=None, **kw):
    """This rank's block C[rows, cols] = A_rows @ Bt_cols of a product whose B
    has n_total columns over all ranks."""
    out = torch.empty(A_rows.size(0), Bt_cols.size(1), dtype=torch.float64, device=A_rows.device)
    return ShardedProduct(A_rows, Bt_cols, True, n_total, A_rows.size(1), group=group, **kw).run(out)


def bmm_nt_sharded(A_b, Bt_b, batch_total, group=None, **kw):
    """This rank's members C[b] = A[b] @ Bt[b] of a batch of batch_total."""
    out = torch.empty(A_b.size(0), A_b.size(1), Bt_b.size(2), dtype=torch.float64, device=A_b.device)
    return ShardedProduct(A_b, Bt_b, True, batch_total * Bt_b.size(2), A_b.size(2), group=group, **kw).run(out)
