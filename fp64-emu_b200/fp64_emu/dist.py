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


def host_share_ranges(rank, world, M, N, K, b_kn):
    """The host shares rank copies in for a ShardedHostStream product: the
    global rows [a0, a1) of A (a slice of its row block, split over the pc
    ranks of its grid row, ceil-sized so only the last slices are short) and
    the range [b0, b1) of the first dimension of B's column block ([K, nb]
    when b_kn, else [nb, K]), split over the pr ranks of its grid column."""
    pr, pc = grid_shape(world)
    gi, gj = divmod(rank, pc)
    (r0, r1), (c0, c1) = rank_block(rank, world, M, N)
    mb, nb = r1 - r0, c1 - c0
    a_rows = -(-mb // pc)
    a0 = min(mb, gj * a_rows)
    ext = K if b_kn else nb
    b_rows = -(-ext // pr)
    b0 = min(ext, gi * b_rows)
    return (r0 + a0, r0 + min(mb, a0 + a_rows)), (b0, min(ext, b0 + b_rows))


class ShardedHostStream:
    """A stream of partitioned products whose operands and results live in host
    memory, one process per GPU.

    Rank (i, j) of the pr x pc grid owns C's block (i, j) and needs A's row
    block i and B's column block j.  Over PCIe each rank copies in only a
    disjoint share of those blocks (A's row block split over the pc ranks of
    grid row i, B's column block split over the pr ranks of grid column j), so
    the whole job moves each operand byte across PCIe once, as on one GPU; two
    NCCL all-gathers over NVLink (within the grid row and within the grid
    column) complete the blocks on the device.  Then the usual sizing
    (+ MAX all-reduce) and product, and the copy of the rank's C block back.
    With `depth` buffer sets in rotation on four streams (copy in, gather,
    compute, copy out), neighbouring products overlap stage by stage.

    Batched products ("bmm_nt", "bmm"; batch > 1) are split by batch member
    instead: each rank copies in its own members' operands, so nothing needs
    gathering, and the stages are copy in, sizing with the MAX all-reduce and
    product, copy out.

    Host layout: `host_shares(A, B)` cuts a full host A and B into this rank's
    shares (once, outside any timed loop); submit(a_share, b_share, c_block)
    takes page-locked CPU tensors shaped like those shares and this rank's C
    block.  kind: "mm_nt" (B given as [K, N]) or "mm" (B as [N, K]), or their
    batched forms "bmm_nt" ([batch, K, N]) and "bmm" ([batch, N, K])."""

    def __init__(self, kind, M, N, K, nprimes=None, exact=True, bits=53, corr=None, depth=2, batch=1):
        if kind not in ("mm", "mm_nt", "bmm", "bmm_nt"):
            raise ValueError("kind must be mm, mm_nt, bmm or bmm_nt")
        self.batched = kind in ("bmm", "bmm_nt")
        if self.batched != (batch > 1):
            raise ValueError("bmm / bmm_nt take batch > 1, mm / mm_nt batch = 1")
        self.kind, self.b_kn = kind, kind in ("mm_nt", "bmm_nt")
        self.M, self.N, self.K, self.batch = M, N, K, batch
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        if self.batched:
            self.m0, self.m1 = block_range(batch, self.world, self.rank)
            self.nprimes, self.exact, self.bits, self.corr = nprimes, exact, bits, corr
            self.depth = max(1, int(depth))
            self.dev = torch.device("cuda", torch.cuda.current_device())
            self.streams = [torch.cuda.Stream(self.dev) for _ in range(4)]
            self.slots = [None] * self.depth
            self.n = 0
            return
        self.pr, self.pc = grid_shape(self.world)
        self.gi, self.gj = divmod(self.rank, self.pc)
        (self.r0, self.r1), (self.c0, self.c1) = rank_block(self.rank, self.world, M, N)
        self.mb, self.nb = self.r1 - self.r0, self.c1 - self.c0
        # every rank creates every row and column group, in the same order
        self.row_groups = [dist.new_group([i * self.pc + j for j in range(self.pc)]) for i in range(self.pr)]
        self.col_groups = [dist.new_group([i * self.pc + j for i in range(self.pr)]) for j in range(self.pc)]
        self.row_group, self.col_group = self.row_groups[self.gi], self.col_groups[self.gj]
        # shares: A rows of the row block over the pc ranks of the grid row;
        # B's block (as [K, nb] or [nb, K]) split along its first dimension
        # over the pr ranks of the grid column; padded to equal sizes for the
        # all-gathers
        self.a_rows = -(-self.mb // self.pc)
        self.b_rows = -(-(K if self.b_kn else self.nb) // self.pr)
        self.nprimes, self.exact, self.bits, self.corr = nprimes, exact, bits, corr
        self.depth = max(1, int(depth))
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.streams = [torch.cuda.Stream(dev) for _ in range(4)]
        self.slots = [None] * self.depth
        self.n = 0

    def a_share_range(self):
        """Rows of A (global indices) this rank copies in."""
        return host_share_ranges(self.rank, self.world, self.M, self.N, self.K, self.b_kn)[0]

    def b_share_range(self):
        """First-dimension range of B's column block ([K, nb] or [nb, K]) this rank copies in."""
        return host_share_ranges(self.rank, self.world, self.M, self.N, self.K, self.b_kn)[1]

    def host_shares(self, A, B):
        """This rank's page-locked shares of full host operands A [M, K] and
        B ([K, N] or [N, K]), and a page-locked C block to receive results
        (batched: this rank's members of A, B and C)."""
        if self.batched:
            m0, m1 = self.m0, self.m1
            a = A[m0:m1].contiguous().pin_memory()
            b = B[m0:m1].contiguous().pin_memory()
            c = torch.empty(m1 - m0, self.M, self.N, dtype=torch.float64).pin_memory()
            return a, b, c
        a0, a1 = self.a_share_range()
        b0, b1 = self.b_share_range()
        blk = B[:, self.c0:self.c1] if self.b_kn else B[self.c0:self.c1]
        a = A[a0:a1].contiguous().pin_memory()
        b = blk[b0:b1].contiguous().pin_memory()
        c = torch.empty(self.mb, self.nb, dtype=torch.float64).pin_memory()
        return a, b, c

    def _slot(self, k):
        s = self.slots[k]
        if s is not None:
            return s
        if self.batched:
            return self._batch_slot(k)
        dev, K = self.dev, self.K
        bshape_full = (K, self.nb) if self.b_kn else (self.nb, K)
        with torch.cuda.stream(self.streams[2]):
            s = {"a_sh": torch.empty(self.a_rows, K, dtype=torch.float64, device=dev),
                 "b_sh": torch.empty((self.b_rows,) + bshape_full[1:], dtype=torch.float64, device=dev),
                 "a_all": torch.empty(self.pc * self.a_rows, K, dtype=torch.float64, device=dev),
                 "b_all": torch.empty((self.pr * self.b_rows,) + bshape_full[1:], dtype=torch.float64, device=dev),
                 "C": torch.empty(self.mb, self.nb, dtype=torch.float64, device=dev)}
            s["A"] = s["a_all"][:self.mb]
            s["B"] = s["b_all"][:bshape_full[0]]
            s["sp"] = ShardedProduct(s["A"], s["B"], self.b_kn, self.N, K, nprimes=self.nprimes, exact=self.exact,
                                     bits=self.bits, corr=self.corr)
        for name in ("loaded", "gathered", "computed", "done"):
            s[name] = torch.cuda.Event()
        s["used"] = False
        self.slots[k] = s
        return s

    def _batch_slot(self, k):
        dev, K, M, N = self.dev, self.K, self.M, self.N
        nb = self.m1 - self.m0
        with torch.cuda.stream(self.streams[2]):
            s = {"A": torch.empty(nb, M, K, dtype=torch.float64, device=dev),
                 "B": torch.empty((nb, K, N) if self.b_kn else (nb, N, K), dtype=torch.float64, device=dev),
                 "C": torch.empty(nb, M, N, dtype=torch.float64, device=dev)}
            # the column-slab rule runs over all members' columns, as on one GPU
            s["sp"] = ShardedProduct(s["A"], s["B"], self.b_kn, self.batch * N, K, nprimes=self.nprimes,
                                     exact=self.exact, bits=self.bits, corr=self.corr)
        for name in ("loaded", "computed", "done"):
            s[name] = torch.cuda.Event()
        s["used"] = False
        self.slots[k] = s
        return s

    def _submit_batched(self, a_share, b_share, c_block):
        h2d, _, comp, d2h = self.streams
        s = self._slot(self.n % self.depth)
        cur = torch.cuda.current_stream(self.dev)
        for st in self.streams:
            st.wait_stream(cur)
        if s["used"]:
            h2d.wait_event(s["computed"])   # the operands were read by the product
            comp.wait_event(s["done"])      # the C members left the device
        with torch.cuda.stream(h2d):
            s["A"].copy_(a_share, non_blocking=True)
            s["B"].copy_(b_share, non_blocking=True)
            s["loaded"].record(h2d)
        comp.wait_event(s["loaded"])
        with torch.cuda.stream(comp):
            sp = s["sp"]
            sp.sizing(s["C"])    # MAX all-reduce of the operand maxima over all ranks
            sp._phase(s["C"], PHASE_COMPUTE)
            s["computed"].record(comp)
        d2h.wait_event(s["computed"])
        with torch.cuda.stream(d2h):
            c_block.copy_(s["C"], non_blocking=True)
            s["done"].record(d2h)
        s["used"] = True
        self.n += 1
        return c_block

    def submit(self, a_share, b_share, c_block):
        """Queue this rank's part of one product; every rank calls submit in
        the same order.  Returns at once; c_block holds the rank's C block
        after synchronize()."""
        if self.batched:
            return self._submit_batched(a_share, b_share, c_block)
        h2d, comm, comp, d2h = self.streams
        s = self._slot(self.n % self.depth)
        cur = torch.cuda.current_stream(self.dev)
        for st in self.streams:
            st.wait_stream(cur)
        if s["used"]:
            h2d.wait_event(s["gathered"])    # the share buffers were gathered from
            comm.wait_event(s["computed"])   # the blocks were read by the product
            comp.wait_event(s["done"])       # the C block left the device
        with torch.cuda.stream(h2d):
            s["a_sh"][:a_share.size(0)].copy_(a_share, non_blocking=True)
            s["b_sh"][:b_share.size(0)].copy_(b_share, non_blocking=True)
            s["loaded"].record(h2d)
        comm.wait_event(s["loaded"])
        with torch.cuda.stream(comm):
            dist.all_gather_into_tensor(s["a_all"], s["a_sh"], group=self.row_group)
            dist.all_gather_into_tensor(s["b_all"], s["b_sh"], group=self.col_group)
            s["gathered"].record(comm)
        comp.wait_event(s["gathered"])
        with torch.cuda.stream(comp):
            sp = s["sp"]
            sp.sizing(s["C"])
            sp._phase(s["C"], PHASE_COMPUTE)
            s["computed"].record(comp)
        d2h.wait_event(s["computed"])
        with torch.cuda.stream(d2h):
            c_block.copy_(s["C"], non_blocking=True)
            s["done"].record(d2h)
        s["used"] = True
        self.n += 1
        return c_block

    def join(self, stream=None):
        st = stream or torch.cuda.current_stream(self.dev)
        for s in self.slots:
            if s is not None and s["used"]:
                st.wait_event(s["done"])

    def synchronize(self):
        for s in self.slots:
            if s is not None and s["used"]:
                s["done"].synchronize()
