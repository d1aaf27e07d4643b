"""A stream of products whose operands and results live in host memory.

Each submitted product goes through three stages on three CUDA streams:
host-to-device copies of its operands, the emulated product on the device,
and the device-to-host copy of its result.  With `depth` sets of device
buffers in rotation, the copies of one product overlap the computation of
its neighbours, so a stream of host-resident products runs at the rate of its
slowest stage (on one B200 over PCIe: the operand copies) instead of the sum
of the three.  The single-call form of the same idea is fp64_emu.mm_nt_host
(result blocks copied back while later blocks compute).

    hs = HostStream("mm_nt")
    for A, Bt, C in jobs:            # page-locked CPU tensors
        hs.submit(A, Bt, C)          # returns at once
    hs.synchronize()                 # every C now holds its product

Results are bit-identical to the device-resident call of the same kind.
"""
import torch

from . import _defaults, _tables
from ._ops import ops

_KINDS = {"mm": False, "mm_nt": True, "bmm": False, "bmm_nt": True}


class HostStream:
    def __init__(self, kind="mm_nt", nprimes=None, exact=True, bits=53, corr=None, depth=2, device=None):
        if kind not in _KINDS:
            raise ValueError(f"kind must be one of {sorted(_KINDS)}")
        self.kind, self.b_kn = kind, _KINDS[kind]
        self.nprimes, self.exact, self.bits, self.corr = nprimes, exact, bits, corr
        self.depth = max(1, int(depth))
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.h2d = torch.cuda.Stream(self.device)
        self.comp = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self.slots = [None] * self.depth
        self.n = 0

    def _slot(self, i, A, B):
        """Device buffers of slot i for operands shaped like A and B."""
        s = self.slots[i]
        if s is None or s["A"].shape != A.shape or s["B"].shape != B.shape:
            if s is not None:
                s["done"].synchronize()
            dev = self.device
            if A.dim() == 3:
                cshape = (A.size(0), A.size(1), B.size(2) if self.b_kn else B.size(1))
            else:
                cshape = (A.size(0), B.size(1) if self.b_kn else B.size(0))
            K = A.size(-1)
            nprimes, corr = _defaults(K, self.nprimes, self.corr)
            primes = _tables(nprimes)[0]
            with torch.cuda.stream(self.comp):
                Ad = torch.empty(A.shape, dtype=torch.float64, device=dev)
                Bd = torch.empty(B.shape, dtype=torch.float64, device=dev)
                Cd = torch.empty(cshape, dtype=torch.float64, device=dev)
                ws = torch.empty(ops.fp64_emu_workspace_bytes(Ad, Bd, primes, self.b_kn, corr), dtype=torch.uint8,
                                 device=dev)
            s = {"A": Ad, "B": Bd, "C": Cd, "ws": ws, "primes": primes, "corr": corr,
                 "loaded": torch.cuda.Event(), "computed": torch.cuda.Event(), "done": torch.cuda.Event(),
                 "used": False}
            self.slots[i] = s
        return s

    def submit(self, A, B, out):
        """Queue out = op(A, B) for CPU tensors A, B, out (page-locked for the
        copies to overlap).  Returns at once; the inputs must stay unchanged
        and `out` unread until synchronize()."""
        if A.is_cuda or B.is_cuda or out.is_cuda:
            raise RuntimeError("HostStream.submit takes CPU tensors")
        s = self._slot(self.n % self.depth, A, B)
        cur = torch.cuda.current_stream(self.device)
        for st in (self.h2d, self.comp, self.d2h):
            st.wait_stream(cur)                       # work the caller queued before this call
        if s["used"]:
            self.h2d.wait_event(s["computed"])        # the slot's previous product has read its operands
            self.comp.wait_event(s["done"])           # ... and its result has left the device
        with torch.cuda.stream(self.h2d):
            s["A"].copy_(A, non_blocking=True)
            s["B"].copy_(B, non_blocking=True)
            s["loaded"].record(self.h2d)
        self.comp.wait_event(s["loaded"])
        with torch.cuda.stream(self.comp):
            ops.fp64_emu_gemm_ws(s["C"], s["ws"], s["A"], s["B"], s["primes"], self.b_kn, self.exact, self.bits,
                                 s["corr"], 15, 0)
            s["computed"].record(self.comp)
        self.d2h.wait_event(s["computed"])
        with torch.cuda.stream(self.d2h):
            out.copy_(s["C"], non_blocking=True)
            s["done"].record(self.d2h)
        s["used"] = True
        self.n += 1
        return out

    def join(self, stream=None):
        """Make `stream` (default: the current stream) wait for every submitted product."""
        st = stream or torch.cuda.current_stream(self.device)
        for s in self.slots:
            if s is not None and s["used"]:
                st.wait_event(s["done"])

    def synchronize(self):
        for s in self.slots:
            if s is not None and s["used"]:
                s["done"].synchronize()
