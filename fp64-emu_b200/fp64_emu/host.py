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
import os

import torch

from . import _defaults, _tables
from ._ops import ops


def gpu_local_cpus(device=None):
    """The CPU cores NVML reports as local to `device` (its NUMA node's
    cores), or None when NVML cannot tell.  Read only: no GPU setting is
    touched."""
    try:
        import pynvml
        idx = torch.cuda.current_device() if device is None else torch.device(device).index
        uuid = str(torch.cuda.get_device_properties(idx).uuid)
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            words = (os.cpu_count() + 63) // 64
            mask = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        finally:
            pynvml.nvmlShutdown()
        cpus = [64 * w + b for w, m in enumerate(mask) for b in range(64) if (int(m) >> b) & 1]
        cpus = [c for c in cpus if c < os.cpu_count()]
        return cpus or None
    except Exception:  # noqa: BLE001  (no NVML, no permission, unknown device)
        return None


class gpu_local_allocation:
    """Context manager: while active, this process runs on the cores local to
    `device`, so page-locked buffers allocated inside it are placed on the
    GPU's NUMA node; the previous CPU affinity is restored on exit (copies
    keep using the buffers' placement, whichever cores later run).
    .cpus: the cores used, or None when NVML could not tell."""

    def __init__(self, device=None):
        self.device = device
        self.cpus = None
        self._old = None

    def __enter__(self):
        self._old = os.sched_getaffinity(0)
        self.cpus = bind_to_gpu_cpus(self.device)
        return self

    def __exit__(self, *exc):
        if self._old is not None:
            os.sched_setaffinity(0, self._old)
        return False


def bind_to_gpu_cpus(device=None):
    """Restrict this process to the cores local to `device`, so page-locked
    buffers allocated afterwards are first touched on the GPU's NUMA node and
    host-device copies do not cross the socket link.  Returns the cores, or
    None (affinity unchanged) when they are unknown."""
    cpus = gpu_local_cpus(device)
    if cpus:
        os.sched_setaffinity(0, cpus)
    return cpus

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
        self._streams = [self.h2d.cuda_stream, self.comp.cuda_stream, self.d2h.cuda_stream]
        self._caller = self._event()
        self.slots = [None] * self.depth
        self.n = 0

    def _event(self):
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))   # creates the CUDA event
        return ev

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
                 "loaded": self._event(), "computed": self._event(), "done": self._event(), "used": False}
            self.slots[i] = s
        return s

    def submit(self, A, B, out):
        """Queue out = op(A, B) for CPU tensors A, B, out (page-locked for the
        copies to overlap).  Returns at once; the inputs must stay unchanged
        and `out` unread until synchronize()."""
        if A.is_cuda or B.is_cuda or out.is_cuda:
            raise RuntimeError("HostStream.submit takes CPU tensors")
        if A.dtype != torch.float64 or B.dtype != torch.float64 or out.dtype != torch.float64:
            raise RuntimeError("HostStream.submit takes float64 tensors")
        A, B = A.contiguous(), B.contiguous()
        s = self._slot(self.n % self.depth, A, B)
        # one native call queues the operand copies, the product and the
        # result copy on the three streams, ordered by the slot's events
        ops.fp64_emu_host_submit(out, A, B, s["A"], s["B"], s["C"], s["ws"], s["primes"], self.b_kn, self.exact,
                                 self.bits, s["corr"], self._streams,
                                 [self._caller.cuda_event, s["loaded"].cuda_event, s["computed"].cuda_event,
                                  s["done"].cuda_event], s["used"])
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
