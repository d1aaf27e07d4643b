"""Loads the in-tree torch op library (_fp64_emu_b200.so, which links libf64e.so)
and exposes its op namespace as `ops`.  There is no fallback: if the CUDA
extension is missing, importing the package fails with the build command."""
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
EXT_PATH = os.path.join(_HERE, "_fp64_emu_b200.so")
LIB_PATH = os.path.join(_HERE, "libf64e.so")


def _load():
    ns = getattr(torch.ops, "fp64_emu_b200")
    try:
        getattr(ns, "fp64_emu_mm")
        return ns
    except (AttributeError, RuntimeError):
        pass
    if not os.path.exists(EXT_PATH):
        raise ImportError(
            "fp64_emu: the CUDA extension is not built (missing %s); run "
            "`python fp64-emu_b200/build.py`" % EXT_PATH)
    torch.ops.load_library(EXT_PATH)
    return getattr(torch.ops, "fp64_emu_b200")


ops = _load()
