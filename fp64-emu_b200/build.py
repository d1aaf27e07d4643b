"""In-tree build of the fp64-emu B200 libraries.

  fp64_emu/libf64e.so          CUDA kernels + C ABI (include/f64e.h), sm_100a
  fp64_emu/_fp64_emu_b200.so   torch op binding (namespace fp64_emu_b200),
                               linked against libf64e.so
  fp64_emu/libf64e_debug.so    the same C ABI built with F64E_DEBUG_BOUNDS:
                               every extraction, GEMM-epilogue and
                               reconstruction access checked against its
                               buffer, misses recorded in the status word and
                               skipped (a checking build for callers of the C
                               ABI; nothing loads it by default)

Both land inside the package directory, so they travel with the working tree
and are found without any install step.  Usage: python fp64-emu_b200/build.py
[--force] [-v]
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
PKG = HERE / "fp64_emu"
OBJ = HERE / "_build"
INCLUDE = ROOT / "include"
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
CXX = "/usr/bin/g++"

CUDA_SOURCES = ["f64e_api.cu", "f64e_sizing.cu", "f64e_extract.cu", "f64e_gemm.cu", "f64e_gemm_check.cu",
                "f64e_recon.cu", "f64e_deepk.cu", "f64e_noalloc.cu"]
HEADERS = ["f64e_device.cuh", "f64e_params.h", "f64e_kernels.h", "f64e_crt64.cuh"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-ccbin", CXX,
              f"-I{INCLUDE}", f"-I{CSRC}"]
LIB = PKG / "libf64e.so"
LIB_DEBUG = PKG / "libf64e_debug.so"
EXT = PKG / "_fp64_emu_b200.so"


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(Path(d).stat().st_mtime <= t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")
    return r


def build_lib(force=False, verbose=False, extra_nvcc=(), debug=False):
    obj_dir = OBJ / "debug" if debug else OBJ
    lib = LIB_DEBUG if debug else LIB
    flags = NVCC_FLAGS + (["-DF64E_DEBUG_BOUNDS"] if debug else []) + list(extra_nvcc)
    obj_dir.mkdir(parents=True, exist_ok=True)
    hdrs = [CSRC / h for h in HEADERS] + [INCLUDE / "f64e.h"]
    jobs = []
    for src in CUDA_SOURCES:
        o = obj_dir / (Path(src).stem + ".o")
        if force or not _newer(o, [CSRC / src] + hdrs):
            jobs.append([NVCC, "-c", CSRC / src, "-o", o] + flags)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda c: _run(c, verbose), jobs))
    objs = [obj_dir / (Path(s).stem + ".o") for s in CUDA_SOURCES]
    if force or jobs or not _newer(lib, objs):
        _run([NVCC, "-shared", "-o", lib] + objs + ["-gencode", "arch=compute_100a,code=sm_100a",
                                                     "-cudart", "shared", "-ccbin", CXX], verbose)
    return lib


def build_ext(force=False, verbose=False):
    import torch
    import torch.utils.cpp_extension as ce
    src = CSRC / "torch_binding.cpp"
    if not force and _newer(EXT, [src, INCLUDE / "f64e.h", LIB]):
        return EXT
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], str(INCLUDE)]
    libs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [CXX, "-shared", "-fPIC", "-O2", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", src, "-o", EXT]
    cmd += [f"-I{p}" for p in inc] + [f"-L{p}" for p in libs] + [f"-Wl,-rpath,{p}" for p in libs]
    cmd += [f"-L{PKG}", "-Wl,-rpath,$ORIGIN", "-lf64e", "-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda",
            "-ltorch_cuda", "-lcudart"]
    _run(cmd, verbose)
    return EXT


def build(force=False, verbose=False):
    build_lib(force, verbose)
    build_ext(force, verbose)
    build_lib(force, verbose, debug=True)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--lib-only", action="store_true")
    a = ap.parse_args()
    if a.lib_only:
        build_lib(a.force, a.v)
    else:
        build(a.force, a.v)
    print("built", LIB, "" if a.lib_only else f"{EXT} {LIB_DEBUG}")
