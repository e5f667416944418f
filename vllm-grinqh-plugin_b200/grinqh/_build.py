"""Build the native parts of the plugin in-tree.

* ``libgrinqh_b200.so`` -- the sm_100a CUDA kernels behind the C ABI declared in
  ``include/grinqh_b200.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``);
* ``_grinqh_ops.so`` -- the ``torch.ops.grinqh`` registrations (g++ against the
  installed torch), linked to the library above.

Both land next to this file. ``python -m grinqh._build`` (or ``build()``) rebuilds
whatever is older than its sources.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
PLUGIN_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PLUGIN_DIR, "csrc")
INCLUDE = os.path.join(os.path.dirname(PLUGIN_DIR), "include")
LIB = os.path.join(PKG_DIR, "libgrinqh_b200.so")
OPS = os.path.join(PKG_DIR, "_grinqh_ops.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> str:
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if home:
        return home
    nvcc = shutil.which("nvcc")
    if nvcc:
        return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))
    return "/usr/local/cuda"


def _stale(target: str, sources) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


OBJ_DIR = os.path.join(PLUGIN_DIR, "_build")


def build_lib(force: bool = False, verbose: bool = True) -> str:
    """Each .cu compiles to its own object (in parallel; a source recompiles when it or
    any header is newer than its object), then nvcc links the shared library."""
    from concurrent.futures import ThreadPoolExecutor

    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    if not (force or _stale(LIB, cu + headers)):
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    nvcc = os.path.join(_cuda_home(), "bin", "nvcc")
    flags = [*ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}",
             "--expt-relaxed-constexpr", "-diag-suppress", "177"]
    objs, jobs = [], []
    for src in cu:
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs.append([nvcc, *flags, "-c", src, "-o", obj])
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for f in [ex.submit(_run, j, verbose) for j in jobs]:
            f.result()
    # no -lcuda: the library must load on hosts without a driver (CPU CI);
    # cudart is linked statically by nvcc and finds the driver at first use.
    _run([nvcc, *ARCH_FLAGS, "-shared", *objs, "-o", LIB + ".tmp"], verbose)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_ops(force: bool = False, verbose: bool = True) -> str:
    import torch
    from torch.utils.cpp_extension import include_paths, library_paths

    src = os.path.join(CSRC, "torch_ops.cpp")
    deps = [src, LIB] + glob.glob(os.path.join(INCLUDE, "*.h"))
    if force or _stale(OPS, deps):
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
               "-DTORCH_API_INCLUDE_EXTENSION_H", "-Wno-deprecated-declarations",
               *[f"-I{p}" for p in include_paths()], f"-I{os.path.join(_cuda_home(), 'include')}",
               f"-I{INCLUDE}", src, "-o", OPS + ".tmp",
               *[f"-L{p}" for p in library_paths()], f"-L{PKG_DIR}",
               "-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda", "-lgrinqh_b200",
               "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{p}" for p in library_paths()]]
        _run(cmd, verbose)
        os.replace(OPS + ".tmp", OPS)
    return OPS


def build(force: bool = False, verbose: bool = True):
    build_lib(force, verbose)
    build_ops(force, verbose)
    return LIB, OPS


if __name__ == "__main__":
    build(force="--force" in sys.argv)
