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


def build_lib(force: bool = False, verbose: bool = True) -> str:
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = cu + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    if force or _stale(LIB, deps):
        nvcc = os.path.join(_cuda_home(), "bin", "nvcc")
        cmd = [nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
               f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr", "-diag-suppress", "177",
               *cu, "-o", LIB + ".tmp"]
        # no -lcuda: the library must load on hosts without a driver (CPU CI);
        # cudart is linked statically by nvcc and finds the driver at first use.
        _run(cmd, verbose)
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
