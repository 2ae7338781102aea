"""Build the in-tree native libraries of the package.

* ``libnsa_sel.so`` -- the sm_100a kernel family and its C ABI (include/nsa_sel.h), compiled
  by nvcc with ``-gencode arch=compute_100a,code=sm_100a``.  It links the CUDA runtime
  dynamically so that, inside a PyTorch process, it shares torch's runtime (same current
  device, same streams).
* ``_C*.so`` -- the PyTorch extension (nsa_sel_torch.cpp) exposing the reference's op
  signature; host code only, it opens libnsa_sel.so at first use.

Both land next to this file so they travel with the source tree.  ``python -m
nsa_hopper_b200.build`` builds whatever is out of date.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from typing import List

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
REPO = os.path.dirname(PKG)
INCLUDE = os.path.join(REPO, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
LIB = os.path.join(PKG, "libnsa_sel.so")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _ext_path() -> str:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(PKG, "_C" + suffix)


def _stale(target: str, sources: List[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd: List[str]) -> None:
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {r.returncode})")


def build_kernel_lib(force: bool = False, extra: List[str] = ()) -> str:
    # the translation unit first, then every header it may include (staleness check)
    srcs = [os.path.join(CSRC, "nsa_sel_api.cu")] + sorted(
        os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh"))
    srcs.append(os.path.join(INCLUDE, "nsa_sel.h"))
    if not force and not _stale(LIB, srcs):
        return LIB
    cmd = [NVCC, *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
           "-cudart", "shared", f"-I{INCLUDE}", f"-I{CSRC}", "-Xlinker", f"-rpath={CUDA_HOME}/lib64",
           *extra, "-o", LIB + ".tmp", srcs[0]]
    _run(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_peaks_lib(force: bool = False) -> str:
    """libnsa_peaks.so: the on-chip ceiling microbenchmarks behind bench.py's roofline (measurement
    code, not on the product path)."""
    out = os.path.join(PKG, "libnsa_peaks.so")
    srcs = [os.path.join(CSRC, "nsa_peaks.cu")] + sorted(
        os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh"))
    if not force and not _stale(out, srcs):
        return out
    cmd = [NVCC, *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
           "-cudart", "shared", f"-I{INCLUDE}", f"-I{CSRC}", "-Xlinker", f"-rpath={CUDA_HOME}/lib64",
           "-o", out + ".tmp", srcs[0]]
    _run(cmd)
    os.replace(out + ".tmp", out)
    return out


def build_torch_ext(force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    out = _ext_path()
    srcs = [os.path.join(CSRC, "nsa_sel_torch.cpp"), os.path.join(INCLUDE, "nsa_sel.h")]
    if not force and not _stale(out, srcs):
        return out
    inc = cpp_extension.include_paths() + [sysconfig.get_paths()["include"], os.path.join(CUDA_HOME, "include"), INCLUDE]
    libdirs = cpp_extension.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in inc], srcs[0],
           *[f"-L{p}" for p in libdirs], *[f"-Wl,-rpath,{p}" for p in libdirs],
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-ldl",
           "-o", out + ".tmp"]
    _run(cmd)
    os.replace(out + ".tmp", out)
    return out


def build_all(force: bool = False) -> None:
    build_kernel_lib(force)
    build_peaks_lib(force)
    build_torch_ext(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print("built", LIB, _ext_path())
