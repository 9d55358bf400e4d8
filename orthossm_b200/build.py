"""Build the orthossm_b200 C-ABI shared library in-tree with nvcc (sm_100a).

    python -m orthossm_b200.build            # -> orthossm_b200/_lib/liborthossm_b200.so

The library links the CUDA runtime dynamically (libcudart.so.12), so inside a
PyTorch process it shares torch's runtime and streams.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(PKG, "_lib")
LIBNAME = "liborthossm_b200.so"
SOURCES = ["ossm_capi.cu", "ossm_forward.cu", "ossm_forward_3p.cu", "ossm_forward_grp.cu", "ossm_host.cu", "ossm_lion.cu", "ossm_noalloc.cu", "ossm_reverse.cu", "ossm_ttt.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def lib_path() -> str:
    return os.path.join(LIBDIR, LIBNAME)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    out = lib_path()
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(INCLUDE, "orthossm_b200.h"))
    if not force and os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(d) for d in deps):
        return out
    cuda_lib = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "lib64")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-cudart", "shared", f"-I{INCLUDE}", f"-I{CSRC}", "-Xlinker", f"-rpath,{cuda_lib}",
           "-o", out + ".tmp", *srcs]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
