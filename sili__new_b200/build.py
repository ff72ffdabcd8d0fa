"""Build recipe for the sili__new_b200 native extension (in-tree).

Produces, next to this file:
  libsili_b200.so   CUDA kernels + C ABI (include/sili_b200.h), sm_100a only
  _cuda<ext>        pybind11 module mirroring sili._cpu's SparseLinearLayer,
                    linked against libsili_b200.so (rpath $ORIGIN)

nvcc cross-compiles for sm_100a without a GPU, so this runs anywhere the
CUDA toolkit is installed.  Objects go to sili__new_b200/_build/.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
NVCC = os.environ.get("NVCC", "nvcc")

CU_SOURCES = ["kernels_compute.cu", "kernels_update.cu", "kernels_forward.cu", "kernels_struct.cu", "block4.cu", "block4_tc.cu", "synap.cu", "topk.cu", "peak.cu", "csr_ops.cu", "attention.cu", "layer.cu"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "--fmad=false",
              "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INCLUDE]
LIB = os.path.join(HERE, "libsili_b200.so")
EXT = os.path.join(HERE, "_cuda" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, "sili_b200.h")]


def build(verbose: bool = False, force: bool = False) -> None:
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    hdrs = _headers()
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [NVCC] + NVCC_FLAGS + ["-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a"] + objs + ["-o", LIB]
        subprocess.run(cmd, check=True)
    pym = os.path.join(CSRC, "pymod.cpp")
    if force or _stale(EXT, [pym, LIB] + hdrs):
        import pybind11
        cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I" + pybind11.get_include(),
               "-I" + sysconfig.get_paths()["include"], "-I" + INCLUDE, pym, "-o", EXT,
               "-L" + HERE, "-lsili_b200", "-Wl,-rpath,$ORIGIN"]
        subprocess.run(cmd, check=True)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print("built", LIB, EXT)
