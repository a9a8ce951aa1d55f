"""In-tree build of the native library and the `_kvops` Python module.

    python -m kv_offload_proto_b200._build

produces
  kv_offload_proto_b200/libkvops_b200.so             (nvcc, sm_100a, the C ABI of include/kvops_b200.h)
  kv_offload_proto_b200/kvops_ext/_kvops<EXT_SUFFIX>  (g++, pybind11, links the library via $ORIGIN)

Both are plain compiler invocations (no CMake, no torch JIT cache), so the built files
sit next to the sources and travel with the tree.
"""
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libkvops_b200.so")
EXT = os.path.join(PKG, "kvops_ext", "_kvops" + sysconfig.get_config_var("EXT_SUFFIX"))
CU_SOURCES = ["capi.cu", "sieve.cu", "rows.cu", "noalloc.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def build_lib(force=False, verbose_ptxas=False):
    deps = [os.path.join(CSRC, f) for f in CU_SOURCES + ["kvops_internal.cuh", "rows_common.cuh", "sieve_big.cuh"]]
    deps.append(os.path.join(ROOT, "include", "kvops_b200.h"))
    if not force and not _newer(LIB, deps):
        return LIB
    cmd = [NVCC, "-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC", "-shared",
           "-Xlinker", "--no-undefined", "-I", os.path.join(ROOT, "include"), "-o", LIB]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, f) for f in CU_SOURCES]
    _run(cmd)
    return LIB


def build_ext(force=False):
    src = os.path.join(CSRC, "kvops_pybind.cpp")
    deps = [src, os.path.join(ROOT, "include", "kvops_b200.h"), LIB]
    if not force and not _newer(EXT, deps):
        return EXT
    import pybind11
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall",
           "-I", pybind11.get_include(), "-I", sysconfig.get_paths()["include"], "-I", os.path.join(ROOT, "include"),
           src, "-o", EXT, "-L", PKG, "-lkvops_b200", "-Wl,-rpath,$ORIGIN/.."]
    _run(cmd)
    return EXT


def build(force=False, verbose_ptxas=False):
    build_lib(force=force, verbose_ptxas=verbose_ptxas)
    build_ext(force=force)
    return LIB, EXT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="--ptxas-v" in sys.argv)
