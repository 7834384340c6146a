"""Build the native parts in-tree: libabft_b200.so (kernels, C ABI, pipeline)
and the abft_gemm driver.

    python asynchronous_abft_for_mpi-cuda_architectures_b200/build.py

Device code is compiled for sm_100a only (B200). Host code is compiled with
-ffp-contract=off and no -march flag, so that threshold arithmetic rounds like
the reference's x86-64 host code.
"""
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
LIB = os.path.join(PKG_DIR, "libabft_b200.so")
DRIVER = os.path.join(PKG_DIR, "abft_gemm")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
CUDA_LIB = os.path.join(CUDA_HOME, "lib64")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HOST_FLAGS = "-fPIC,-ffp-contract=off,-O2"

LIB_CU = ["abft_kernels.cu", "abft_capi.cu", "abft_pipeline.cu"]
LIB_CPP = ["abft_host.cpp", "abft_report.cpp"]
DRIVER_SRC = ["abft_gemm_main.cpp", "abft_comm.cpp"]


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _objects(verbose_ptxas=False):
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".h")]
    headers.append(os.path.join(INCLUDE, "abft_b200.h"))
    objs = []
    for src in LIB_CU:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD_DIR, src + ".o")
        if _stale(o, [s] + headers):
            cmd = [NVCC, "-c", "-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", HOST_FLAGS, "-I", INCLUDE,
                   "-I", CSRC, "--expt-relaxed-constexpr", "-o", o, s]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd)
        objs.append(o)
    for src in LIB_CPP:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD_DIR, src + ".o")
        if _stale(o, [s] + headers):
            _run(["g++", "-c", "-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-I", INCLUDE, "-I", CSRC,
                  "-I", os.path.join(CUDA_HOME, "include"), "-o", o, s])
        objs.append(o)
    return objs


def build_library(verbose_ptxas=False):
    objs = _objects(verbose_ptxas)
    if _stale(LIB, objs):
        _run([NVCC, "-shared", *ARCH, "-o", LIB, *objs, "-L", CUDA_LIB, "-lcublas",
              "-Xlinker", "-rpath=" + CUDA_LIB])
    return LIB


def build_driver():
    """abft_gemm: the reference-compatible command-line driver (C++17, NCCL)."""
    srcs = [os.path.join(CSRC, s) for s in DRIVER_SRC]
    if not all(os.path.exists(s) for s in srcs):
        return None
    deps = srcs + [LIB] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".h")]
    if _stale(DRIVER, deps):
        _run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I", INCLUDE, "-I", CSRC,
              "-I", os.path.join(CUDA_HOME, "include"), "-o", DRIVER, *srcs, "-L", PKG_DIR, "-labft_b200",
              "-L", CUDA_LIB, "-lcudart", "-lnccl", "-lpthread",
              "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + CUDA_LIB])
    return DRIVER


def build(verbose_ptxas=False):
    if not os.path.exists(NVCC):
        raise RuntimeError(f"nvcc not found at {NVCC}")
    build_library(verbose_ptxas)
    build_driver()


def clean():
    shutil.rmtree(BUILD_DIR, ignore_errors=True)
    for p in (LIB, DRIVER):
        if os.path.exists(p):
            os.remove(p)


if __name__ == "__main__":
    if "--clean" in sys.argv:
        clean()
    build(verbose_ptxas="--ptxas-v" in sys.argv)
