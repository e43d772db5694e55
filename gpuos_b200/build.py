"""Build the B200 runtime in-tree.

Outputs (git-ignored, shipped with the source tree):
  gpuos_b200/lib/libgpuos_b200.so   C ABI: device worker (sm_100a) + host runtime
  gpuos_b200/lib/gpuos_worker_rdc.cubin  the worker as relocatable sm_100a code, linked at run
                                    time with operators compiled by NVRTC
  gpuos_b200/_gpuos_ext<EXT_SUFFIX> CPython binding (the gpuos_ext drop-in)

Usage: python -m gpuos_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIBDIR = os.path.join(PKG, "lib")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = os.path.join(LIBDIR, "libgpuos_b200.so")
WORKER_RDC = os.path.join(LIBDIR, "gpuos_worker_rdc.cubin")
EXT = os.path.join(PKG, "_gpuos_ext" + sysconfig.get_config_var("EXT_SUFFIX"))

DEVICE_HEADERS = [
    os.path.join(CSRC, "internal.h"),
    os.path.join(INCLUDE, "gpuos_b200.h"),
] + [os.path.join(CSRC, "device", f) for f in sorted(os.listdir(os.path.join(CSRC, "device")))]


def _newer(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {r.returncode})")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)


def _worker_obj(force: bool, verbose: bool) -> list[str]:
    """The library's worker: relocatable device code plus its device link.  Every function is
    held to the worker's register budget (512 threads per CTA: 128 registers), so the device
    link accounts for every callee reached through the function tables, exactly as the run-time
    link does for modules with compiled operators (whole-program compilation of this file takes
    ptxas 10-20 minutes for the same code)."""
    src = os.path.join(CSRC, "worker.cu")
    out = os.path.join(BUILD, "worker.o")
    dlink = os.path.join(BUILD, "worker_dlink.o")
    if force or _newer(out, [src] + DEVICE_HEADERS):
        _run([NVCC, *ARCH, "-O3", "-std=c++17", "-fmad=false", "-rdc=true", "-maxrregcount=128", "-lineinfo",
              "-Xcompiler", "-fPIC", "-I" + INCLUDE, "-I" + CSRC, "-c", src, "-o", out], verbose)
    if force or _newer(dlink, [out]):
        _run([NVCC, *ARCH, "-dlink", "-Xcompiler", "-fPIC", out, "-o", dlink], verbose)
    return [out, dlink]


def _worker_rdc(force: bool, verbose: bool) -> str:
    """The worker as relocatable device code.  Every function is held to the worker's register
    budget (512 threads per CTA: 128 registers), so that the device link with run-time
    compiled operators accounts for every callee."""
    src = os.path.join(CSRC, "worker.cu")
    if force or _newer(WORKER_RDC, [src] + DEVICE_HEADERS):
        _run([NVCC, *ARCH, "-O3", "-std=c++17", "-fmad=false", "-rdc=true", "-maxrregcount=128", "-cubin",
              "-DGPUOS_JIT_WORKER", "-I" + INCLUDE, "-I" + CSRC, src, "-o", WORKER_RDC], verbose)
    return WORKER_RDC


def _jit_obj(force: bool, verbose: bool) -> str:
    src = os.path.join(CSRC, "jit.cpp")
    out = os.path.join(BUILD, "jit.o")
    if force or _newer(out, [src, os.path.join(CSRC, "jit.h"), os.path.join(INCLUDE, "gpuos_b200.h"),
                             os.path.join(CSRC, "device", "ew_math.inc")]):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-deprecated-declarations", "-I" + INCLUDE,
              "-I" + CSRC, "-I" + os.path.join(CUDA_HOME, "include"), "-c", src, "-o", out], verbose)
    return out


def _expr_obj(force: bool, verbose: bool) -> str:
    src = os.path.join(CSRC, "expr.cpp")
    out = os.path.join(BUILD, "expr.o")
    if force or _newer(out, [src, os.path.join(CSRC, "internal.h"), os.path.join(INCLUDE, "gpuos_b200.h")]):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-Wall", "-I" + INCLUDE, "-I" + CSRC,
              "-I" + os.path.join(CUDA_HOME, "include"), "-c", src, "-o", out], verbose)
    return out


def _runtime_obj(force: bool, verbose: bool) -> str:
    src = os.path.join(CSRC, "runtime.cpp")
    out = os.path.join(BUILD, "runtime.o")
    if force or _newer(out, [src, os.path.join(CSRC, "internal.h"), os.path.join(CSRC, "jit.h"),
                             os.path.join(INCLUDE, "gpuos_b200.h")]):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function",
              "-I" + INCLUDE, "-I" + CSRC, "-I" + os.path.join(CUDA_HOME, "include"),
              "-c", src, "-o", out], verbose)
    return out


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension as ce
    inc = [f"-I{p}" for p in ce.include_paths()]
    libdir = ce.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = inc + [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    lflags = [f"-L{libdir}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
              f"-Wl,-rpath,{libdir}"]
    return cflags, lflags


def _ext(force: bool, verbose: bool) -> str:
    src = os.path.join(CSRC, "pyext.cpp")
    icp = os.path.join(CSRC, "intercept.cpp")
    if force or _newer(EXT, [src, icp, os.path.join(CSRC, "intercept.h"), os.path.join(INCLUDE, "gpuos_b200.h"), LIB]):
        cflags, lflags = _torch_flags()
        py_inc = sysconfig.get_paths()["include"]
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w",
              "-I" + py_inc, "-I" + INCLUDE, "-I" + CSRC, "-I" + os.path.join(CUDA_HOME, "include"), *cflags,
              src, icp, "-o", EXT, "-L" + LIBDIR, "-lgpuos_b200", "-Wl,-rpath,$ORIGIN/lib", *lflags], verbose)
    return EXT


def build(force: bool = False, verbose: bool = False) -> None:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=5) as ex:
        fw = ex.submit(_worker_obj, force, verbose)
        fd = ex.submit(_worker_rdc, force, verbose)
        fr = ex.submit(_runtime_obj, force, verbose)
        fx = ex.submit(_expr_obj, force, verbose)
        fj = ex.submit(_jit_obj, force, verbose)
        objs = [*fw.result(), fr.result(), fx.result(), fj.result()]
        fd.result()
    if force or _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", *objs, "-o", LIB,
              "-lpthread", "-ldl", "-lrt"], verbose)
    _ext(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print("built", LIB, EXT)
