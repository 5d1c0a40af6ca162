"""Build the ferrum-gpu B200 libraries in-tree.

Outputs (next to the Python package so they travel with the source tree):
  ferrum_gpu/libferrum_fft.so                    C ABI (include/ferrum_fft.h) + sm_100a kernels
  ferrum_gpu/_native.<python-ext-suffix>         pybind11 module over the C ABI

Every .cu is compiled with
  nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3
and the CUDA runtime is linked statically. Objects go to _build/. A target
is rebuilt only when a source or header is newer than it.

Usage: python ferrum-gpu_b200/build.py [-j JOBS] [--force]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "ferrum_gpu")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(REPO, "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = shutil.which("nvcc") or os.path.join(CUDA_HOME, "bin", "nvcc")
# The system g++ builds the pybind11 module: it must match the libstdc++ the
# interpreter loads at run time.
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else (shutil.which("g++") or "g++")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", f"-I{INCLUDE}"] + ARCH

CU_SOURCES = ["launch_rows.cu", "launch_pass.cu", "launch_misc.cu", "launch_tile.cu", "capi.cu", "host_path.cu", "dist.cu",
              "no_alloc.cu", "substrate.cu"]
LIB = os.path.join(PKG, "libferrum_fft.so")
EXT = os.path.join(PKG, "_native" + sysconfig.get_config_var("EXT_SUFFIX"))


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"command failed ({r.returncode}): {cmd[0]} ... {cmd[-1]}")


def _compile_cu(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    if force or _stale(obj, [src] + _headers()):
        _run([NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj])
    return obj


def build(jobs: int = 4, force: bool = False) -> None:
    os.makedirs(BUILD, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile_cu(s, force), srcs))
    if force or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs
             + ["-ldl", "-lpthread", "-lrt"])
    native_src = os.path.join(CSRC, "native_py.cpp")
    if force or _stale(EXT, [native_src, LIB] + _headers()):
        import pybind11

        py_inc = sysconfig.get_paths()["include"]
        _run([CXX, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
              f"-I{pybind11.get_include()}", f"-I{py_inc}", f"-I{INCLUDE}", native_src,
              "-o", EXT, f"-L{PKG}", "-lferrum_fft", "-Wl,-rpath,$ORIGIN"])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", "--jobs", type=int, default=4)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build(a.jobs, a.force)
    print(LIB)
    print(EXT)


if __name__ == "__main__":
    main()
