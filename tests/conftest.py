"""Shared fixtures.

Markers: ``gpu`` tests need a B200 and call the CUDA path through the C ABI
(or the Python API over it); everything else runs on CPU. The CPU oracle
(``oracle/``) and the kernel emulator (``tests/emulator/``) are test
infrastructure and are built here on first use.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "ferrum-gpu_b200")
for p in (REPO, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

EMU_DIR = os.path.join(REPO, "tests", "emulator")
EMU_SRC = os.path.join(EMU_DIR, "emulate.cu")
EMU_LIB = os.path.join(EMU_DIR, "libemulate.so")
CSRC = os.path.join(PKG_DIR, "csrc")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and runs the CUDA path")


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def build_emulator() -> str:
    deps = [EMU_SRC] + [os.path.join(CSRC, f) for f in os.listdir(CSRC)
                        if f.endswith((".h", ".cuh"))]
    if not os.path.exists(EMU_LIB) or os.path.getmtime(EMU_LIB) < _newest(deps):
        subprocess.run(["nvcc", "-std=c++17", "-O2", "--expt-relaxed-constexpr",
                        "-Wno-deprecated-gpu-targets", "-Xcompiler", "-fPIC", "-shared",
                        EMU_SRC, "-o", EMU_LIB], check=True)
    return EMU_LIB


@pytest.fixture(scope="session")
def emulator():
    lib = ctypes.CDLL(build_emulator())
    for fn in ("emu_fft_1d", "emu_fft_2d"):
        getattr(lib, fn).argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                     ctypes.c_int, ctypes.c_int]
        getattr(lib, fn).restype = ctypes.c_int
    lib.emu_fft_2d_dist.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int]
    lib.emu_fft_2d_dist.restype = ctypes.c_int
    lib.emu_fft_2d_dist_layout.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.emu_fft_2d_dist_layout.restype = ctypes.c_int
    lib.emu_fft_2d_dist_p2p.argtypes = lib.emu_fft_2d_dist_layout.argtypes
    lib.emu_fft_2d_dist_p2p.restype = ctypes.c_int
    lib.emu_group_lp.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    lib.emu_group_lp.restype = ctypes.c_int
    lib.emu_plan_1d_passes.argtypes = [ctypes.c_int]
    lib.emu_plan_1d_passes.restype = ctypes.c_int
    return lib


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    oracle.build()
    return oracle


def rand_c64(rng: np.random.Generator, shape, dist: str = "uniform") -> np.ndarray:
    """re/im i.i.d. uniform[-1, 1) or standard normal, as complex64."""
    if dist == "uniform":
        re, im = rng.uniform(-1.0, 1.0, shape), rng.uniform(-1.0, 1.0, shape)
    else:
        re, im = rng.standard_normal(shape), rng.standard_normal(shape)
    return (re + 1j * im).astype(np.complex64)


def max_rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max|out - ref| / max|ref| (crates/ferrum-gpu-py/python/tests/test_fft_vs_numpy.py:61-63)."""
    out = np.asarray(out).reshape(-1)
    ref = np.asarray(ref).reshape(-1)
    return float(np.max(np.abs(out.astype(np.complex128) - ref.astype(np.complex128)))
                 / max(1e-30, float(np.max(np.abs(ref)))))


def gpu_available() -> bool:
    try:
        import torch

        if not torch.cuda.is_available():
            return False
        return torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False
