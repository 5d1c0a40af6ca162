"""CPU oracle — test infrastructure only.

ctypes wrapper over ``liboracle_stockham.so``, the plain-C restatement of the
reference's CPU radix-2 Stockham FFT (crates/ferrum-gpu-fft/src/cpu.rs:15-124,
cpu_2d.rs:9-73, twiddles.rs:10-23). Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference legs import this module; the CUDA
product path never does.

Parity is pinned by the reference's own known-answer tests (cpu.rs:141-170,
tests/twiddles.rs, tests/cpu_roundtrip.rs, tests/cpu_2d_roundtrip.rs) and by
numpy float64 cross-checks on the reference's pytest inputs
(python/tests/test_fft_vs_numpy.py, test_fft_2d_vs_numpy.py); see
tests/test_oracle.py and tests/golden/.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_stockham.so")
_lib = None


def build() -> str:
    """Compile the oracle library with its Makefile; returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    c_float_p = ctypes.POINTER(ctypes.c_float)
    lib.oracle_twiddle_count.argtypes = [ctypes.c_uint32]
    lib.oracle_twiddle_count.restype = ctypes.c_size_t
    lib.oracle_twiddles.argtypes = [ctypes.c_uint32, c_float_p]
    lib.oracle_twiddles.restype = None
    lib.oracle_fft_1d_mt.argtypes = [c_float_p, ctypes.c_uint32, ctypes.c_size_t,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.oracle_fft_1d_mt.restype = ctypes.c_int
    lib.oracle_fft_2d.argtypes = [c_float_p, ctypes.c_uint32, ctypes.c_size_t,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.oracle_fft_2d.restype = ctypes.c_int
    _lib = lib
    return lib


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _dir(direction: str) -> int:
    if direction == "forward":
        return 1
    if direction == "inverse":
        return -1
    raise ValueError(f"direction must be 'forward' or 'inverse', got {direction!r}")


def twiddles(log_n: int) -> np.ndarray:
    """Radix-2 stage twiddle table (twiddles.rs:10-23), complex64, length N-1."""
    lib = _load()
    out = np.empty(int(lib.oracle_twiddle_count(log_n)), dtype=np.complex64)
    lib.oracle_twiddles(log_n, _fptr(out))
    return out


def fft_1d(arr: np.ndarray, log_n: int, direction: str = "forward",
           normalize: bool = False, threads: int = 1) -> np.ndarray:
    """Batched 1D C2C on a flat complex64 array of length batch * 2^log_n.

    Returns a new array; ``arr`` is not modified.
    """
    lib = _load()
    n = 1 << log_n
    buf = np.array(arr, dtype=np.complex64, copy=True).reshape(-1)
    if buf.size == 0 or buf.size % n:
        raise ValueError(f"arr len {buf.size} must be a positive multiple of N = {n}")
    rc = lib.oracle_fft_1d_mt(_fptr(buf), log_n, buf.size // n, _dir(direction),
                              int(bool(normalize)), int(threads))
    if rc != 0:
        raise ValueError("oracle_fft_1d_mt failed")
    return buf.reshape(np.shape(arr))


def fft_2d(arr: np.ndarray, log_n: int, direction: str = "forward",
           normalize: bool = False, threads: int = 1) -> np.ndarray:
    """2D C2C on (N, N) or (B, N, N) complex64 (cpu_2d.rs:9-73 per image)."""
    lib = _load()
    n = 1 << log_n
    buf = np.array(arr, dtype=np.complex64, copy=True)
    if buf.shape[-2:] != (n, n):
        raise ValueError(f"arr shape {buf.shape} != (..., {n}, {n})")
    batch = buf.size // (n * n)
    flat = buf.reshape(-1)
    rc = lib.oracle_fft_2d(_fptr(flat), log_n, batch, _dir(direction),
                           int(bool(normalize)), int(threads))
    if rc != 0:
        raise ValueError("oracle_fft_2d failed")
    return flat.reshape(buf.shape)


def library_path() -> str:
    return _LIB_PATH
