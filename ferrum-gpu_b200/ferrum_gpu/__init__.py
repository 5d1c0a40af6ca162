"""ferrum-gpu Python bindings — B200 (sm_100a) FFT path.

Mirrors the reference package (crates/ferrum-gpu-py/python/ferrum_gpu/__init__.py):
``version``, ``cuda`` (``Device``) and ``fft`` (``fft_1d_c2c_pow2``,
``fft_2d_c2c_pow2``). Added by this build: ``device`` runs the same
transforms zero-copy on torch CUDA tensors and other CUDA Array Interface /
DLPack arrays, ``capi`` binds the C ABI (include/ferrum_fft.h) for callers
that hold raw device pointers, and ``dist`` runs the distributed 2D transform
across ranks.
"""

from ferrum_gpu._native import version
from ferrum_gpu import cuda, fft

__all__ = ["version", "cuda", "fft"]
