"""ferrum_gpu.cuda submodule.

The native ``Device`` class lives in the ``cuda`` submodule of the compiled
``_native`` module, which is not importable as a package path, so it is
re-exported by attribute (as in crates/ferrum-gpu-py/python/ferrum_gpu/cuda.py).
"""

from ferrum_gpu._native import cuda as _cuda_native

Device = _cuda_native.Device

__all__ = ["Device"]
