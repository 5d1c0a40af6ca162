"""ferrum_gpu.fft submodule.

``fft_1d_c2c_pow2`` and ``fft_2d_c2c_pow2`` take and return numpy complex64
arrays, exactly like the reference
(crates/ferrum-gpu-py/python/ferrum_gpu/fft.py, src/lib.rs:445-588). They are
the compiled functions of ``_native.fft``, re-exported by attribute.
"""

from ferrum_gpu._native import fft as _fft_native

fft_1d_c2c_pow2 = _fft_native.fft_1d_c2c_pow2
fft_2d_c2c_pow2 = _fft_native.fft_2d_c2c_pow2

__all__ = ["fft_1d_c2c_pow2", "fft_2d_c2c_pow2"]
