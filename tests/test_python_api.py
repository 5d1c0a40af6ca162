"""The Python boundary mirrors the reference's PyO3 module
(crates/ferrum-gpu-py/src/lib.rs:445-604): names, defaults, validation order
and ValueError messages. Runs on CPU: every check here fails before any GPU
work."""

from __future__ import annotations

import inspect

import numpy as np
import pytest

from conftest import gpu_available


@pytest.fixture(scope="module")
def fg():
    import ferrum_gpu

    return ferrum_gpu


def test_module_layout(fg):
    assert callable(fg.version)
    assert hasattr(fg.cuda, "Device")
    assert callable(fg.fft.fft_1d_c2c_pow2) and callable(fg.fft.fft_2d_c2c_pow2)
    from ferrum_gpu import _native

    assert _native.fft.fft_1d_c2c_pow2 is fg.fft.fft_1d_c2c_pow2


def test_signature_defaults(fg):
    doc = fg.fft.fft_1d_c2c_pow2.__doc__
    assert "direction: str = 'forward'" in doc and "normalize: bool = False" in doc
    assert "device: object = None" in doc


@pytest.mark.parametrize("log_n", [0, 1, 27])
def test_1d_log_n_range(fg, log_n):
    with pytest.raises(ValueError, match=rf"log_n must be in \[2, 26\], got {log_n}"):
        fg.fft.fft_1d_c2c_pow2(np.zeros(16, np.complex64), log_n)


@pytest.mark.parametrize("length", [0, 6, 17])
def test_1d_length_multiple(fg, length):
    with pytest.raises(ValueError, match=rf"arr len {length} must be a positive multiple of N = 4"):
        fg.fft.fft_1d_c2c_pow2(np.zeros(length, np.complex64), 2)


def test_1d_direction(fg):
    with pytest.raises(ValueError, match=r"direction must be 'forward' or 'inverse', got \"up\""):
        fg.fft.fft_1d_c2c_pow2(np.zeros(8, np.complex64), 2, direction="up")


def test_1d_dtype_and_rank(fg):
    with pytest.raises(TypeError):
        fg.fft.fft_1d_c2c_pow2(np.zeros(8, np.complex128), 2)
    with pytest.raises(TypeError):
        fg.fft.fft_1d_c2c_pow2(np.zeros((2, 4), np.complex64), 2)


@pytest.mark.parametrize("log_n", [1, 15])
def test_2d_log_n_range(fg, log_n):
    with pytest.raises(ValueError, match=rf"2D requires log_n in \[2, 14\]; got {log_n}"):
        fg.fft.fft_2d_c2c_pow2(np.zeros((4, 4), np.complex64), log_n)


def test_2d_shape(fg):
    with pytest.raises(ValueError, match=r"arr shape \[3, 4\] != \(16, 16\)"):
        fg.fft.fft_2d_c2c_pow2(np.zeros((3, 4), np.complex64), 4)
    with pytest.raises(ValueError, match=r"arr shape \[16\] != \(4, 4\)"):
        fg.fft.fft_2d_c2c_pow2(np.zeros(16, np.complex64), 2)


def test_2d_direction(fg):
    with pytest.raises(ValueError, match=r"direction must be 'forward' or 'inverse'"):
        fg.fft.fft_2d_c2c_pow2(np.zeros((4, 4), np.complex64), 2, direction="back")


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure mode")
def test_fails_loudly_without_gpu(fg):
    with pytest.raises(ValueError, match=r"CudaContext::new\(0\)"):
        fg.cuda.Device(0)
    with pytest.raises(ValueError):
        fg.fft.fft_1d_c2c_pow2(np.zeros(16, np.complex64), 2)
