"""The reference's own Python tests, run against this build's public API.

Restates crates/ferrum-gpu-py/python/tests/test_fft_vs_numpy.py and
test_fft_2d_vs_numpy.py: the same inputs, cases, tolerances and the
``use_device`` matrix (device=None vs a persistent ``Device``), plus the same
cases against the CPU oracle and the golden fixtures. The reference's 2D API
stops at N=1024 in its tests and crashes at N=4096 on its GPU path; the
matrix here adds N=4096, batched (B, N, N) images and 1D lengths beyond 4096.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import max_rel_err

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

import ferrum_gpu as fgpu  # noqa: E402

GOLDEN = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                              "numpy_f64.npz"))


@pytest.fixture(scope="module")
def device():
    return fgpu.cuda.Device(0)


def _input_signal(n: int, batch: int) -> np.ndarray:
    # test_fft_vs_numpy.py:14-19
    i = np.arange(n, dtype=np.float64)
    return np.tile((np.sin(i) + 1j * np.cos(i)).astype(np.complex64), batch)


def _reference(arr, n, batch, direction, normalize):
    lanes = arr.reshape(batch, n)
    if direction == "forward":
        out = np.fft.fft(lanes, axis=1)
    else:
        out = np.fft.ifft(lanes, axis=1)
        if not normalize:
            out = out * n
    return out.astype(np.complex64).reshape(-1)


CASES = [
    (2, 1, "forward", False, "N=4 fwd"),
    (3, 1, "forward", False, "N=8 fwd"),
    (6, 1, "forward", False, "N=64 fwd"),
    (8, 1, "forward", False, "N=256 fwd"),
    (10, 1, "forward", False, "N=1024 fwd"),
    (12, 1, "forward", False, "N=4096 fwd"),
    (8, 8, "forward", False, "N=256 fwd batch=8"),
    (8, 1, "inverse", True, "N=256 inv normalize"),
]


@pytest.mark.parametrize("log_n,batch,direction,normalize,label", CASES)
@pytest.mark.parametrize("use_device", [False, True])
def test_gpu_fft_matches_numpy(device, oracle_mod, log_n, batch, direction, normalize, label,
                               use_device):
    n = 1 << log_n
    inp = _input_signal(n, batch)
    expected = _reference(inp, n, batch, direction, normalize)
    kwargs = {"log_n": log_n, "direction": direction, "normalize": normalize}
    if use_device:
        kwargs["device"] = device
    out = fgpu.fft.fft_1d_c2c_pow2(inp, **kwargs)
    assert out.shape == inp.shape and out.dtype == np.complex64
    assert max_rel_err(out, expected) < 1e-4, label
    golden = GOLDEN[f"x1d_{log_n}_{batch}_{direction}_{int(normalize)}"]
    assert max_rel_err(out, golden) < 1e-4, label
    assert max_rel_err(out, oracle_mod.fft_1d(inp, log_n, direction, normalize)) < 1e-4, label


# test_fft_vs_numpy.py:71-75 (the reference's large-batch radix-16 path, 1e-3
# there); this build holds them to 1e-4 like every other case.
R16S_CASES = [
    (8, 4096, "forward", False),
    (8, 4096, "inverse", True),
    (12, 4096, "forward", False),
]


@pytest.mark.parametrize("log_n,batch,direction,normalize", R16S_CASES)
@pytest.mark.parametrize("use_device", [False, True])
def test_large_batch_matches_numpy(device, log_n, batch, direction, normalize, use_device):
    n = 1 << log_n
    inp = _input_signal(n, batch)
    expected = _reference(inp, n, batch, direction, normalize)
    kwargs = {"log_n": log_n, "direction": direction, "normalize": normalize}
    if use_device:
        kwargs["device"] = device
    out = fgpu.fft.fft_1d_c2c_pow2(inp, **kwargs)
    assert max_rel_err(out, expected) < 1e-4


@pytest.mark.parametrize("log_n", [13, 14, 16, 20])
def test_beyond_reference_lengths(device, oracle_mod, log_n):
    rng = np.random.default_rng(log_n)
    n = 1 << log_n
    inp = (rng.uniform(-1, 1, 2 * n) + 1j * rng.uniform(-1, 1, 2 * n)).astype(np.complex64)
    out = fgpu.fft.fft_1d_c2c_pow2(inp, log_n, device=device)
    assert max_rel_err(out, oracle_mod.fft_1d(inp, log_n, threads=8)) < 1e-4
    back = fgpu.fft.fft_1d_c2c_pow2(out, log_n, "inverse", True, device)
    assert max_rel_err(back, inp) < 1e-4


def _input_2d(n: int) -> np.ndarray:
    # test_fft_2d_vs_numpy.py:9-12
    base = np.arange(n * n, dtype=np.float32).reshape(n, n)
    return (np.sin(base * 0.1) + 1j * np.cos(base * 0.07)).astype(np.complex64)


@pytest.mark.parametrize("log_n,label", [(4, "N=16"), (5, "N=32"), (6, "N=64"), (8, "N=256"),
                                         (10, "N=1024"), (12, "N=4096")])
@pytest.mark.parametrize("use_device", [False, True])
def test_gpu_fft2d_matches_numpy(device, log_n, label, use_device):
    n = 1 << log_n
    arr = _input_2d(n)
    expected = np.fft.fft2(arr).astype(np.complex64)
    kwargs = {"log_n": log_n, "direction": "forward", "normalize": False}
    if use_device:
        kwargs["device"] = device
    out = fgpu.fft.fft_2d_c2c_pow2(arr, **kwargs)
    assert out.shape == arr.shape
    # The reference gates this at 1e-3 (test_fft_2d_vs_numpy.py:41); the
    # north_star bar for this build is 1e-4.
    assert max_rel_err(out, expected) < 1e-4, label


@pytest.mark.parametrize("log_n,label", [(4, "N=16"), (6, "N=64"), (8, "N=256")])
def test_gpu_fft2d_inverse_roundtrip(device, log_n, label):
    n = 1 << log_n
    arr = _input_2d(n)
    fwd = fgpu.fft.fft_2d_c2c_pow2(arr, log_n=log_n, direction="forward", device=device)
    inv = fgpu.fft.fft_2d_c2c_pow2(fwd, log_n=log_n, direction="inverse", normalize=True,
                                   device=device)
    assert max_rel_err(inv, arr) < 1e-4, label


def test_2d_batched_images_and_golden(device, oracle_mod):
    for log_n in (3, 4, 5, 6):
        n = 1 << log_n
        arr = np.stack([_input_2d(n)] * 3)
        out = fgpu.fft.fft_2d_c2c_pow2(arr, log_n, device=device)
        assert out.shape == (3, n, n)
        for b in range(3):
            assert max_rel_err(out[b], GOLDEN[f"x2d_{log_n}"]) < 1e-4
        assert max_rel_err(out, oracle_mod.fft_2d(arr, log_n)) < 1e-4


def test_kernel_cross_check_inputs(device, oracle_mod):
    # crates/ferrum-gpu-bench/src/bin/kernel-cross-check.rs:20,33-58 at batch 4:
    # per-bin err / max(|ref|, 1) <= REL_TOL = 1e-3 (the reference's gate; the
    # CPU oracle itself reaches 1.7e-4 on this metric), plus the suite-wide
    # max|err| / max|ref| < 1e-4 against both float64 numpy and the oracle.
    for log_n in (8, 10, 12):
        n = 1 << log_n
        t = (np.arange(n * 4) % n).astype(np.float32)
        x = (np.sin(t * np.float32(0.013)) + 1j * np.cos(t * np.float32(0.021))).astype(np.complex64)
        out = fgpu.fft.fft_1d_c2c_pow2(x, log_n, device=device)
        ref = GOLDEN[f"xcheck_{log_n}"]
        assert float(np.max(np.abs(out - ref) / np.maximum(np.abs(ref), 1.0))) <= 1e-3
        assert max_rel_err(out, ref) < 1e-4
        assert max_rel_err(out, oracle_mod.fft_1d(x, log_n)) < 1e-4


def test_input_not_modified_and_noncontiguous(device):
    x = _input_signal(1024, 4)
    keep = x.copy()
    out = fgpu.fft.fft_1d_c2c_pow2(x, 10, device=device)
    assert np.array_equal(x, keep)
    strided = np.repeat(x, 2)[::2]
    assert not strided.flags["C_CONTIGUOUS"]
    out2 = fgpu.fft.fft_1d_c2c_pow2(strided, 10, device=device)
    assert np.array_equal(out, out2)


def test_device_sync(device):
    device.sync()
    assert device.ordinal == 0
