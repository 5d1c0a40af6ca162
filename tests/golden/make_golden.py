"""Generate the golden fixtures under tests/golden/.

The reference (Rust + cuda-oxide) cannot be built or imported in this
environment (no cargo/rustc, git-pinned codegen backend, no network), so its
outputs cannot be recorded directly. The fixtures therefore hold:

* ``kat.json`` — the reference's hand-written known answers:
  - DFT of [1, 2, 3, 4] = [10, -2+2i, -2, -2-2i]
    (crates/ferrum-gpu-fft/src/cpu.rs:141-170, README.md:18-21);
  - twiddle-table invariants (crates/ferrum-gpu-fft/tests/twiddles.rs).
* ``numpy_f64.npz`` — float64 numpy.fft results, rounded to complex64, on the
  exact inputs the reference's own tests use. numpy stands in for rustfft
  6.4.1 (Cargo.lock:888-890), the reference's dev-dependency oracle, whose
  source is not vendored:
  - ``x1d_*``: ``sin(i) + i*cos(i)`` lanes, the CASES matrix of
    crates/ferrum-gpu-py/python/tests/test_fft_vs_numpy.py:14-19,37-46;
  - ``rustfft_*``: ``(sin(i), cos(i))``, tests/rustfft_cross_check.rs:21-47
    at log_n in {2, 3, 6};
  - ``x2d_*``: ``sin(0.1*i) + i*cos(0.07*i)`` images,
    python/tests/test_fft_2d_vs_numpy.py:9-12 and tests/cpu_2d_vs_rustfft.rs:41-67;
  - ``xcheck_*``: ``(sin(0.013*t), cos(0.021*t))`` lanes, batch 4,
    crates/ferrum-gpu-bench/src/bin/kernel-cross-check.rs:33-40.

Run from the repository root: ``python tests/golden/make_golden.py``.
"""

from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def input_signal(n: int, batch: int) -> np.ndarray:
    """test_fft_vs_numpy.py:14-19 (float64 sin/cos rounded to complex64)."""
    i = np.arange(n, dtype=np.float64)
    lane = (np.sin(i) + 1j * np.cos(i)).astype(np.complex64)
    return np.tile(lane, batch)


def input_rustfft(n: int) -> np.ndarray:
    """rustfft_cross_check.rs:21-25: f32 sin/cos of i as f32."""
    i = np.arange(n, dtype=np.float32)
    return (np.sin(i) + 1j * np.cos(i)).astype(np.complex64)


def input_2d(n: int) -> np.ndarray:
    """test_fft_2d_vs_numpy.py:9-12."""
    base = np.arange(n * n, dtype=np.float32).reshape(n, n)
    return (np.sin(base * 0.1) + 1j * np.cos(base * 0.07)).astype(np.complex64)


def input_xcheck(n: int, batch: int) -> np.ndarray:
    """kernel-cross-check.rs:33-40: t = i mod n as f32."""
    t = (np.arange(n * batch) % n).astype(np.float32)
    return (np.sin(t * np.float32(0.013)) + 1j * np.cos(t * np.float32(0.021))).astype(np.complex64)


CASES_1D = [
    (2, 1, "forward", False),
    (3, 1, "forward", False),
    (6, 1, "forward", False),
    (8, 1, "forward", False),
    (10, 1, "forward", False),
    (12, 1, "forward", False),
    (8, 8, "forward", False),
    (8, 1, "inverse", True),
]


def ref_1d(arr: np.ndarray, n: int, direction: str, normalize: bool) -> np.ndarray:
    lanes = arr.reshape(-1, n).astype(np.complex128)
    if direction == "forward":
        out = np.fft.fft(lanes, axis=1)
    else:
        out = np.fft.ifft(lanes, axis=1)
        if not normalize:
            out = out * n
    return out.astype(np.complex64).reshape(-1)


def main() -> None:
    kat = {
        "dft4_input": [[1.0, 0.0], [2.0, 0.0], [3.0, 0.0], [4.0, 0.0]],
        "dft4_expected": [[10.0, 0.0], [-2.0, 2.0], [-2.0, 0.0], [-2.0, -2.0]],
        "dft4_tol": 1e-5,
        "twiddle_count_log_n": [2, 3, 6, 8, 10, 12],
        "twiddle_first_log_n": 3,
        "twiddle_last_log_n": 2,
        "twiddle_tol": 1e-6,
        "roundtrip_1d": [
            {"log_n": 2, "input": "i+1, 2i-1", "tol": 1e-4},
            {"log_n": 3, "input": "i, n-i", "tol": 1e-4},
            {"log_n": 8, "input": "i, n-i", "tol": 1e-3},
        ],
        "roundtrip_2d": [
            {"log_n": 2, "input": "i+1, 2i-0.5", "tol": 1e-4},
            {"log_n": 6, "input": "sin(i mod n), cos(i div n)", "tol": 1e-3},
        ],
    }
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(kat, f, indent=1)

    arrays = {}
    for log_n, batch, direction, normalize in CASES_1D:
        n = 1 << log_n
        key = f"x1d_{log_n}_{batch}_{direction}_{int(normalize)}"
        arrays[key] = ref_1d(input_signal(n, batch), n, direction, normalize)
    for log_n in (2, 3, 6):
        n = 1 << log_n
        arrays[f"rustfft_{log_n}"] = ref_1d(input_rustfft(n), n, "forward", False)
    for log_n in (3, 4, 5, 6):
        n = 1 << log_n
        arrays[f"x2d_{log_n}"] = np.fft.fft2(input_2d(n).astype(np.complex128)).astype(np.complex64)
    for log_n in (8, 10, 12):
        n = 1 << log_n
        arrays[f"xcheck_{log_n}"] = ref_1d(input_xcheck(n, 4), n, "forward", False)
    np.savez_compressed(os.path.join(HERE, "numpy_f64.npz"), **arrays)


if __name__ == "__main__":
    main()
