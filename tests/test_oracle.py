"""Pins the CPU oracle before anything is compared with it.

Every check here restates a known answer or fixture from the reference's own
tests (see tests/golden/make_golden.py for the file:line of each); numpy
float64 stands in for the reference's rustfft dev-dependency.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import max_rel_err, rand_c64

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def kat():
    with open(os.path.join(GOLDEN, "kat.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def npz():
    return np.load(os.path.join(GOLDEN, "numpy_f64.npz"))


def test_dft4_known_answer(oracle_mod, kat):
    # crates/ferrum-gpu-fft/src/cpu.rs:141-170
    x = np.array([complex(*c) for c in kat["dft4_input"]], dtype=np.complex64)
    want = np.array([complex(*c) for c in kat["dft4_expected"]], dtype=np.complex64)
    got = oracle_mod.fft_1d(x, 2)
    assert np.all(np.abs(got.real - want.real) < kat["dft4_tol"])
    assert np.all(np.abs(got.imag - want.imag) < kat["dft4_tol"])


def test_twiddle_table_invariants(oracle_mod, kat):
    # crates/ferrum-gpu-fft/tests/twiddles.rs
    for log_n in kat["twiddle_count_log_n"]:
        assert len(oracle_mod.twiddles(log_n)) == (1 << log_n) - 1
    first = oracle_mod.twiddles(kat["twiddle_first_log_n"])[0]
    last = oracle_mod.twiddles(kat["twiddle_last_log_n"])[-1]
    for w in (first, last):
        assert abs(w.real - 1.0) < kat["twiddle_tol"] and abs(w.imag) < kat["twiddle_tol"]


def test_twiddle_layout_stage_descending(oracle_mod):
    # twiddles.rs:10-23: [W_8^0..3, W_4^0..1, W_2^0] for log_n = 3
    tw = oracle_mod.twiddles(3)
    want = [np.exp(-2j * np.pi * k / 8) for k in range(4)] + \
           [np.exp(-2j * np.pi * k / 4) for k in range(2)] + [1.0]
    assert np.max(np.abs(tw - np.array(want))) < 1e-6


@pytest.mark.parametrize("log_n,tol", [(2, 1e-4), (3, 1e-4), (8, 1e-3)])
def test_roundtrip_1d(oracle_mod, log_n, tol):
    # crates/ferrum-gpu-fft/tests/cpu_roundtrip.rs
    n = 1 << log_n
    i = np.arange(n, dtype=np.float32)
    if log_n == 2:
        x = (i + 1) + 1j * (2 * i - 1)
    else:
        x = i + 1j * (n - i)
    x = x.astype(np.complex64)
    y = oracle_mod.fft_1d(oracle_mod.fft_1d(x, log_n), log_n, "inverse", True)
    assert np.all(np.abs(y.real - x.real) < tol) and np.all(np.abs(y.imag - x.imag) < tol)


@pytest.mark.parametrize("log_n,tol", [(2, 1e-4), (6, 1e-3)])
def test_roundtrip_2d(oracle_mod, log_n, tol):
    # crates/ferrum-gpu-fft/tests/cpu_2d_roundtrip.rs
    n = 1 << log_n
    i = np.arange(n * n)
    if log_n == 2:
        x = (i + 1.0) + 1j * (2.0 * i - 0.5)
    else:
        x = np.sin((i % n).astype(np.float32)) + 1j * np.cos((i // n).astype(np.float32))
    x = x.astype(np.complex64).reshape(n, n)
    y = oracle_mod.fft_2d(oracle_mod.fft_2d(x, log_n), log_n, "inverse", True)
    assert np.all(np.abs(y - x) < tol * 1.5)


@pytest.mark.parametrize("log_n", [2, 3, 6])
def test_cross_check_rustfft_inputs(oracle_mod, npz, log_n):
    # tests/rustfft_cross_check.rs:21-47, metric (|dre|+|dim|)/(|re|+|im|+1) < 1e-4
    n = 1 << log_n
    i = np.arange(n, dtype=np.float32)
    x = (np.sin(i) + 1j * np.cos(i)).astype(np.complex64)
    got = oracle_mod.fft_1d(x, log_n)
    ref = npz[f"rustfft_{log_n}"]
    rel = (np.abs(got.real - ref.real) + np.abs(got.imag - ref.imag)) / \
          (np.abs(ref.real) + np.abs(ref.imag) + 1.0)
    assert float(np.max(rel)) < 1e-4


@pytest.mark.parametrize("log_n", [3, 4, 5, 6])
def test_cross_check_2d_inputs(oracle_mod, npz, log_n):
    # tests/cpu_2d_vs_rustfft.rs:41-67 and python/tests/test_fft_2d_vs_numpy.py
    n = 1 << log_n
    base = np.arange(n * n, dtype=np.float32).reshape(n, n)
    x = (np.sin(base * 0.1) + 1j * np.cos(base * 0.07)).astype(np.complex64)
    got = oracle_mod.fft_2d(x, log_n)
    ref = npz[f"x2d_{log_n}"]
    rel = (np.abs(got.real - ref.real) + np.abs(got.imag - ref.imag)) / \
          (np.abs(ref.real) + np.abs(ref.imag) + 1.0)
    assert float(np.max(rel)) < 1e-4


CASES_1D = [(2, 1, "forward", False), (3, 1, "forward", False), (6, 1, "forward", False),
            (8, 1, "forward", False), (10, 1, "forward", False), (12, 1, "forward", False),
            (8, 8, "forward", False), (8, 1, "inverse", True)]


@pytest.mark.parametrize("log_n,batch,direction,normalize", CASES_1D)
def test_python_cases_vs_numpy(oracle_mod, npz, log_n, batch, direction, normalize):
    # python/tests/test_fft_vs_numpy.py:37-63: max rel err < 1e-4
    n = 1 << log_n
    i = np.arange(n, dtype=np.float64)
    x = np.tile((np.sin(i) + 1j * np.cos(i)).astype(np.complex64), batch)
    got = oracle_mod.fft_1d(x, log_n, direction, normalize)
    ref = npz[f"x1d_{log_n}_{batch}_{direction}_{int(normalize)}"]
    assert max_rel_err(got, ref) < 1e-4


@pytest.mark.parametrize("log_n", [8, 10, 12])
def test_kernel_cross_check_inputs(oracle_mod, npz, log_n):
    # crates/ferrum-gpu-bench/src/bin/kernel-cross-check.rs:20,33-58: per-bin
    # err / max(|ref|, 1) <= REL_TOL = 1e-3
    n = 1 << log_n
    t = (np.arange(n * 4) % n).astype(np.float32)
    x = (np.sin(t * np.float32(0.013)) + 1j * np.cos(t * np.float32(0.021))).astype(np.complex64)
    got = oracle_mod.fft_1d(x, log_n)
    ref = npz[f"xcheck_{log_n}"]
    per_bin = np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)
    assert float(np.max(per_bin)) <= 1e-3


@pytest.mark.parametrize("log_n", [4, 9, 13, 16])
def test_matches_numpy_f64_seeded(oracle_mod, log_n):
    rng = np.random.default_rng(log_n)
    n = 1 << log_n
    x = rand_c64(rng, 3 * n)
    ref = np.fft.fft(x.reshape(3, n).astype(np.complex128), axis=1)
    assert max_rel_err(oracle_mod.fft_1d(x, log_n), ref) < 1e-5


def test_threaded_is_bitwise_single_threaded(oracle_mod):
    rng = np.random.default_rng(7)
    x = rand_c64(rng, 64 * 1024)
    a = oracle_mod.fft_1d(x, 10, threads=1)
    b = oracle_mod.fft_1d(x, 10, threads=4)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_rejects_bad_lengths(oracle_mod):
    with pytest.raises(ValueError):
        oracle_mod.fft_1d(np.zeros(6, np.complex64), 2)
    with pytest.raises(ValueError):
        oracle_mod.fft_1d(np.zeros(0, np.complex64), 2)
