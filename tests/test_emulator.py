"""CPU emulation of the sm_100a kernels' own index arithmetic and butterflies
(tests/emulator/emulate.cu) against the CPU oracle.

The emulator runs the kernel helpers from ferrum-gpu_b200/csrc (radix plans,
twiddle tables, stage_compute / stage_out_pos / smem_pad, the four-step
twiddle lookup and the distributed blocked layout) thread by thread and
returns a negative code when a shared-memory exchange is not a permutation.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import max_rel_err, rand_c64

TOL = 1e-4  # north_star: max relative error vs the CPU reference


def _dir(d):
    return 1 if d == "forward" else -1


@pytest.mark.parametrize("log_n", list(range(2, 15)))
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True),
                                                  ("inverse", False)])
def test_single_pass_matches_oracle(emulator, oracle_mod, log_n, direction, normalize):
    rng = np.random.default_rng(100 + log_n)
    batch = 3
    x = rand_c64(rng, batch << log_n)
    y = x.copy()
    assert emulator.emu_fft_1d(y.ctypes.data, log_n, batch, _dir(direction), int(normalize)) == 0
    ref = oracle_mod.fft_1d(x, log_n, direction, normalize)
    assert max_rel_err(y, ref) < TOL


@pytest.mark.parametrize("log_n,log_p", [(9, 5), (10, 5), (11, 5), (12, 5)])
def test_tile_value_splits_match_oracle(emulator, oracle_mod, log_n, log_p):
    # the tile kernels run these lengths with 32 values per thread
    rng = np.random.default_rng(700 + 8 * log_n + log_p)
    x = rand_c64(rng, 1 << log_n)
    y = x.copy()
    assert emulator.emu_group_lp(y.ctypes.data, log_n, log_p) == 0
    ref = oracle_mod.fft_1d(x, log_n, "forward", False)
    assert max_rel_err(y, ref) < TOL


@pytest.mark.parametrize("log_n", [15, 16, 17, 18, 20, 21, 22, 23, 24])
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_multi_pass_matches_oracle(emulator, oracle_mod, log_n, direction, normalize):
    # two passes up to 2^23, three passes from 2^24
    rng = np.random.default_rng(200 + log_n)
    batch = 2 if log_n <= 18 else 1
    x = rand_c64(rng, batch << log_n, "normal")
    y = x.copy()
    assert emulator.emu_fft_1d(y.ctypes.data, log_n, batch, _dir(direction), int(normalize)) == 0
    ref = oracle_mod.fft_1d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(y, ref) < TOL


def test_pass_counts(emulator):
    assert [emulator.emu_plan_1d_passes(l) for l in (2, 14, 15, 21, 22, 23, 24, 26)] == \
        [1, 1, 2, 2, 2, 2, 3, 3]


@pytest.mark.parametrize("log_n", [2, 3, 4, 5, 6, 8, 10, 11, 12])
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_2d_matches_oracle(emulator, oracle_mod, log_n, direction, normalize):
    # N = 2048 runs one 4-column strided pass; N >= 4096 runs the columns as two
    # sub-passes before the row pass
    rng = np.random.default_rng(300 + log_n)
    n = 1 << log_n
    x = rand_c64(rng, (2 if log_n <= 10 else 1, n, n))
    y = x.copy()
    assert emulator.emu_fft_2d(y.ctypes.data, log_n, x.shape[0], _dir(direction),
                               int(normalize)) == 0
    ref = oracle_mod.fft_2d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(y, ref) < TOL


@pytest.mark.parametrize("log_n,ranks", [(4, 2), (5, 8), (6, 4), (8, 8), (10, 2), (10, 8),
                                          (11, 2), (12, 4)])
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_distributed_2d_decomposition(emulator, oracle_mod, log_n, ranks, direction, normalize):
    rng = np.random.default_rng(400 + log_n + ranks)
    n = 1 << log_n
    x = rand_c64(rng, (n, n), "normal")
    y = x.copy()
    assert emulator.emu_fft_2d_dist(y.ctypes.data, log_n, ranks, _dir(direction),
                                    int(normalize)) == 0
    ref = oracle_mod.fft_2d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(y, ref) < TOL


@pytest.mark.parametrize("log_n,ranks", [(4, 2), (6, 8), (10, 4), (11, 2), (12, 8)])
@pytest.mark.parametrize("layouts", [(0, 1), (1, 0)])
def test_distributed_2d_transposed_layouts(emulator, oracle_mod, log_n, ranks, layouts):
    """Row slabs in -> column slabs out (one exchange) for the forward, and
    column slabs in -> row slabs out for the inverse; the emulator splits and
    reassembles the whole image, so the result compares with the 2D oracle."""
    rng = np.random.default_rng(500 + log_n + ranks)
    n = 1 << log_n
    x = rand_c64(rng, (n, n), "normal")
    fwd = x.copy()
    assert emulator.emu_fft_2d_dist_layout(fwd.ctypes.data, log_n, ranks, 1, 0, *layouts) == 0
    assert max_rel_err(fwd, oracle_mod.fft_2d(x, log_n, threads=8)) < TOL
    inv = fwd.copy()
    back = layouts[::-1]
    assert emulator.emu_fft_2d_dist_layout(inv.ctypes.data, log_n, ranks, -1, 1, *back) == 0
    assert max_rel_err(inv, x) < TOL


@pytest.mark.parametrize("log_n,ranks", [(4, 2), (6, 8), (10, 4), (11, 2), (12, 8), (12, 2)])
@pytest.mark.parametrize("layouts", [(0, 0), (0, 1), (1, 0)])
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_distributed_2d_peer_path(emulator, oracle_mod, log_n, ranks, layouts, direction,
                                  normalize):
    """The peer-memory path of the distributed transform (row-FFT scatter into
    the ranks' receive slabs, column passes, row-FFT gather / block gather),
    with the kernels' index arithmetic, against the 2D oracle."""
    rng = np.random.default_rng(600 + log_n + ranks)
    n = 1 << log_n
    x = rand_c64(rng, (n, n), "normal")
    y = x.copy()
    assert emulator.emu_fft_2d_dist_p2p(y.ctypes.data, log_n, ranks, _dir(direction),
                                        int(normalize), *layouts) == 0
    ref = oracle_mod.fft_2d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(y, ref) < TOL
