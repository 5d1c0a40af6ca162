"""GPU parity: the sm_100a kernels, called through the C ABI, against the CPU
oracle on the same seeded inputs.

Tolerance (north_star): max|gpu - ref| / max|ref| <= 1e-4 for forward and
inverse. Batches include ragged counts (not a multiple of the transforms per
CTA) and >= 512 CTAs, the reference's race-exposing size
(crates/ferrum-gpu-bench/src/bin/batch-sweep-4096.rs:39-41,80). At the full
config sizes, where the oracle would take minutes, size-independent
properties are checked instead: forward/inverse round trip, linearity,
Parseval, plus oracle parity on a sample of rows.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import gpu_available, max_rel_err, rand_c64

pytestmark = pytest.mark.gpu
TOL = 1e-4
THREADS = max(1, min(32, os.cpu_count() or 1))  # oracle lanes in parallel

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)


@pytest.fixture(scope="module")
def capi():
    from ferrum_gpu import capi as c

    return c


@pytest.fixture(scope="module")
def dev(capi):
    assert gpu_available(), "GPU tests need a B200 (sm_100)"
    d = capi.DeviceHandle(0)
    yield d
    d.close()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def run_1d(capi, dev, x: np.ndarray, log_n: int, direction: str, normalize: bool,
           inplace: bool = False) -> np.ndarray:
    batch = x.size >> log_n
    t_in = torch.from_numpy(np.ascontiguousarray(x)).to("cuda")
    t_out = t_in if inplace else torch.empty_like(t_in)
    capi.fft_1d(dev, t_in.data_ptr(), t_out.data_ptr(), log_n, batch, direction, normalize,
                _stream())
    torch.cuda.synchronize()
    return t_out.cpu().numpy()


def run_2d(capi, dev, x: np.ndarray, log_n: int, direction: str, normalize: bool,
           inplace: bool = False) -> np.ndarray:
    n = 1 << log_n
    batch = x.size // (n * n)
    t_in = torch.from_numpy(np.ascontiguousarray(x)).to("cuda")
    t_out = t_in if inplace else torch.empty_like(t_in)
    capi.fft_2d(dev, t_in.data_ptr(), t_out.data_ptr(), log_n, batch, direction, normalize,
                _stream())
    torch.cuda.synchronize()
    return t_out.cpu().numpy()


def rows_per_cta(log_n: int) -> int:
    t = 1 << (log_n - min(log_n, 4))
    return 256 // t if t <= 256 else 1


DIRS = [("forward", False), ("inverse", True), ("inverse", False)]


@pytest.mark.parametrize("log_n", list(range(2, 15)))
@pytest.mark.parametrize("direction,normalize", DIRS)
def test_single_pass_small_batches(capi, dev, oracle_mod, log_n, direction, normalize):
    rng = np.random.default_rng(1000 + log_n)
    for batch in (1, 3):
        x = rand_c64(rng, batch << log_n)
        got = run_1d(capi, dev, x, log_n, direction, normalize)
        ref = oracle_mod.fft_1d(x, log_n, direction, normalize)
        assert max_rel_err(got, ref) < TOL, (log_n, batch)


@pytest.mark.parametrize("log_n", list(range(2, 15)))
def test_single_pass_many_ctas_ragged(capi, dev, oracle_mod, log_n):
    # >= 512 CTAs and a partial last CTA.
    rng = np.random.default_rng(2000 + log_n)
    batch = 512 * rows_per_cta(log_n) + 3
    x = rand_c64(rng, batch << log_n)
    for direction, normalize in (("forward", False), ("inverse", True)):
        got = run_1d(capi, dev, x, log_n, direction, normalize)
        ref = oracle_mod.fft_1d(x, log_n, direction, normalize, threads=8)
        assert max_rel_err(got, ref) < TOL


@pytest.mark.parametrize("log_n", [2, 8, 10, 12, 14])
def test_single_pass_in_place(capi, dev, oracle_mod, log_n):
    rng = np.random.default_rng(3000 + log_n)
    x = rand_c64(rng, 700 << log_n)
    got = run_1d(capi, dev, x, log_n, "forward", False, inplace=True)
    ref = oracle_mod.fft_1d(x, log_n, "forward", False, threads=8)
    assert max_rel_err(got, ref) < TOL


@pytest.mark.parametrize("log_n", [4, 8, 12])
def test_single_pass_unaligned_input_uses_plain_kernel(capi, dev, oracle_mod, log_n):
    # An input that is 8- but not 16-byte aligned cannot feed the TMA bulk
    # copies; the call must take the plain kernel and give the same result.
    rng = np.random.default_rng(3500 + log_n)
    batch = 600
    x = rand_c64(rng, batch << log_n)
    buf = torch.zeros(x.size + 1, dtype=torch.complex64, device="cuda")
    buf[1:] = torch.from_numpy(x).to("cuda")
    out = torch.empty(x.size, dtype=torch.complex64, device="cuda")
    assert (buf[1:].data_ptr() % 16) == 8
    capi.fft_1d(dev, buf[1:].data_ptr(), out.data_ptr(), log_n, batch, "forward", False, _stream())
    torch.cuda.synchronize()
    ref = oracle_mod.fft_1d(x, log_n, threads=8)
    assert max_rel_err(out.cpu().numpy(), ref) < TOL
    dev.sync()


@pytest.mark.parametrize("log_n", list(range(15, 25)))
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_four_step(capi, dev, oracle_mod, log_n, direction, normalize):
    rng = np.random.default_rng(4000 + log_n)
    batch = 3 if log_n <= 20 else 1
    x = rand_c64(rng, batch << log_n, "normal")
    got = run_1d(capi, dev, x, log_n, direction, normalize)
    ref = oracle_mod.fft_1d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(got, ref) < TOL


@pytest.mark.parametrize("log_n", [19, 20, 22, 23])
def test_four_step_unaligned_buffers_use_plain_kernels(capi, dev, oracle_mod, log_n):
    # The tile kernels of the 2^19..2^23 plans read and write through TMA
    # tensor maps, which need 16-byte aligned buffers. An input and a
    # workspace that are 8- but not 16-byte aligned must take the plain
    # kernels of the same passes and give the same result.
    rng = np.random.default_rng(4400 + log_n)
    batch = 2
    x = rand_c64(rng, batch << log_n, "normal")
    buf = torch.zeros(x.size + 1, dtype=torch.complex64, device="cuda")
    buf[1:] = torch.from_numpy(x).to("cuda")
    assert (buf[1:].data_ptr() % 16) == 8
    out = torch.empty(x.size, dtype=torch.complex64, device="cuda")
    ws_bytes = capi.workspace_bytes(log_n, batch, 1)
    ws = torch.empty(ws_bytes + 8, dtype=torch.uint8, device="cuda")
    ref = oracle_mod.fft_1d(x, log_n, threads=THREADS)
    for ws_ptr in (ws.data_ptr(), ws.data_ptr() + 8):
        capi.fft_1d_ws(dev, buf[1:].data_ptr(), out.data_ptr(), log_n, batch, "forward", False,
                       ws_ptr, ws_bytes, _stream())
        torch.cuda.synchronize()
        assert max_rel_err(out.cpu().numpy(), ref) < TOL
    aligned = torch.from_numpy(x).to("cuda")
    capi.fft_1d(dev, aligned.data_ptr(), out.data_ptr(), log_n, batch, "forward", False, _stream())
    torch.cuda.synchronize()
    assert max_rel_err(out.cpu().numpy(), ref) < TOL
    dev.sync()


@pytest.mark.parametrize("log_n", [15, 18, 19, 21, 22, 23, 24, 26])
def test_four_step_accuracy_budget(capi, dev, log_n):
    # The multi-pass 1D takes its four-step twiddle factors from the SFU
    # (sin/cos within ~7e-7 per component instead of a correctly rounded
    # table). The whole transform must stay far inside the 1e-4 contract:
    # measured 5e-7 .. 1.1e-6 against a float64 FFT of the same inputs.
    rng = np.random.default_rng(4300 + log_n)
    x = rand_c64(rng, 1 << log_n, "normal")
    got = run_1d(capi, dev, x, log_n, "forward", False)
    ref = np.fft.fft(x.astype(np.complex128))
    assert max_rel_err(got, ref) < 3e-6


def test_four_step_in_place_and_caller_workspace(capi, dev, oracle_mod):
    rng = np.random.default_rng(4100)
    log_n, batch = 20, 2
    x = rand_c64(rng, batch << log_n, "normal")
    ref = oracle_mod.fft_1d(x, log_n, threads=8)
    assert max_rel_err(run_1d(capi, dev, x, log_n, "forward", False, inplace=True), ref) < TOL
    t_in = torch.from_numpy(x).to("cuda")
    t_out = torch.empty_like(t_in)
    ws_bytes = capi.workspace_bytes(log_n, batch, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    capi.fft_1d_ws(dev, t_in.data_ptr(), t_out.data_ptr(), log_n, batch, "forward", False,
                   ws.data_ptr(), ws_bytes, _stream())
    torch.cuda.synchronize()
    assert max_rel_err(t_out.cpu().numpy(), ref) < TOL
    with pytest.raises(capi.FerrumError) as e:
        capi.fft_1d_ws(dev, t_in.data_ptr(), t_out.data_ptr(), log_n, batch, "forward", False,
                       ws.data_ptr(), ws_bytes - 8, _stream())
    assert e.value.status == capi.FERRUM_ERR_INVALID_ARG


def test_four_step_2_26_roundtrip(capi, dev):
    # Largest 1D length: round trip and a DC check instead of the oracle.
    log_n = 26
    rng = np.random.default_rng(4200)
    x = rand_c64(rng, 1 << log_n, "normal")
    t = torch.from_numpy(x).to("cuda")
    y = torch.empty_like(t)
    capi.fft_1d(dev, t.data_ptr(), y.data_ptr(), log_n, 1, "forward", False, _stream())
    torch.cuda.synchronize()
    dc = complex(y[0].item())
    want = complex(np.sum(x.astype(np.complex128)))
    assert abs(dc - want) / max(1.0, abs(want)) < 1e-4 * np.sqrt(1 << log_n)
    capi.fft_1d(dev, y.data_ptr(), y.data_ptr(), log_n, 1, "inverse", True, _stream())
    torch.cuda.synchronize()
    assert max_rel_err(y.cpu().numpy(), x) < TOL


@pytest.mark.parametrize("log_n", list(range(2, 13)))
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_2d(capi, dev, oracle_mod, log_n, direction, normalize):
    rng = np.random.default_rng(5000 + log_n)
    n = 1 << log_n
    batch = 3 if log_n <= 10 else 1
    x = rand_c64(rng, (batch, n, n))
    got = run_2d(capi, dev, x, log_n, direction, normalize)
    ref = oracle_mod.fft_2d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(got, ref) < TOL


@pytest.mark.parametrize("log_n,batch", [(11, 2), (12, 3), (13, 1)])
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_2d_in_place(capi, dev, oracle_mod, log_n, batch, direction, normalize):
    # N = 2048: one column pass; N = 4096: the fused two-sub-pass column
    # kernel (three images: tiles of more than one image per CTA); N = 8192:
    # separate sub-passes; every plan then runs the rows in place.
    rng = np.random.default_rng(5100 + log_n)
    n = 1 << log_n
    x = rand_c64(rng, (batch, n, n), "normal")
    got = run_2d(capi, dev, x, log_n, direction, normalize, inplace=True)
    ref = oracle_mod.fft_2d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(got, ref) < TOL


def test_2d_16384_full_image(capi, dev, oracle_mod):
    """16384 x 16384 (the distributed config, here on one GPU, standard normal
    inputs): the whole forward image against the oracle's 2D (row pass,
    transpose, row pass, transpose), then the inverse with 1/N^2 against the
    oracle's inverse of the same spectrum, and the round trip."""
    log_n = 14
    n = 1 << log_n
    g = torch.Generator(device="cuda").manual_seed(14)
    x = torch.complex(torch.randn(n, n, device="cuda", generator=g),
                      torch.randn(n, n, device="cuda", generator=g))
    y = torch.empty_like(x)
    s = _stream()
    capi.fft_2d(dev, x.data_ptr(), y.data_ptr(), log_n, 1, "forward", False, s)
    torch.cuda.synchronize()
    xh = x.cpu().numpy()
    ref = oracle_mod.fft_2d(xh, log_n, "forward", False, threads=THREADS)
    assert max_rel_err(y.cpu().numpy(), ref) < TOL
    # the inverse from the oracle's own spectrum, so both see the same input
    yr = torch.from_numpy(ref).to("cuda")
    capi.fft_2d(dev, yr.data_ptr(), y.data_ptr(), log_n, 1, "inverse", True, s)
    torch.cuda.synchronize()
    ref_inv = oracle_mod.fft_2d(ref, log_n, "inverse", True, threads=THREADS)
    del ref
    assert max_rel_err(y.cpu().numpy(), ref_inv) < TOL
    assert max_rel_err(ref_inv, xh) < TOL
    assert float((y - x).abs().max() / x.abs().max()) < TOL


@pytest.mark.parametrize("log_n,batch", [(10, 1 << 15), (12, 3000), (20, 5)])
def test_host_pointer_path(capi, dev, oracle_mod, log_n, batch):
    # Spans several 64 MiB chunks; pageable (numpy) and pinned (torch) buffers.
    rng = np.random.default_rng(6000 + log_n)
    x = rand_c64(rng, batch << log_n)
    ref_rows = np.r_[0:3, batch - 3:batch]
    ref = oracle_mod.fft_1d(x.reshape(batch, -1)[ref_rows].reshape(-1), log_n, threads=8)
    out = np.empty_like(x)
    capi.fft_1d_host(dev, x.ctypes.data, out.ctypes.data, log_n, batch, "forward", False)
    assert max_rel_err(out.reshape(batch, -1)[ref_rows], ref) < TOL
    pin_in = torch.from_numpy(x).pin_memory()
    pin_out = torch.empty_like(pin_in).pin_memory()
    capi.fft_1d_host(dev, pin_in.data_ptr(), pin_out.data_ptr(), log_n, batch, "forward", False)
    assert np.array_equal(pin_out.numpy().view(np.uint64), out.view(np.uint64))


@pytest.mark.parametrize("log_n,batch,direction,normalize", [(11, 5, "inverse", True),
                                                            (12, 4, "forward", False)])
def test_host_pointer_2d(capi, dev, oracle_mod, log_n, batch, direction, normalize):
    # N = 4096: one 128 MiB image per chunk, so the three pipeline streams run
    # the fused column kernel concurrently, each with its own scratch slots.
    rng = np.random.default_rng(6100 + log_n)
    n = 1 << log_n
    x = rand_c64(rng, (batch, n, n))
    out = np.empty_like(x)
    capi.fft_2d_host(dev, x.ctypes.data, out.ctypes.data, log_n, batch, direction, normalize)
    pick = [0, batch - 1]
    ref = oracle_mod.fft_2d(x[pick], log_n, direction, normalize, threads=8)
    assert max_rel_err(out[pick], ref) < TOL


@pytest.mark.parametrize("log_n,batch", [(8, 1 << 20), (10, 1 << 18), (12, 1 << 16), (14, 1 << 14)])
def test_config_sizes_properties(capi, dev, oracle_mod, log_n, batch):
    """2 GiB sweep sizes (N = 256..16384): sampled-row parity, round trip,
    linearity and Parseval on the full batch."""
    n = 1 << log_n
    g = torch.Generator(device="cuda").manual_seed(log_n)
    x = torch.complex(torch.rand(batch, n, device="cuda", generator=g) * 2 - 1,
                      torch.rand(batch, n, device="cuda", generator=g) * 2 - 1)
    y = torch.empty_like(x)
    s = _stream()
    capi.fft_1d(dev, x.data_ptr(), y.data_ptr(), log_n, batch, "forward", False, s)
    torch.cuda.synchronize()
    # 64 rows spread over the batch (the first, the last and 62 between,
    # seeded) against the oracle
    pick = np.random.default_rng(100 + log_n).choice(np.arange(1, batch - 1), 62, replace=False)
    rows = torch.tensor(np.r_[0, np.sort(pick), batch - 1], device="cuda")
    ref = oracle_mod.fft_1d(x[rows].cpu().numpy().reshape(-1), log_n, threads=THREADS)
    assert max_rel_err(y[rows].cpu().numpy().reshape(-1), ref) < TOL
    # Parseval: sum |X|^2 = N sum |x|^2 (per row, in float64)
    ex = (x.abs().double() ** 2).sum(dim=1) * n
    ey = (y.abs().double() ** 2).sum(dim=1)
    assert float(((ey - ex).abs() / ex).max()) < 1e-4
    # linearity on a slice: F(a x0 + b x1) = a F(x0) + b F(x1)
    a, b = 0.75 - 0.5j, -1.25 + 0.25j
    k = 4096 if batch > 8192 else batch // 2
    z = (a * x[:k] + b * x[k:2 * k]).contiguous()
    fz = torch.empty_like(z)
    capi.fft_1d(dev, z.data_ptr(), fz.data_ptr(), log_n, k, "forward", False, s)
    torch.cuda.synchronize()
    lin = a * y[:k] + b * y[k:2 * k]
    assert float((fz - lin).abs().max() / lin.abs().max()) < TOL
    # round trip in place
    capi.fft_1d(dev, y.data_ptr(), y.data_ptr(), log_n, batch, "inverse", True, s)
    torch.cuda.synchronize()
    assert float((y - x).abs().max() / x.abs().max()) < TOL


@pytest.mark.parametrize("log_n,batch", [(20, 64), (24, 4)])
def test_large_n_config_properties(capi, dev, oracle_mod, log_n, batch):
    """Large-N sizes 2^20 x 64 and 2^24 x 4 (standard normal inputs): every transform
    against the oracle, forward and inverse (1/N), and the full batch through a round trip."""
    n = 1 << log_n
    g = torch.Generator(device="cuda").manual_seed(log_n)
    x = torch.complex(torch.randn(batch, n, device="cuda", generator=g),
                      torch.randn(batch, n, device="cuda", generator=g))
    y = torch.empty_like(x)
    s = _stream()
    capi.fft_1d(dev, x.data_ptr(), y.data_ptr(), log_n, batch, "forward", False, s)
    torch.cuda.synchronize()
    xh = x.cpu().numpy()
    ref = oracle_mod.fft_1d(xh.reshape(-1), log_n, threads=THREADS).reshape(batch, n)
    yh = y.cpu().numpy()
    for i in range(batch):
        assert max_rel_err(yh[i], ref[i]) < TOL, i
    yr = torch.from_numpy(ref).to("cuda")
    z = torch.empty_like(yr)
    capi.fft_1d(dev, yr.data_ptr(), z.data_ptr(), log_n, batch, "inverse", True, s)
    torch.cuda.synchronize()
    ref_inv = oracle_mod.fft_1d(ref.reshape(-1), log_n, "inverse", True,
                                threads=THREADS).reshape(batch, n)
    zh = z.cpu().numpy()
    for i in range(batch):
        assert max_rel_err(zh[i], ref_inv[i]) < TOL, i
    capi.fft_1d(dev, y.data_ptr(), y.data_ptr(), log_n, batch, "inverse", True, s)
    torch.cuda.synchronize()
    assert float((y - x).abs().max() / x.abs().max()) < TOL


def test_2d_config4_properties(capi, dev, oracle_mod):
    """2D 4096 x 4096 x 16 images: one image against the
    oracle, all through a round trip."""
    log_n, batch = 12, 16
    n = 1 << log_n
    g = torch.Generator(device="cuda").manual_seed(44)
    x = torch.complex(torch.rand(batch, n, n, device="cuda", generator=g) * 2 - 1,
                      torch.rand(batch, n, n, device="cuda", generator=g) * 2 - 1)
    y = torch.empty_like(x)
    s = _stream()
    capi.fft_2d(dev, x.data_ptr(), y.data_ptr(), log_n, batch, "forward", False, s)
    torch.cuda.synchronize()
    ref = oracle_mod.fft_2d(x[7].cpu().numpy(), log_n, threads=8)
    assert max_rel_err(y[7].cpu().numpy(), ref) < TOL
    capi.fft_2d(dev, y.data_ptr(), y.data_ptr(), log_n, batch, "inverse", True, s)
    torch.cuda.synchronize()
    assert float((y - x).abs().max() / x.abs().max()) < TOL


def test_invalid_arguments_with_device(capi, dev):
    t = torch.zeros(64, dtype=torch.complex64, device="cuda")
    lib = capi.lib()
    s = _stream()
    assert lib.ferrum_fft_1d_c2c_pow2(dev.ptr, t.data_ptr() + 4, t.data_ptr(), 4, 1, 1, 0, s) \
        == capi.FERRUM_ERR_INVALID_ARG
    assert lib.ferrum_fft_1d_c2c_pow2(dev.ptr, t.data_ptr(), t.data_ptr(), 4, 1, 2, 0, s) \
        == capi.FERRUM_ERR_INVALID_ARG
    assert lib.ferrum_fft_1d_c2c_pow2(dev.ptr, t.data_ptr(), t.data_ptr(), 27, 1, 1, 0, s) \
        == capi.FERRUM_ERR_INVALID_ARG
    assert lib.ferrum_fft_2d_c2c_pow2(dev.ptr, t.data_ptr(), t.data_ptr(), 15, 1, 1, 0, s) \
        == capi.FERRUM_ERR_INVALID_ARG
    assert lib.ferrum_fft_1d_c2c_pow2(dev.ptr, None, t.data_ptr(), 4, 1, 1, 0, s) \
        == capi.FERRUM_ERR_INVALID_ARG
