"""Split (planar) layout entry points and the complex helpers.

Mirrors the reference's split twins and layout kernels
(crates/ferrum-gpu-fft-kernels/src/kernels_body.rs:508-626, 1614-1672). CPU:
argument validation through the C ABI (no compute is launched). GPU: the
split transform equals the interleaved one bit for bit (same butterflies),
the interleaved transform is checked against the oracle elsewhere; cmul
equals float32 arithmetic with separate roundings; (de)interleave are exact.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import gpu_available, max_rel_err, rand_c64

from ferrum_gpu import capi

ERR_INVALID = capi.FERRUM_ERR_INVALID_ARG


def test_split_argument_checks():
    lib = capi.lib()
    assert lib.ferrum_fft_1d_c2c_pow2_split(None, 1, 1, 1, 1, 4, 1, 1, 0, None) == ERR_INVALID
    assert lib.ferrum_cmul_interleaved(None, 8, 8, 8, 4, None) == ERR_INVALID
    assert lib.ferrum_cmul_split(None, 4, 4, 4, 4, 4, 4, 4, None) == ERR_INVALID
    assert lib.ferrum_deinterleave(None, 8, 4, 4, 4, None) == ERR_INVALID
    assert lib.ferrum_interleave(None, 4, 4, 8, 4, None) == ERR_INVALID
    assert "device handle" in capi.last_error()


# ---------------------------------------------------------------------------
torch = None


@pytest.fixture(scope="module")
def gpu():
    global torch
    torch = pytest.importorskip("torch")
    if not gpu_available():
        pytest.skip("no B200")
    return capi.DeviceHandle(0)


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.gpu
@pytest.mark.parametrize("log_n,batch", [(2, 7), (4, 33), (5, 17), (6, 9), (10, 5), (12, 3),
                                         (13, 2), (14, 2)])
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_split_transform_equals_interleaved(gpu, oracle_mod, log_n, batch, direction, normalize):
    n = 1 << log_n
    x = rand_c64(np.random.default_rng(7000 + log_n), batch * n)
    t = torch.from_numpy(x).cuda()
    y = torch.empty_like(t)
    capi.fft_1d(gpu, t.data_ptr(), y.data_ptr(), log_n, batch, direction, normalize, _stream())
    re = torch.from_numpy(np.ascontiguousarray(x.real)).cuda()
    im = torch.from_numpy(np.ascontiguousarray(x.imag)).cuda()
    ore, oim = torch.empty_like(re), torch.empty_like(im)
    capi.fft_1d_split(gpu, re.data_ptr(), im.data_ptr(), ore.data_ptr(), oim.data_ptr(), log_n,
                      batch, direction, normalize, _stream())
    torch.cuda.synchronize()
    yi = y.cpu().numpy()
    assert np.array_equal(ore.cpu().numpy(), yi.real) and np.array_equal(oim.cpu().numpy(), yi.imag)
    # in place on the split arrays
    capi.fft_1d_split(gpu, re.data_ptr(), im.data_ptr(), re.data_ptr(), im.data_ptr(), log_n,
                      batch, direction, normalize, _stream())
    torch.cuda.synchronize()
    assert np.array_equal(re.cpu().numpy(), yi.real) and np.array_equal(im.cpu().numpy(), yi.imag)
    ref = oracle_mod.fft_1d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(yi, ref) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 255, 4096, 1 << 20])
def test_cmul_and_interleave(gpu, n):
    rng = np.random.default_rng(n)
    a = rand_c64(rng, n)
    b = rand_c64(rng, n)
    ar, ai = a.real.astype(np.float32), a.imag.astype(np.float32)
    br, bi = b.real.astype(np.float32), b.imag.astype(np.float32)
    want_re = ar * br - ai * bi   # each float32 product and difference rounded
    want_im = ar * bi + ai * br
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    to = torch.empty_like(ta)
    capi.cmul_interleaved(gpu, ta.data_ptr(), tb.data_ptr(), to.data_ptr(), n, _stream())
    s = [torch.from_numpy(np.ascontiguousarray(v)).cuda() for v in (ar, ai, br, bi)]
    ore, oim = torch.empty_like(s[0]), torch.empty_like(s[0])
    capi.cmul_split(gpu, *(v.data_ptr() for v in s), ore.data_ptr(), oim.data_ptr(), n, _stream())
    dre, dim = torch.empty_like(s[0]), torch.empty_like(s[0])
    capi.deinterleave(gpu, ta.data_ptr(), dre.data_ptr(), dim.data_ptr(), n, _stream())
    back = torch.empty_like(ta)
    capi.interleave(gpu, dre.data_ptr(), dim.data_ptr(), back.data_ptr(), n, _stream())
    torch.cuda.synchronize()
    o = to.cpu().numpy()
    assert np.array_equal(o.real, want_re) and np.array_equal(o.imag, want_im)
    assert np.array_equal(ore.cpu().numpy(), want_re) and np.array_equal(oim.cpu().numpy(), want_im)
    assert np.array_equal(dre.cpu().numpy(), ar) and np.array_equal(dim.cpu().numpy(), ai)
    assert np.array_equal(back.cpu().numpy(), a)


@pytest.mark.gpu
def test_split_rejects_bad_shapes(gpu):
    lib = capi.lib()
    t = torch.zeros(64, device="cuda")
    p = t.data_ptr()
    assert lib.ferrum_fft_1d_c2c_pow2_split(gpu.ptr, p, p, p, p, 15, 1, 1, 0, None) == ERR_INVALID
    assert lib.ferrum_fft_1d_c2c_pow2_split(gpu.ptr, p, p, p, p, 4, 0, 1, 0, None) == ERR_INVALID
    assert lib.ferrum_fft_1d_c2c_pow2_split(gpu.ptr, p, p + 4, p + 4, p, 4, 1, 1, 0, None) == ERR_INVALID
