"""ferrum_gpu.device: the zero-copy API over device arrays.

CPU tests check argument handling with stand-in CUDA Array Interface objects
(no compute is launched). GPU tests run torch tensors, a generic CUDA Array
Interface object and a DLPack-only object through the C ABI and compare with
the CPU oracle (max relative error < 1e-4).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import gpu_available, max_rel_err, rand_c64

from ferrum_gpu import device as fdev


class FakeCAI:
    """Carries a __cuda_array_interface__ dict; its pointer is never used."""

    def __init__(self, shape, typestr="<c8", strides=None, ptr=0, stream=None):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "strides": strides,
                                         "version": 3, "stream": stream}


def test_validation_order_and_messages():
    with pytest.raises(ValueError, match=r"log_n must be in \[2, 26\], got 27"):
        fdev.fft_1d_c2c_pow2(FakeCAI((8,)), 27)
    with pytest.raises(ValueError, match=r"log_n must be in \[2, 26\], got 1"):
        fdev.fft_1d_c2c_pow2(FakeCAI((8,)), 1)
    with pytest.raises(ValueError, match="complex64"):
        fdev.fft_1d_c2c_pow2(FakeCAI((8,), typestr="<f4"), 3)
    with pytest.raises(ValueError, match="C-contiguous"):
        fdev.fft_1d_c2c_pow2(FakeCAI((4, 8), strides=(8, 32)), 3)
    with pytest.raises(ValueError, match="arr len 12 must be a positive multiple of N = 8"):
        fdev.fft_1d_c2c_pow2(FakeCAI((12,)), 3)
    with pytest.raises(ValueError, match="arr len 0 must be a positive multiple of N = 8"):
        fdev.fft_1d_c2c_pow2(FakeCAI((0,)), 3)
    with pytest.raises(ValueError, match="direction must be 'forward' or 'inverse', got \"up\""):
        fdev.fft_1d_c2c_pow2(FakeCAI((16,)), 3, "up")
    with pytest.raises(ValueError, match=r"2D requires log_n in \[2, 14\]; got 15"):
        fdev.fft_2d_c2c_pow2(FakeCAI((4, 4)), 15)
    with pytest.raises(ValueError, match=r"arr shape \[4, 8\] != \(4, 4\)"):
        fdev.fft_2d_c2c_pow2(FakeCAI((4, 8)), 2)
    with pytest.raises(ValueError, match=r"arr shape \[16\] != \(4, 4\)"):
        fdev.fft_2d_c2c_pow2(FakeCAI((16,)), 2)


def test_rejects_host_arrays():
    with pytest.raises(ValueError, match="use ferrum_gpu.fft for numpy arrays"):
        fdev.fft_1d_c2c_pow2(np.zeros(8, np.complex64), 3)
    torch = pytest.importorskip("torch")
    with pytest.raises(ValueError, match="CPU tensor"):
        fdev.fft_1d_c2c_pow2(torch.zeros(8, dtype=torch.complex64), 3)


def test_out_shape_checked_before_launch():
    with pytest.raises(ValueError, match=r"out shape \[8\] != input shape \[16\]"):
        fdev.fft_1d_c2c_pow2(FakeCAI((16,)), 3, out=FakeCAI((8,)))


def test_stream_selection():
    v = fdev._view(FakeCAI((8,), stream=2), "arr")
    assert fdev._stream_handle(None, v) == 2          # announced by the array (v3)
    assert fdev._stream_handle(77, v) == 77            # explicit argument wins

    class S:
        cuda_stream = 99

    assert fdev._stream_handle(S(), v) == 99           # torch.cuda.Stream-like
    assert fdev._stream_handle(None, fdev._view(FakeCAI((8,)), "arr")) == 0


# ---------------------------------------------------------------------------
gpu = pytest.mark.gpu


def _torch_cuda():
    torch = pytest.importorskip("torch")
    if not gpu_available():
        pytest.skip("no B200")
    return torch


@gpu
@pytest.mark.parametrize("log_n,batch", [(2, 5), (8, 33), (12, 7), (14, 2), (18, 3), (22, 1)])
@pytest.mark.parametrize("direction,normalize", [("forward", False), ("inverse", True)])
def test_torch_1d_matches_oracle(oracle_mod, log_n, batch, direction, normalize):
    torch = _torch_cuda()
    rng = np.random.default_rng(900 + log_n)
    x = rand_c64(rng, batch << log_n)
    t = torch.from_numpy(x).cuda()
    y = fdev.fft_1d_c2c_pow2(t, log_n, direction, normalize)
    torch.cuda.synchronize()
    assert isinstance(y, torch.Tensor) and y.shape == t.shape and y.is_cuda
    ref = oracle_mod.fft_1d(x, log_n, direction, normalize, threads=8)
    assert max_rel_err(y.cpu().numpy(), ref) < 1e-4
    assert np.array_equal(t.cpu().numpy(), x)  # input untouched


@gpu
@pytest.mark.parametrize("log_n,batch", [(4, 3), (10, 2), (11, 1), (12, 1)])
def test_torch_2d_matches_oracle(oracle_mod, log_n, batch):
    torch = _torch_cuda()
    n = 1 << log_n
    x = rand_c64(np.random.default_rng(950 + log_n), (batch, n, n))
    t = torch.from_numpy(x).cuda()
    y = fdev.fft_2d_c2c_pow2(t, log_n)
    ref = oracle_mod.fft_2d(x, log_n, threads=8)
    assert y.shape == (batch, n, n)
    assert max_rel_err(y.cpu().numpy(), ref) < 1e-4
    back = fdev.fft_2d_c2c_pow2(y[0], log_n, "inverse", True)
    assert max_rel_err(back.cpu().numpy(), x[0]) < 1e-4


@gpu
def test_out_in_place_and_side_stream(oracle_mod):
    torch = _torch_cuda()
    log_n, batch = 13, 9
    x = rand_c64(np.random.default_rng(5), batch << log_n)
    ref = oracle_mod.fft_1d(x, log_n, threads=8)
    t = torch.from_numpy(x).cuda()
    out = torch.empty_like(t)
    assert fdev.fft_1d_c2c_pow2(t, log_n, out=out) is out
    assert max_rel_err(out.cpu().numpy(), ref) < 1e-4
    s = torch.cuda.Stream()
    u = t.clone()
    torch.cuda.current_stream().synchronize()
    with torch.cuda.stream(s):
        fdev.fft_1d_c2c_pow2(u, log_n, out=u)      # in place, on the side stream
        u2 = u * 2                                   # stream ordered after it
    s.synchronize()
    assert max_rel_err(u.cpu().numpy(), ref) < 1e-4
    assert max_rel_err(u2.cpu().numpy(), 2 * ref) < 1e-4


@gpu
def test_cuda_array_interface_and_dlpack_objects(oracle_mod):
    torch = _torch_cuda()
    log_n, batch = 10, 4
    x = rand_c64(np.random.default_rng(6), batch << log_n)
    ref = oracle_mod.fft_1d(x, log_n, threads=8)
    t = torch.from_numpy(x).cuda()

    class CAIOnly:
        def __init__(self, tensor):
            self._t = tensor
            self.__cuda_array_interface__ = {
                "shape": tuple(tensor.shape), "typestr": "<c8",
                "data": (tensor.data_ptr(), False), "strides": None, "version": 3,
                "stream": torch.cuda.current_stream().cuda_stream}

    class DLPackOnly:
        def __init__(self, tensor):
            self._t = tensor

        def __dlpack__(self, stream=None):
            return self._t.__dlpack__(stream=stream)

        def __dlpack_device__(self):
            return self._t.__dlpack_device__()

    out = torch.empty_like(t)
    r = fdev.fft_1d_c2c_pow2(CAIOnly(t), log_n, out=CAIOnly(out))
    torch.cuda.synchronize()
    assert isinstance(r, CAIOnly)
    assert max_rel_err(out.cpu().numpy(), ref) < 1e-4
    y = fdev.fft_1d_c2c_pow2(DLPackOnly(t), log_n)
    torch.cuda.synchronize()
    assert max_rel_err(y.cpu().numpy(), ref) < 1e-4


@gpu
def test_explicit_device_object(oracle_mod):
    torch = _torch_cuda()
    import ferrum_gpu as fg

    dev = fg.cuda.Device(0)
    x = rand_c64(np.random.default_rng(7), 3 << 9)
    y = fdev.fft_1d_c2c_pow2(torch.from_numpy(x).cuda(), 9, device=dev)
    assert max_rel_err(y.cpu().numpy(), oracle_mod.fft_1d(x, 9)) < 1e-4
