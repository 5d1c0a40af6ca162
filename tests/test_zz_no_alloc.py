"""ferrum_fft_1d_c2c_pow2_noalloc, the allocation-free 1D entry point.

Callers whose device memory belongs to their own allocator, or that run in
latency-critical loops where an allocation may block, use this entry point:
lengths above 2^14 take their multi-pass intermediate from a static 32 MiB
device array instead of a workspace. Calls in a row (different lengths, so
each later call sees the previous call's leftovers in the shared array) must
match the pool-backed entry point ferrum_fft_1d_c2c_pow2 within the suite's
1e-4 tolerance; the largest case (one 2^22 transform, the whole scratch and
the longest length it takes) is also compared with the CPU oracle directly. A request
larger than the array, or a batch whose size would overflow, is rejected.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import max_rel_err, rand_c64

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

TOL = 1e-4


def _run(fn, dev, x, log_n, direction, normalize):
    batch = x.size >> log_n
    t_in = torch.from_numpy(x).to("cuda")
    t_out = torch.empty_like(t_in)
    fn(dev, t_in.data_ptr(), t_out.data_ptr(), log_n, batch, direction, normalize,
       torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return t_out.cpu().numpy()


def test_no_alloc_matches_pool_entry_point(oracle_mod):
    from ferrum_gpu import capi

    dev = capi.DeviceHandle(0)
    try:
        cases = [(20, 4, "forward", False),   # fills the whole 2^22 scratch
                 (18, 3, "inverse", True),    # second call over stale contents
                 (22, 1, "forward", False),   # the longest length, whole scratch again
                 (12, 5, "forward", False)]   # single pass, no scratch
        for i, (log_n, batch, direction, normalize) in enumerate(cases):
            x = rand_c64(np.random.default_rng(77 + i), batch << log_n, "normal")
            want = _run(capi.fft_1d, dev, x, log_n, direction, normalize)
            got = _run(capi.fft_1d_noalloc, dev, x, log_n, direction, normalize)
            assert max_rel_err(got, want) < TOL, (log_n, batch, direction)
            if log_n == 22:
                ref = oracle_mod.fft_1d(x, log_n, direction, normalize)
                assert max_rel_err(got, ref) < TOL

        t = torch.zeros(1 << 23, dtype=torch.complex64, device="cuda")
        st = capi.lib().ferrum_fft_1d_c2c_pow2_noalloc(
            dev.ptr, t.data_ptr(), t.data_ptr(), 22, 2, 1, 0,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert st == capi.FERRUM_ERR_INVALID_ARG
        assert "exceed the static scratch" in capi.last_error()
        st = capi.lib().ferrum_fft_1d_c2c_pow2_noalloc(
            dev.ptr, t.data_ptr(), t.data_ptr(), 20, (1 << 44) + 1, 1, 0,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert st == capi.FERRUM_ERR_INVALID_ARG
        assert "exceeds 2^36" in capi.last_error()
    finally:
        dev.close()
