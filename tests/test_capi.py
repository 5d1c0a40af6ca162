"""The C ABI library loads and exports every symbol include/ferrum_fft.h
declares; argument validation works without a GPU, and compute entry points
fail loudly (no CPU fallback) when no B200 is present."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import REPO, gpu_available

HEADER = os.path.join(REPO, "include", "ferrum_fft.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(ferrum_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def capi():
    from ferrum_gpu import capi as c

    c.lib()
    return c


def test_header_and_binding_agree(capi):
    assert declared_symbols() == sorted(capi.SIGNATURES)


def test_library_exports_every_declared_symbol(capi):
    lib = ctypes.CDLL(capi.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert missing == []


def test_version(capi):
    import ferrum_gpu

    assert capi.version() == "0.3.0-b200"
    assert ferrum_gpu.version() == capi.version()


def test_workspace_and_launch_counts(capi):
    assert capi.workspace_bytes(12, 65536, 1) == 0
    assert capi.workspace_bytes(20, 64, 1) == (1 << 20) * 64 * 8
    assert capi.workspace_bytes(24, 4, 1) == (1 << 24) * 4 * 8
    # 2D up to 512^2: row pass + one column pass in place, no workspace;
    # 1024^2..4096^2: two transposed-row passes through an image-sized
    # workspace; from 8192^2 two column sub-passes and the row pass.
    assert capi.workspace_bytes(9, 16, 2) == 0
    assert capi.workspace_bytes(10, 16, 2) == 16 * (1 << 20) * 8
    assert capi.workspace_bytes(12, 16, 2) == 16 * (1 << 24) * 8
    assert capi.workspace_bytes(13, 4, 2) == 4 * (1 << 26) * 8
    assert capi.workspace_bytes(14, 1, 2) == (1 << 28) * 8
    assert capi.launch_count(10, 256, 1) == 1
    assert capi.launch_count(14, 1, 1) == 1
    assert capi.launch_count(15, 1, 1) == 2
    assert capi.launch_count(21, 1, 1) == 2
    assert capi.launch_count(22, 1, 1) == 2
    assert capi.launch_count(23, 1, 1) == 2
    assert capi.launch_count(24, 1, 1) == 3
    assert capi.launch_count(26, 1, 1) == 3
    assert capi.launch_count(10, 16, 2) == 2
    assert capi.launch_count(11, 64, 2) == 2
    assert capi.launch_count(9, 64, 2) == 2
    assert capi.launch_count(12, 16, 2) == 2
    assert capi.launch_count(14, 1, 2) == 3
    assert capi.launch_count(13, 4, 2) == 3


@pytest.mark.parametrize("log_n,batch,kind", [(1, 1, 1), (27, 1, 1), (10, 0, 1), (15, 1, 2),
                                              (10, 1, 3),
                                              # N * batch above 2^36 complex values: rejected
                                              # before any size is formed (2^44 + 1 would wrap
                                              # the byte count at 2^20)
                                              (20, (1 << 44) + 1, 1), (20, (1 << 16) + 1, 1),
                                              (14, (1 << 8) + 1, 2), (2, (1 << 34) + 1, 1)])
def test_invalid_sizes_rejected(capi, log_n, batch, kind):
    with pytest.raises(capi.FerrumError) as e:
        capi.workspace_bytes(log_n, batch, kind)
    assert e.value.status == capi.FERRUM_ERR_INVALID_ARG


def test_largest_allowed_batch_sizes(capi):
    # exactly 2^36 complex values per call is still accepted
    assert capi.workspace_bytes(20, 1 << 16, 1) == (1 << 36) * 8
    assert capi.workspace_bytes(2, 1 << 34, 1) == 0


def test_null_device_rejected(capi):
    lib = capi.lib()
    st = lib.ferrum_fft_1d_c2c_pow2(None, 16, 16, 10, 1, 1, 0, None)
    assert st == capi.FERRUM_ERR_INVALID_ARG
    assert "device handle" in capi.last_error()
    st = lib.ferrum_fft_2d_c2c_pow2_host(None, 16, 16, 10, 1, 1, 0)
    assert st == capi.FERRUM_ERR_INVALID_ARG


def test_dist_shape_check(capi):
    lib = capi.lib()
    assert lib.ferrum_dist_check(14, 8) == capi.FERRUM_OK
    assert lib.ferrum_dist_check(14, 3) == capi.FERRUM_ERR_INVALID_ARG
    assert lib.ferrum_dist_check(3, 2) == capi.FERRUM_ERR_INVALID_ARG
    assert lib.ferrum_dist_check(4, 16) == capi.FERRUM_ERR_INVALID_ARG


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure mode")
def test_no_cpu_fallback_without_gpu(capi):
    with pytest.raises(capi.FerrumError) as e:
        capi.DeviceHandle(0)
    assert e.value.status in (capi.FERRUM_ERR_CUDA, capi.FERRUM_ERR_UNSUPPORTED,
                              capi.FERRUM_ERR_INVALID_ARG)
