"""The kernel-module substrate (the reference's backend contract,
crates/ferrum-gpu-core/src/backend.rs:12-77) and its vector-add example.

CPU: argument validation through the C ABI. GPU: a hand-written PTX
vector-add kernel is loaded, looked up by name and launched on zeroed buffers
filled by synchronous copies, as the reference's vector-add examples do.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import gpu_available

from ferrum_gpu import capi

# c[i] = a[i] + b[i] for i < n, one thread per element (written for this test).
VECTOR_ADD_PTX = r"""
.version 8.6
.target sm_100a
.address_size 64

.visible .entry vector_add(
    .param .u64 pa,
    .param .u64 pb,
    .param .u64 pc,
    .param .u32 n)
{
    .reg .pred %p;
    .reg .b32 %idx, %cta, %ntd, %thr, %cnt;
    .reg .b64 %a, %b, %c, %off;
    .reg .f32 %x, %y, %z;

    ld.param.u64 %a, [pa];
    ld.param.u64 %b, [pb];
    ld.param.u64 %c, [pc];
    ld.param.u32 %cnt, [n];
    mov.u32 %cta, %ctaid.x;
    mov.u32 %ntd, %ntid.x;
    mov.u32 %thr, %tid.x;
    mad.lo.u32 %idx, %cta, %ntd, %thr;
    setp.ge.u32 %p, %idx, %cnt;
    @%p bra DONE;
    cvta.to.global.u64 %a, %a;
    cvta.to.global.u64 %b, %b;
    cvta.to.global.u64 %c, %c;
    mul.wide.u32 %off, %idx, 4;
    add.s64 %a, %a, %off;
    add.s64 %b, %b, %off;
    add.s64 %c, %c, %off;
    ld.global.f32 %x, [%a];
    ld.global.f32 %y, [%b];
    add.f32 %z, %x, %y;
    st.global.f32 [%c], %z;
DONE:
    ret;
}
"""


def test_substrate_argument_checks():
    lib = capi.lib()
    out = ctypes.c_void_p()
    inv = capi.FERRUM_ERR_INVALID_ARG
    assert lib.ferrum_buffer_alloc_zeros(None, 16, ctypes.byref(out)) == inv
    assert lib.ferrum_copy_h2d(None, 1, 1, 4) == inv
    assert lib.ferrum_copy_d2h(None, 1, 1, 4) == inv
    assert lib.ferrum_module_load(None, b"x\0", ctypes.byref(out)) == inv
    assert lib.ferrum_module_kernel(None, b"k", ctypes.byref(out)) == inv
    g = (ctypes.c_uint * 3)(1, 1, 1)
    assert lib.ferrum_launch(None, 1, g, g, 0, None, None) == inv
    assert lib.ferrum_stream_sync(None, None) == inv
    assert lib.ferrum_module_unload(None) == capi.FERRUM_OK


@pytest.mark.gpu
def test_vector_add_module():
    if not gpu_available():
        pytest.skip("no B200")
    dev = capi.DeviceHandle(0)
    lib = capi.lib()
    n = 1_000_003
    rng = np.random.default_rng(11)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    bufs = []
    for _ in range(3):
        p = ctypes.c_void_p()
        capi.check(lib.ferrum_buffer_alloc_zeros(dev.ptr, n * 4, ctypes.byref(p)))
        bufs.append(p)
    zeros = np.ones(n, np.float32)
    capi.check(lib.ferrum_copy_d2h(dev.ptr, zeros.ctypes.data, bufs[2], n * 4))
    assert not zeros.any()  # zero-filled
    capi.check(lib.ferrum_copy_h2d(dev.ptr, bufs[0], a.ctypes.data, n * 4))
    capi.check(lib.ferrum_copy_h2d(dev.ptr, bufs[1], b.ctypes.data, n * 4))
    mod = capi.Module(dev, VECTOR_ADD_PTX)
    k = mod.kernel("vector_add")
    mod.launch(k, ((n + 255) // 256,), (256,),
               [ctypes.c_void_p(bufs[0].value), ctypes.c_void_p(bufs[1].value),
                ctypes.c_void_p(bufs[2].value), ctypes.c_uint(n)])
    capi.check(lib.ferrum_stream_sync(dev.ptr, None))
    c = np.empty(n, np.float32)
    capi.check(lib.ferrum_copy_d2h(dev.ptr, c.ctypes.data, bufs[2], n * 4))
    assert np.array_equal(c, a + b)
    with pytest.raises(capi.FerrumError):
        mod.kernel("no_such_kernel")
    mod.close()
    for p in bufs:
        capi.check(lib.ferrum_buffer_free(dev.ptr, p))
