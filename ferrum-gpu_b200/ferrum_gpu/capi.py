"""ctypes binding of the C ABI in include/ferrum_fft.h.

This is the binding a caller of the reference would add to reach the B200
kernels through plain pointers: device-resident buffers (for example
``torch.Tensor.data_ptr()`` of a CUDA complex64 tensor), a ``cudaStream_t``
and sizes. Every function raises :class:`FerrumError` with the library's
status code and ``ferrum_last_error()`` message on failure. There is no CPU
fallback: on a machine without a B200 the compute calls fail with
``FERRUM_ERR_CUDA`` / ``FERRUM_ERR_UNSUPPORTED``.
"""

from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libferrum_fft.so")

FERRUM_OK = 0
FERRUM_ERR_INVALID_ARG = 1
FERRUM_ERR_CUDA = 2
FERRUM_ERR_NCCL = 3
FERRUM_ERR_TIMEOUT = 4
FERRUM_ERR_ALLOC = 5
FERRUM_ERR_UNSUPPORTED = 6
FORWARD = 1
INVERSE = -1
DIST_ID_BYTES = 128
DIST_ROW_SLAB = 0
DIST_COL_SLAB = 1

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_i = ctypes.c_int

# name -> (restype, argtypes); mirrors include/ferrum_fft.h one to one.
SIGNATURES = {
    "ferrum_version": (ctypes.c_char_p, []),
    "ferrum_last_error": (ctypes.c_char_p, []),
    "ferrum_device_create": (_i, [_i, ctypes.POINTER(_vp)]),
    "ferrum_device_destroy": (_i, [_vp]),
    "ferrum_device_sync": (_i, [_vp]),
    "ferrum_device_ordinal": (_i, [_vp, ctypes.POINTER(_i)]),
    "ferrum_fft_1d_c2c_pow2": (_i, [_vp, _vp, _vp, _i, _sz, _i, _i, _vp]),
    "ferrum_fft_1d_c2c_pow2_ws": (_i, [_vp, _vp, _vp, _i, _sz, _i, _i, _vp, _sz, _vp]),
    "ferrum_fft_1d_c2c_pow2_noalloc": (_i, [_vp, _vp, _vp, _i, _sz, _i, _i, _vp]),
    "ferrum_fft_2d_c2c_pow2": (_i, [_vp, _vp, _vp, _i, _sz, _i, _i, _vp]),
    "ferrum_fft_1d_c2c_pow2_host": (_i, [_vp, _vp, _vp, _i, _sz, _i, _i]),
    "ferrum_fft_1d_c2c_pow2_split": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _sz, _i, _i, _vp]),
    "ferrum_cmul_interleaved": (_i, [_vp, _vp, _vp, _vp, _sz, _vp]),
    "ferrum_cmul_split": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ferrum_deinterleave": (_i, [_vp, _vp, _vp, _vp, _sz, _vp]),
    "ferrum_interleave": (_i, [_vp, _vp, _vp, _vp, _sz, _vp]),
    "ferrum_buffer_alloc_zeros": (_i, [_vp, _sz, ctypes.POINTER(_vp)]),
    "ferrum_buffer_free": (_i, [_vp, _vp]),
    "ferrum_copy_h2d": (_i, [_vp, _vp, _vp, _sz]),
    "ferrum_copy_d2h": (_i, [_vp, _vp, _vp, _sz]),
    "ferrum_module_load": (_i, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "ferrum_module_unload": (_i, [_vp]),
    "ferrum_module_kernel": (_i, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "ferrum_launch": (_i, [_vp, _vp, ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_uint),
                           ctypes.c_uint, ctypes.POINTER(_vp), _vp]),
    "ferrum_stream_sync": (_i, [_vp, _vp]),
    "ferrum_fft_2d_c2c_pow2_host": (_i, [_vp, _vp, _vp, _i, _sz, _i, _i]),
    "ferrum_fft_workspace_bytes": (_i, [_i, _sz, _i, ctypes.POINTER(_sz)]),
    "ferrum_fft_launch_count": (_i, [_i, _sz, _i, ctypes.POINTER(_i)]),
    "ferrum_dist_get_unique_id": (_i, [ctypes.c_char_p]),
    "ferrum_dist_init": (_i, [_vp, ctypes.c_char_p, _i, _i, _i, ctypes.POINTER(_vp)]),
    "ferrum_dist_destroy": (_i, [_vp]),
    "ferrum_dist_world": (_i, [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "ferrum_dist_workspace_bytes": (_i, [_vp, _i, ctypes.POINTER(_sz)]),
    "ferrum_fft_2d_c2c_pow2_dist": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "ferrum_fft_2d_c2c_pow2_dist_layout": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "ferrum_dist_sync": (_i, [_vp, _vp]),
    "ferrum_dist_barrier": (_i, [_vp, _vp]),
    "ferrum_dist_peer_path": (_i, [_vp]),
    "ferrum_dist_set_timeout": (_i, [_vp, _i]),
    "ferrum_dist_abort": (_i, [_vp]),
    "ferrum_dist_check": (_i, [_i, _i]),
}


class FerrumError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"ferrum status {status}: {message}")
        self.status = status
        self.message = message


_lib = None


def lib() -> ctypes.CDLL:
    """Load libferrum_fft.so (raises if the library has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python ferrum-gpu_b200/build.py`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    return lib().ferrum_last_error().decode()


def check(status: int) -> None:
    if status != FERRUM_OK:
        raise FerrumError(status, last_error())


def version() -> str:
    return lib().ferrum_version().decode()


class DeviceHandle:
    """Owning wrapper of a ``ferrum_device*``."""

    def __init__(self, ordinal: int = 0):
        h = _vp()
        check(lib().ferrum_device_create(ordinal, ctypes.byref(h)))
        self.ptr = h
        self.ordinal = ordinal

    def sync(self) -> None:
        check(lib().ferrum_device_sync(self.ptr))

    def close(self) -> None:
        if self.ptr:
            lib().ferrum_device_destroy(self.ptr)
            self.ptr = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _dir(direction) -> int:
    if direction in (1, "forward"):
        return FORWARD
    if direction in (-1, "inverse"):
        return INVERSE
    raise ValueError(f"direction must be 'forward' or 'inverse', got {direction!r}")


def fft_1d(dev: DeviceHandle, in_ptr: int, out_ptr: int, log_n: int, batch: int,
           direction="forward", normalize: bool = False, stream: int = 0) -> None:
    """Enqueue a batched 1D C2C transform on device pointers."""
    check(lib().ferrum_fft_1d_c2c_pow2(dev.ptr, in_ptr, out_ptr, log_n, batch, _dir(direction),
                                       int(bool(normalize)), stream))


def fft_1d_ws(dev: DeviceHandle, in_ptr: int, out_ptr: int, log_n: int, batch: int,
              direction, normalize: bool, ws_ptr: int, ws_bytes: int, stream: int = 0) -> None:
    check(lib().ferrum_fft_1d_c2c_pow2_ws(dev.ptr, in_ptr, out_ptr, log_n, batch,
                                          _dir(direction), int(bool(normalize)), ws_ptr,
                                          ws_bytes, stream))


def fft_1d_noalloc(dev: DeviceHandle, in_ptr: int, out_ptr: int, log_n: int, batch: int,
                   direction="forward", normalize: bool = False, stream: int = 0) -> None:
    """Allocation-free 1D transform: lengths above 2^14 use the library's
    static 32 MiB device scratch (N * batch <= 2^22) instead of a workspace."""
    check(lib().ferrum_fft_1d_c2c_pow2_noalloc(dev.ptr, in_ptr, out_ptr, log_n, batch,
                                               _dir(direction), int(bool(normalize)), stream))


def fft_2d(dev: DeviceHandle, in_ptr: int, out_ptr: int, log_n: int, batch: int,
           direction="forward", normalize: bool = False, stream: int = 0) -> None:
    """Enqueue a batched 2D C2C transform on device pointers."""
    check(lib().ferrum_fft_2d_c2c_pow2(dev.ptr, in_ptr, out_ptr, log_n, batch, _dir(direction),
                                       int(bool(normalize)), stream))


def fft_1d_host(dev: DeviceHandle, in_ptr: int, out_ptr: int, log_n: int, batch: int,
                direction="forward", normalize: bool = False) -> None:
    check(lib().ferrum_fft_1d_c2c_pow2_host(dev.ptr, in_ptr, out_ptr, log_n, batch,
                                            _dir(direction), int(bool(normalize))))


def fft_2d_host(dev: DeviceHandle, in_ptr: int, out_ptr: int, log_n: int, batch: int,
                direction="forward", normalize: bool = False) -> None:
    check(lib().ferrum_fft_2d_c2c_pow2_host(dev.ptr, in_ptr, out_ptr, log_n, batch,
                                            _dir(direction), int(bool(normalize))))


def fft_1d_split(dev: DeviceHandle, in_re: int, in_im: int, out_re: int, out_im: int,
                 log_n: int, batch: int, direction="forward", normalize: bool = False,
                 stream: int = 0) -> None:
    """Batched 1D transform on split (planar) float arrays (2 <= log_n <= 14)."""
    check(lib().ferrum_fft_1d_c2c_pow2_split(dev.ptr, in_re, in_im, out_re, out_im, log_n, batch,
                                             _dir(direction), int(bool(normalize)), stream))


def cmul_interleaved(dev: DeviceHandle, a: int, b: int, out: int, n: int, stream: int = 0) -> None:
    check(lib().ferrum_cmul_interleaved(dev.ptr, a, b, out, n, stream))


def cmul_split(dev: DeviceHandle, a_re: int, a_im: int, b_re: int, b_im: int, out_re: int,
               out_im: int, n: int, stream: int = 0) -> None:
    check(lib().ferrum_cmul_split(dev.ptr, a_re, a_im, b_re, b_im, out_re, out_im, n, stream))


def deinterleave(dev: DeviceHandle, inp: int, out_re: int, out_im: int, n: int,
                 stream: int = 0) -> None:
    check(lib().ferrum_deinterleave(dev.ptr, inp, out_re, out_im, n, stream))


def interleave(dev: DeviceHandle, re: int, im: int, out: int, n: int, stream: int = 0) -> None:
    check(lib().ferrum_interleave(dev.ptr, re, im, out, n, stream))


class Module:
    """A loaded kernel module (PTX text or a cubin / fatbin image)."""

    def __init__(self, dev: DeviceHandle, image: bytes):
        if isinstance(image, str):
            image = image.encode()
        if not image.endswith(b"\0") and image[:4] != b"\x7fELF":
            image = image + b"\0"   # PTX text is read up to its NUL
        self._image = image
        h = _vp()
        check(lib().ferrum_module_load(dev.ptr, image, ctypes.byref(h)))
        self.ptr = h
        self.dev = dev

    def kernel(self, name: str) -> int:
        k = _vp()
        check(lib().ferrum_module_kernel(self.ptr, name.encode(), ctypes.byref(k)))
        return k.value

    def launch(self, kernel: int, grid, block, args, shared_bytes: int = 0,
               stream: int = 0) -> None:
        """`args`: ctypes values (c_void_p, c_int, c_float, ...) in kernel order."""
        g = (ctypes.c_uint * 3)(*(tuple(grid) + (1,) * (3 - len(grid))))
        b = (ctypes.c_uint * 3)(*(tuple(block) + (1,) * (3 - len(block))))
        ptrs = (_vp * len(args))(*(ctypes.cast(ctypes.pointer(a), _vp) for a in args))
        check(lib().ferrum_launch(self.dev.ptr, kernel, g, b, shared_bytes, ptrs, stream))

    def close(self) -> None:
        if getattr(self, "ptr", None) and self.ptr.value:
            lib().ferrum_module_unload(self.ptr)
            self.ptr = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def workspace_bytes(log_n: int, batch: int, kind: int = 1) -> int:
    out = _sz()
    check(lib().ferrum_fft_workspace_bytes(log_n, batch, kind, ctypes.byref(out)))
    return out.value


def launch_count(log_n: int, batch: int, kind: int = 1) -> int:
    out = _i()
    check(lib().ferrum_fft_launch_count(log_n, batch, kind, ctypes.byref(out)))
    return out.value
