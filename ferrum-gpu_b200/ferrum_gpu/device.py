"""Device-resident FFT on arrays that already live in GPU memory.

New in this build (the reference's Python API takes and returns numpy arrays
only, crates/ferrum-gpu-py/src/lib.rs:445-588, and copies both ways on every
call). These functions take a torch CUDA tensor, or any object exporting the
CUDA Array Interface (``__cuda_array_interface__``, e.g. CuPy or Numba
arrays) or DLPack (``__dlpack__``), and run the transform in place in HBM with
no host copies:

    out = ferrum_gpu.device.fft_1d_c2c_pow2(x, log_n, "forward")

Arguments mean what they mean in ``ferrum_gpu.fft``: ``log_n`` in [2, 26]
(1D) or [2, 14] (2D), ``direction`` "forward" | "inverse", ``normalize``
scales the inverse by 1/N (1/N^2 for 2D), ``device`` an optional
``ferrum_gpu.cuda.Device``. Input: complex64, C-contiguous, batch * N
elements for 1D, shape (N, N) or (B, N, N) for 2D.

Semantics differ from the numpy API in one way: the call is stream ordered and
returns without waiting. The work is enqueued on ``stream`` (a
``cudaStream_t`` as int, or a torch stream), else on the stream the array
announces (CUDA Array Interface v3), else on torch's current stream for torch
tensors, else on the legacy default stream. ``out`` (same shape and type) may
be given, and may be the input itself; otherwise a torch tensor is allocated
(for torch inputs, and for other inputs when torch is importable).

Errors: the validation messages of ``ferrum_gpu.fft`` as ``ValueError``;
failures of the library as ``ferrum_gpu.capi.FerrumError``.
"""

from __future__ import annotations

import threading
from typing import Any, Optional

from ferrum_gpu import capi

_MAX_LOG_N_1D = 26
_MAX_LOG_N_2D = 14

_handles: dict[int, "capi.DeviceHandle"] = {}
_handles_lock = threading.Lock()


class _View:
    """Pointer, element count, shape, device ordinal and stream of an input."""

    def __init__(self, ptr: int, shape: tuple, ordinal: int, stream: Optional[int],
                 owner: Any, torch_tensor: Any = None):
        self.ptr = ptr
        self.shape = tuple(int(s) for s in shape)
        self.ordinal = ordinal
        self.stream = stream
        self.owner = owner
        self.tensor = torch_tensor
        n = 1
        for s in self.shape:
            n *= s
        self.size = n


def _torch():
    try:
        import torch

        return torch
    except ImportError:  # pragma: no cover - torch is part of this image
        return None


def _is_torch_tensor(x) -> bool:
    torch = _torch()
    return torch is not None and isinstance(x, torch.Tensor)


def _contiguous_strides(shape, itemsize):
    strides, acc = [], itemsize
    for s in reversed(shape):
        strides.append(acc)
        acc *= int(s)
    return tuple(reversed(strides))


def _cai_stream(value) -> Optional[int]:
    # CUDA Array Interface v3: None = no synchronisation requested, 1 = legacy
    # default stream, 2 = per-thread default stream, otherwise a cudaStream_t.
    if value is None:
        return None
    return int(value)


def _view(x, what: str) -> _View:
    if _is_torch_tensor(x):
        torch = _torch()
        if not x.is_cuda:
            raise ValueError(f"{what} must be a CUDA array (got a CPU tensor)")
        if x.dtype != torch.complex64:
            raise ValueError(f"{what} must be complex64, got {x.dtype}")
        if not x.is_contiguous():
            raise ValueError(f"{what} must be C-contiguous")
        return _View(x.data_ptr(), tuple(x.shape), x.device.index, None, x, x)
    cai = getattr(x, "__cuda_array_interface__", None)
    dl_device = getattr(x, "__dlpack_device__", None)
    # DLPack device type 2 is kDLCUDA; host arrays (numpy: type 1) fall through.
    if cai is None and hasattr(x, "__dlpack__") and dl_device is not None and dl_device()[0] == 2:
        torch = _torch()
        if torch is None:
            raise ValueError(f"{what}: DLPack inputs need torch to be importable")
        return _view(torch.from_dlpack(x), what)
    if cai is None:
        raise ValueError(f"{what} must be a CUDA array (torch tensor, __cuda_array_interface__ "
                         "or __dlpack__); use ferrum_gpu.fft for numpy arrays")
    typestr = cai.get("typestr")
    if typestr not in ("<c8", "|c8", "=c8"):
        raise ValueError(f"{what} must be complex64 (typestr '<c8'), got {typestr!r}")
    shape = tuple(cai.get("shape", ()))
    strides = cai.get("strides")
    if strides is not None and tuple(strides) != _contiguous_strides(shape, 8):
        raise ValueError(f"{what} must be C-contiguous")
    if cai.get("mask") is not None:
        raise ValueError(f"{what}: masked arrays are not supported")
    ptr = int(cai["data"][0]) if cai.get("data") else 0
    ordinal = _pointer_ordinal(ptr)
    return _View(ptr, shape, ordinal, _cai_stream(cai.get("stream")), x)


def _pointer_ordinal(ptr: int) -> int:
    """Device ordinal owning `ptr` (0 when it cannot be asked)."""
    if ptr == 0:
        return 0
    try:
        from cuda.bindings import runtime as cudart  # cuda-python
    except ImportError:
        try:
            from cuda import cudart  # older cuda-python layout
        except ImportError:
            return 0
    err, attrs = cudart.cudaPointerGetAttributes(ptr)
    if int(err) != 0:
        return 0
    return int(attrs.device)


def _handle(device, ordinal: int) -> int:
    """ferrum_device* address for `device` (a cuda.Device) or the cached
    per-ordinal handle."""
    if device is not None:
        addr = getattr(device, "handle_address", None)
        if addr is None:
            raise ValueError("device must be a ferrum_gpu.cuda.Device")
        if getattr(device, "ordinal", ordinal) != ordinal:
            raise ValueError(f"array is on cuda:{ordinal}, device is cuda:{device.ordinal}")
        return int(addr)
    with _handles_lock:
        h = _handles.get(ordinal)
        if h is None:
            h = capi.DeviceHandle(ordinal)
            _handles[ordinal] = h
        return h.ptr.value


def _stream_handle(stream, view: _View) -> int:
    if stream is not None:
        return int(getattr(stream, "cuda_stream", stream))
    if view.stream is not None:
        return view.stream
    if view.tensor is not None:
        torch = _torch()
        return int(torch.cuda.current_stream(view.tensor.device).cuda_stream)
    return 0


def _output(view: _View, out, what: str = "out") -> _View:
    if out is not None:
        o = _view(out, what)
        if o.shape != view.shape:
            raise ValueError(f"out shape {list(o.shape)} != input shape {list(view.shape)}")
        if o.ordinal != view.ordinal:
            raise ValueError("out must be on the same device as the input")
        return o
    torch = _torch()
    if torch is None:
        raise ValueError("out= is required when torch is not importable")
    t = torch.empty(view.shape, dtype=torch.complex64, device=f"cuda:{view.ordinal}")
    return _View(t.data_ptr(), view.shape, view.ordinal, None, t, t)


def _check_direction(direction) -> int:
    if direction not in ("forward", "inverse"):
        raise ValueError(f'direction must be \'forward\' or \'inverse\', got "{direction}"')
    return capi.FORWARD if direction == "forward" else capi.INVERSE


def fft_1d_c2c_pow2(arr, log_n: int, direction: str = "forward", normalize: bool = False,
                    device=None, out=None, stream=None):
    """Batched 1D C2C transform of a device array (batch * 2^log_n elements)."""
    if not 2 <= log_n <= _MAX_LOG_N_1D:
        raise ValueError(f"log_n must be in [2, {_MAX_LOG_N_1D}], got {log_n}")
    v = _view(arr, "arr")
    n = 1 << log_n
    if v.size == 0 or v.size % n:
        raise ValueError(f"arr len {v.size} must be a positive multiple of N = {n}")
    d = _check_direction(direction)
    o = _output(v, out)
    s = _stream_handle(stream, v)
    h = _handle(device, v.ordinal)
    capi.check(capi.lib().ferrum_fft_1d_c2c_pow2(h, v.ptr, o.ptr, log_n, v.size // n, d,
                                                 int(bool(normalize)), s))
    return o.owner


def fft_2d_c2c_pow2(arr, log_n: int, direction: str = "forward", normalize: bool = False,
                    device=None, out=None, stream=None):
    """2D C2C transform of a device array of shape (N, N) or (B, N, N)."""
    if not 2 <= log_n <= _MAX_LOG_N_2D:
        raise ValueError(f"2D requires log_n in [2, {_MAX_LOG_N_2D}]; got {log_n}")
    v = _view(arr, "arr")
    n = 1 << log_n
    if len(v.shape) not in (2, 3) or v.shape[-2:] != (n, n) or v.size == 0:
        dims = ", ".join(str(d) for d in v.shape)
        raise ValueError(f"arr shape [{dims}] != ({n}, {n})")
    d = _check_direction(direction)
    o = _output(v, out)
    s = _stream_handle(stream, v)
    h = _handle(device, v.ordinal)
    batch = v.shape[0] if len(v.shape) == 3 else 1
    capi.check(capi.lib().ferrum_fft_2d_c2c_pow2(h, v.ptr, o.ptr, log_n, batch, d,
                                                 int(bool(normalize)), s))
    return o.owner


__all__ = ["fft_1d_c2c_pow2", "fft_2d_c2c_pow2"]
