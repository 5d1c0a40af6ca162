"""Distributed 2D C2C FFT across GPUs (one process per GPU).

New in this build: the reference is single-GPU (every context is
``CudaContext::new(0)``, crates/ferrum-gpu-py/src/lib.rs:261,385). A single
N x N image is split into row slabs of N/P rows, one per rank; each rank
passes its slab to :meth:`Dist2D.fft_2d` and gets its slab of the 2D result
back. The data path (row FFTs, NCCL all-to-all, column FFTs, all-to-all,
block gather) runs in libferrum_fft.so (ferrum_fft_2d_c2c_pow2_dist);
Python only sets up the communicator: rank 0 creates the NCCL unique id and
``torch.distributed`` broadcasts it. On up to 8 ranks whose GPUs can map each
other's memory the library fuses the exchange into the FFT kernels (peer
stores and loads over NVLink, :attr:`Dist2D.peer_path` is 1 after the first
transform); otherwise, or with ``FERRUM_DIST_P2P=0``, NCCL moves the blocks.

Failure handling: communicator set-up, :meth:`Dist2D.sync` and the device-side
peer barriers are bounded by ``timeout_ms``; on expiry the communicator is
aborted and :class:`ferrum_gpu.capi.FerrumError` (status FERRUM_ERR_TIMEOUT)
is raised by the next :meth:`Dist2D.sync`.
A rank that never reaches set-up makes the id broadcast fail after the
process group's own timeout.
"""

from __future__ import annotations

import ctypes
from typing import Callable, Optional, Sequence

from ferrum_gpu import capi


def slab_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s slab of an n x n image."""
    if world < 1 or world & (world - 1):
        raise ValueError(f"world size must be a power of two, got {world}")
    if n % world:
        raise ValueError(f"N = {n} is not divisible by the world size {world}")
    rows = n // world
    return rank * rows, rows


def split_rows(image, world: int) -> list:
    """Row slabs of an (N, N) array, in rank order (views, not copies)."""
    n = image.shape[0]
    return [image[r0:r0 + rows] for r0, rows in (slab_bounds(n, world, r) for r in range(world))]


def join_rows(slabs: Sequence):
    """Inverse of split_rows for numpy arrays or torch tensors."""
    first = slabs[0]
    if hasattr(first, "numpy") and not hasattr(first, "__array_interface__"):
        import torch

        return torch.cat(list(slabs), dim=0)
    import numpy as np

    return np.concatenate(list(slabs), axis=0)


def _layout(name: str) -> int:
    if name == "rows":
        return capi.DIST_ROW_SLAB
    if name == "cols":
        return capi.DIST_COL_SLAB
    raise ValueError(f"layout must be 'rows' or 'cols', got {name!r}")


def split_cols(image, world: int) -> list:
    """Column slabs (N x N/P) of an (N, N) array, in rank order (copies)."""
    n = image.shape[1]
    out = []
    for r in range(world):
        c0, cols = slab_bounds(n, world, r)
        sl = image[:, c0:c0 + cols]
        out.append(sl.contiguous() if hasattr(sl, "contiguous") else sl.copy())
    return out


def exchange_unique_id(make_id: Callable[[], bytes], group=None) -> bytes:
    """Rank 0 calls `make_id()`; every rank returns rank 0's bytes."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    payload = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(payload, src=0, group=group)
    uid = payload[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != capi.DIST_ID_BYTES:
        raise RuntimeError("distributed set-up: malformed communicator id from rank 0")
    return bytes(uid)


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(capi.DIST_ID_BYTES)
    capi.check(capi.lib().ferrum_dist_get_unique_id(buf))
    return buf.raw


class Dist2D:
    """NCCL communicator plus the distributed 2D transform for one rank."""

    def __init__(self, device: "capi.DeviceHandle", group=None, timeout_ms: int = 60000,
                 make_id: Optional[Callable[[], bytes]] = None):
        import torch.distributed as dist

        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device
        uid = exchange_unique_id(make_id or nccl_unique_id, group)
        ctx = ctypes.c_void_p()
        capi.check(capi.lib().ferrum_dist_init(device.ptr, uid, self.world, self.rank,
                                               int(timeout_ms), ctypes.byref(ctx)))
        self.ctx = ctx

    def check_shape(self, log_n: int) -> None:
        capi.check(capi.lib().ferrum_dist_check(log_n, self.world))

    def workspace_bytes(self, log_n: int) -> int:
        out = ctypes.c_size_t()
        capi.check(capi.lib().ferrum_dist_workspace_bytes(self.ctx, log_n, ctypes.byref(out)))
        return out.value

    def fft_2d(self, in_ptr: int, out_ptr: int, log_n: int, direction="forward",
               normalize: bool = False, stream: int = 0, in_layout: str = "rows",
               out_layout: str = "rows") -> None:
        """Enqueue the collective transform. Layout "rows": this rank's
        (N/P) x N row slab; "cols": its N x (N/P) column slab (columns
        [rank*N/P, (rank+1)*N/P) of every row). rows->cols and cols->rows need
        one all-to-all, rows->rows two."""
        capi.check(capi.lib().ferrum_fft_2d_c2c_pow2_dist_layout(
            self.ctx, in_ptr, out_ptr, log_n, capi._dir(direction), int(bool(normalize)),
            _layout(in_layout), _layout(out_layout), stream))

    def fft_2d_tensor(self, slab, log_n: int, direction="forward", normalize: bool = False,
                      out=None, in_layout: str = "rows", out_layout: str = "rows"):
        """Torch convenience: `slab` is this rank's contiguous complex64 CUDA
        tensor in `in_layout`. Returns `out` (a new tensor in `out_layout` by
        default) after the collective has completed on the current stream."""
        import torch

        n = 1 << log_n
        _, rows = slab_bounds(n, self.world, self.rank)
        shape = {"rows": (rows, n), "cols": (n, rows)}
        if (tuple(slab.shape) != shape[in_layout] or slab.dtype != torch.complex64
                or not slab.is_cuda):
            raise ValueError(f"slab must be a CUDA complex64 tensor of shape {shape[in_layout]}")
        slab = slab.contiguous()
        if out is None:
            out = torch.empty(shape[out_layout], dtype=torch.complex64, device=slab.device)
        stream = torch.cuda.current_stream().cuda_stream
        self.fft_2d(slab.data_ptr(), out.data_ptr(), log_n, direction, normalize, stream,
                    in_layout, out_layout)
        self.sync(stream)
        return out

    def sync(self, stream: int = 0) -> None:
        capi.check(capi.lib().ferrum_dist_sync(self.ctx, stream))

    def barrier(self, stream: int = 0) -> None:
        """Stream-ordered barrier across the ranks (collective)."""
        capi.check(capi.lib().ferrum_dist_barrier(self.ctx, stream))

    def abort(self) -> None:
        """Abandon the collective without waiting for other ranks (after a
        peer failure learned on the host); close() then frees local state."""
        capi.check(capi.lib().ferrum_dist_abort(self.ctx))

    def set_timeout(self, timeout_ms: int) -> None:
        """Bound for later waits and device-side peer barriers."""
        capi.check(capi.lib().ferrum_dist_set_timeout(self.ctx, int(timeout_ms)))

    @property
    def peer_path(self) -> int:
        """1: exchange over peer memory, 0: NCCL, -1: not decided yet."""
        return int(capi.lib().ferrum_dist_peer_path(self.ctx))

    def close(self) -> None:
        if getattr(self, "ctx", None):
            capi.lib().ferrum_dist_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
