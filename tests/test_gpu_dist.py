"""Distributed 2D FFT on 2..4 GPUs (skipped with fewer than 2).

One process per GPU. The communicator id travels over a gloo process group;
the data path is ferrum_fft_2d_c2c_pow2_dist (row FFTs, NCCL all-to-all,
column FFTs, all-to-all, block gather). Each rank checks its output slab
against the CPU oracle's 2D result (max rel err <= 1e-4), and a forward +
inverse round trip recovers its input slab. NVLS is disabled so that a rank
that fails cannot leave an NVLink multicast object bound.
"""

from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

from conftest import PKG_DIR, REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("distributed tests need at least 2 GPUs", allow_module_level=True)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cases, q):
    import datetime

    import torch
    import torch.distributed as dist

    for p in (REPO, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        torch.cuda.set_device(rank)
        import oracle
        from ferrum_gpu import capi
        from ferrum_gpu import dist as fdist

        dev = capi.DeviceHandle(rank)
        ctx = fdist.Dist2D(dev, timeout_ms=120000)
        results = []
        for log_n in cases:
            n = 1 << log_n
            rng = np.random.default_rng(log_n)
            img = (rng.standard_normal((n, n)) + 1j * rng.standard_normal((n, n))).astype(np.complex64)
            r0, rows = fdist.slab_bounds(n, world, rank)
            slab = torch.from_numpy(np.ascontiguousarray(img[r0:r0 + rows])).cuda()
            out = ctx.fft_2d_tensor(slab, log_n, "forward", False)
            ref = oracle.fft_2d(img, log_n, threads=4)[r0:r0 + rows]
            err = float(np.max(np.abs(out.cpu().numpy() - ref)) / np.max(np.abs(ref)))
            back = ctx.fft_2d_tensor(out, log_n, "inverse", True)
            rt = float((back - slab).abs().max() / slab.abs().max())
            # One-exchange pair: rows -> column slab (forward), column slab ->
            # rows (inverse).
            cols = ctx.fft_2d_tensor(slab, log_n, "forward", False, out_layout="cols")
            ref_full = oracle.fft_2d(img, log_n, threads=4)
            ref_cols = ref_full[:, r0:r0 + rows]
            err_c = float(np.max(np.abs(cols.cpu().numpy() - ref_cols)) / np.max(np.abs(ref_cols)))
            back_c = ctx.fft_2d_tensor(cols, log_n, "inverse", True, in_layout="cols")
            rt_c = float((back_c - slab).abs().max() / slab.abs().max())
            results.append((log_n, max(err, err_c), max(rt, rt_c)))
        ctx.close()
        dev.close()
        dist.destroy_process_group()
        q.put((rank, "ok", results))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_distributed_2d_matches_oracle(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    cases = [6, 10, 12]
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, status, payload in out:
        assert status == "ok", f"rank {rank}: {payload}"
        for log_n, err, rt in payload:
            assert err < 1e-4, (rank, log_n, err)
            assert rt < 1e-4, (rank, log_n, rt)
