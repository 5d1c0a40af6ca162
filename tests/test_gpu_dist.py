"""Distributed 2D FFT on 2, 4 and 8 GPUs (each case skipped without enough GPUs).

One process per GPU. The communicator id travels over a gloo process group;
the data path is ferrum_fft_2d_c2c_pow2_dist_layout, run both ways: over peer
memory (the exchange fused into the FFT kernels; the test checks that this
path was taken) and with FERRUM_DIST_P2P=0 over NCCL send/recv. Each rank
checks its output slab against the CPU oracle's 2D result (max rel err <=
1e-4) for every layout pair, and forward + inverse round trips recover its
input slab. NVLS is disabled so that a rank that fails cannot leave an NVLink
multicast object bound.

The barrier test makes one rank's device-side wait run out (its peer never
arrives) and checks that ferrum_dist_sync reports FERRUM_ERR_TIMEOUT; the
waiting kernel returns on its own after the context's timeout. The other rank
learns of the failure on the host (the gloo group) between steps, with no
kernel or collective in flight, and aborts its context instead of meeting
the failed rank again.
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


def _worker(rank, world, port, cases, q, p2p):
    import datetime

    import torch
    import torch.distributed as dist

    for p in (REPO, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["FERRUM_DIST_P2P"] = "1" if p2p else "0"
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
        path = ctx.peer_path
        ctx.close()
        dev.close()
        dist.destroy_process_group()
        q.put((rank, "ok", (path, results)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))


def _spawn(target, world, *args, wait_s: float = 600):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = [q.get(timeout=wait_s) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


def _worker_entry(rank, world, port, cases, p2p, q):
    _worker(rank, world, port, cases, q, p2p)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("p2p", [True, False], ids=["peer", "nccl"])
def test_distributed_2d_matches_oracle(world, p2p):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = _spawn(_worker_entry, world, [6, 10, 12], p2p)
    for rank, status, payload in out:
        assert status == "ok", f"rank {rank}: {payload}"
        path, results = payload
        assert path == (1 if p2p else 0), (rank, path)
        for log_n, err, rt in results:
            assert err < 1e-4, (rank, log_n, err)
            assert rt < 1e-4, (rank, log_n, rt)


def _sampled_rows(n, world, per_rank=2):
    """Output rows checked at 16384^2: `per_rank` rows inside every rank's row slab."""
    b = n // world
    rows = []
    for q in range(world):
        rows += [q * b + (37 * q + 5) % b, q * b + b - 1 - (11 * q) % b][:per_rank]
    return np.array(sorted(set(rows)))


def _worker_16384(rank, world, port, p2p, q):
    """16384^2 on `world` ranks. Each rank makes only its own row slab (seeded
    per rank). The reference for a sample of output rows k is built without
    any rank holding the whole image: each rank forms the column DFT of its
    slab at the sampled frequencies in float64, sum_n1 W_N^(k n1) x[n1, :]
    over its rows, the partial sums are added over the ranks (gloo), and the
    oracle's 1D FFT of each summed row gives output row k of the 2D
    transform (rows first or columns first give the same result)."""
    import datetime

    import torch
    import torch.distributed as dist

    for p in (REPO, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["FERRUM_DIST_P2P"] = "1" if p2p else "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=300))
        torch.cuda.set_device(rank)
        import oracle
        from ferrum_gpu import capi
        from ferrum_gpu import dist as fdist

        log_n = 14
        n = 1 << log_n
        r0, rows = fdist.slab_bounds(n, world, rank)
        rng = np.random.default_rng([log_n, rank])
        slab_h = (rng.standard_normal((rows, n), dtype=np.float32)
                  + 1j * rng.standard_normal((rows, n), dtype=np.float32)).astype(np.complex64)
        ks = _sampled_rows(n, world)
        n1 = np.arange(r0, r0 + rows, dtype=np.float64)
        w = np.exp(-2j * np.pi * np.outer(ks, n1) / n)          # (|S|, rows)
        part = torch.from_numpy(w @ slab_h.astype(np.complex128))  # (|S|, n)
        part = torch.view_as_real(part).contiguous()
        dist.all_reduce(part)
        colsum = torch.view_as_complex(part).numpy().astype(np.complex64)
        ref = oracle.fft_1d(colsum.reshape(-1), log_n, threads=2).reshape(len(ks), n)

        dev = capi.DeviceHandle(rank)
        ctx = fdist.Dist2D(dev, timeout_ms=60000)
        slab = torch.from_numpy(slab_h).cuda()
        errs = []
        out = ctx.fft_2d_tensor(slab, log_n, "forward", False)            # rows -> rows
        mine = [i for i, k in enumerate(ks) if r0 <= k < r0 + rows]
        got = out.cpu().numpy()
        for i in mine:
            errs.append(float(np.max(np.abs(got[ks[i] - r0] - ref[i])) / np.max(np.abs(ref[i]))))
        cols = ctx.fft_2d_tensor(slab, log_n, "forward", False, out_layout="cols")  # rows -> cols
        got_c = cols.cpu().numpy()                                        # (n, rows)
        for i, k in enumerate(ks):
            seg = ref[i, r0:r0 + rows]
            errs.append(float(np.max(np.abs(got_c[k] - seg)) / np.max(np.abs(ref[i]))))
        back = ctx.fft_2d_tensor(cols, log_n, "inverse", True, in_layout="cols")
        rt = float((back - slab).abs().max() / slab.abs().max())
        back_r = ctx.fft_2d_tensor(out, log_n, "inverse", True)
        rt = max(rt, float((back_r - slab).abs().max() / slab.abs().max()))
        path = ctx.peer_path
        ctx.close()
        dev.close()
        dist.destroy_process_group()
        q.put((rank, "ok", (path, len(mine), max(errs), rt)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("p2p", [True, False], ids=["peer", "nccl"])
def test_distributed_2d_16384_sampled(world, p2p):
    """BASELINE config 5 at its full size: sampled output rows (every rank's
    row slab holds some) of the 16384^2 transform against the oracle, both
    output layouts, and the round trips."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = _spawn(_worker_16384, world, p2p, wait_s=900)
    for rank, status, payload in out:
        assert status == "ok", f"rank {rank}: {payload}"
        path, n_mine, err, rt = payload
        assert path == (1 if p2p else 0), (rank, path)
        assert n_mine >= 1, rank
        assert err < 1e-4, (rank, err)
        assert rt < 1e-4, (rank, rt)


def _barrier_worker(rank, world, port, q):
    import datetime
    import faulthandler

    faulthandler.dump_traceback_later(100, exit=True)

    import torch
    import torch.distributed as dist

    for p in (REPO, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["FERRUM_DIST_P2P"] = "1"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        torch.cuda.set_device(rank)
        from ferrum_gpu import capi
        from ferrum_gpu import dist as fdist

        dev = capi.DeviceHandle(rank)
        ctx = fdist.Dist2D(dev, timeout_ms=120000)
        slab = torch.zeros((32, 64), dtype=torch.complex64, device="cuda")
        ctx.fft_2d_tensor(slab, 6)           # sets up the peer path, completes
        ctx.set_timeout(1500)                 # short bound for the barrier waits
        ok_barrier = None
        if ctx.peer_path == 1:
            ctx.barrier()                     # both ranks: met
            ctx.sync()
            ok_barrier = True
        dist.barrier()
        status = None
        if rank == 0 and ctx.peer_path == 1:
            ctx.barrier()                     # rank 1 never arrives
            try:
                ctx.sync()
                status = capi.FERRUM_OK
            except capi.FerrumError as e:
                status = e.status
        dist.barrier()
        path = ctx.peer_path
        if rank != 0:
            ctx.abort()                       # rank 0 failed: do not meet it again
        ctx.close()
        dev.close()
        dist.destroy_process_group()
        q.put((rank, "ok", (path, ok_barrier, status)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))


def test_peer_barrier_timeout_is_reported():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from ferrum_gpu import capi

    out = dict((r, (st, pl)) for r, st, pl in _spawn(_barrier_worker, 2, wait_s=150))
    for rank, (status, payload) in out.items():
        assert status == "ok", f"rank {rank}: {payload}"
    path, ok_barrier, status = out[0][1]
    assert path == 1 and ok_barrier
    assert status == capi.FERRUM_ERR_TIMEOUT
