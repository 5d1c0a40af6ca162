"""Host-side logic of the distributed 2D path on CPU ranks (gloo, world 2).

No GPU: the communicator-id exchange, slab partitioning and the failure path
(a rank that dies before set-up) run as real processes over gloo. The
distributed data path itself is covered by the CPU emulator
(test_emulator.py::test_distributed_2d_decomposition) and, on GPUs, by
test_gpu_dist.py.
"""

from __future__ import annotations

import os
import socket
import sys
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG_DIR, REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import datetime

    import torch.distributed as dist

    for p in (REPO, PKG_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _worker_exchange(rank, world, port, q):
    dist = _init(rank, world, port)
    from ferrum_gpu import dist as fdist

    made = []

    def make_id():
        made.append(rank)
        return bytes(range(128))

    uid = fdist.exchange_unique_id(make_id)
    q.put((rank, uid == bytes(range(128)), made))
    # each rank owns its slab; reassembly in rank order restores the image
    img = np.arange(16 * 16, dtype=np.float32).reshape(16, 16)
    mine = fdist.split_rows(img, world)[rank]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    q.put((rank, "join", bool(np.array_equal(fdist.join_rows(gathered), img))))
    dist.destroy_process_group()


def test_unique_id_exchange_and_slabs():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_exchange, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2 * world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    exchange = {r: (ok, made) for r, ok, made in results if ok != "join"}
    joins = [ok for r, tag, ok in results if tag == "join"]
    # every rank received rank 0's id, and only rank 0 created one
    assert exchange == {0: (True, [0]), 1: (True, [])}
    assert joins == [True, True]


def _worker_dead_peer(rank, world, port, q):
    dist = _init(rank, world, port, timeout_s=5)
    from ferrum_gpu import dist as fdist

    if rank == 1:
        # This rank fails on the host before communicator set-up and leaves.
        os._exit(3)
    t0 = time.time()
    try:
        fdist.exchange_unique_id(lambda: bytes(128))
        # rank 0 may finish its send before rank 1 exits; a second collective
        # that needs rank 1 must then fail.
        dist.barrier()
        q.put(("no-error", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((type(e).__name__, time.time() - t0))


def test_dead_rank_is_detected_on_host():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_dead_peer, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    kind, elapsed = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert kind != "no-error"
    assert elapsed < 60
    assert procs[1].exitcode == 3


def test_slab_bounds_validation():
    from ferrum_gpu import dist as fdist

    assert fdist.slab_bounds(16384, 8, 3) == (6144, 2048)
    with pytest.raises(ValueError):
        fdist.slab_bounds(16, 3, 0)
    with pytest.raises(ValueError):
        fdist.slab_bounds(4, 8, 0)
