"""Multi-process host logic of the data-parallel replicas, on CPU with gloo (world size 2):
sharding, gathering, and failure detection of a replica that leaves between steps."""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import rldx_b200  # noqa: F401
from rldx_b200.replicas import Heartbeat, serve_sharded, shard, shard_bounds


def test_shard_bounds_partition():
    for n in (0, 1, 7, 256):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def test_shard_rejects_ragged_batch():
    with pytest.raises(ValueError):
        shard({"a": torch.zeros(4, 2), "b": torch.zeros(3, 2)}, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker_gather(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        obs = {"vl": torch.arange(7 * 3, dtype=torch.float32).view(7, 3),
               "state": torch.arange(7, dtype=torch.float32).view(7, 1)}
        out = serve_sharded(lambda o: o["vl"].sum(-1, keepdim=True) + o["state"], obs, world, rank)
        if rank == 0:
            q.put(out.tolist())
    finally:
        dist.destroy_process_group()


def test_serve_sharded_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_gather, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    got = torch.tensor(q.get(timeout=5))
    vl = torch.arange(21, dtype=torch.float32).view(7, 3)
    expect = vl.sum(-1, keepdim=True) + torch.arange(7, dtype=torch.float32).view(7, 1)
    assert torch.equal(got, expect)


def _worker_heartbeat(rank, world, port, q):
    store = dist.TCPStore("127.0.0.1", port, world, is_master=(rank == 0),
                          timeout=datetime.timedelta(seconds=30))
    hb = Heartbeat(store, world, rank, timeout_s=1.0)
    if rank == 1:
        return  # the replica leaves between steps (no kernel in flight)
    time.sleep(2.5)
    q.put(hb.dead_peers())


def test_heartbeat_detects_a_replica_that_left():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_heartbeat, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    dead = q.get(timeout=60)
    for p in procs:
        p.join(timeout=60)
    assert dead == [1]
