"""Failure handling of the multi-rank host logic on CPU ranks (gloo), made on
the host as the multi-GPU path would meet it: a shard layout the gather cannot
assemble is refused before any collective, a rank that never joins makes the
others' rendezvous end with an error instead of a hang, and a rank that dies
between steps makes the survivors' next collective end with an error within
the process group's timeout."""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fp8imma_b200.sharded import ColumnParallelFP8Gemm, shard_bounds


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _uneven_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        N, K = 100, 32  # 100 columns over 3 ranks: not an even split
        B = torch.zeros(N // world, K, dtype=torch.uint8)
        s = torch.ones(N // world, dtype=torch.float16)
        try:
            ColumnParallelFP8Gemm(B, s, N_total=N, local_fn=lambda *a: None)
            q.put((rank, "no error"))
        except ValueError as e:
            q.put((rank, "ValueError: %s" % e))
    finally:
        dist.destroy_process_group()


def test_uneven_shard_is_refused_before_any_collective():
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_uneven_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=5) for _ in range(world))
    assert all(v.startswith("ValueError") for v in res.values()), res
    assert all(p.exitcode == 0 for p in procs)


def _lonely_worker(port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        q.put(("joined", time.time() - t0))
        dist.destroy_process_group()
    except Exception as e:  # the store rendezvous times out: rank 1 never came
        q.put((type(e).__name__, time.time() - t0))


def test_rank_that_never_joins_ends_rendezvous_with_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_worker, args=(_free_port(), q))
    p.start()
    p.join(timeout=120)
    assert p.exitcode == 0
    kind, dt = q.get(timeout=5)
    assert kind != "joined"
    assert dt < 60


def _dying_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # a timeout long enough for both ranks to start on a loaded machine; the
    # survivor learns of the dead peer from its closed connection, not from it
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    M, N, K = 4, 32 * world, 32
    rng = np.random.default_rng(0)
    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float16))
    B = torch.from_numpy(rng.integers(0, 0x78, (N, K), dtype=np.uint8))
    s = torch.from_numpy(rng.uniform(0.5, 2, N).astype(np.float16))
    n0, n1 = shard_bounds(N, world, rank)

    def local(A_, B_, s_, cs, gs, ainv, aq, out):
        out.zero_()
        return out

    layer = ColumnParallelFP8Gemm(B[n0:n1], s[n0:n1], N_total=N, local_fn=local)
    layer(A, 1.0, 1.0)  # one good step on every rank
    if rank == world - 1:
        os._exit(3)  # leaves between steps, with nothing in flight
    t0 = time.time()
    try:
        layer(A, 1.0, 1.0)
        q.put((rank, "completed", time.time() - t0))
    except Exception as e:
        q.put((rank, type(e).__name__, time.time() - t0))
    # os._exit skips the queue's feeder thread: flush the report first
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_dying_between_steps_fails_the_next_collective():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[-1].exitcode == 3
    rank, kind, dt = q.get(timeout=5)
    assert rank == 0 and kind != "completed", (rank, kind)
    assert dt < 45
