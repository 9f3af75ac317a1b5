"""Column-parallel (N-sharded) host logic on CPU ranks (gloo, world size 2
and 3): shard bounds, in-order assembly of the col-major output, equality with
the unsharded result. The local GEMM is the CPU oracle, so no GPU is used."""
import os
import socket

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


def oracle_local(A, B, scales, col_scales_f32, gs, ainv, act_quant, out):
    from oracle import oracle as O

    D, _ = O.gemm_ex(A.numpy().view(np.uint16), B.numpy(), scales.numpy().view(np.uint16),
                     row_quant=(act_quant == "row"), global_scale=gs, a_inv_scale=ainv)
    out.copy_(torch.from_numpy(D.view(np.int16)).view(torch.float16))
    return out


def _worker(rank, world, port, M, N, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float16))
        B = torch.from_numpy(rng.integers(0, 256, (N, K), dtype=np.uint8))
        s = torch.from_numpy(rng.uniform(0.25, 4, N).astype(np.float16))
        n0, n1 = shard_bounds(N, world, rank)
        layer = ColumnParallelFP8Gemm(B[n0:n1], s[n0:n1], N_total=N, local_fn=oracle_local)
        D = layer(A, 0.5, 8.0, "row" if rank >= 0 else "tensor")
        full = oracle_local(A, B, s, None, 0.5, 8.0, "row", torch.empty(N, M, dtype=torch.float16))
        q.put((rank, bool(torch.equal(D.view(torch.int16), full.view(torch.int16)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_column_parallel_gloo(world):
    M, N, K = 8, 96 * world, 64
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=5) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert all(res.values()), res


def test_shard_bounds_cover_exactly():
    for N in (16, 96, 4096, 28672, 100, 4097):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(N, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == N
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0 and a0 <= a1
