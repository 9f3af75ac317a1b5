"""Column-parallel GEMM over NCCL on 2 GPUs (skipped with fewer): every
rank's assembled output equals the single-GPU result bit for bit (the int8
path is exact, so sharding by N cannot change any value)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, N, K, q):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "cuda-fp8-ampere_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import fp8imma_b200 as F
        from fp8imma_b200 import workloads as WL
        from fp8imma_b200.sharded import ColumnParallelFP8Gemm, shard_bounds

        inp = WL.make_inputs(M, N, K, seed=3)  # same seed on every rank -> same full tensors
        n0, n1 = shard_bounds(N, world, rank)
        layer = ColumnParallelFP8Gemm(inp.B[n0:n1], inp.scales_u16[n0:n1], N_total=N)
        D = layer(inp.A, 1.0 / 16, 16.0)
        full, _ = F.ext().imma_fp8_gemm(inp.A, inp.B, inp.scales_u16, None, 1.0 / 16, 16.0, "tensor", "e4m3", "int8",
                                        "float16", "col", False, None)
        torch.cuda.synchronize()
        ok = bool(torch.equal(D.view(torch.int16), full.view(torch.int16)))
        if M <= 64:
            # fused in-kernel gather over NVLink: same bits, several calls in a row
            from fp8imma_b200.sharded import FusedGatherFP8Gemm

            fused = FusedGatherFP8Gemm(inp.B[n0:n1], inp.scales_u16[n0:n1], M)
            L = F.lib()
            # gather kernel, then in the GEMM epilogue, then the kernel again: each
            # form keeps its own counters, so switching between calls is safe
            for mode in (0, 1, 0):
                assert L.fp8imma_set_fused_gather(mode) == 0
                for _ in range(2):
                    Df = fused(inp.A, 1.0 / 16, 16.0)
                    torch.cuda.synchronize()
                    ok = ok and bool(torch.equal(Df.view(torch.int16), full.view(torch.int16)))
            L.fp8imma_set_fused_gather(0)
            ok = ok and L.fp8imma_device_error(0) == 0
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K", [(16, 4096, 4096), (37, 4004, 1024), (300, 2048, 1024)])
def test_column_parallel_nccl_2gpu(cuda, M, N, K):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=5) for _ in range(world))
    assert all(res.values()), res
