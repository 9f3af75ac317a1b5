"""Bounded waits on one GPU: a wait that runs out ends its kernel with an
error code instead of hanging, the host reads the code, and the context stays
usable. The failure is a flag that nothing sets: the column-parallel gather
is called as rank 0 of a world of 2 whose "peer" is a local buffer pair that
no rank ever signals. The wait limit is lowered to 50 ms for the test and
restored after it. No GPU fault, trap or endless loop is involved."""
import ctypes
import time

import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from helpers import bits_equal, stream_ptr, to_np_bits
from test_gpu_ext import inputs

pytestmark = pytest.mark.gpu

ERR_WAIT_PEER = 5


@pytest.fixture
def short_waits(cuda):
    L = F.lib()
    L.fp8imma_device_error(1)
    assert L.fp8imma_set_wait_limit_ns(50_000_000) == 0
    yield L
    assert L.fp8imma_set_wait_limit_ns(2_000_000_000) == 0
    L.fp8imma_device_error(1)
    L.fp8imma_set_fused_gather(0)


@pytest.mark.parametrize("fused", [0, 1])
def test_unsignalled_peer_times_out_with_error_code(short_waits, fused):
    L = short_waits
    M, N, K = 16, 512, 1024  # this rank's shard: N columns
    A, B, s, _ = inputs(M, N, K, seed=2)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    dB = torch.from_numpy(B).cuda()
    ds = torch.from_numpy(s.view(np.int16)).cuda()
    world, rank = 2, 0
    outs = [torch.full((world * N, M), float("nan"), dtype=torch.float16, device="cuda") for _ in range(world)]
    pads = [torch.zeros(64, dtype=torch.int32, device="cuda") for _ in range(world)]
    a = F.FP8ImmaGemmArgs()
    a.path, a.a_type, a.b_format, a.act_quant, a.out_type, a.out_layout = 0, 0, 0, 0, 0, 0
    a.M, a.N, a.K = M, N, K
    a.A, a.B, a.col_scales_u16, a.col_scales_f32 = dA.data_ptr(), dB.data_ptr(), ds.data_ptr(), None
    a.global_scale, a.a_inv_scale = 0.05, 20.0
    a.D, a.acc_out = None, None
    out_ptrs = (ctypes.c_void_p * world)(*[o.data_ptr() for o in outs])
    pad_ptrs = (ctypes.c_void_p * world)(*[p.data_ptr() for p in pads])
    assert L.fp8imma_set_fused_gather(fused) == 0
    t0 = time.time()
    assert L.fp8imma_gemm_allgather(ctypes.byref(a), out_ptrs, pad_ptrs, world, rank, 0, stream_ptr()) == 0
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert dt < 1.5, "the wait should give up after about 50 ms, took %.2f s" % dt
    assert L.fp8imma_device_error(1) == ERR_WAIT_PEER
    # the context is still usable and this rank's own rows are right
    ref, _ = F.ext().imma_fp8_gemm(dA, dB, ds, None, 0.05, 20.0, "tensor", "e4m3", "int8", "float16", "col", False,
                                   None)
    torch.cuda.synchronize()
    assert bits_equal(to_np_bits(outs[rank][:N]), to_np_bits(ref)).all()
    assert L.fp8imma_device_error(0) == 0
