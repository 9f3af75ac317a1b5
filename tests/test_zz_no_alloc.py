"""The allocation-free entry point fp8imma_gemm_rowquant_noalloc.

It exists for callers that may not allocate device memory while they run a
GEMM (runtimes that reserve HBM for their own pool, serving loops that forbid
allocation on the request path, plugin hosts that only pass caller-owned
buffers). Its results must be those of the allocating entry point
fp8imma_gemm with per-row activation quantisation; both are called here
through the C ABI, twice in a row with different shapes, so that values left
in the shared fixed array by the first call cannot leak into the second.
This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from helpers import ptr, stream_ptr, bits_equal, to_np_bits
from oracle import oracle as O
from test_gpu_ext import inputs

pytestmark = pytest.mark.gpu


def make_args(A, B, s16, D, M, N, K, a_bf16, acc=None):
    a = F.FP8ImmaGemmArgs()
    a.path, a.a_type, a.b_format, a.act_quant = 0, 1 if a_bf16 else 0, 0, 1  # int8-exact, per-row quant
    a.out_type, a.out_layout = 0, 0
    a.M, a.N, a.K = M, N, K
    a.A, a.B, a.col_scales_u16 = A.data_ptr(), B.data_ptr(), s16.data_ptr()
    a.col_scales_f32 = None
    a.global_scale, a.a_inv_scale = 1.0, 1.0
    a.D = D.data_ptr()
    a.acc_out = None if acc is None else acc.data_ptr()
    return a


def one_case(M, N, K, a_bf16, seed):
    L = F.lib()
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = (torch.randn(M, K, generator=g, device="cuda") * 3).to(torch.bfloat16 if a_bf16 else torch.float16)
    B = torch.randint(0, 256, (N, K), generator=g, device="cuda", dtype=torch.uint8)
    s16 = (torch.rand(N, generator=g, device="cuda") * 3.5 + 0.25).to(torch.float16).view(torch.int16)
    D_ref = torch.full((N, M), float("nan"), dtype=torch.float16, device="cuda")
    D_new = torch.full((N, M), float("nan"), dtype=torch.float16, device="cuda")
    acc_ref = torch.zeros(N, M, dtype=torch.int32, device="cuda")
    acc_new = torch.zeros(N, M, dtype=torch.int32, device="cuda")
    r = make_args(A, B, s16, D_ref, M, N, K, a_bf16, acc_ref)
    n = make_args(A, B, s16, D_new, M, N, K, a_bf16, acc_new)
    assert L.fp8imma_gemm(ctypes.byref(r), stream_ptr()) == 0
    assert L.fp8imma_gemm_rowquant_noalloc(ctypes.byref(n), stream_ptr()) == 0
    torch.cuda.synchronize()
    assert torch.equal(acc_new, acc_ref)
    assert bits_equal(to_np_bits(D_new), to_np_bits(D_ref)).all()


def test_noalloc_matches_allocating_entry_two_calls(cuda):
    # first call: more rows, so the second call's rows were all written before
    one_case(37, 640, 1024, a_bf16=False, seed=1)
    one_case(16, 4096, 4096, a_bf16=True, seed=2)


def test_noalloc_rejects_too_many_rows(cuda):
    L = F.lib()
    M, N, K = 4097, 16, 16
    A = torch.zeros(M, K, dtype=torch.float16, device="cuda")
    B = torch.zeros(N, K, dtype=torch.uint8, device="cuda")
    s16 = torch.ones(N, dtype=torch.float16, device="cuda").view(torch.int16)
    D = torch.empty(N, M, dtype=torch.float16, device="cuda")
    a = make_args(A, B, s16, D, M, N, K, False)
    assert L.fp8imma_gemm_rowquant_noalloc(ctypes.byref(a), stream_ptr()) == 1  # cudaErrorInvalidValue


@pytest.mark.parametrize("M,N,K", [(65, 96, 256), (1024, 64, 128), (4096, 32, 128), (12, 200, 1000)])
def test_noalloc_matches_oracle(cuda, M, N, K):
    """Against the CPU oracle's per-row quantisation directly (not only against
    the allocating entry): M above the small-M range, where this entry still
    runs the split-K kernel, and K = 1000 (not a multiple of 16: the generic
    kernel)."""
    L = F.lib()
    A, B, s, _ = inputs(M, N, K, seed=M + K)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    dB = torch.from_numpy(B).cuda()
    ds = torch.from_numpy(s.view(np.int16)).cuda()
    D = torch.full((N, M), float("nan"), dtype=torch.float16, device="cuda")
    acc = torch.zeros(N, M, dtype=torch.int32, device="cuda")
    a = make_args(dA, dB, ds, D, M, N, K, False, acc)
    a.global_scale = 0.05
    assert L.fp8imma_gemm_rowquant_noalloc(ctypes.byref(a), stream_ptr()) == 0
    torch.cuda.synchronize()
    D_o, acc_o = O.gemm_ex(A, B, s, row_quant=True, global_scale=0.05, nthreads=16)
    assert (acc.cpu().numpy() == acc_o).all(), "int32 accumulators differ"
    assert bits_equal(to_np_bits(D), D_o).all()
