"""The two forms of the small-M kernel: stream-K (persistent CTAs, an even
share of 64-wide K halves each, partial tiles finished by the last arriving
CTA; forced with fp8imma_set_stream_k(2)) and clusters of K slices (forced
with fp8imma_set_stream_k(0)); the default picks stream-K only where the
cluster form would need more than one wave of CTAs. Shapes are
chosen so that segments start and end on odd halves, tiles have one to many
contributors, the unit count is below the grid size, and the last m-chunk and
column tile are ragged. The int8 path must be bit-exact against the oracle in
both forms; the fp32-accumulating paths (native FP8, fp8wgt) within their
stated tolerances; repeated and graph-replayed calls must give identical bits
(the arrival counters re-arm)."""
import ctypes

import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from helpers import bits_equal, ptr, stream_ptr, to_np_bits
from oracle import oracle as O
from test_gpu_ext import inputs

pytestmark = pytest.mark.gpu

# (32, 8192, 8192): M*K*tiles >= 16M, so activations are quantised once by a pre-pass
SHAPES = [(1, 128, 64), (3, 200, 528), (16, 4096, 4096), (37, 300, 1040), (64, 1000, 8192), (8, 28672, 1024),
          (33, 130, 1088), (2, 8192, 16384), (32, 8192, 8192)]


@pytest.fixture(params=[2, 0], ids=["streamk", "cluster"])
def sk_mode(request, cuda):
    L = F.lib()
    assert L.fp8imma_set_stream_k(request.param) == 0
    L.fp8imma_set_decode_kernel(0)  # these forms, not the balanced decode kernel
    yield request.param
    L.fp8imma_set_decode_kernel(1)
    L.fp8imma_set_stream_k(1)


def run_int8(M, N, K, seed, row_quant=False, a_bf16=False):
    e = F.ext()
    A, B, s, sig = inputs(M, N, K, seed=seed, a_bf16=a_bf16)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.bfloat16 if a_bf16 else torch.float16)
    D, acc = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
                             torch.from_numpy(sig).cuda(), 0.05, 20.0, "row" if row_quant else "tensor", "e4m3",
                             "int8", "float16", "col", True, None)
    torch.cuda.synchronize()
    return A, B, s, sig, D, acc


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_int8_bitexact_both_forms(sk_mode, M, N, K):
    A, B, s, sig, D, acc = run_int8(M, N, K, seed=M * 3 + K)
    assert F.ext().last_path() == 1
    D_o, acc_o = O.gemm_ex(A, B, s, col_scale_f32=sig, global_scale=0.05, a_inv_scale=20.0, nthreads=16)
    assert (acc.cpu().numpy() == acc_o).all(), "int32 accumulators differ"
    assert bits_equal(to_np_bits(D), D_o).all()


@pytest.mark.parametrize("M,N,K", [(5, 384, 2112), (48, 640, 640), (48, 8192, 6144)])
def test_int8_row_quant_bf16_both_forms(sk_mode, M, N, K):
    A, B, s, sig, D, acc = run_int8(M, N, K, seed=7, row_quant=True, a_bf16=True)
    D_o, acc_o = O.gemm_ex(A, B, s, a_bf16=True, row_quant=True, col_scale_f32=sig, global_scale=0.05,
                           a_inv_scale=20.0, nthreads=16)
    assert (acc.cpu().numpy() == acc_o).all()
    assert bits_equal(to_np_bits(D), D_o).all()


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (16, 1000, 1040), (40, 640, 8192)])
def test_native_fp8_both_forms(sk_mode, M, N, K):
    e = F.ext()
    A, B, s, sig = inputs(M, N, K, seed=M + K)
    D_o, _, _ = O.fp8_native(A, B, sig, b_fmt=O.FMT_E4M3FN)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    D, _ = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), None, torch.from_numpy(sig).cuda(), 1.0, 1.0, "row",
                           "e4m3", "fp8", "float16", "col", False, None)
    torch.cuda.synchronize()
    got = D.cpu().float().numpy()
    ref = D_o.view(np.float16).astype(np.float32)
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max() + 1e-6


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (16, 1000, 1040), (64, 256, 8192)])
def test_fp8wgt_both_forms(sk_mode, M, N, K):
    rng = np.random.default_rng(M + N)
    A = rng.standard_normal((M, K)).astype(np.float16)
    B = rng.integers(0, 0x78, (N, K), dtype=np.uint8) | (rng.integers(0, 2, (N, K), dtype=np.uint8) << 7)
    C_o = O.fp8wgt(A.view(np.uint16), B, 0.03, nthreads=16)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.full((M, N), float("nan"), device="cuda")
    assert F.lib().fp8imma_fp8wgt_linear_forward(ptr(dA), ptr(dB), 0.03, ptr(C), M, N, K, stream_ptr()) == 0
    torch.cuda.synchronize()
    C = C.cpu().numpy()
    assert np.abs(C - C_o).max() <= 1e-3 * np.abs(C_o).max()


def test_repeated_and_interleaved_calls_identical(cuda):
    e = F.ext()
    cases = [(16, 4096, 4096), (3, 200, 528), (37, 300, 1040)]
    data = []
    for i, (M, N, K) in enumerate(cases):
        A, B, s, sig = inputs(M, N, K, seed=i)
        data.append((torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16), torch.from_numpy(B).cuda(),
                     torch.from_numpy(s.view(np.int16)).cuda()))
    first = [e.imma_fp8_gemm(a, b, s, None, 0.5, 8.0, "tensor", "e4m3", "int8", "float16", "col", True, None)
             for a, b, s in data]
    for _ in range(4):
        for (a, b, s), (D0, acc0) in zip(data, first):
            D, acc = e.imma_fp8_gemm(a, b, s, None, 0.5, 8.0, "tensor", "e4m3", "int8", "float16", "col", True, None)
            assert torch.equal(acc, acc0) and torch.equal(D.view(torch.int16), D0.view(torch.int16))


def test_graph_replay_streamk(cuda):
    e = F.ext()
    M, N, K = 16, 4096, 4096
    A, B, s, _ = inputs(M, N, K, seed=3)
    a = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    b, sc = torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda()
    outs = [torch.empty(N, M, dtype=torch.float16, device="cuda") for _ in range(3)]
    ref, _ = e.imma_fp8_gemm(a, b, sc, None, 0.5, 8.0, "tensor", "e4m3", "int8", "float16", "col", False, None)
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=st):
        for o in outs:
            e.imma_fp8_gemm(a, b, sc, None, 0.5, 8.0, "tensor", "e4m3", "int8", "float16", "col", False, o)
    for _ in range(3):
        for o in outs:
            o.fill_(0)
        g.replay()
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o.view(torch.int16), ref.view(torch.int16))
