"""Split-K form of the CTA-pair tcgen05 kernel (mid-size M, where 256 x 256
tiles would leave most CTA pairs idle): every K split writes its raw
accumulators, a second kernel sums them in a fixed order and applies the
epilogue. Forced split counts (including ones that do not divide the K blocks
evenly) and the automatic choice; int8 path bit-exact against the oracle
(fp16/bf16 outputs, both layouts, int32 accumulators), native FP8 and fp8wgt
within their stated tolerances."""
import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from helpers import bits_equal, ptr, stream_ptr, to_np_bits
from oracle import oracle as O
from test_gpu_ext import inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[-1, 1, 3, 5], ids=["auto", "s1", "s3", "s5"])
def tc_splits(request, cuda):
    L = F.lib()
    assert L.fp8imma_set_tc_pair(1) == 0
    assert L.fp8imma_set_tc_splitk(request.param) == 0
    yield request.param
    L.fp8imma_set_tc_splitk(-1)


@pytest.mark.parametrize("M,N,K,a_bf16,row_quant,out_row", [(128, 1024, 2048, False, False, False),
                                                             (200, 640, 1408, True, True, True),
                                                             (65, 384, 1024, False, True, False),
                                                             (512, 512, 2560, True, False, True)])
def test_int8_splitk_bitexact(tc_splits, M, N, K, a_bf16, row_quant, out_row):
    e = F.ext()
    A, B, s, sig = inputs(M, N, K, seed=M + K, a_bf16=a_bf16)
    D_o, acc_o = O.gemm_ex(A, B, s, a_bf16=a_bf16, row_quant=row_quant, col_scale_f32=sig, global_scale=0.05,
                           a_inv_scale=20.0, out_bf16=a_bf16, out_row_major=out_row, nthreads=16)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.bfloat16 if a_bf16 else torch.float16)
    D, acc = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
                             torch.from_numpy(sig).cuda(), 0.05, 20.0, "row" if row_quant else "tensor", "e4m3",
                             "int8", "bfloat16" if a_bf16 else "float16", "row" if out_row else "col", True, None)
    assert e.last_path() == 3
    torch.cuda.synchronize()
    assert (acc.cpu().numpy() == acc_o).all(), "int32 accumulators differ"
    assert bits_equal(to_np_bits(D), D_o, is_bf16=a_bf16).all()


@pytest.mark.parametrize("M,N,K,out_row", [(128, 1024, 2048, False), (300, 512, 1536, True)])
def test_native_splitk(tc_splits, M, N, K, out_row):
    e = F.ext()
    A, B, s, sig = inputs(M, N, K, seed=M + 3)
    D_o, _, _ = O.fp8_native(A, B, sig, b_fmt=O.FMT_E4M3FN, out_row_major=out_row)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    D, _ = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), None, torch.from_numpy(sig).cuda(), 1.0, 1.0, "row",
                           "e4m3", "fp8", "float16", "row" if out_row else "col", False, None)
    assert e.last_path() == 4
    torch.cuda.synchronize()
    got = D.cpu().float().numpy()
    ref = D_o.view(np.float16).astype(np.float32)
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max() + 1e-6


@pytest.mark.parametrize("M,N,K", [(128, 1024, 2048), (96, 640, 512)])
def test_fp8wgt_splitk(tc_splits, M, N, K):
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


def test_splitk_setter_rejects_bad_values(cuda):
    L = F.lib()
    assert L.fp8imma_set_tc_splitk(0) == 1
    assert L.fp8imma_set_tc_splitk(-2) == 1
    assert L.fp8imma_set_tc_splitk(-1) == 0


@pytest.fixture(params=[192, 128, 0], ids=["x192", "x128", "auto"])
def tile_x(request, cuda):
    L = F.lib()
    assert L.fp8imma_set_tc_pair(1) == 0
    assert L.fp8imma_set_tc_tile_x(request.param) == 0
    yield request.param
    L.fp8imma_set_tc_tile_x(0)


@pytest.mark.parametrize("M,N,K,out_row", [(300, 640, 1024, False), (1024, 512, 512, True), (97, 256, 2048, False)])
def test_int8_tile_widths_bitexact(tile_x, M, N, K, out_row):
    """Activation rows per CTA-pair tile (MMA N = 256 / 192 / 128): same
    bits whatever the width, including ragged last tiles."""
    e = F.ext()
    A, B, s, sig = inputs(M, N, K, seed=M * 5 + N)
    D_o, acc_o = O.gemm_ex(A, B, s, col_scale_f32=sig, global_scale=0.05, a_inv_scale=20.0, out_row_major=out_row,
                           nthreads=16)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    D, acc = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
                             torch.from_numpy(sig).cuda(), 0.05, 20.0, "tensor", "e4m3", "int8", "float16",
                             "row" if out_row else "col", True, None)
    assert e.last_path() == 3
    torch.cuda.synchronize()
    assert (acc.cpu().numpy() == acc_o).all()
    assert bits_equal(to_np_bits(D), D_o).all()


def test_native_and_fp8wgt_tile_widths(tile_x):
    e = F.ext()
    M, N, K = 513, 384, 768
    A, B, s, sig = inputs(M, N, K, seed=7)
    D_o, _, _ = O.fp8_native(A, B, sig, b_fmt=O.FMT_E4M3FN)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    D, _ = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), None, torch.from_numpy(sig).cuda(), 1.0, 1.0, "row",
                           "e4m3", "fp8", "float16", "col", False, None)
    torch.cuda.synchronize()
    got, ref = D.cpu().float().numpy(), D_o.view(np.float16).astype(np.float32)
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max() + 1e-6
    rng = np.random.default_rng(3)
    Aw = rng.standard_normal((256, 512)).astype(np.float16)
    Bw = rng.integers(0, 0x78, (512, 512), dtype=np.uint8)
    C_o = O.fp8wgt(Aw.view(np.uint16), Bw, 0.03, nthreads=16)
    C = F.wgt_ext().fp8_linear_forward(torch.from_numpy(Aw).cuda(), torch.from_numpy(Bw).cuda(), 0.03)
    torch.cuda.synchronize()
    C = C.cpu().numpy()
    assert np.abs(C - C_o).max() <= 1e-3 * np.abs(C_o).max()


@pytest.mark.parametrize("half_tail", [1, 0])
@pytest.mark.parametrize("M,N,K,fmt", [(2560, 2048, 256, "e4m3"), (2304, 2560, 384, "e5m2")])
def test_int8_half_width_tail_bitexact(cuda, half_tail, M, N, K, fmt):
    """More tiles than CTA pairs with a short last round (80 tiles on 74
    pairs): its tiles run as two half-width items each; bit-exact either way."""
    L = F.lib()
    assert L.fp8imma_set_tc_pair(1) == 0 and L.fp8imma_set_tc_half_tail(half_tail) == 0
    try:
        e = F.ext()
        A, B, s, sig = inputs(M, N, K, seed=M + N, fmt=fmt)
        b_fmt = O.FMT_E5M2 if fmt == "e5m2" else O.FMT_E4M3_REF
        D_o, acc_o = O.gemm_ex(A, B, s, b_fmt=b_fmt, col_scale_f32=sig, global_scale=0.05, a_inv_scale=20.0,
                               nthreads=16)
        dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
        D, acc = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
                                 torch.from_numpy(sig).cuda(), 0.05, 20.0, "tensor", fmt, "int8", "float16", "col",
                                 True, None)
        torch.cuda.synchronize()
        assert (acc.cpu().numpy() == acc_o).all()
        assert bits_equal(to_np_bits(D), D_o).all()
        D_o, _, _ = O.fp8_native(A, B, sig, b_fmt=O.FMT_E5M2 if fmt == "e5m2" else O.FMT_E4M3FN)
        D, _ = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), None, torch.from_numpy(sig).cuda(), 1.0, 1.0, "row",
                               fmt, "fp8", "float16", "col", False, None)
        torch.cuda.synchronize()
        got, ref = D.cpu().float().numpy(), D_o.view(np.float16).astype(np.float32)
        assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max() + 1e-6
    finally:
        L.fp8imma_set_tc_half_tail(1)
