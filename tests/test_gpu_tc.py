"""GPU parity of the large-M tensor-core path (tcgen05 kind::i8 and
kind::f8f6f4): bit-exact against the CPU oracle on the int8 path (fp16
outputs and int32 accumulators), within a stated tolerance on the native FP8
path, and at full BASELINE sizes through size-independent checks (row slices
against the oracle, agreement with the independent split-K kernel)."""
import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from helpers import bits_equal, to_np_bits
from oracle import oracle as O
from test_gpu_parity import REF_FUNCS, np_inputs, to_dev
from helpers import cabi_ref_launch

pytestmark = pytest.mark.gpu

TC_PATH, NATIVE_PATH, NATIVE_SK_PATH = 3, 4, 5
GEMV_PATHS = (1, 6)  # small-M split-K kernel, balanced decode kernel


@pytest.fixture(params=[1, 0], ids=["pair", "single"])
def tc_mode(request, cuda):
    L = F.lib()
    L.fp8imma_set_tc_pair(request.param)
    yield request.param
    L.fp8imma_set_tc_pair(1)


@pytest.mark.parametrize("variant", ["v4_f16", "v4_bf16", "v3_f16", "v2"])
@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (256, 128, 1024), (300, 200, 256), (513, 384, 2048),
                                   (1024, 1024, 1024), (65, 640, 128)])
def test_tc_reference_api_bitexact(tc_mode, variant, M, N, K):
    L = F.lib()
    A, B, s = np_inputs(variant, M, N, K, seed=M + N + K)
    err_o, D_o, _ = O.imma_fp8(variant, 32, A, B, s, 0.37, 9.5, nthreads=16)
    dA, dB, ds = to_dev(A, B, s, variant)
    err, D = cabi_ref_launch(REF_FUNCS[variant], 32, dA, dB, ds, M, N, K, 0.37,
                             None if variant.startswith("v2") else 9.5)
    assert err == 0
    assert L.fp8imma_last_path() in ((TC_PATH,) if M > 64 else GEMV_PATHS)
    torch.cuda.synchronize()
    assert L.fp8imma_device_error(0) == 0
    eq = bits_equal(to_np_bits(D), D_o)
    assert eq.all(), "%d / %d mismatches" % ((~eq).sum(), eq.size)


def test_tc_special_scales_and_codes(cuda):
    run = np_inputs("v4_f16", 256, 160, 512, seed=3, scale_mode="special", codes="all")
    A, B, s = run
    _, D_o, _ = O.imma_fp8("v4_f16", 32, A, B, s, 1.0, 4.0, nthreads=16)
    dA, dB, ds = to_dev(A, B, s, "v4_f16")
    err, D = cabi_ref_launch(REF_FUNCS["v4_f16"], 32, dA, dB, ds, 256, 160, 512, 1.0, 4.0)
    torch.cuda.synchronize()
    assert err == 0
    assert bits_equal(to_np_bits(D), D_o).all()


@pytest.mark.parametrize("a_bf16,fmt,row_quant,out_row", [(False, "e4m3", False, False), (True, "e4m3", True, True),
                                                           (False, "e5m2", True, False), (True, "e5m2", False, True)])
def test_tc_extended_args_and_accumulators(tc_mode, a_bf16, fmt, row_quant, out_row):
    e = F.ext()
    from test_gpu_ext import inputs

    M, N, K = 320, 384, 768
    A, B, s, sig = inputs(M, N, K, seed=11, a_bf16=a_bf16, fmt=fmt)
    D_o, acc_o = O.gemm_ex(A, B, s, a_bf16=a_bf16, b_fmt=O.FMT_E5M2 if fmt == "e5m2" else O.FMT_E4M3_REF,
                           row_quant=row_quant, col_scale_f32=sig, global_scale=0.05, a_inv_scale=20.0,
                           out_bf16=a_bf16, out_row_major=out_row, nthreads=16)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.bfloat16 if a_bf16 else torch.float16)
    D, acc = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
                             torch.from_numpy(sig).cuda(), 0.05, 20.0, "row" if row_quant else "tensor", fmt, "int8",
                             "bfloat16" if a_bf16 else "float16", "row" if out_row else "col", True, None)
    assert e.last_path() == TC_PATH
    torch.cuda.synchronize()
    assert (acc.cpu().numpy() == acc_o).all()
    assert bits_equal(to_np_bits(D), D_o, is_bf16=a_bf16).all()


def test_tc_full_size_square4096_row_slices_and_splitk_agreement(tc_mode):
    """M=N=K=4096 (square config): every output checked bitwise against the
    independent split-K kernel, and 48 rows against the CPU oracle."""
    from fp8imma_b200 import workloads as WL

    e = F.ext()
    L = F.lib()
    M = N = K = 4096
    inp = WL.make_inputs(M, N, K, dist="uniform4", seed=5)
    gs, ainv = 1.0 / 32.0, 32.0
    D_tc, acc_tc = e.imma_fp8_gemm(inp.A, inp.B, inp.scales_u16, None, gs, ainv, "tensor", "e4m3", "int8", "float16",
                                   "col", True, None)
    assert e.last_path() == TC_PATH
    L.fp8imma_set_small_m_max(1 << 30)
    try:
        D_sk, acc_sk = e.imma_fp8_gemm(inp.A, inp.B, inp.scales_u16, None, gs, ainv, "tensor", "e4m3", "int8",
                                       "float16", "col", True, None)
        assert e.last_path() in GEMV_PATHS
    finally:
        L.fp8imma_set_small_m_max(64)
    torch.cuda.synchronize()
    assert torch.equal(acc_tc, acc_sk)
    assert torch.equal(D_tc.view(torch.int16), D_sk.view(torch.int16))
    rows = np.random.default_rng(0).choice(M, 48, replace=False)
    A_np = inp.A.cpu().view(torch.int16).numpy().view(np.uint16)[rows]
    _, D_o, _ = O.imma_fp8("v4_f16", 32, A_np, inp.B.cpu().numpy(), inp.scales_u16.cpu().numpy().view(np.uint16),
                           gs, ainv, nthreads=16)
    got = to_np_bits(D_tc)[:, rows]
    assert bits_equal(got, D_o).all()


@pytest.mark.parametrize("M,N,K,fmt,a_bf16", [(256, 256, 512, "e4m3", False), (300, 200, 1024, "e5m2", False),
                                               (1024, 512, 2048, "e4m3", True), (64, 384, 256, "e4m3", False),
                                               (1, 4096, 4096, "e4m3", False), (16, 1000, 1024, "e5m2", True),
                                               (33, 640, 512, "e4m3", False)])
def test_native_fp8_matches_oracle(tc_mode, M, N, K, fmt, a_bf16):
    """Native FP8 path tolerance: fp16 outputs within 2e-3 relative (to the
    output's max magnitude) of the oracle, which uses the same quantised
    activations and exact (double) accumulation."""
    e = F.ext()
    from test_gpu_ext import inputs

    A, B, s, sig = inputs(M, N, K, seed=M + K, a_bf16=a_bf16, fmt=fmt)
    D_o, _, _ = O.fp8_native(A, B, sig, b_fmt=O.FMT_E5M2 if fmt == "e5m2" else O.FMT_E4M3FN, a_bf16=a_bf16)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.bfloat16 if a_bf16 else torch.float16)
    D, _ = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), None, torch.from_numpy(sig).cuda(), 1.0, 1.0, "row", fmt,
                           "fp8", "float16", "col", False, None)
    assert e.last_path() == (NATIVE_PATH if M > 64 else NATIVE_SK_PATH)
    torch.cuda.synchronize()
    got = D.cpu().float().numpy()
    ref = D_o.view(np.float16).astype(np.float32)
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 2e-3 * scale + 1e-6


def test_native_fp8_vs_fp32_matmul_of_decoded_weights(cuda):
    """Native path against a plain fp32 torch matmul of the decoded weights
    and unquantised activations: the per-row E4M3 activation quantisation is
    the only approximation; stated tolerance rel-L2 <= 3e-2."""
    from fp8imma_b200 import workloads as WL

    e = F.ext()
    inp = WL.make_inputs(512, 1024, 1024, seed=9)
    D, _ = e.imma_fp8_gemm(inp.A, inp.B, None, inp.sigma_c, 1.0, 1.0, "row", "e4m3", "fp8", "float16", "row", False,
                           None)
    W = inp.B.view(torch.float8_e4m3fn).float() * inp.sigma_c[:, None]
    ref = inp.A.float() @ W.t()
    rel = (D.float() - ref).norm() / ref.norm()
    assert rel.item() < 3e-2, rel.item()
