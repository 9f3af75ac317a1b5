"""Parity at the benchmark definition's full-size configurations, where the
tile schedules (half-width tail, split-K, stream-K, the decode kernel's CTA
pairs) differ most from small cases. Checks that do not depend on size: every
output and int32 accumulator of the tensor-core path equals an independent
second kernel (the small-M kernels forced on the same inputs); sampled rows
against the CPU oracle bit for bit (int8 path) or within the native path's
stated tolerance; decode shapes against the oracle in full.

Configurations: prefill up-projection 2048 x 11008 x 4096 with per-row
activation quantisation and bf16 output; square 8192^3 with E4M3 and E5M2
weights on the int8 path and on the native FP8 path; the 70B-style
up-projection K = 8192, N = 28672 at M = 1, 32 and 4096. Inputs are seeded
synthetic tensors with the configurations' distributions."""
import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from fp8imma_b200 import workloads as WL
from helpers import bits_equal, to_np_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TC_PATH = 3
SMALL_M_PATHS = (1, 6)


def _np16(t):
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _two_kernels(A, B, s16, sig, aq, fmt, out_dtype, layout, gs=1.0 / 16, ainv=16.0):
    """The tensor-core result and the small-M kernels' result of one call."""
    e, L = F.ext(), F.lib()
    D_tc, acc_tc = e.imma_fp8_gemm(A, B, s16, sig, gs, ainv, aq, fmt, "int8", out_dtype, layout, True, None)
    assert e.last_path() == TC_PATH
    L.fp8imma_set_small_m_max(1 << 30)
    try:
        D_sk, acc_sk = e.imma_fp8_gemm(A, B, s16, sig, gs, ainv, aq, fmt, "int8", out_dtype, layout, True, None)
        assert e.last_path() in SMALL_M_PATHS
    finally:
        L.fp8imma_set_small_m_max(64)
    torch.cuda.synchronize()
    assert L.fp8imma_device_error(1) == 0
    return D_tc, acc_tc, D_sk, acc_sk


def _oracle_rows(inp, rows, aq, fmt, out_bf16, row_major, sig, gs=1.0 / 16, ainv=16.0):
    a_bf16 = inp.A.dtype == torch.bfloat16
    A_np = _np16(inp.A)[rows]
    D_o, acc_o = O.gemm_ex(A_np, inp.B.cpu().numpy(), _np16(inp.scales_u16),
                           a_bf16=a_bf16, b_fmt=O.FMT_E5M2 if fmt == "e5m2" else O.FMT_E4M3_REF,
                           row_quant=aq == "row", col_scale_f32=None if sig is None else sig.cpu().numpy(),
                           global_scale=gs, a_inv_scale=ainv, out_bf16=out_bf16, out_row_major=row_major,
                           nthreads=16)
    return D_o, acc_o


def test_prefill_2048x11008x4096_rowquant_bf16(cuda):
    M, N, K = 2048, 11008, 4096
    inp = WL.make_inputs(M, N, K, dtype=torch.bfloat16, seed=21)
    D_tc, acc_tc, D_sk, acc_sk = _two_kernels(inp.A, inp.B, inp.scales_u16, inp.sigma_c, "row", "e4m3", "bfloat16",
                                              "row")
    assert torch.equal(acc_tc, acc_sk)
    assert torch.equal(D_tc.view(torch.int16), D_sk.view(torch.int16))
    rows = np.random.default_rng(1).choice(M, 12, replace=False)
    D_o, acc_o = _oracle_rows(inp, rows, "row", "e4m3", True, True, inp.sigma_c)
    assert (acc_tc.cpu().numpy()[:, rows] == acc_o).all()
    assert bits_equal(_np16(D_tc)[rows], D_o, is_bf16=True).all()


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_square8192_int8_path(cuda, fmt):
    M = N = K = 8192
    inp = WL.make_inputs(M, N, K, fmt=fmt, dist="uniform4", seed=31)
    D_tc, acc_tc, D_sk, acc_sk = _two_kernels(inp.A, inp.B, inp.scales_u16, None, "tensor", fmt, "float16", "col",
                                              gs=1.0 / 32, ainv=32.0)
    assert torch.equal(acc_tc, acc_sk)
    assert torch.equal(D_tc.view(torch.int16), D_sk.view(torch.int16))
    rows = np.random.default_rng(2).choice(M, 8, replace=False)
    D_o, acc_o = _oracle_rows(inp, rows, "tensor", fmt, False, False, None, gs=1.0 / 32, ainv=32.0)
    assert (acc_tc.cpu().numpy()[:, rows] == acc_o).all()
    assert bits_equal(_np16(D_tc)[:, rows], D_o).all()


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_square8192_native_fp8_path(cuda, fmt):
    """Native path tolerance (as at small sizes): within 2e-3 of the output's
    largest magnitude, against the oracle on the same per-row E4M3 activations
    with exact accumulation, on sampled rows."""
    e = F.ext()
    M = N = K = 8192
    inp = WL.make_inputs(M, N, K, fmt=fmt, dist="uniform4", seed=41)
    D, _ = e.imma_fp8_gemm(inp.A, inp.B, None, inp.sigma_c, 1.0, 1.0, "row", fmt, "fp8", "float16", "col", False,
                           None)
    assert e.last_path() == 4
    torch.cuda.synchronize()
    rows = np.random.default_rng(3).choice(M, 4, replace=False)
    D_o, _, _ = O.fp8_native(_np16(inp.A)[rows], inp.B.cpu().numpy(), inp.sigma_c.cpu().numpy(),
                             b_fmt=O.FMT_E5M2 if fmt == "e5m2" else O.FMT_E4M3FN)
    got = D.cpu().float().numpy()[:, rows]
    ref = D_o.view(np.float16).astype(np.float32)
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max() + 1e-6


@pytest.mark.parametrize("M", [1, 32])
def test_up70b_decode_shapes_full_oracle(cuda, M):
    e = F.ext()
    N, K = 28672, 8192
    inp = WL.make_inputs(M, N, K, sigma_w=0.015, seed=51 + M)
    D, acc = e.imma_fp8_gemm(inp.A, inp.B, inp.scales_u16, None, 1.0 / 16, 16.0, "tensor", "e4m3", "int8",
                             "float16", "col", True, None)
    assert e.last_path() in SMALL_M_PATHS
    torch.cuda.synchronize()
    assert F.lib().fp8imma_device_error(1) == 0
    D_o, acc_o = _oracle_rows(inp, np.arange(M), "tensor", "e4m3", False, False, None)
    assert (acc.cpu().numpy() == acc_o).all()
    assert bits_equal(_np16(D), D_o).all()


def test_up70b_m4096(cuda):
    M, N, K = 4096, 28672, 8192
    inp = WL.make_inputs(M, N, K, sigma_w=0.015, seed=61)
    D_tc, acc_tc, D_sk, acc_sk = _two_kernels(inp.A, inp.B, inp.scales_u16, None, "tensor", "e4m3", "float16", "col")
    assert torch.equal(acc_tc, acc_sk)
    assert torch.equal(D_tc.view(torch.int16), D_sk.view(torch.int16))
    rows = np.random.default_rng(4).choice(M, 4, replace=False)
    D_o, acc_o = _oracle_rows(inp, rows, "tensor", "e4m3", False, False, None)
    assert (acc_tc.cpu().numpy()[:, rows] == acc_o).all()
    assert bits_equal(_np16(D_tc)[:, rows], D_o).all()
