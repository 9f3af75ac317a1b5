"""The balanced decode kernel (one CTA per SM, CTA pairs splitting K; path 6)
must be bit-exact against the CPU oracle on every argument it takes: per-tensor
and per-row activation quantisation, fp16 / bf16 / int8 activations, E4M3 and
E5M2 weights, fp32 column scale, bf16 and row-major output, int32 accumulator
export, fused bias + activation, K tails, N not a multiple of the 8-column
group, one CTA or a CTA pair per cluster, the exact per-byte path (special
scales, all 256 codes); and equal, bit for bit, to the split-K cluster kernel
it replaces, with and without programmatic dependent launch, on repeated and
graph-replayed calls."""
import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from fp8imma_b200 import workloads as WL
from helpers import bits_equal, guarded, guards_intact, to_np_bits
from oracle import oracle as O
from test_gpu_ext import _epilogue_ref, inputs
from test_gpu_parity import run_case

pytestmark = pytest.mark.gpu

DECODE_PATH = 6

# (M, N, K): the 4096^2 decode shapes (7 / 6 groups per CTA pair), a 70B-style
# shard (N = 3584, K = 8192; it fits only with the activation pre-pass of
# M >= 8), K not a multiple of 128 or 64, N not a multiple of 8, fewer groups
# than SMs, K = 128 (no pair: one CTA per cluster), M = 9..15 (rows 8..15
# partly live), 8 groups per CTA (the 17-warp instantiation: N = 9000, one CTA
# per cluster)
SHAPES = [(1, 4096, 4096), (16, 4096, 4096), (4, 4096, 4096), (16, 3584, 8192), (3, 200, 528), (9, 1003, 1040),
          (16, 8, 256), (2, 24, 4160), (12, 7168, 1024), (8, 513, 128), (15, 1200, 2112), (4, 9000, 1024)]


@pytest.fixture
def decode_on(cuda):
    L = F.lib()
    assert L.fp8imma_set_decode_kernel(1) == 0
    yield L
    L.fp8imma_set_decode_kernel(1)
    L.fp8imma_set_pdl(1)


def _gemm(A, B, s, sig, M, N, K, a_bf16=False, fmt="e4m3", row_quant=False, bias=None, act="none"):
    e = F.ext()
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.bfloat16 if a_bf16 else torch.float16)
    kw = {} if bias is None else dict(bias=torch.from_numpy(bias).cuda(), act=act)
    out = guarded(M, N, torch.bfloat16) if a_bf16 else guarded(N, M)  # bf16 tests use the row-major layout
    D, acc = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
                             torch.from_numpy(sig).cuda(), 0.05, 20.0, "row" if row_quant else "tensor", fmt, "int8",
                             "bfloat16" if a_bf16 else "float16", "row" if a_bf16 else "col", True, out, **kw)
    path = e.last_path()
    torch.cuda.synchronize()
    assert guards_intact(out), "writes outside the output"
    return D, acc, path


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("a_bf16,fmt,row_quant", [(False, "e4m3", False), (True, "e5m2", True), (False, "e4m3", True)])
def test_decode_matches_oracle(decode_on, M, N, K, a_bf16, fmt, row_quant):
    A, B, s, sig = inputs(M, N, K, seed=M * 7 + N + K, a_bf16=a_bf16, fmt=fmt)
    D, acc, path = _gemm(A, B, s, sig, M, N, K, a_bf16, fmt, row_quant)
    assert path == DECODE_PATH
    assert decode_on.fp8imma_device_error(1) == 0
    b_fmt = O.FMT_E5M2 if fmt == "e5m2" else O.FMT_E4M3_REF
    D_o, acc_o = O.gemm_ex(A, B, s, a_bf16=a_bf16, b_fmt=b_fmt, row_quant=row_quant, col_scale_f32=sig,
                           global_scale=0.05, a_inv_scale=20.0, out_bf16=a_bf16, out_row_major=a_bf16, nthreads=16)
    assert (acc.cpu().numpy() == acc_o).all(), "int32 accumulators differ"
    assert bits_equal(to_np_bits(D), D_o, is_bf16=a_bf16).all()


@pytest.mark.parametrize("M,N,K", [(8, 256, 512), (16, 1000, 4096)])
def test_decode_int8_activations(decode_on, M, N, K):
    e = F.ext()
    rng = np.random.default_rng(M + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    _, B, s, _ = inputs(M, N, K, seed=K)
    D, acc = e.imma_fp8_gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(),
                             torch.from_numpy(s.view(np.int16)).cuda(), None, 0.01, 1.0, "tensor", "e4m3", "int8",
                             "float16", "col", True, None)
    assert e.last_path() == DECODE_PATH
    torch.cuda.synchronize()
    D_o, acc_o = O.gemm_ex(A, B, s, global_scale=0.01, nthreads=16)
    assert (acc.cpu().numpy() == acc_o).all()
    assert bits_equal(to_np_bits(D), D_o).all()


@pytest.mark.parametrize("act", ["none", "relu", "silu"])
def test_decode_fused_epilogue(decode_on, act):
    M, N, K = 16, 1024, 2048
    A, B, s, sig = inputs(M, N, K, seed=11)
    bias = np.random.default_rng(2).standard_normal(N).astype(np.float32) * 0.5
    D, acc, path = _gemm(A, B, s, sig, M, N, K, bias=bias, act=act)
    assert path == DECODE_PATH
    ref = _epilogue_ref(acc.cpu().numpy(), s, sig, np.float32(0.05), bias, act)
    got = D.cpu().numpy()
    if act in ("none", "relu"):
        assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    else:
        g, r = got.astype(np.float32), ref.astype(np.float32)
        assert (np.abs(g - r) <= 2 * (np.abs(r) * 2.0 ** -10 + 2.0 ** -24) + 1e-6).all()


@pytest.mark.parametrize("variant", ["v4_f16", "v4_bf16", "v2"])
def test_decode_special_scales_all_codes(decode_on, variant):
    """Special column scales (0, 1e-9, +-Inf, NaN, negative, tiny, huge) put
    CTAs on the exact per-byte path; every weight code appears in every column."""
    run_case(variant, 16, 160, 512, seed=9, scale_mode="special", codes="all")
    run_case(variant, 5, 1000, 1024, seed=10, scale_mode="normal", codes="all")


@pytest.mark.parametrize("M", [1, 4, 16])
@pytest.mark.parametrize("pdl", [0, 1])
def test_decode_equals_split_k_kernel_graph_replay(decode_on, M, pdl):
    """Benchmark recipe (E4M3 weights with NaN/Inf-table codes, outlier
    activation channels): the decode kernel equals the split-K cluster kernel
    bit for bit, and three graph replays of ten back-to-back calls each give the
    same bits."""
    L = decode_on
    e = F.ext()
    N = K = 4096
    inp = WL.make_inputs(M, N, K, outlier_frac=0.01, seed=M)
    L.fp8imma_set_pdl(pdl)
    L.fp8imma_set_decode_kernel(0)
    D_ref, acc_ref = e.imma_fp8_gemm(inp.A, inp.B, inp.scales_u16, None, 1.0 / 16, 16.0, "tensor", "e4m3", "int8",
                                     "float16", "col", True, None)
    assert e.last_path() == 1
    L.fp8imma_set_decode_kernel(1)
    outs = [torch.empty(N, M, dtype=torch.float16, device="cuda") for _ in range(10)]
    st = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):  # first call on the capture stream: its scratch exists before capture
        e.imma_fp8_gemm(inp.A, inp.B, inp.scales_u16, None, 1.0 / 16, 16.0, "tensor", "e4m3", "int8", "float16",
                        "col", False, outs[0])
    assert e.last_path() == DECODE_PATH
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=st):
        for o in outs:
            e.imma_fp8_gemm(inp.A, inp.B, inp.scales_u16, None, 1.0 / 16, 16.0, "tensor", "e4m3", "int8", "float16",
                            "col", False, o)
    for _ in range(3):
        for o in outs:
            o.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o.view(torch.int16), D_ref.view(torch.int16))
    assert L.fp8imma_device_error(1) == 0


@pytest.mark.parametrize("M,N,K", [(4, 512, 12288), (16, 1000, 12288)])
def test_decode_rowquant_long_rows(decode_on, M, N, K):
    """Per-row quantisation with rows longer than the pre-pass keeps in
    registers (K > 8192: the rest of the row is read a second time)."""
    A, B, s, sig = inputs(M, N, K, seed=K + M)
    D, acc, path = _gemm(A, B, s, sig, M, N, K, row_quant=True)
    assert path == DECODE_PATH
    D_o, acc_o = O.gemm_ex(A, B, s, row_quant=True, col_scale_f32=sig, global_scale=0.05, a_inv_scale=20.0,
                           nthreads=16)
    assert (acc.cpu().numpy() == acc_o).all()
    assert bits_equal(to_np_bits(D), D_o).all()
