"""GPU parity of the extension entry point fp8imma_gemm (int8-exact path):
per-row activation quantisation, fp32 column scale, bf16 and row-major
output, E5M2 weights, int32 accumulator export; and the fp8wgt linear."""
import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from helpers import bits_equal, to_np_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def inputs(M, N, K, seed, a_bf16=False, fmt="e4m3"):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((M, K)) * 2.0).astype(np.float32)
    if a_bf16:
        A = (a.view(np.uint32) >> 16).astype(np.uint16)
    else:
        A = a.astype(np.float16).view(np.uint16)
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    sig = np.abs(w).max(axis=1) / (448.0 if fmt == "e4m3" else 57344.0)
    enc = O.e4m3fn_encode if fmt == "e4m3" else O.e5m2_encode
    B = enc(w / sig[:, None])
    s = rng.uniform(0.5, 3.5, N).astype(np.float16).view(np.uint16)
    return A, B, s, sig.astype(np.float32)


@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (16, 4096, 1024), (37, 300, 256), (64, 128, 2048)])
@pytest.mark.parametrize("a_bf16", [False, True])
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("row_quant", [False, True])
def test_gemm_ex_matches_oracle(cuda, M, N, K, a_bf16, fmt, row_quant):
    e = F.ext()
    A, B, s, sig = inputs(M, N, K, seed=M + N + K, a_bf16=a_bf16, fmt=fmt)
    b_fmt = O.FMT_E5M2 if fmt == "e5m2" else O.FMT_E4M3_REF
    D_o, acc_o = O.gemm_ex(A, B, s, a_bf16=a_bf16, b_fmt=b_fmt, row_quant=row_quant, col_scale_f32=sig,
                           global_scale=0.05, a_inv_scale=20.0, out_bf16=a_bf16, out_row_major=a_bf16,
                           nthreads=8)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.bfloat16 if a_bf16 else torch.float16)
    D, acc = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
                             torch.from_numpy(sig).cuda(), 0.05, 20.0, "row" if row_quant else "tensor", fmt, "int8",
                             "bfloat16" if a_bf16 else "float16", "row" if a_bf16 else "col", True, None)
    torch.cuda.synchronize()
    assert (acc.cpu().numpy() == acc_o).all(), "int32 accumulators differ"
    assert bits_equal(to_np_bits(D), D_o, is_bf16=a_bf16).all()


def test_gemm_ex_default_equals_reference_api(cuda):
    e = F.ext()
    A, B, s, _ = inputs(16, 512, 1024, seed=1)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    dB = torch.from_numpy(B).cuda()
    ds = torch.from_numpy(s.view(np.int16)).cuda()
    D1 = e.imma_fp8_v4_act(dA, dB, ds.view(torch.float16), 0.3, 7.0, 32)
    D2, _ = e.imma_fp8_gemm(dA, dB, ds, None, 0.3, 7.0, "tensor", "e4m3", "int8", "float16", "col", False, None)
    assert torch.equal(D1.view(torch.int16), D2.view(torch.int16))


def test_int8_activation_api(cuda):
    e = F.ext()
    rng = np.random.default_rng(4)
    A = rng.integers(-128, 128, (8, 256), dtype=np.int8)
    _, B, s, _ = inputs(8, 64, 256, seed=4)
    D_o, acc_o = O.gemm_ex(A, B, s, global_scale=0.01)
    D, acc = e.imma_fp8_gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(),
                             torch.from_numpy(s.view(np.int16)).cuda(), None, 0.01, 1.0, "tensor", "e4m3", "int8",
                             "float16", "col", True, None)
    assert (acc.cpu().numpy() == acc_o).all()
    assert bits_equal(to_np_bits(D), D_o).all()


@pytest.mark.parametrize("M,N,K", [(16, 64, 64), (32, 256, 512), (64, 128, 1024), (48, 80, 96), (128, 256, 512),
                                   (304, 400, 1024), (1024, 512, 2048)])
def test_fp8wgt_linear(cuda, M, N, K):
    w = F.wgt_ext()
    rng = np.random.default_rng(M * N)
    A = (rng.standard_normal((M, K))).astype(np.float16)
    B = rng.integers(0, 0x78, (N, K), dtype=np.uint8)   # finite codes
    B |= (rng.integers(0, 2, (N, K), dtype=np.uint8) << 7)
    C_o = O.fp8wgt(A.view(np.uint16), B, 0.05)
    C = w.fp8_linear_forward(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), 0.05)
    torch.cuda.synchronize()
    C = C.cpu().numpy()
    assert C.shape == (M, N) and C.dtype == np.float32
    # fp32 accumulation in a different order: relative tolerance on the output scale
    err = np.abs(C - C_o).max() / max(np.abs(C_o).max(), 1e-6)
    assert err < 1e-3, err


@pytest.mark.parametrize("M", [16, 48, 64])
@pytest.mark.parametrize("scale_b", [0.05, -3.0, 0.0, 1e-40, 3e-36, 7.0e4])
def test_fp8wgt_decode_exact_all_codes(cuda, M, scale_b):
    """One-hot activations (A[m,k] = 1 for k == m) make every output a single
    decoded weight plus exact zeros, so the small-M path's decode and the scale
    rounding are checked bit for bit, on both the packed and the scalar decode.
    Columns 0..239 cycle through the 240 finite codes; columns 240..255 hold
    one exponent-15 code each (Inf / NaN) at k = 0 and zeros elsewhere, so row
    0 sees +-Inf or NaN and the other rows 0 * Inf = NaN (NaN against NaN)."""
    w = F.wgt_ext()
    N, K = 256, 256
    A = np.zeros((M, K), np.float16)
    A[np.arange(M), np.arange(M)] = 1.0
    codes = np.arange(256, dtype=np.uint8)
    finite = codes[(codes & 0x78) != 0x78]
    special = codes[(codes & 0x78) == 0x78]
    B = np.zeros((N, K), np.uint8)
    for n in range(240):
        B[n] = np.roll(np.resize(finite, K), n)
    B[240:, 0] = special
    C_o = O.fp8wgt(A.view(np.uint16), B, scale_b)
    C = w.fp8_linear_forward(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), scale_b)
    torch.cuda.synchronize()
    C = C.cpu().numpy()
    nan_o, nan_g = np.isnan(C_o), np.isnan(C)
    assert (nan_o == nan_g).all(), (nan_o != nan_g).sum()
    assert (C.view(np.uint32)[~nan_g] == C_o.view(np.uint32)[~nan_o]).all()


@pytest.mark.parametrize("M,N,K,boff", [(1, 4096, 1024, 0), (5, 200, 528, 0), (40, 300, 256, 0),
                                        (7, 64, 128, 8)])
def test_fp8wgt_cabi_ragged_rows(cuda, M, N, K, boff):
    """The C entry point takes any M (the torch wrapper asks for multiples of
    16 like the reference); boff = 8 gives 8-byte aligned weights, which take
    the unstaged kernel instead of the TMA one."""
    import ctypes
    from helpers import ptr, stream_ptr

    rng = np.random.default_rng(M + K)
    A = rng.standard_normal((M, K)).astype(np.float16)
    B = rng.integers(0, 0x78, (N, K), dtype=np.uint8) | (rng.integers(0, 2, (N, K), dtype=np.uint8) << 7)
    C_o = O.fp8wgt(A.view(np.uint16), B, 0.125)
    dA = torch.from_numpy(A).cuda()
    raw = torch.zeros(N * K + 16, dtype=torch.uint8, device="cuda")
    dB = raw[boff:boff + N * K].view(N, K)
    dB.copy_(torch.from_numpy(B))
    C = torch.full((M, N), float("nan"), device="cuda")
    err = F.lib().fp8imma_fp8wgt_linear_forward(ptr(dA), ptr(dB), 0.125, ptr(C), M, N, K, stream_ptr())
    assert err == 0
    torch.cuda.synchronize()
    C = C.cpu().numpy()
    err = np.abs(C - C_o).max() / max(np.abs(C_o).max(), 1e-6)
    assert err < 1e-3, err


def test_fp8linear_module(cuda):
    import fp8_linear

    rng = np.random.default_rng(0)
    B = torch.from_numpy(rng.integers(0, 0x70, (128, 256), dtype=np.uint8)).cuda()
    mod = fp8_linear.FP8Linear(B, 0.1)
    A = torch.randn(32, 256, device="cuda", dtype=torch.float16)
    out = mod(A)
    C_o = O.fp8wgt(A.cpu().numpy().view(np.uint16), B.cpu().numpy(), 0.1)
    assert np.abs(out.cpu().numpy() - C_o).max() / np.abs(C_o).max() < 1e-3


@pytest.mark.parametrize("M,N,K,pinned", [(16, 4096, 1024, True), (3, 200, 528, True), (256, 512, 512, True),
                                          (16, 256, 512, False), (5, 130, 96, False)])
def test_host_io_entry_matches_device_entry(cuda, M, N, K, pinned):
    """fp8imma_gemm_host_io: host activations in, host result out, on the
    caller's stream; bit-identical to fp8imma_gemm on device buffers. Pinned
    host memory is moved by a kernel through its mapped address, pageable
    memory by the copy engine; on decode shapes, once the stream's pre-pass
    buffer exists (the second call), the decode kernel's pre-pass reads the
    pinned rows and its epilogue writes the pinned result in place. The
    device output buffer receives the result either way."""
    e = F.ext()
    A, B, s, _ = inputs(M, N, K, seed=M + 5)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    dB, ds = torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda()
    D_ref, _ = e.imma_fp8_gemm(dA, dB, ds, None, 0.5, 8.0, "tensor", "e4m3", "int8", "float16", "col", False, None)
    a_host = torch.from_numpy(A.view(np.int16)).view(torch.float16).clone()
    d_host = torch.full((N, M), float("nan"), dtype=torch.float16)
    if pinned:
        a_host, d_host = a_host.pin_memory(), d_host.pin_memory()
    a_stage = torch.zeros(M, K, dtype=torch.float16, device="cuda")
    d_stage = torch.empty(N, M, dtype=torch.float16, device="cuda")
    st = torch.cuda.Stream()
    for _ in range(2):
        d_host.fill_(float("nan"))
        d_stage.fill_(float("nan"))
        with torch.cuda.stream(st):
            e.imma_fp8_gemm(a_stage, dB, ds, None, 0.5, 8.0, "tensor", "e4m3", "int8", "float16", "col", False,
                            d_stage, a_host=a_host, out_host=d_host)
        st.synchronize()
        assert torch.equal(d_host.view(torch.int16), D_ref.cpu().view(torch.int16))
        assert torch.equal(d_stage.view(torch.int16), D_ref.view(torch.int16))
    with pytest.raises(RuntimeError, match="go together"):
        e.imma_fp8_gemm(a_stage, dB, ds, None, 0.5, 8.0, "tensor", "e4m3", "int8", "float16", "col", False, d_stage,
                        a_host=a_host)


def _epilogue_ref(acc, s_u16, sig, gs, bias, act, row_g=None):
    """Same fp32 op order as the kernels: se = cs * g (* sig); v = acc * se;
    v += bias; activation; round to fp16."""
    cs = s_u16.view(np.float16).astype(np.float32)
    g = np.float32(gs) if row_g is None else row_g.astype(np.float32)[None, :]
    se = (cs[:, None] * g).astype(np.float32)
    if sig is not None:
        se = (se * sig.astype(np.float32)[:, None]).astype(np.float32)
    v = (acc.astype(np.float32) * se).astype(np.float32)
    if bias is not None:
        v = (v + bias.astype(np.float32)[:, None]).astype(np.float32)
    v64 = v.astype(np.float64)
    if act == "relu":
        v = np.maximum(v, np.float32(0.0))
    elif act == "gelu":
        v = (0.5 * v64 * (1.0 + np.tanh(0.7978845608 * (v64 + 0.044715 * v64 ** 3)))).astype(np.float32)
    elif act == "silu":
        v = (v64 / (1.0 + np.exp(-v64))).astype(np.float32)
    return v.astype(np.float16)


@pytest.mark.parametrize("M,N,K", [(16, 512, 1024), (37, 300, 256), (300, 640, 512), (128, 1024, 2048)])
@pytest.mark.parametrize("act", ["none", "relu", "gelu", "silu"])
def test_fused_bias_activation_epilogue(cuda, M, N, K, act):
    """fp8imma_gemm_epilogue on the int8-exact path (split-K, tcgen05, split-K
    tcgen05): bias and ReLU are exact in fp32, so bit-exact against the same
    op order on the int32 accumulators; GELU / SiLU use the math library's
    tanhf / expf, within 2 fp16 ulps."""
    e = F.ext()
    A, B, s, sig = inputs(M, N, K, seed=M + N)
    bias = np.random.default_rng(1).standard_normal(N).astype(np.float32) * 0.5
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    D, acc = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
                             torch.from_numpy(sig).cuda(), 0.05, 20.0, "tensor", "e4m3", "int8", "float16", "col", True,
                             None, bias=torch.from_numpy(bias).cuda(), act=act)
    torch.cuda.synchronize()
    acc = acc.cpu().numpy()
    ref = _epilogue_ref(acc, s, sig, np.float32(0.05), bias, act)
    got = D.cpu().numpy()
    if act in ("none", "relu"):
        assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    else:
        g, r = got.astype(np.float32), ref.astype(np.float32)
        ulp = np.abs(r) * 2.0 ** -10 + 2.0 ** -24
        assert (np.abs(g - r) <= 2 * ulp + 1e-6).all()


@pytest.mark.parametrize("M", [16, 300])
def test_fused_epilogue_native_path(cuda, M):
    e = F.ext()
    N, K = 640, 512
    A, B, s, sig = inputs(M, N, K, seed=3)
    bias = np.linspace(-1, 1, N).astype(np.float32)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.float16)
    D0, _ = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), None, torch.from_numpy(sig).cuda(), 1.0, 1.0, "row",
                            "e4m3", "fp8", "float16", "col", False, None)
    D1, _ = e.imma_fp8_gemm(dA, torch.from_numpy(B).cuda(), None, torch.from_numpy(sig).cuda(), 1.0, 1.0, "row",
                            "e4m3", "fp8", "float16", "col", False, None, bias=torch.from_numpy(bias).cuda(), act="relu")
    torch.cuda.synchronize()
    ref = np.maximum(D0.cpu().float().numpy() + bias[:, None], 0.0)
    assert np.abs(D1.cpu().float().numpy() - ref).max() <= 2e-3 * np.abs(ref).max() + 1e-3
