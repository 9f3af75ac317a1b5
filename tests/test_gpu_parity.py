"""GPU parity of the reference API (C ABI) against the CPU oracle: bit-exact
fp16 outputs and int32 accumulators, every variant, odd shapes, K tails,
special scales and all 256 weight codes."""
import ctypes

import numpy as np
import pytest
import torch

import fp8imma_b200 as F
from helpers import bits_equal, cabi_ref_launch, guards_intact, ptr, stream_ptr, to_np_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REF_FUNCS = {
    "v2": "fp8imma_launch_imma_fp8_jit_v2",
    "v2_i8lut": "fp8imma_launch_imma_fp8_jit_v2_i8lut",
    "v3_f16": "fp8imma_launch_imma_fp8_actquant_v3_f16",
    "v3_bf16": "fp8imma_launch_imma_fp8_actquant_v3_bf16",
    "v4_f16": "fp8imma_launch_imma_fp8_actquant_v4_f16",
    "v4_bf16": "fp8imma_launch_imma_fp8_actquant_v4_bf16",
}


def np_inputs(variant, M, N, K, seed=0, scale_mode="normal", codes="uniform"):
    rng = np.random.default_rng(seed)
    if variant.startswith("v2"):
        A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    elif variant.endswith("bf16"):
        a = (rng.standard_normal((M, K)) * 1.5).astype(np.float32)
        A = (a.view(np.uint32) >> 16).astype(np.uint16)  # truncation is a valid bf16 bit pattern
    else:
        A = (rng.standard_normal((M, K)) * 1.5).astype(np.float16).view(np.uint16)
    if codes == "uniform":
        B = rng.integers(0, 256, (N, K), dtype=np.uint8)
    else:
        B = np.tile(np.arange(256, dtype=np.uint8), (N, (K + 255) // 256))[:, :K].copy()
        for n in range(N):
            B[n] = np.roll(B[n], n)
    if scale_mode == "normal":
        s = rng.uniform(0.25, 4.0, N).astype(np.float16)
    elif scale_mode == "special":
        pool = np.array([0.0, 1e-9, 3e-5, 6e-5, 1e-3, 0.02, 0.5, 1.0, 3.5, 64.0, 1000.0, -2.0, -0.3,
                         np.inf, -np.inf, np.nan], np.float32)
        s = pool[rng.integers(0, len(pool), N)].astype(np.float16)
    else:
        raise ValueError(scale_mode)
    return A, B, s.view(np.uint16)


def to_dev(A, B, s, variant):
    dA = torch.from_numpy(A.view(np.int8) if variant.startswith("v2") else A.view(np.int16)).cuda()
    return dA, torch.from_numpy(B).cuda(), torch.from_numpy(s.view(np.int16)).cuda()


def run_case(variant, M, N, K, seed=0, scale_mode="normal", codes="uniform", kchunk=32, gs=0.37, ainv=9.5):
    A, B, s = np_inputs(variant, M, N, K, seed, scale_mode, codes)
    err_o, D_o, _ = O.imma_fp8(variant, kchunk, A, B, s, gs, ainv, nthreads=8)
    assert err_o == 0
    dA, dB, ds = to_dev(A, B, s, variant)
    name = REF_FUNCS[variant]
    err, D = cabi_ref_launch(name, kchunk, dA, dB, ds, M, N, K, gs, None if variant.startswith("v2") else ainv)
    assert err == 0
    torch.cuda.synchronize()
    eq = bits_equal(to_np_bits(D), D_o)
    assert eq.all(), "%s M=%d N=%d K=%d: %d / %d mismatches" % (variant, M, N, K, (~eq).sum(), eq.size)
    assert guards_intact(D), "writes outside the output"


@pytest.mark.parametrize("variant", list(REF_FUNCS))
@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (4, 128, 64), (16, 96, 528), (17, 200, 256), (33, 64, 1024),
                                   (64, 130, 128), (65, 16, 48), (128, 256, 512)])
def test_reference_variants_bitexact(cuda, variant, M, N, K):
    run_case(variant, M, N, K, seed=M * 7 + N)


@pytest.mark.parametrize("variant", ["v4_f16", "v4_bf16", "v2"])
def test_all_codes_and_special_scales(cuda, variant):
    run_case(variant, 24, 160, 512, seed=5, scale_mode="special", codes="all")


@pytest.mark.parametrize("variant", ["v4_f16", "v3_f16", "v3_bf16", "v2"])
@pytest.mark.parametrize("K", [8, 24, 40, 100, 4])
def test_k_tails_generic_path(cuda, variant, K):
    if variant.startswith("v2") and K % 4:
        pytest.skip("v2 reads int8 activations in 16-byte vectors")
    run_case(variant, 9, 37, K, seed=K)


@pytest.mark.parametrize("kchunk", [32, 64])
def test_kchunk_values_give_same_result(cuda, kchunk):
    run_case("v4_f16", 16, 256, 1024, seed=11, kchunk=kchunk)


def test_decode_shape_full_size(cuda):
    run_case("v4_f16", 16, 4096, 4096, seed=3)


def test_decode_shape_m1_70b_columns(cuda):
    run_case("v4_bf16", 1, 28672, 1024, seed=4)


@pytest.mark.parametrize("splits", [1, 2, 4, 8])
def test_forced_splitk(cuda, splits):
    L = F.lib()
    assert L.fp8imma_set_splitk(splits) == 0
    try:
        run_case("v4_f16", 8, 512, 2048, seed=splits)
    finally:
        L.fp8imma_set_splitk(0)


def test_invalid_arguments(cuda):
    A, B, s = np_inputs("v4_f16", 16, 16, 16)
    dA, dB, ds = to_dev(A, B, s, "v4_f16")
    err, _ = cabi_ref_launch(REF_FUNCS["v4_f16"], 48, dA, dB, ds, 16, 16, 16, 1.0, 1.0)
    assert err == 1  # cudaErrorInvalidValue, as the reference
    err, _ = cabi_ref_launch(REF_FUNCS["v4_f16"], 32, dA, dB, ds, 0, 16, 16, 1.0, 1.0)
    assert err == 9  # cudaErrorInvalidConfiguration (empty grid in the reference)
    L = F.lib()
    D = torch.empty(16, 16, dtype=torch.float16, device="cuda")
    err = L.fp8imma_launch_imma_fp8_actquant_v4_f16(32, None, ptr(dB), ptr(ds), ptr(D), 16, 16, 16, 1.0, 1.0,
                                                    stream_ptr())
    assert err == 1


def make_texture(ds: torch.Tensor):
    from cuda.bindings import runtime as rt

    res = rt.cudaResourceDesc()
    res.resType = rt.cudaResourceType.cudaResourceTypeLinear
    res.res.linear.devPtr = ds.data_ptr()
    res.res.linear.sizeInBytes = ds.numel() * 2
    err, fmt = rt.cudaCreateChannelDesc(16, 0, 0, 0, rt.cudaChannelFormatKind.cudaChannelFormatKindUnsigned)
    res.res.linear.desc = fmt
    td = rt.cudaTextureDesc()
    td.addressMode = [rt.cudaTextureAddressMode.cudaAddressModeClamp] * 3
    td.filterMode = rt.cudaTextureFilterMode.cudaFilterModePoint
    td.readMode = rt.cudaTextureReadMode.cudaReadModeElementType
    td.normalizedCoords = 0
    err, tex = rt.cudaCreateTextureObject(res, td, None)
    assert err == rt.cudaError_t.cudaSuccess
    return tex


@pytest.mark.parametrize("variant", ["v4_f16", "v4_bf16"])
def test_texscale_variants(cuda, variant):
    from cuda.bindings import runtime as rt

    M, N, K = 16, 200, 512
    A, B, s = np_inputs(variant, M, N, K, seed=21)
    _, D_o, _ = O.imma_fp8(variant, 32, A, B, s, 0.5, 4.0)
    dA, dB, ds = to_dev(A, B, s, variant)
    tex = make_texture(ds)
    try:
        L = F.lib()
        D = torch.empty(N, M, dtype=torch.float16, device="cuda")
        f = getattr(L, "fp8imma_launch_imma_fp8_actquant_v4_texscale_" + variant.split("_")[1])
        err = f(32, ptr(dA), ptr(dB), ctypes.c_void_p(int(tex)), ptr(D), M, N, K, 0.5, 4.0, stream_ptr())
        assert err == 0
        torch.cuda.synchronize()
        assert bits_equal(to_np_bits(D), D_o).all()
    finally:
        rt.cudaDestroyTextureObject(tex)


def test_torch_ext_v4_act_matches_oracle(cuda):
    e = F.ext()
    A, B, s = np_inputs("v4_f16", 32, 256, 512, seed=9)
    _, D_o, _ = O.imma_fp8("v4_f16", 32, A, B, s, 0.25, 16.0)
    dA, dB, ds = to_dev(A, B, s, "v4_f16")
    D = e.imma_fp8_v4_act(dA.view(torch.float16), dB, ds.view(torch.float16), 0.25, 16.0, 64)
    assert D.shape == (256, 32) and D.dtype == torch.float16 and D.is_contiguous()
    assert bits_equal(to_np_bits(D), D_o).all()
    with pytest.raises(RuntimeError, match="multiples of 16"):
        e.imma_fp8_v4_act(dA[:8].view(torch.float16), dB, ds.view(torch.float16), 1.0, 1.0, 32)


def test_torch_ext_uses_current_stream(cuda):
    e = F.ext()
    A, B, s = np_inputs("v4_f16", 16, 128, 256, seed=10)
    _, D_o, _ = O.imma_fp8("v4_f16", 32, A, B, s, 1.0, 8.0)
    dA, dB, ds = to_dev(A, B, s, "v4_f16")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        D = e.imma_fp8_v4_act(dA.view(torch.float16), dB, ds.view(torch.float16), 1.0, 8.0, 32)
    st.synchronize()
    assert bits_equal(to_np_bits(D), D_o).all()
