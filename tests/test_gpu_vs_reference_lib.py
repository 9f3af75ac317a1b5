"""A/B against the reference library itself (its WMMA kernels compiled for
sm_100a from the reference sources): identical seeded inputs through both
C ABIs must give bit-identical fp16 outputs."""
import ctypes

import numpy as np
import pytest
import torch

import reflib
from helpers import bits_equal, cabi_ref_launch, ptr, stream_ptr, to_np_bits
from test_gpu_parity import REF_FUNCS, np_inputs, to_dev

pytestmark = pytest.mark.gpu


def run_ref(name, kchunk, dA, dB, ds, M, N, K, gs, ainv):
    L = reflib.lib()
    D = torch.full((N, M), float("nan"), dtype=torch.float16, device="cuda")
    f = getattr(L, name)
    if ainv is None:
        err = f(kchunk, ptr(dA), ptr(dB), ptr(ds), ptr(D), M, N, K, float(gs), stream_ptr())
    else:
        err = f(kchunk, ptr(dA), ptr(dB), ptr(ds), ptr(D), M, N, K, float(gs), float(ainv), stream_ptr())
    assert err == 0
    return D


@pytest.fixture(scope="module")
def ref_available(cuda):
    if not reflib.available():
        pytest.skip("reference library not built (make -C oracle ref)")
    # the reference initialises its constant table on the current device once
    torch.cuda.set_device(0)
    reflib.lib().fp8imma_init_fp8_e4m3_lut()
    return True


# v2_i8lut is compared at kChunk=32 only: at 64 the reference leaves half of
# every K chunk of B stale (src/fp8imma/impl/v2_kernels.inl:99-104).
@pytest.mark.parametrize("variant", list(REF_FUNCS))
@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (16, 4096, 4096), (64, 128, 256), (100, 200, 512), (128, 256, 512)])
def test_bitexact_vs_reference_library(ref_available, variant, M, N, K):
    A, B, s = np_inputs(variant, M, N, K, seed=M + K)
    dA, dB, ds = to_dev(A, B, s, variant)
    ainv = None if variant.startswith("v2") else 9.5
    D_ref = run_ref(REF_FUNCS[variant], 32, dA, dB, ds, M, N, K, 0.37, ainv)
    err, D = cabi_ref_launch(REF_FUNCS[variant], 32, dA, dB, ds, M, N, K, 0.37, ainv)
    assert err == 0
    torch.cuda.synchronize()
    eq = bits_equal(to_np_bits(D), to_np_bits(D_ref))
    assert eq.all(), "%d mismatches" % (~eq).sum()


@pytest.mark.parametrize("scale_mode,codes", [("special", "all"), ("normal", "all")])
def test_special_values_vs_reference_library(ref_available, scale_mode, codes):
    variant = "v4_f16"
    M, N, K = 32, 160, 512
    A, B, s = np_inputs(variant, M, N, K, seed=7, scale_mode=scale_mode, codes=codes)
    dA, dB, ds = to_dev(A, B, s, variant)
    D_ref = run_ref(REF_FUNCS[variant], 64, dA, dB, ds, M, N, K, 1.0, 4.0)
    err, D = cabi_ref_launch(REF_FUNCS[variant], 64, dA, dB, ds, M, N, K, 1.0, 4.0)
    torch.cuda.synchronize()
    assert bits_equal(to_np_bits(D), to_np_bits(D_ref)).all()
