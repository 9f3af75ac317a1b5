"""CPU checks of the drop-in boundary: the shared library loads and exports
every symbol the public headers declare; the torch extension modules import
and carry the reference's entry points. No compute is launched."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for h in ("imma_fp8.h", "fp8imma_ext.h"):
        txt = open(os.path.join(ROOT, "include", "fp8imma", h)).read()
        # C ABI section: extern "C" declarations of fp8imma_* functions
        c_part = txt.split('extern "C" {', 1)[1]
        syms |= set(re.findall(r"^(?:int|void|const char\s*\*)\s+(fp8imma_[a-z0-9_]+)\s*\(", c_part, re.M))
    return sorted(syms)


def test_headers_declare_reference_abi():
    syms = declared_symbols()
    for s in ["fp8imma_init_fp8_e4m3_lut", "fp8imma_launch_imma_fp8_jit_v2", "fp8imma_launch_imma_fp8_jit_v2_i8lut",
              "fp8imma_launch_imma_fp8_actquant_v3_f16", "fp8imma_launch_imma_fp8_actquant_v3_bf16",
              "fp8imma_launch_imma_fp8_actquant_v4_texscale_f16", "fp8imma_launch_imma_fp8_actquant_v4_texscale_bf16",
              "fp8imma_launch_imma_fp8_actquant_v4_f16", "fp8imma_launch_imma_fp8_actquant_v4_bf16"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    import fp8imma_b200 as F

    L = F.lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert b"sm_100a" in L.fp8imma_version()


def test_library_is_sm100a_only():
    import subprocess

    out = subprocess.run(["cuobjdump", "--list-elf", os.path.join(ROOT, "cuda-fp8-ampere_b200", "libfp8imma.so")],
                         capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


def test_torch_extensions_import():
    import fp8imma_b200 as F

    e = F.ext()
    assert hasattr(e, "imma_fp8_v4_act") and hasattr(e, "imma_fp8_gemm")
    w = F.wgt_ext()
    assert hasattr(w, "fp8_linear_forward")
    import fp8_linear

    assert hasattr(fp8_linear, "FP8Linear")


def test_torch_ext_rejects_cpu_tensors():
    import torch

    import fp8imma_b200 as F

    e = F.ext()
    A = torch.zeros(16, 16, dtype=torch.float16)
    B = torch.zeros(16, 16, dtype=torch.uint8)
    s = torch.zeros(16, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="A must be a CUDA tensor"):
        e.imma_fp8_v4_act(A, B, s, 1.0, 1.0, 32)


def test_extension_entries_reject_bad_arguments_before_any_launch():
    """Host-side validation of the extension entry points and tuning knobs:
    these return the CUDA error code without touching a device, so they run
    here."""
    import ctypes

    import fp8imma_b200 as F

    L = F.lib()
    INVALID_VALUE, INVALID_CONFIG = 1, 9
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    assert L.fp8imma_quantize_weights(p, 0, 0, 16, 0, p, None, None, None) == INVALID_CONFIG
    assert L.fp8imma_quantize_weights(None, 0, 4, 16, 0, p, None, None, None) == INVALID_VALUE
    assert L.fp8imma_quantize_weights(p, 3, 4, 16, 0, p, None, None, None) == INVALID_VALUE
    assert L.fp8imma_quantize_weights(p, 0, 4, 16, 3, p, None, None, None) == INVALID_VALUE
    a = F.FP8ImmaGemmArgs()
    assert L.fp8imma_gemm_epilogue(ctypes.byref(a), None, 4, None) == INVALID_VALUE
    assert L.fp8imma_gemm_epilogue(ctypes.byref(a), None, -1, None) == INVALID_VALUE
    assert L.fp8imma_gemm_host_io(ctypes.byref(a), None, None, None) == INVALID_VALUE
    for setter, bad, good in [(L.fp8imma_set_stream_k, 3, 1), (L.fp8imma_set_tc_splitk, 0, -1),
                              (L.fp8imma_set_tc_tile_x, 100, 0), (L.fp8imma_set_fused_gather, 2, 0),
                              (L.fp8imma_set_tc_half_tail, 2, 1), (L.fp8imma_set_splitk, 3, 0)]:
        assert setter(bad) == INVALID_VALUE
        assert setter(good) == 0
