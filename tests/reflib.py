"""ctypes handle on the reference fp8imma library compiled for sm_100a from
the reference sources (oracle/_ref/libfp8imma_ref.so, built by
`make -C oracle ref`). Test and benchmark infrastructure only: it is the
reference implementation being compared against, never the product."""
from __future__ import annotations

import ctypes
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libfp8imma_ref.so")
_ref = None


def available() -> bool:
    return os.path.exists(REF_LIB)


def lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_LIB)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        for name in ("fp8imma_launch_imma_fp8_jit_v2", "fp8imma_launch_imma_fp8_jit_v2_i8lut"):
            getattr(L, name).restype = I
            getattr(L, name).argtypes = [I, P, P, P, P, I, I, I, F, P]
        for name in ("fp8imma_launch_imma_fp8_actquant_v3_f16", "fp8imma_launch_imma_fp8_actquant_v3_bf16",
                     "fp8imma_launch_imma_fp8_actquant_v4_f16", "fp8imma_launch_imma_fp8_actquant_v4_bf16",
                     "fp8imma_launch_imma_fp8_actquant_v4_texscale_f16",
                     "fp8imma_launch_imma_fp8_actquant_v4_texscale_bf16"):
            getattr(L, name).restype = I
            getattr(L, name).argtypes = [I, P, P, P, P, I, I, I, F, F, P]
        L.fp8imma_init_fp8_e4m3_lut.restype = None
        _ref = L
    return _ref
