"""fp8imma on B200 (sm_100a): Python side of the drop-in.

The product is ``libfp8imma.so`` (CUDA kernels + the reference C ABI, see
``include/fp8imma/imma_fp8.h`` and ``fp8imma_ext.h``) and the torch extension
modules ``fp8imma_ext`` / ``fp8wgt_ext`` that call it. This package loads them
(failing loudly when they are missing), exposes a ctypes handle on the C ABI,
and holds the column-parallel multi-GPU wrapper (``sharded``).

There is no CPU fallback: every entry point runs the sm_100a kernels.
"""
from __future__ import annotations

import ctypes
import os
import sys

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))  # cuda-fp8-ampere_b200/
LIB_PATH = os.path.join(PKG_DIR, "libfp8imma.so")

if PKG_DIR not in sys.path:
    sys.path.insert(0, PKG_DIR)

_lib = None

# reference C ABI entry points (include/fp8imma/imma_fp8.h) and extensions
REF_SYMBOLS = [
    "fp8imma_init_fp8_e4m3_lut",
    "fp8imma_launch_imma_fp8_jit_v2",
    "fp8imma_launch_imma_fp8_jit_v2_i8lut",
    "fp8imma_launch_imma_fp8_actquant_v3_f16",
    "fp8imma_launch_imma_fp8_actquant_v3_bf16",
    "fp8imma_launch_imma_fp8_actquant_v4_texscale_f16",
    "fp8imma_launch_imma_fp8_actquant_v4_texscale_bf16",
    "fp8imma_launch_imma_fp8_actquant_v4_f16",
    "fp8imma_launch_imma_fp8_actquant_v4_bf16",
]
EXT_SYMBOLS = [
    "fp8imma_gemm",
    "fp8imma_gemm_host_io",
    "fp8imma_gemm_epilogue",
    "fp8imma_gemm_rowquant_noalloc",
    "fp8imma_gemm_allgather",
    "fp8imma_set_fused_gather",
    "fp8imma_fp8wgt_linear_forward",
    "fp8imma_quantize_weights",
    "fp8imma_set_splitk",
    "fp8imma_set_stream_k",
    "fp8imma_set_small_m_max",
    "fp8imma_last_path",
    "fp8imma_set_pdl",
    "fp8imma_set_decode_kernel",
    "fp8imma_set_wait_limit_ns",
    "fp8imma_set_tc_pair",
    "fp8imma_set_tc_splitk",
    "fp8imma_set_tc_tile_x",
    "fp8imma_set_tc_half_tail",
    "fp8imma_device_error",
    "fp8imma_version",
]


class FP8ImmaGemmArgs(ctypes.Structure):
    """Mirror of ``fp8imma_gemm_args`` (include/fp8imma/fp8imma_ext.h)."""

    _fields_ = [
        ("path", ctypes.c_int), ("a_type", ctypes.c_int), ("b_format", ctypes.c_int),
        ("act_quant", ctypes.c_int), ("out_type", ctypes.c_int), ("out_layout", ctypes.c_int),
        ("M", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int),
        ("A", ctypes.c_void_p), ("B", ctypes.c_void_p), ("col_scales_u16", ctypes.c_void_p),
        ("col_scales_f32", ctypes.c_void_p), ("global_scale", ctypes.c_float),
        ("a_inv_scale", ctypes.c_float), ("D", ctypes.c_void_p), ("acc_out", ctypes.c_void_p),
    ]


def lib() -> ctypes.CDLL:
    """ctypes handle on libfp8imma.so with argument types declared."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError("libfp8imma.so is not built (%s); run cuda-fp8-ampere_b200/build.py" % LIB_PATH)
    L = ctypes.CDLL(LIB_PATH)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.fp8imma_init_fp8_e4m3_lut.restype = None
    L.fp8imma_init_fp8_e4m3_lut.argtypes = []
    for name in ("fp8imma_launch_imma_fp8_jit_v2", "fp8imma_launch_imma_fp8_jit_v2_i8lut"):
        f = getattr(L, name)
        f.restype = I
        f.argtypes = [I, P, P, P, P, I, I, I, F, P]
    for name in REF_SYMBOLS[3:]:
        f = getattr(L, name)
        f.restype = I
        f.argtypes = [I, P, P, P, P, I, I, I, F, F, P]
    L.fp8imma_gemm.restype = I
    L.fp8imma_gemm.argtypes = [ctypes.POINTER(FP8ImmaGemmArgs), P]
    L.fp8imma_gemm_host_io.restype = I
    L.fp8imma_gemm_epilogue.restype = I
    L.fp8imma_gemm_epilogue.argtypes = [ctypes.POINTER(FP8ImmaGemmArgs), P, I, P]
    L.fp8imma_gemm_host_io.argtypes = [ctypes.POINTER(FP8ImmaGemmArgs), P, P, P]
    L.fp8imma_gemm_allgather.restype = I
    L.fp8imma_set_fused_gather.restype = I
    L.fp8imma_set_fused_gather.argtypes = [I]
    L.fp8imma_gemm_allgather.argtypes = [ctypes.POINTER(FP8ImmaGemmArgs), P, P, I, I, ctypes.c_uint, P]
    L.fp8imma_gemm_rowquant_noalloc.restype = I
    L.fp8imma_gemm_rowquant_noalloc.argtypes = [ctypes.POINTER(FP8ImmaGemmArgs), P]
    L.fp8imma_quantize_weights.restype = I
    L.fp8imma_quantize_weights.argtypes = [P, I, I, I, I, P, P, P, P]
    L.fp8imma_fp8wgt_linear_forward.restype = I
    L.fp8imma_fp8wgt_linear_forward.argtypes = [P, P, F, P, I, I, I, P]
    L.fp8imma_set_splitk.restype = I
    L.fp8imma_set_splitk.argtypes = [I]
    L.fp8imma_set_stream_k.restype = I
    L.fp8imma_set_stream_k.argtypes = [I]
    L.fp8imma_set_small_m_max.restype = I
    L.fp8imma_set_small_m_max.argtypes = [I]
    L.fp8imma_set_tc_pair.restype = I
    L.fp8imma_set_tc_pair.argtypes = [I]
    L.fp8imma_set_tc_splitk.restype = I
    L.fp8imma_set_tc_splitk.argtypes = [I]
    L.fp8imma_set_tc_tile_x.restype = I
    L.fp8imma_set_tc_tile_x.argtypes = [I]
    L.fp8imma_set_tc_half_tail.restype = I
    L.fp8imma_set_tc_half_tail.argtypes = [I]
    L.fp8imma_set_pdl.restype = I
    L.fp8imma_set_pdl.argtypes = [I]
    L.fp8imma_set_decode_kernel.restype = I
    L.fp8imma_set_decode_kernel.argtypes = [I]
    L.fp8imma_set_wait_limit_ns.restype = I
    L.fp8imma_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
    L.fp8imma_device_error.restype = ctypes.c_uint
    L.fp8imma_device_error.argtypes = [I]
    L.fp8imma_last_path.restype = I
    L.fp8imma_last_path.argtypes = []
    L.fp8imma_version.restype = ctypes.c_char_p
    L.fp8imma_version.argtypes = []
    _lib = L
    return L


def ext():
    """The compiled torch extension ``fp8imma_ext`` (reference module name)."""
    import torch  # noqa: F401  (loads libtorch before the extension)
    import fp8imma_ext

    return fp8imma_ext


def wgt_ext():
    import torch  # noqa: F401
    import fp8wgt_ext

    return fp8wgt_ext
