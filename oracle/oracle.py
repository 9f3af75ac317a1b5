"""ctypes/numpy front end of the fp8imma CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this module. It checks (or, for the CPU baseline, stands in for) the
reference fp8imma arithmetic; the product library never calls it.

The C code it wraps (``fp8imma_oracle.c``) restates the reference rounding
chain; each C function cites the reference file:line it follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

VARIANTS = {"v2": 0, "v2_i8lut": 1, "v3_f16": 2, "v3_bf16": 3, "v4_f16": 4, "v4_bf16": 5,
            "v4_texscale_f16": 4, "v4_texscale_bf16": 5}
FMT_E4M3_REF, FMT_E5M2, FMT_E4M3FN = 0, 1, 2
A_F16, A_BF16, A_S8 = 0, 1, 2

_lib = None


def build() -> str:
    """Compile the C oracle (gcc) into oracle/_build/liboracle.so."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "fp8imma_oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [F]
        L.orc_f16_to_f32.restype = F
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_hmul.restype = ctypes.c_uint16
        L.orc_hmul.argtypes = [ctypes.c_uint16, ctypes.c_uint16]
        L.orc_cvt_rni_sat_s8_f16.restype = I
        L.orc_cvt_rni_sat_s8_f16.argtypes = [ctypes.c_uint16]
        L.orc_inv_scale_h.restype = ctypes.c_uint16
        L.orc_inv_scale_h.argtypes = [ctypes.c_uint16]
        L.orc_lut_e4m3_ref.argtypes = [P]
        L.orc_lut_e5m2.argtypes = [P]
        L.orc_f32_to_e4m3fn_sat.restype = ctypes.c_uint8
        L.orc_f32_to_e4m3fn_sat.argtypes = [F]
        L.orc_f32_to_e5m2_sat.restype = ctypes.c_uint8
        L.orc_f32_to_e5m2_sat.argtypes = [F]
        L.orc_e4m3fn_to_f32.restype = F
        L.orc_e4m3fn_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_quant_a.argtypes = [P, I, I, I, I, P, ctypes.c_uint16, P]
        L.orc_transcode_b.argtypes = [P, P, I, I, I, P]
        L.orc_gemm_s8.argtypes = [P, P, I, I, I, I, P, I]
        L.orc_imma_fp8.restype = I
        L.orc_imma_fp8.argtypes = [I, I, P, P, P, P, I, I, I, F, F, P, I]
        L.orc_gemm_ex.restype = I
        L.orc_gemm_ex.argtypes = [I, I, I, P, P, P, P, P, I, I, I, F, F, I, I, P, I]
        L.orc_row_scales.argtypes = [P, I, I, I, P, P, P]
        L.orc_fp8wgt.argtypes = [P, P, F, I, I, I, P, I]
        L.orc_fp8_native.argtypes = [I, P, I, P, P, I, I, I, I, I, P, P, P, I]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _bits16(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint16)


def lut_e4m3_ref() -> np.ndarray:
    out = np.zeros(256, np.uint16)
    lib().orc_lut_e4m3_ref(_p(out))
    return out


def lut_e5m2() -> np.ndarray:
    out = np.zeros(256, np.uint16)
    lib().orc_lut_e5m2(_p(out))
    return out


def f32_to_f16_bits(x: float) -> int:
    return int(lib().orc_f32_to_f16(float(x)))


def cvt_rni_sat_s8_f16(bits: int) -> int:
    return int(lib().orc_cvt_rni_sat_s8_f16(int(bits)))


def hmul_bits(a: int, b: int) -> int:
    return int(lib().orc_hmul(int(a), int(b)))


def inv_scale_bits(scale_bits: int) -> int:
    return int(lib().orc_inv_scale_h(int(scale_bits)))


def _atype(A: np.ndarray, bf16: bool) -> int:
    if A.dtype == np.int8:
        return A_S8
    return A_BF16 if bf16 else A_F16


def imma_fp8(variant: str, kChunk: int, A: np.ndarray, B: np.ndarray, scales_u16: np.ndarray,
             global_scale: float, a_inv_scale: float = 1.0, nthreads: int = 1):
    """Reference launch semantics. A: [M,K] (int8, or fp16 / bf16 as uint16
    bits), B: [N,K] uint8, scales_u16: [N] fp16 bits. Returns (err, D_col[N,M]
    fp16 bits, acc[N,M] int32)."""
    A = np.ascontiguousarray(A)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    s = np.ascontiguousarray(scales_u16).view(np.uint16)
    M, K = A.shape
    N = B.shape[0]
    D = np.zeros((N, M), np.uint16)
    acc = np.zeros((N, M), np.int32)
    err = lib().orc_imma_fp8(VARIANTS[variant], kChunk, _p(A), _p(B), _p(s), _p(D), M, N, K,
                             float(global_scale), float(a_inv_scale), _p(acc), nthreads)
    return err, D, acc


def gemm_ex(A: np.ndarray, B: np.ndarray, scales_u16: np.ndarray, *, a_bf16: bool = False,
            b_fmt: int = FMT_E4M3_REF, row_quant: bool = False, col_scale_f32=None,
            global_scale: float = 1.0, a_inv_scale: float = 1.0, out_bf16: bool = False,
            out_row_major: bool = False, nthreads: int = 1):
    """Extended int8-exact path. Returns (D bits, acc[N,M] int32)."""
    A = np.ascontiguousarray(A)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    s = np.ascontiguousarray(scales_u16).view(np.uint16)
    M, K = A.shape
    N = B.shape[0]
    D = np.zeros((M, N) if out_row_major else (N, M), np.uint16)
    acc = np.zeros((N, M), np.int32)
    cs = None if col_scale_f32 is None else np.ascontiguousarray(col_scale_f32, np.float32)
    lib().orc_gemm_ex(_atype(A, a_bf16), b_fmt, int(row_quant), _p(A), _p(B), _p(s), _p(cs),
                      _p(D), M, N, K, float(global_scale), float(a_inv_scale), int(out_bf16),
                      int(out_row_major), _p(acc), nthreads)
    return D, acc


def row_scales(A: np.ndarray, a_bf16: bool = False):
    A = np.ascontiguousarray(A)
    M, K = A.shape
    inv = np.zeros(M, np.float32)
    invh = np.zeros(M, np.uint16)
    g = np.zeros(M, np.float32)
    lib().orc_row_scales(_p(A), A_BF16 if a_bf16 else A_F16, M, K, _p(inv), _p(invh), _p(g))
    return inv, invh, g


def quant_a(A: np.ndarray, a_inv_bits: int, group: int = 8, a_bf16: bool = False) -> np.ndarray:
    A = np.ascontiguousarray(A)
    M, K = A.shape
    out = np.zeros((M, K), np.int8)
    lib().orc_quant_a(_p(A), _atype(A, a_bf16), M, K, group, None, int(a_inv_bits), _p(out))
    return out


def transcode_b(B: np.ndarray, scales_u16: np.ndarray, fmt: int = FMT_E4M3_REF) -> np.ndarray:
    B = np.ascontiguousarray(B, dtype=np.uint8)
    s = np.ascontiguousarray(scales_u16).view(np.uint16)
    N, K = B.shape
    out = np.zeros((N, K), np.int8)
    lib().orc_transcode_b(_p(B), _p(s), N, K, fmt, _p(out))
    return out


def gemm_s8(Aq: np.ndarray, Bq: np.ndarray, keff: int | None = None, nthreads: int = 1):
    M, K = Aq.shape
    N = Bq.shape[0]
    acc = np.zeros((N, M), np.int32)
    lib().orc_gemm_s8(_p(np.ascontiguousarray(Aq)), _p(np.ascontiguousarray(Bq)), M, N, K,
                      K if keff is None else keff, _p(acc), nthreads)
    return acc


def fp8wgt(A: np.ndarray, B: np.ndarray, scale_b: float, nthreads: int = 4) -> np.ndarray:
    A = _bits16(A)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    M, K = A.shape
    N = B.shape[0]
    C = np.zeros((M, N), np.float32)
    lib().orc_fp8wgt(_p(A), _p(B), float(scale_b), M, N, K, _p(C), nthreads)
    return C


def fp8_native(A: np.ndarray, B: np.ndarray, col_scale_f32, *, b_fmt: int = FMT_E4M3FN,
               a_bf16: bool = False, out_bf16: bool = False, out_row_major: bool = False):
    A = _bits16(A)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    M, K = A.shape
    N = B.shape[0]
    D = np.zeros((M, N) if out_row_major else (N, M), np.uint16)
    Aq = np.zeros((M, K), np.uint8)
    rs = np.zeros(M, np.float32)
    cs = None if col_scale_f32 is None else np.ascontiguousarray(col_scale_f32, np.float32)
    lib().orc_fp8_native(b_fmt, _p(A), A_BF16 if a_bf16 else A_F16, _p(B), _p(cs), M, N, K,
                         int(out_bf16), int(out_row_major), _p(D), _p(Aq), _p(rs), 1)
    return D, Aq, rs


def e4m3fn_encode(x: np.ndarray) -> np.ndarray:
    """Vectorised RNE-satfinite encode to E4M3FN bytes (numpy, exact)."""
    return _encode_fp8(np.asarray(x, np.float32), 3, 7, 448.0)


def e5m2_encode(x: np.ndarray) -> np.ndarray:
    return _encode_fp8(np.asarray(x, np.float32), 2, 15, 57344.0)


def _encode_fp8(x: np.ndarray, mbits: int, bias: int, maxv: float) -> np.ndarray:
    x = x.astype(np.float64)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.minimum(np.abs(x), maxv)
    nan = np.isnan(x)
    a = np.where(nan, 0.0, a)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    # guard log2 rounding at exact powers of two
    e = np.where(np.ldexp(1.0, e.astype(np.int64)) > a, e - 1, e)
    e = np.where(np.ldexp(1.0, (e + 1).astype(np.int64)) <= a, e + 1, e)
    e = np.maximum(e, 1 - bias)
    quantum = np.ldexp(1.0, (e - mbits).astype(np.int64))
    v = np.rint(a / quantum) * quantum  # rint: ties to even
    v = np.minimum(v, maxv)
    with np.errstate(divide="ignore"):
        e2 = np.floor(np.log2(np.where(v > 0, v, 1.0)))
    e2 = np.where(np.ldexp(1.0, e2.astype(np.int64)) > v, e2 - 1, e2)
    sub = e2 < (1 - bias)
    m_sub = np.rint(v / np.ldexp(1.0, 1 - bias - mbits))
    m_norm = np.rint((v / np.ldexp(1.0, e2.astype(np.int64)) - 1.0) * (1 << mbits))
    code = np.where(sub, m_sub, ((e2 + bias).astype(np.int64) << mbits) + m_norm)
    code = np.where(v == 0, 0, code).astype(np.uint8)
    out = sign | code
    return np.where(nan, np.uint8(0x7F), out).astype(np.uint8)


def e4m3fn_decode(b: np.ndarray) -> np.ndarray:
    """E4M3FN bytes -> float32 (OCP semantics: exponent 15 finite except 0x7F/0xFF NaN)."""
    b = np.asarray(b, np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 7
    v = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, e - 7))
    v = np.where((b & 0x7F) == 0x7F, np.nan, v)
    return (s * v).astype(np.float32)


def e5m2_decode(b: np.ndarray) -> np.ndarray:
    """E5M2 bytes -> float32 (fp16 bits b << 8)."""
    return (np.asarray(b, np.uint8).astype(np.uint16) << 8).view(np.float16).astype(np.float32)


def quantize_weights(W: np.ndarray, fmt: str = "e4m3"):
    """Per-column FP8 weight quantiser, restated from the GEMM path's weight
    recipe (finite weights): sigma_n = float32(max(absmax_n, 1e-30) / fmax),
    B = fp8_rne_satfinite(float32(W / sigma_n)) (E4M3FN 448, E5M2 57344, or
    E4M3 clamped at 240, the largest value the reference decode table reads
    as finite; the reference's own benchmark encoder clamps there too,
    src/bench/bench_fp8_quant_cublas.inl:2-38, but is per tensor and
    approximate), step_n = fp16(float32(max |decode(B_n)|) / 127).
    Returns (B uint8 [N,K], sigma float32 [N], step uint16 fp16 bits [N])."""
    W = np.asarray(W, np.float32)
    fmax = {"e4m3": 448.0, "e5m2": 57344.0, "e4m3_ref": 240.0}[fmt]
    amax = np.maximum(np.abs(W).max(axis=1), np.float32(1e-30)).astype(np.float32)
    sigma = (amax / np.float32(fmax)).astype(np.float32)
    x = (W / sigma[:, None]).astype(np.float32)
    if fmt == "e4m3_ref":
        x = np.clip(x, np.float32(-240.0), np.float32(240.0))
    if fmt == "e5m2":
        B = e5m2_encode(x)
        dec = e5m2_decode(B)
    else:
        B = e4m3fn_encode(x)
        dec = e4m3fn_decode(B)
    dmax = np.abs(dec).max(axis=1).astype(np.float32)
    step = (dmax / np.float32(127.0)).astype(np.float16).view(np.uint16)
    return B, sigma, step
