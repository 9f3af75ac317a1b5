"""Shared test helpers: call the library through its C ABI with torch-owned
device buffers, and compare fp16/bf16 bit patterns NaN-aware."""
from __future__ import annotations

import ctypes

import numpy as np
import torch

import fp8imma_b200 as F


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


# Guard bands: an output tensor is the middle of a larger buffer whose first
# and last GUARD elements hold a canary pattern; a kernel that writes outside
# its output (a stray index, a wrong stride) changes them.
GUARD = 4096
CANARY = 0x5A5A
_guards = {}


def guarded(rows: int, cols: int, dtype=torch.float16, device="cuda") -> torch.Tensor:
    """[rows, cols] 16-bit tensor (NaN-filled) between two canary bands."""
    n = rows * cols
    raw = torch.full((n + 2 * GUARD,), CANARY, dtype=torch.int16, device=device)
    body = raw[GUARD:GUARD + n]
    body.fill_(0x7E00 if dtype == torch.float16 else 0x7FC0)  # quiet NaN
    t = body.view(dtype).view(rows, cols)
    _guards[t.data_ptr()] = raw
    return t


def guards_intact(t: torch.Tensor) -> bool:
    raw = _guards.pop(t.data_ptr())
    torch.cuda.synchronize()
    return bool((raw[:GUARD] == CANARY).all()) and bool((raw[-GUARD:] == CANARY).all())


def cabi_ref_launch(name: str, kChunk: int, A, B, scales, M, N, K, gs, ainv=None, D=None):
    """Call a reference-API C entry point; returns (err, D[N,M] fp16). A D
    allocated here sits between guard bands (check with guards_intact)."""
    L = F.lib()
    if D is None:
        D = guarded(N, M, device=A.device)
    f = getattr(L, name)
    if ainv is None:
        err = f(kChunk, ptr(A), ptr(B), ptr(scales), ptr(D), M, N, K, float(gs), stream_ptr())
    else:
        err = f(kChunk, ptr(A), ptr(B), ptr(scales), ptr(D), M, N, K, float(gs), float(ainv), stream_ptr())
    return err, D


def bits_equal(a: np.ndarray, b: np.ndarray, is_bf16: bool = False) -> np.ndarray:
    """Elementwise equality of 16-bit float patterns, all NaNs equal."""
    a = a.view(np.uint16)
    b = b.view(np.uint16)
    if is_bf16:
        na = ((a & 0x7F80) == 0x7F80) & ((a & 0x7F) != 0)
        nb = ((b & 0x7F80) == 0x7F80) & ((b & 0x7F) != 0)
    else:
        na = ((a & 0x7C00) == 0x7C00) & ((a & 0x3FF) != 0)
        nb = ((b & 0x7C00) == 0x7C00) & ((b & 0x3FF) != 0)
    return (a == b) | (na & nb)


def to_np_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
