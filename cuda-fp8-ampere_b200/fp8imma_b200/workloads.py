"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (weights FP8 bytes + per-column scales, fp16/bf16
activations). No dataset is involved; every tensor is generated from a seed.

Weight recipe (all configs): w ~ N(0, sigma_w) in fp32, per-column
sigma_c = absmax_c / 448 (E4M3) or absmax_c / 57344 (E5M2), bytes =
round-to-nearest-even FP8 of w / sigma_c. For the reference API the int8 step
of each column is fp16(max|decoded byte| / 127); its inverse is what the
reference multiplies the decoded byte by before rounding to int8.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class GemmInputs:
    A: torch.Tensor              # [M,K] fp16 / bf16
    B: torch.Tensor              # [N,K] uint8
    scales_u16: torch.Tensor     # [N] fp16 int8-step scales (reference API)
    sigma_c: torch.Tensor        # [N] fp32 per-column weight scale
    b_format: str                # "e4m3" | "e5m2"


def make_weights(N: int, K: int, sigma_w: float = 0.02, fmt: str = "e4m3", seed: int = 0,
                 device: str = "cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn(N, K, generator=g, device=device, dtype=torch.float32) * sigma_w
    fmax = 448.0 if fmt == "e4m3" else 57344.0
    absmax = w.abs().amax(dim=1).clamp_min(1e-30)
    sigma_c = absmax / fmax
    x = (w / sigma_c[:, None]).clamp(-fmax, fmax)
    dt = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    q = x.to(dt)
    B = q.view(torch.uint8).contiguous()
    dec_max = q.float().abs().amax(dim=1)
    step = (dec_max / 127.0).to(torch.float16)
    return B, step.view(torch.int16).contiguous(), sigma_c.contiguous()


def make_activations(M: int, K: int, dist: str = "normal", outlier_frac: float = 0.0, seed: int = 1,
                     dtype=torch.float16, device: str = "cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    if dist == "uniform4":
        a = (torch.rand(M, K, generator=g, device=device) * 8.0 - 4.0)
    else:
        a = torch.randn(M, K, generator=g, device=device)
    if outlier_frac > 0:
        n_out = max(1, int(round(K * outlier_frac)))
        idx = torch.randperm(K, generator=g, device=device)[:n_out]
        a[:, idx] *= 20.0
    return a.to(dtype).contiguous()


def make_inputs(M: int, N: int, K: int, *, sigma_w: float = 0.02, fmt: str = "e4m3", dist: str = "normal",
                outlier_frac: float = 0.0, dtype=torch.float16, seed: int = 0, device: str = "cuda") -> GemmInputs:
    B, s16, sc = make_weights(N, K, sigma_w, fmt, seed, device)
    A = make_activations(M, K, dist, outlier_frac, seed + 1, dtype, device)
    return GemmInputs(A, B, s16, sc, fmt)


# Benchmark configurations (shapes and distributions), indexed like the
# benchmark definition: 0 smoke, 1 decode, 2 prefill up-proj, 3 square sweep,
# 4 column-parallel 70B-style up-proj.
CONFIGS = {
    "smoke": dict(M=128, N=256, K=512, sigma_w=0.02, dist="normal"),
    "decode_m1": dict(M=1, N=4096, K=4096, sigma_w=0.02, dist="normal", outlier_frac=0.01),
    "decode_m4": dict(M=4, N=4096, K=4096, sigma_w=0.02, dist="normal", outlier_frac=0.01),
    "decode_m16": dict(M=16, N=4096, K=4096, sigma_w=0.02, dist="normal", outlier_frac=0.01),
    "prefill": dict(M=2048, N=11008, K=4096, sigma_w=0.02, dist="normal"),
    "square2048": dict(M=2048, N=2048, K=2048, sigma_w=0.02, dist="uniform4"),
    "square4096": dict(M=4096, N=4096, K=4096, sigma_w=0.02, dist="uniform4"),
    "square8192": dict(M=8192, N=8192, K=8192, sigma_w=0.02, dist="uniform4"),
    "up70b_m1": dict(M=1, N=28672, K=8192, sigma_w=0.015, dist="normal"),
    "up70b_m32": dict(M=32, N=28672, K=8192, sigma_w=0.015, dist="normal"),
    "up70b_m4096": dict(M=4096, N=28672, K=8192, sigma_w=0.015, dist="normal"),
}


def algorithmic_bytes(M: int, N: int, K: int) -> int:
    """Bytes one GEMM call must move at minimum: weights N*K, fp32 column
    scale 4N, activations 2MK, output 2MN."""
    return N * K + 4 * N + 2 * M * K + 2 * M * N


def flops(M: int, N: int, K: int) -> int:
    return 2 * M * N * K
