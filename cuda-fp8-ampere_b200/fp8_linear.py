"""FP8Linear — inference-only linear layer over fp8wgt_ext.

Mirrors the reference module torch_ext/fp8wgt/fp8_linear.py:4-26: fp16
activations, FP8(E4M3) weights stored as a [N,K] uint8 buffer (col-major KxN,
ld = K), fp32 [M,N] output, forward only. The kernel behind it is the sm_100a
one in libfp8imma.so.
"""
import torch

import fp8wgt_ext


class FP8Linear(torch.nn.Module):
    def __init__(self, B_fp8_u8: torch.Tensor, scale_b: float = 1.0):
        super().__init__()
        assert B_fp8_u8.is_cuda and B_fp8_u8.dtype == torch.uint8 and B_fp8_u8.dim() == 2
        self.register_buffer("B_fp8_u8", B_fp8_u8.contiguous())
        self.scale_b = float(scale_b)

    def forward(self, A_fp16: torch.Tensor) -> torch.Tensor:
        assert A_fp16.is_cuda and A_fp16.dtype == torch.float16 and A_fp16.dim() == 2
        return fp8wgt_ext.fp8_linear_forward(A_fp16.contiguous(), self.B_fp8_u8, self.scale_b)
