// PyTorch binding fp8wgt_ext.fp8_linear_forward — mirrors the reference
// torch_ext/fp8wgt/fp8wgt_ext.cpp:1-9 and fp8wgt_ext_cuda.cu:223-258 (same
// argument checks and result: fp32 [M,N]); the kernel is the sm_100a one in
// libfp8imma.so (fp8imma_fp8wgt_linear_forward). It launches on the current
// stream (the reference used the default stream).
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "fp8imma/fp8imma_ext.h"

torch::Tensor fp8_linear_forward(torch::Tensor A_fp16, torch::Tensor B_fp8_u8, double scale_b) {
  TORCH_CHECK(A_fp16.is_cuda(), "A must be CUDA");
  TORCH_CHECK(B_fp8_u8.is_cuda(), "B must be CUDA");
  TORCH_CHECK(A_fp16.scalar_type() == at::kHalf, "A must be FP16");
  TORCH_CHECK(B_fp8_u8.scalar_type() == at::kByte, "B must be uint8");
  TORCH_CHECK(A_fp16.is_contiguous(), "A must be contiguous");
  TORCH_CHECK(B_fp8_u8.is_contiguous(), "B must be contiguous");
  TORCH_CHECK(A_fp16.dim() == 2, "A must be 2D");
  TORCH_CHECK(B_fp8_u8.dim() == 2, "B must be 2D");
  const int64_t M = A_fp16.size(0), K = A_fp16.size(1), N = B_fp8_u8.size(0);
  TORCH_CHECK(B_fp8_u8.size(1) == K, "B must have shape [N,K] (col-major KxN with ld=K)");
  TORCH_CHECK((M % 16) == 0 && (N % 16) == 0 && (K % 16) == 0, "M,N,K must be multiples of 16 for WMMA");
  const c10::cuda::CUDAGuard guard(A_fp16.device());
  auto C = torch::empty({M, N}, torch::TensorOptions().device(A_fp16.device()).dtype(torch::kFloat32));
  int err = fp8imma_fp8wgt_linear_forward(A_fp16.data_ptr(), B_fp8_u8.data_ptr(), (float)scale_b, C.data_ptr(),
                                          (int)M, (int)N, (int)K, (void*)at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(err == 0, "CUDA error: fp8imma_fp8wgt_linear_forward returned ", err);
  return C;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("fp8_linear_forward", &fp8_linear_forward,
        "FP8(E4M3) weight-only linear forward (FP16 compute, fused decode), sm_100a");
}
