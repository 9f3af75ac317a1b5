/* A plain C caller of the reference C ABI (include/fp8imma/imma_fp8.h), the
 * way a C / FFI user links the library: deterministic inputs from a 32-bit
 * LCG, device buffers from the CUDA runtime, one call per reference variant,
 * and the raw outputs written to a file for the test to compare against the
 * CPU oracle. Usage: fp8imma_c_caller M N K out_path
 * Exit status: 0 ok, 2 bad arguments, 3 CUDA runtime error, 4 launcher error. */
#include <cuda_runtime_api.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "fp8imma/imma_fp8.h"

static uint32_t lcg(uint32_t* s) {
  *s = *s * 1664525u + 1013904223u;
  return *s;
}

int main(int argc, char** argv) {
  if (argc != 5) return 2;
  const int M = atoi(argv[1]), N = atoi(argv[2]), K = atoi(argv[3]);
  if (M <= 0 || N <= 0 || K <= 0) return 2;
  uint16_t* A = (uint16_t*)malloc((size_t)M * K * 2);
  uint8_t* B = (uint8_t*)malloc((size_t)N * K);
  uint16_t* S = (uint16_t*)malloc((size_t)N * 2);
  uint16_t* D = (uint16_t*)malloc((size_t)N * M * 2);
  uint32_t seed = 12345u;
  /* activations: fp16 bits of small values (sign, exponent 12..16, any mantissa) */
  for (size_t i = 0; i < (size_t)M * K; ++i) {
    uint32_t r = lcg(&seed);
    A[i] = (uint16_t)(((r >> 31) << 15) | ((12u + (r >> 8) % 5u) << 10) | (r & 0x3FFu));
  }
  for (size_t i = 0; i < (size_t)N * K; ++i) B[i] = (uint8_t)(lcg(&seed) >> 24);
  for (int n = 0; n < N; ++n) S[n] = (uint16_t)(0x3800u + (lcg(&seed) >> 22)); /* fp16 in [0.5, 2) */
  void *dA, *dB, *dS, *dD;
  if (cudaMalloc(&dA, (size_t)M * K * 2) || cudaMalloc(&dB, (size_t)N * K) || cudaMalloc(&dS, (size_t)N * 2) ||
      cudaMalloc(&dD, (size_t)N * M * 2))
    return 3;
  if (cudaMemcpy(dA, A, (size_t)M * K * 2, cudaMemcpyHostToDevice) ||
      cudaMemcpy(dB, B, (size_t)N * K, cudaMemcpyHostToDevice) ||
      cudaMemcpy(dS, S, (size_t)N * 2, cudaMemcpyHostToDevice))
    return 3;
  fp8imma_init_fp8_e4m3_lut();
  FILE* f = fopen(argv[4], "wb");
  if (!f) return 2;
  /* v4 f16, v3 f16, then v4 f16 with kChunk 64: (global_scale, a_inv_scale) = (0.125, 8) */
  int err = fp8imma_launch_imma_fp8_actquant_v4_f16(32, dA, dB, dS, dD, M, N, K, 0.125f, 8.0f, 0);
  if (err) return 4;
  if (cudaMemcpy(D, dD, (size_t)N * M * 2, cudaMemcpyDeviceToHost)) return 3;
  fwrite(D, 2, (size_t)N * M, f);
  err = fp8imma_launch_imma_fp8_actquant_v3_f16(32, dA, dB, dS, dD, M, N, K, 0.125f, 8.0f, 0);
  if (err) return 4;
  if (cudaMemcpy(D, dD, (size_t)N * M * 2, cudaMemcpyDeviceToHost)) return 3;
  fwrite(D, 2, (size_t)N * M, f);
  err = fp8imma_launch_imma_fp8_actquant_v4_f16(64, dA, dB, dS, dD, M, N, K, 0.125f, 8.0f, 0);
  if (err) return 4;
  if (cudaMemcpy(D, dD, (size_t)N * M * 2, cudaMemcpyDeviceToHost)) return 3;
  fwrite(D, 2, (size_t)N * M, f);
  fclose(f);
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dS);
  cudaFree(dD);
  free(A);
  free(B);
  free(S);
  free(D);
  return 0;
}
