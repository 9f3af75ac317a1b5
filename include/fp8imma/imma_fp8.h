// fp8imma public API — B200 (sm_100a) implementation.
//
// Drop-in for the reference header include/fp8imma/imma_fp8.h of
// Zzzxkxz/cuda-fp8-ampere: the same C++ launchers (namespace fp8imma) and the
// same C ABI (fp8imma_* symbols, void* pointers, void* stream, int return =
// cudaError_t, 0 = success), with the same argument order, layouts and
// numerical results. Each declaration names the reference declaration it
// replaces (reference header line numbers).
//
// Layouts (unchanged from the reference):
//   A        [M,K] row-major (int8 for v2, fp16/bf16 for v3/v4)
//   B_col    [N,K] row-major uint8 = col-major KxN FP8(E4M3) weight bytes
//   scales   [N] fp16 bits (uint16), the int8 step of each weight column
//   D_col    col-major MxN fp16, i.e. D[n*M + m]
// kChunk must be 32 or 64 (cudaErrorInvalidValue otherwise); it selects the
// reference kernel's K step and does not change results here.
//
// Differences from the reference, all on inputs the reference mishandles:
//   * arguments are validated on the host (null pointers, negative K:
//     cudaErrorInvalidValue; M or N <= 0: cudaErrorInvalidConfiguration, the
//     code the reference's empty grid launch returns);
//   * no device table has to be initialised: init_fp8_e4m3_lut() is a no-op
//     kept for API compatibility, and every device works without it (the
//     reference initialises only the device current at its first call);
//   * v2_i8lut at kChunk=64 returns the correct result (the reference leaves
//     half of each K chunk of B stale there).
#pragma once

#ifdef __cplusplus
#include <cstddef>
#include <cstdint>
#else
/* plain C callers (FFI bindings, cgo) see only the C ABI below */
#include <stddef.h>
#include <stdint.h>
#endif

#ifdef __CUDACC__
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#endif

#ifdef __cplusplus
namespace fp8imma {

// reference imma_fp8.h:23
void init_fp8_e4m3_lut();

#ifdef __CUDACC__
// reference imma_fp8.h:29 — int8 activations, FP8 weights.
cudaError_t launch_imma_fp8_jit_v2(int kChunk, const int8_t* A_row_i8, const uint8_t* B_col_fp8,
                                   const uint16_t* col_scales_u16, half* D_col_f16, int M, int N,
                                   int K, float global_scale, cudaStream_t stream);
// reference imma_fp8.h:42
cudaError_t launch_imma_fp8_jit_v2_i8lut(int kChunk, const int8_t* A_row_i8,
                                         const uint8_t* B_col_fp8, const uint16_t* col_scales_u16,
                                         half* D_col_f16, int M, int N, int K, float global_scale,
                                         cudaStream_t stream);
// reference imma_fp8.h:55 — fused fp16 activation quant (16-element groups).
cudaError_t launch_imma_fp8_actquant_v3_f16(int kChunk, const half* A_row_f16,
                                            const uint8_t* B_col_fp8,
                                            const uint16_t* col_scales_u16, half* D_col_f16, int M,
                                            int N, int K, float global_scale, float a_inv_scale,
                                            cudaStream_t stream);
// reference imma_fp8.h:68
cudaError_t launch_imma_fp8_actquant_v3_bf16(int kChunk, const __nv_bfloat16* A_row_bf16,
                                             const uint8_t* B_col_fp8,
                                             const uint16_t* col_scales_u16, half* D_col_f16,
                                             int M, int N, int K, float global_scale,
                                             float a_inv_scale, cudaStream_t stream);
// reference imma_fp8.h:86 — the path the torch extension uses (8-element groups).
cudaError_t launch_imma_fp8_actquant_v4_f16(int kChunk, const half* A_row_f16,
                                            const uint8_t* B_col_fp8,
                                            const uint16_t* col_scales_u16, half* D_col_f16, int M,
                                            int N, int K, float global_scale, float a_inv_scale,
                                            cudaStream_t stream);
// reference imma_fp8.h:99
cudaError_t launch_imma_fp8_actquant_v4_bf16(int kChunk, const __nv_bfloat16* A_row_bf16,
                                             const uint8_t* B_col_fp8,
                                             const uint16_t* col_scales_u16, half* D_col_f16,
                                             int M, int N, int K, float global_scale,
                                             float a_inv_scale, cudaStream_t stream);
// reference imma_fp8.h:113 — column scales read through a texture object.
cudaError_t launch_imma_fp8_actquant_v4_texscale_f16(int kChunk, const half* A_row_f16,
                                                     const uint8_t* B_col_fp8,
                                                     cudaTextureObject_t scale_tex_u16,
                                                     half* D_col_f16, int M, int N, int K,
                                                     float global_scale, float a_inv_scale,
                                                     cudaStream_t stream);
// reference imma_fp8.h:126
cudaError_t launch_imma_fp8_actquant_v4_texscale_bf16(int kChunk, const __nv_bfloat16* A_row_bf16,
                                                      const uint8_t* B_col_fp8,
                                                      cudaTextureObject_t scale_tex_u16,
                                                      half* D_col_f16, int M, int N, int K,
                                                      float global_scale, float a_inv_scale,
                                                      cudaStream_t stream);
#endif

}  // namespace fp8imma
#endif  // __cplusplus

#ifdef __cplusplus
extern "C" {
#endif

// reference imma_fp8.h:152
void fp8imma_init_fp8_e4m3_lut(void);

// reference imma_fp8.h:154
int fp8imma_launch_imma_fp8_jit_v2(int kChunk, const void* A_row_i8, const void* B_col_fp8,
                                   const void* col_scales_u16, void* D_col_f16, int M, int N, int K,
                                   float global_scale, void* stream);
// reference imma_fp8.h:166
int fp8imma_launch_imma_fp8_jit_v2_i8lut(int kChunk, const void* A_row_i8, const void* B_col_fp8,
                                         const void* col_scales_u16, void* D_col_f16, int M, int N,
                                         int K, float global_scale, void* stream);
// reference imma_fp8.h:178
int fp8imma_launch_imma_fp8_actquant_v3_f16(int kChunk, const void* A_row_f16,
                                            const void* B_col_fp8, const void* col_scales_u16,
                                            void* D_col_f16, int M, int N, int K,
                                            float global_scale, float a_inv_scale, void* stream);
// reference imma_fp8.h:191
int fp8imma_launch_imma_fp8_actquant_v3_bf16(int kChunk, const void* A_row_bf16,
                                             const void* B_col_fp8, const void* col_scales_u16,
                                             void* D_col_f16, int M, int N, int K,
                                             float global_scale, float a_inv_scale, void* stream);
// reference imma_fp8.h:204
int fp8imma_launch_imma_fp8_actquant_v4_texscale_f16(int kChunk, const void* A_row_f16,
                                                     const void* B_col_fp8, void* scale_tex_u16,
                                                     void* D_col_f16, int M, int N, int K,
                                                     float global_scale, float a_inv_scale,
                                                     void* stream);
// reference imma_fp8.h:217
int fp8imma_launch_imma_fp8_actquant_v4_texscale_bf16(int kChunk, const void* A_row_bf16,
                                                      const void* B_col_fp8, void* scale_tex_u16,
                                                      void* D_col_f16, int M, int N, int K,
                                                      float global_scale, float a_inv_scale,
                                                      void* stream);
// reference imma_fp8.h:230
int fp8imma_launch_imma_fp8_actquant_v4_f16(int kChunk, const void* A_row_f16,
                                            const void* B_col_fp8, const void* col_scales_u16,
                                            void* D_col_f16, int M, int N, int K,
                                            float global_scale, float a_inv_scale, void* stream);
// reference imma_fp8.h:243
int fp8imma_launch_imma_fp8_actquant_v4_bf16(int kChunk, const void* A_row_bf16,
                                             const void* B_col_fp8, const void* col_scales_u16,
                                             void* D_col_f16, int M, int N, int K,
                                             float global_scale, float a_inv_scale, void* stream);

#ifdef __cplusplus
}  // extern "C"
#endif
