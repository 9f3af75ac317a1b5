// fp8wgt linear: fp16 activations x FP8(E4M3) weights decoded to fp16,
// fp32 accumulation, fp32 row-major output.
//
// Reference: torch_ext/fp8wgt/fp8wgt_ext_cuda.cu:135-258
// (wmma_fp16a_fp8e4m3b_gemm_kernel_tiled_vec4 + fp8_linear_forward):
//   Bdec[n,k] = fp16_rn( float(lut[B[n,k]]) * scale_b )
//   C[m,n]    = sum_k A[m,k] * Bdec[n,k]        (fp32 accumulation)
// Routing (fp8imma_fp8wgt_linear_forward):
//   * M > 64, 16-byte aligned weights: one pass decodes the weights to fp16
//     scratch, then the CTA-pair tcgen05 GEMM with kind::f16 (gemm_tc.cu);
//   * M <= 64, 16-byte aligned weights: the fp16 mode (FMT_WGT) of the TMA
//     split-K kernel (gemv_splitk.cu), weights decoded in registers;
//   * otherwise (8-byte aligned weights) fp8wgt_kernel below: one warp per 16
//     weight columns x 8*MB rows of A, weights streamed with 64-bit loads,
//     decoded in registers and fed to mma.sync m16n8k16 f16 (the decoded fp16
//     weights form the MMA's A operand, the activations its B operand), K
//     split across the 8 warps of a CTA and reduced in shared memory.
#include "fp8imma/fp8imma_ext.h"
#include "fp8imma_device.cuh"
#include "fp8imma_kernels.h"
#include "nvtx_range.h"

using namespace fp8imma_dev;

namespace fp8imma_b200 {
namespace {

constexpr int kWThreads = 256;

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2 weight bytes -> f16x2 of fp16_rn(float(lut[b]) * scale_b)
__device__ __forceinline__ uint32_t decode2(uint32_t two, float sb) {
  uint16_t h0 = ref_e4m3_bits(two & 0xFFu), h1 = ref_e4m3_bits((two >> 8) & 0xFFu);
  float f0 = __half2float(__ushort_as_half(h0)) * sb;
  float f1 = __half2float(__ushort_as_half(h1)) * sb;
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(f1), "f"(f0));
  return r;
}

// CTA: 16 weight columns x 8*MB activation rows; the 8 warps split K.
// Lane (g, t): MMA rows g, g+8 = weight columns; for a 16-wide K step the
// A-fragment wants k = 2t, 2t+1, 2t+8, 2t+9. Each lane loads 8 contiguous
// weight bytes of K per column (logical k = 8t .. 8t+7 of a 32-wide block),
// and the activation fragment is gathered with the same permutation.
template <int MB>
__global__ void __launch_bounds__(kWThreads) fp8wgt_kernel(const uint16_t* __restrict__ A,
                                                           const uint8_t* __restrict__ B, float sb,
                                                           float* __restrict__ C, int M, int N, int K) {
  constexpr int MR = MB * 8;
  __shared__ float red[8][16][MR + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * 16, m0 = blockIdx.y * MR;
  const int c0 = n0 + g, c1 = n0 + g + 8;
  float acc[MB][4];
#pragma unroll
  for (int i = 0; i < MB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  // K blocks of 32, round-robin over warps
  for (int kb = warp * 32; kb < K; kb += 8 * 32) {
    int k = kb + 8 * t;
    uint2 w0 = make_uint2(0u, 0u), w1 = make_uint2(0u, 0u);
    if (k < K) {
      if (c0 < N) w0 = *reinterpret_cast<const uint2*>(B + (size_t)c0 * K + k);
      if (c1 < N) w1 = *reinterpret_cast<const uint2*>(B + (size_t)c1 * K + k);
    }
    // decoded: d0[j] holds logical k = 8t + 2j, 8t + 2j + 1
    uint32_t d0[4], d1[4];
    d0[0] = decode2(w0.x, sb); d0[1] = decode2(w0.x >> 16, sb);
    d0[2] = decode2(w0.y, sb); d0[3] = decode2(w0.y >> 16, sb);
    d1[0] = decode2(w1.x, sb); d1[1] = decode2(w1.x >> 16, sb);
    d1[2] = decode2(w1.y, sb); d1[3] = decode2(w1.y >> 16, sb);
#pragma unroll
    for (int nb = 0; nb < MB; ++nb) {
      int m = m0 + nb * 8 + g;
      uint4 av = make_uint4(0u, 0u, 0u, 0u);
      if (m < M && k < K) av = *reinterpret_cast<const uint4*>(A + (size_t)m * K + k);
      // MMA #1: physical k {2t,2t+1} <- logical {8t, 8t+1}; {2t+8, 2t+9} <- {8t+2, 8t+3}
      mma_f16_16816(acc[nb], d0[0], d1[0], d0[1], d1[1], av.x, av.y);
      // MMA #2: logical {8t+4..8t+7}
      mma_f16_16816(acc[nb], d0[2], d1[2], d0[3], d1[3], av.z, av.w);
    }
  }
#pragma unroll
  for (int nb = 0; nb < MB; ++nb) {
    red[warp][g][nb * 8 + 2 * t] = acc[nb][0];
    red[warp][g][nb * 8 + 2 * t + 1] = acc[nb][1];
    red[warp][g + 8][nb * 8 + 2 * t] = acc[nb][2];
    red[warp][g + 8][nb * 8 + 2 * t + 1] = acc[nb][3];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 16 * MR; e += kWThreads) {
    int mr = e / 16, c = e % 16;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][c][mr];
    int m = m0 + mr, n = n0 + c;
    if (m < M && n < N) C[(size_t)m * N + n] = s;
  }
}

}  // namespace
}  // namespace fp8imma_b200

extern "C" int fp8imma_fp8wgt_linear_forward(const void* A, const void* B, float scale_b, void* C, int M,
                                             int N, int K, void* stream) {
  FP8IMMA_RANGE("fp8imma_fp8wgt_linear_forward");
  using namespace fp8imma_b200;
  if (M <= 0 || N <= 0) return (int)cudaErrorInvalidConfiguration;
  if (!A || !B || !C || K <= 0 || (K % 16) != 0) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(B) & 7u))
    return (int)cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M > 64 && (reinterpret_cast<uintptr_t>(B) & 15u) == 0) {
    // large M: weights decoded once to fp16, then tcgen05 kind::f16 (fp32 accumulate)
    ScopedScratch sc;
    const size_t ws = tc_splitk_ws_bytes(M, N, 2 * K);  // split-K accumulators for mid-size M
    cudaError_t e = sc.get((((size_t)N * K * 2 + 255) & ~size_t(255)) + ws, st, kScratchWgt);
    if (e != cudaSuccess) return (int)e;
    e = launch_gemm_tc_wgt(A, static_cast<const uint8_t*>(B), scale_b, static_cast<float*>(C), M, N, K, sc.ptr, st);
    cudaError_t e2 = sc.release(st);
    return (int)(e != cudaSuccess ? e : e2);
  }
  if ((reinterpret_cast<uintptr_t>(B) & 15u) == 0) {
    // small M: the TMA split-K kernel in its fp16 mode (weights decoded in
    // registers, raw fp16 activations in shared memory, fp32 accumulation)
    GemvParams p = {};
    p.A = A;
    p.B = static_cast<const uint8_t*>(B);
    p.D = C;
    p.M = M;
    p.N = N;
    p.K = K;
    p.keff_a = K;
    p.out_row_major = 1;  // epilogue walks the fp32 output row-major
    // packed decode multiplies by scale_b / 256, exact unless that is an fp32 subnormal
    const float mag = scale_b < 0.0f ? -scale_b : scale_b;
    p.wgt_fast = (mag == 0.0f || !(mag < 0x1p-117f)) ? 1 : 0;
    p.wgt_scale = p.wgt_fast ? scale_b * 0.00390625f : scale_b;
    return (int)launch_gemv_s8(p, A_F16, FMT_WGT, 0, st);
  }
  const int MB = M >= 32 ? 4 : (M + 7) / 8;
  dim3 grid((N + 15) / 16, (M + MB * 8 - 1) / (MB * 8));
  const uint16_t* a = static_cast<const uint16_t*>(A);
  const uint8_t* b = static_cast<const uint8_t*>(B);
  float* c = static_cast<float*>(C);
  switch (MB) {
    case 1: fp8wgt_kernel<1><<<grid, kWThreads, 0, st>>>(a, b, scale_b, c, M, N, K); break;
    case 2: fp8wgt_kernel<2><<<grid, kWThreads, 0, st>>>(a, b, scale_b, c, M, N, K); break;
    case 3: fp8wgt_kernel<3><<<grid, kWThreads, 0, st>>>(a, b, scale_b, c, M, N, K); break;
    default: fp8wgt_kernel<4><<<grid, kWThreads, 0, st>>>(a, b, scale_b, c, M, N, K); break;
  }
  return (int)cudaGetLastError();
}
