// Exact fallback kernel for shapes the fast kernels do not take (K not a
// multiple of 16, unaligned rows), plus the per-row activation-scale kernel.
//
// The fallback keeps the reference's K-tail behaviour: activations are read in
// whole groups (8 fp16 for v4, src/fp8imma/impl/v4_kernels.inl:196; 16 for
// v2/v3, impl/v3_kernels.inl:81) and weights in whole groups of 4 bytes
// (v4_kernels.inl:249); a trailing partial group reads as zero.
#include "fp8imma_kernels.h"
#include "fp8imma_device.cuh"

using namespace fp8imma_dev;

namespace fp8imma_b200 {

namespace {

constexpr int kGCols = 32, kGRows = 8;

template <int AT, int FMT>
__global__ void __launch_bounds__(256) generic_s8_kernel(const __grid_constant__ GemvParams p) {
  __shared__ int8_t tab[kGCols][256];
  const int c = threadIdx.x % kGCols, r = threadIdx.x / kGCols;
  const int n0 = blockIdx.x * kGCols, m0 = blockIdx.y * kGRows;
  // per-column int8 tables: the reference chain applied to all 256 codes
  for (int i = threadIdx.x; i < kGCols * 256; i += 256) {
    int cc = i >> 8, b = i & 255;
    int n = n0 + cc;
    int8_t q = 0;
    if (n < p.N) {
      uint16_t sb = p.scale_tex ? tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n) : p.scale_u16[n];
      uint16_t inv = inv_scale_bits(sb);
      uint16_t h = (FMT == FMT_E5M2) ? e5m2_bits((uint32_t)b) : ref_e4m3_bits((uint32_t)b);
      q = (int8_t)cvt_rni_sat_s8_f16(hmul_rn_bits(h, inv));
    }
    tab[cc][b] = q;
  }
  __syncthreads();
  const int n = n0 + c, m = m0 + r;
  if (n >= p.N || m >= p.M) return;
  const int keff_b = p.K - (p.K & 3);
  const int keff = p.keff_a < keff_b ? p.keff_a : keff_b;
  uint16_t ainv = p.row_inv_h ? p.row_inv_h[m] : p.a_inv_h;
  int32_t s = 0;
  const uint8_t* brow = p.B + (size_t)n * p.K;
  for (int k = 0; k < keff; ++k) {
    int qa;
    if (AT == A_S8) {
      qa = static_cast<const int8_t*>(p.A)[(size_t)m * p.K + k];
    } else {
      uint16_t h = static_cast<const uint16_t*>(p.A)[(size_t)m * p.K + k];
      if (AT == A_BF16) h = __half_as_ushort(__float2half_rn(__uint_as_float((uint32_t)h << 16)));
      qa = cvt_rni_sat_s8_f16(hmul_rn_bits(h, ainv));
    }
    s += qa * (int)tab[c][brow[k]];
  }
  uint16_t sb = p.scale_tex ? tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n) : p.scale_u16[n];
  float se = __half2float(__ushort_as_half(sb)) * (p.row_g ? p.row_g[m] : p.global_scale);
  if (p.col_scale_f32) se = se * p.col_scale_f32[n];
  uint16_t o = store_val(bias_act((float)s * se, p.bias, n, p.act), p.out_bf16);
  uint16_t* D = static_cast<uint16_t*>(p.D);
  if (p.out_row_major) D[(size_t)m * p.N + n] = o;
  else D[(size_t)n * p.M + m] = o;
  if (p.acc_out) p.acc_out[(size_t)n * p.M + m] = s;
}

template <int AT>
__global__ void __launch_bounds__(256) row_scales_kernel(const void* A, int M, int K, uint16_t* a_inv_h, float* g) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x * 8 + warp;
  if (m >= M) return;
  const uint16_t* row = static_cast<const uint16_t*>(A) + (size_t)m * K;
  float amax = 0.0f;
  for (int k = lane; k < K; k += 32) {
    uint16_t h = row[k];
    float v = (AT == A_BF16) ? __half2float(__float2half_rn(__uint_as_float((uint32_t)h << 16)))
                             : __half2float(__ushort_as_half(h));
    amax = fmaxf(amax, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) {
    float inv = 0.0f, gg = 0.0f;
    if (amax > 0.0f && amax <= 3.402823466e38f) {
      inv = __fdiv_rn(127.0f, amax);
      gg = __fdiv_rn(1.0f, inv);
    }
    a_inv_h[m] = __half_as_ushort(__float2half_rn(inv));
    g[m] = gg;
  }
}

}  // namespace

cudaError_t launch_generic_s8(const GemvParams& p, int a_type, int fmt, cudaStream_t stream) {
  dim3 grid((p.N + kGCols - 1) / kGCols, (p.M + kGRows - 1) / kGRows);
  const bool e5 = fmt == FMT_E5M2;
  switch (a_type) {
    case A_F16:
      if (e5) generic_s8_kernel<A_F16, FMT_E5M2><<<grid, 256, 0, stream>>>(p);
      else generic_s8_kernel<A_F16, FMT_E4M3_REF><<<grid, 256, 0, stream>>>(p);
      break;
    case A_BF16:
      if (e5) generic_s8_kernel<A_BF16, FMT_E5M2><<<grid, 256, 0, stream>>>(p);
      else generic_s8_kernel<A_BF16, FMT_E4M3_REF><<<grid, 256, 0, stream>>>(p);
      break;
    case A_S8:
      if (e5) generic_s8_kernel<A_S8, FMT_E5M2><<<grid, 256, 0, stream>>>(p);
      else generic_s8_kernel<A_S8, FMT_E4M3_REF><<<grid, 256, 0, stream>>>(p);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_row_scales(const void* A, int a_type, int M, int K, uint16_t* a_inv_h, float* g,
                              cudaStream_t stream) {
  dim3 grid((M + 7) / 8);
  if (a_type == A_BF16) row_scales_kernel<A_BF16><<<grid, 256, 0, stream>>>(A, M, K, a_inv_h, g);
  else if (a_type == A_F16) row_scales_kernel<A_F16><<<grid, 256, 0, stream>>>(A, M, K, a_inv_h, g);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace fp8imma_b200
