// Device-side arithmetic shared by the fp8imma B200 kernels.
//
// Semantics follow the reference fp8imma chain (Zzzxkxz/cuda-fp8-ampere):
//   weight  q_w = sat_rni_s8( fp16( lut_e4m3[b] * inv_h[n] ) )
//           inv_h[n] = fp16( |s| > 1e-8 ? 1/s : 0 ),  s = float(scale_h[n])
//           (src/fp8imma/impl/v4_kernels.inl:61-70, 146-158)
//   act     q_a = sat_rni_s8( fp16( to_half(a) * a_inv_h ) )
//           (src/fp8imma/impl/v4_kernels.inl:116-131; to_half at
//            src/fp8imma/fp8imma_internal.cuh:44-47)
//   out     D   = fp16_rn( float(acc_s32) * (s_f32[n] * global_scale) )
//           (src/fp8imma/impl/v4_kernels.inl:280-285)
// The reference decodes bytes through a 256-entry table built on the host
// (src/fp8imma/fp8_lut.cu:11-23); these kernels decode arithmetically instead
// and keep the table's exponent-15 behaviour (+-Inf for mantissa 0, NaN
// otherwise), so no table has to be initialised per device.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace fp8imma_dev {

// ----------------------------------------------------------- PTX wrappers --

__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hadd2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t max_s16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.s16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t min_s16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.s16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// two E4M3FN bytes -> f16x2 (hardware decode; exact for exponent <= 14)
__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint32_t two_bytes) {
  uint32_t r;
  uint16_t v = (uint16_t)two_bytes;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}
// 0xFFFF in each half whose f16 value is not NaN
__device__ __forceinline__ uint32_t notnan_mask_f16x2(uint32_t a) {
  uint32_t r;
  asm("set.num.u32.f16x2 %0, %1, %1;" : "=r"(r) : "r"(a));
  return r;
}
__device__ __forceinline__ int cvt_rni_sat_s8_f16(uint16_t h) {
  int32_t r;
  asm("cvt.rni.sat.s8.f16 %0, %1;" : "=r"(r) : "h"(h));
  return (int)(int8_t)r;
}
__device__ __forceinline__ uint16_t hmul_rn_bits(uint16_t a, uint16_t b) {
  uint16_t r;
  asm("mul.rn.f16 %0, %1, %2;" : "=h"(r) : "h"(a), "h"(b));
  return r;
}
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// -------------------------------------------------------- decode (exact) --

// Reference E4M3 byte -> fp16 bits, bit-identical to the reference table
// (fp8_e4m3_to_f32 + host __float2half, src/fp8imma/fp8imma_internal.cuh:54-70).
__host__ __device__ __forceinline__ uint16_t ref_e4m3_bits(uint32_t b) {
  uint32_t s = (b & 0x80u) << 8;
  uint32_t e = (b >> 3) & 15u, m = b & 7u;
  if (e == 15u) return m ? (uint16_t)0x7FFFu : (uint16_t)(s | 0x7C00u);
  if (e == 0u) {
    // m * 2^-9 is a normal fp16: m = 1 -> 2^-9, 2..3 -> 2^-8 * {1, 1.5}, 4..7 -> 2^-7 * {1..1.75}
    if (m == 0u) return (uint16_t)s;
    uint32_t lz = (m >= 4u) ? 2u : (m >= 2u) ? 1u : 0u;          // floor(log2 m)
    uint32_t exp16 = 15u - 9u + lz;                              // fp16 biased exponent
    uint32_t mant = (m << (10u - lz)) & 0x3FFu;
    return (uint16_t)(s | (exp16 << 10) | mant);
  }
  return (uint16_t)(s | (((b & 0x7Fu) << 7) + 0x2000u));
}

// E5M2 byte -> fp16 bits: the byte is the fp16 high byte.
__host__ __device__ __forceinline__ uint16_t e5m2_bits(uint32_t b) { return (uint16_t)(b << 8); }

// Per-column inverse scale exactly as the reference computes it
// (v4_kernels.inl:167-175): fp16( |s| > 1e-8 ? 1/s : 0 ).
__device__ __forceinline__ uint16_t inv_scale_bits(uint16_t scale_bits) {
  float s = __half2float(__ushort_as_half(scale_bits));
  float inv = (fabsf(s) > 1e-8f) ? __fdiv_rn(1.0f, s) : 0.0f;
  return __half_as_ushort(__float2half_rn(inv));
}

// --------------------------------------------- weight transcode, 4 bytes --

// int8-exact formats (transcoded): FMT_E4M3_REF, FMT_E5M2; native FP8 formats
// (fed to the tensor core as bytes): FMT_E4M3FN, FMT_NATIVE_E5M2.
// FMT_WGT: the fp8wgt linear (E4M3 weights decoded to fp16(lut * scale_b),
// fp16 activations, fp32 accumulation).
enum { FMT_E4M3_REF = 0, FMT_E5M2 = 1, FMT_E4M3FN = 2, FMT_NATIVE_E5M2 = 3, FMT_WGT = 4 };

// Exact scalar path (any inverse scale): the reference chain byte by byte.
template <int FMT>
__device__ __forceinline__ uint32_t transcode4_exact(uint32_t x, uint16_t inv_h) {
  uint32_t out = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t b = (x >> (8 * j)) & 0xFFu;
    uint16_t h = (FMT == FMT_E5M2) ? e5m2_bits(b) : ref_e4m3_bits(b);
    int q = cvt_rni_sat_s8_f16(hmul_rn_bits(h, inv_h));
    out |= ((uint32_t)(q & 0xFF)) << (8 * j);
  }
  return out;
}

// Whether a column may take the packed fast path below.
//   E4M3: |inv| >= 2^-6 and finite: inv/256 is then an exact (normal) fp16,
//         so (v*256)*(inv/256) is the exact product v*inv, rounded once.
//   E5M2: inv finite and non-zero.
template <int FMT>
__device__ __forceinline__ bool fast_ok(uint16_t inv_h) {
  uint32_t a = inv_h & 0x7FFFu;
  if (FMT == FMT_E5M2) return a != 0u && a < 0x7C00u;
  return a >= 0x2400u && a < 0x7C00u;
}

// Packed f16x2 constant for the fast path: inv/256 (E4M3) or inv (E5M2).
template <int FMT>
__device__ __forceinline__ uint32_t fast_scale(uint16_t inv_h) {
  uint16_t v = inv_h;
  if (FMT == FMT_E4M3_REF) v = __half_as_ushort(__hmul(__ushort_as_half(inv_h), __ushort_as_half((uint16_t)0x1C00u)));  // * 2^-8, exact
  return (uint32_t)v | ((uint32_t)v << 16);
}

__device__ __forceinline__ uint32_t hmin2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Two f16x2 products -> four saturated int8 = sat_rni(p), packed. Products
// here are never NaN (killed codes are finite, scales are finite
// and non-zero on the fast paths): clamp in fp16 to [-128, 127] first
// (rounding the clamped value equals clamping the rounded one for every
// finite or infinite p), then 1536 + p rounds to the nearest integer (ties to
// even: the fp16 ulp in [1024, 2048) is 1 and 1536 is even), whose low byte
// is the int8 result.
__device__ __forceinline__ uint32_t round_sat_pack(uint32_t p01, uint32_t p23) {
  const uint32_t kMagic = 0x66006600u, kLo = 0xD800D800u, kHi = 0x57F057F0u;  // 1536, -128, 127
  uint32_t r01 = hadd2_rn(hmin2(hmax2(p01, kLo), kHi), kMagic);
  uint32_t r23 = hadd2_rn(hmin2(hmax2(p23, kLo), kHi), kMagic);
  return prmt(r01, r23, 0x6420u);
}

// 0xFF in every byte of t whose bit 7 is set, 0x00 elsewhere (byte permute
// with sign replication)
__device__ __forceinline__ uint32_t byte_sign_mask(uint32_t t) { return prmt(t, 0u, 0xBA98u); }

// two E4M3FN bytes in each half of x -> f16x2 (bytes 0,1 -> lo; 2,3 -> hi)
__device__ __forceinline__ void cvt_e4m3x4_f16x2x2(uint32_t x, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(x));
}

// Fast path, reference-E4M3 semantics, 4 bytes -> 4 int8.
//   1. NaN codes (exponent 15, mantissa != 0) become code 0x00, which gives
//      0 below (the reference gives NaN -> 0).
//   2. Hardware E4M3FN decode is exact for exponent <= 14; the remaining
//      exponent-15 codes (0x78 / 0xF8) decode to +-256.
//   3. *256 is exact for |v| <= 240 and overflows +-256 to +-Inf (the
//      reference table's value for those codes); *(inv/256) then forms the
//      same exact product v*inv as the reference, rounded once.
//   4. round / saturate / pack.
__device__ __forceinline__ uint32_t transcode4_fast_e4m3(uint32_t x, uint32_t inv256x2) {
  const uint32_t t = (x & 0x7F7F7F7Fu) + 0x07070707u;  // bit 7 set iff (b & 0x7F) >= 0x79
  x &= ~byte_sign_mask(t);
  uint32_t h01, h23;
  cvt_e4m3x4_f16x2x2(x, h01, h23);
  const uint32_t k256 = 0x5C005C00u;
  h01 = hmul2_rn(hmul2_rn(h01, k256), inv256x2);
  h23 = hmul2_rn(hmul2_rn(h23, k256), inv256x2);
  return round_sat_pack(h01, h23);
}

// Fast path, E5M2 (fp16 = byte << 8): NaN codes (0x7D..0x7F) become 0x00,
// Inf codes stay Inf.
__device__ __forceinline__ uint32_t transcode4_fast_e5m2(uint32_t x, uint32_t invx2) {
  const uint32_t t = (x & 0x7F7F7F7Fu) + 0x03030303u;  // bit 7 set iff (b & 0x7F) >= 0x7D
  x &= ~byte_sign_mask(t);
  uint32_t h01 = prmt(x, 0u, 0x1404u);
  uint32_t h23 = prmt(x, 0u, 0x3424u);
  h01 = hmul2_rn(h01, invx2);
  h23 = hmul2_rn(h23, invx2);
  return round_sat_pack(h01, h23);
}

template <int FMT>
__device__ __forceinline__ uint32_t transcode4(uint32_t x, bool fast, uint32_t fscale, uint16_t inv_h) {
  if (fast) {
    if (FMT == FMT_E5M2) return transcode4_fast_e5m2(x, fscale);
    return transcode4_fast_e4m3(x, fscale);
  }
  return transcode4_exact<FMT>(x, inv_h);
}

// fp8wgt weight decode, 4 bytes -> two f16x2 (bytes 0,1 -> lo; 2,3 -> hi) of
// fp16_rn(float(lut[b]) * s), lut the reference table (exponent 15: +-Inf for
// mantissa 0, NaN otherwise).
//   1. exponent-15 NaN codes become 0x7F / 0xFF (NaN in hardware E4M3FN);
//   2. hardware decode, exact for exponent <= 14; 0x78 / 0xF8 give +-256;
//   3. *256 in fp16 is exact for |v| <= 240 and turns +-256 into +-Inf;
//   4. fp32 product with s/256 (exact power-of-two rescale of s, which the
//      host guarantees) is the reference's fp32 product v*s, rounded once to
//      fp32 and once to fp16 exactly as the reference does.
__device__ __forceinline__ void wgt_decode4_fast(uint32_t x, float s256, uint32_t& lo, uint32_t& hi) {
  uint32_t t = ((x & 0x7F7F7F7Fu) + 0x07070707u) & 0x80808080u;  // bit 7 set iff (b & 0x7F) >= 0x79
  x |= t - (t >> 7);
  const uint32_t k256 = 0x5C005C00u;
  const uint32_t h01 = hmul2_rn(cvt_e4m3x2_f16x2(x & 0xFFFFu), k256);
  const uint32_t h23 = hmul2_rn(cvt_e4m3x2_f16x2(x >> 16), k256);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(f01.y * s256), "f"(f01.x * s256));
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(f23.y * s256), "f"(f23.x * s256));
}

// Exact scalar form of the same decode (any scale).
__device__ __forceinline__ void wgt_decode4_exact(uint32_t x, float s, uint32_t& lo, uint32_t& hi) {
  float f[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) f[j] = __half2float(__ushort_as_half(ref_e4m3_bits((x >> (8 * j)) & 0xFFu))) * s;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(f[1]), "f"(f[0]));
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(f[3]), "f"(f[2]));
}

// ------------------------------------------------ activation quantisation --

// 4 fp16 values (two f16x2) -> 4 int8: sat_rni(fp16(h * ainv)), NaN -> 0.
__device__ __forceinline__ uint32_t quant4_f16(uint32_t h01, uint32_t h23, uint32_t ainv2) {
  const uint32_t kMagic = 0x66006600u, kLo = 0x65806580u, kHi = 0x667F667Fu;
  uint32_t p01 = hmul2_rn(h01, ainv2), p23 = hmul2_rn(h23, ainv2);
  uint32_t n01 = notnan_mask_f16x2(p01), n23 = notnan_mask_f16x2(p23);
  uint32_t r01 = hadd2_rn(p01, kMagic), r23 = hadd2_rn(p23, kMagic);
  r01 = (r01 & n01) | (kMagic & ~n01);               // NaN lanes -> 1536 -> 0
  r23 = (r23 & n23) | (kMagic & ~n23);
  r01 = min_s16x2(max_s16x2(r01, kLo), kHi);
  r23 = min_s16x2(max_s16x2(r23, kLo), kHi);
  return prmt(r01, r23, 0x6420u);
}

// two bf16 (packed) -> f16x2 via fp32, round to nearest (to_half<bf16>)
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
  float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xFFFF0000u);
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// --------------------------------------------------------------- epilogue --

// Optional fused epilogue after the scales, in fp32: + bias[n], then an
// activation (0 none, 1 ReLU, 2 GELU tanh form, 3 SiLU).
__device__ __forceinline__ float bias_act(float v, const float* bias, int n, int act) {
  if (bias) v = __fadd_rn(v, bias[n]);  // never contracted with the scale product: round, then add
  if (act == 1) {
    v = fmaxf(v, 0.0f);
  } else if (act == 2) {
    const float u = 0.7978845608f * (v + 0.044715f * v * v * v);  // sqrt(2/pi) (v + 0.044715 v^3)
    v = 0.5f * v * (1.0f + tanhf(u));
  } else if (act == 3) {
    v = v / (1.0f + expf(-v));
  }
  return v;
}

__device__ __forceinline__ uint16_t store_val(float v, int out_bf16) {
  return out_bf16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
}

}  // namespace fp8imma_dev
