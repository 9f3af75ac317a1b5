/*
 * fp8imma CPU oracle — TEST INFRASTRUCTURE ONLY (see fp8imma_oracle.h).
 *
 * Scalar restatement of the reference fp8imma arithmetic. Each function names
 * the reference file:line it follows (paths inside Zzzxkxz/cuda-fp8-ampere).
 * Nothing here is used by the shipped library.
 */
#include "fp8imma_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- fp16 --- */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary32 -> binary16, round to nearest even. NaN -> 0x7FFF (the
 * canonical NaN CUDA's __float2half produces on host and device). */
uint16_t orc_f32_to_f16(float f) {
  uint32_t x = f2u(f);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax > 0x7F800000u) return 0x7FFFu;
  if (ax == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 rounds to inf */
  if (ax < 0x33000000u) return sign;                          /* < 2^-25 -> 0 */
  int e = (int)(ax >> 23) - 127;
  uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;               /* 24 significant bits */
  int shift;                                                  /* bits to drop */
  uint32_t base;
  if (e >= -14) {           /* normal fp16 */
    shift = 13;
    base = (uint32_t)(e + 15) << 10;
    mant &= 0x7FFFFFu;      /* drop implicit bit, re-add via exponent */
  } else {                  /* subnormal fp16: value = m * 2^-24 */
    shift = -e - 1;         /* 24-bit significand scaled to units of 2^-24 */
    base = 0;
  }
  uint32_t q = mant >> shift;
  uint32_t rem = mant & ((1u << shift) - 1u);
  uint32_t half = 1u << (shift - 1);
  if (rem > half || (rem == half && (q & 1u))) q++;
  return (uint16_t)(sign | (base + q)); /* carries into exponent are correct */
}

float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
  if (e == 0) {
    float v = ldexpf((float)m, -24);
    return (h & 0x8000u) ? -v : v;
  }
  return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

uint16_t orc_f32_to_bf16(float f) {
  uint32_t x = f2u(f);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFFu;
  uint32_t lsb = (x >> 16) & 1u;
  x += 0x7FFFu + lsb;
  return (uint16_t)(x >> 16);
}

float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* to_half<__nv_bfloat16>: __float2half_rn(__bfloat162float(v))
 * (src/fp8imma/fp8imma_internal.cuh:44-47). */
uint16_t orc_bf16_to_f16(uint16_t b) { return orc_f32_to_f16(orc_bf16_to_f32(b)); }

/* __hmul(a,b): the exact fp16*fp16 product fits in binary32, so one RNE
 * rounding of the binary32 product reproduces the fp16 multiply bit for bit. */
uint16_t orc_hmul(uint16_t a, uint16_t b) {
  return orc_f32_to_f16(orc_f16_to_f32(a) * orc_f16_to_f32(b));
}

/* cvt.rni.sat.s8.f16 (src/fp8imma/fp8imma_internal.cuh:29-34): round to
 * nearest integer, ties to even; saturate to [-128,127]; NaN -> 0. */
int orc_cvt_rni_sat_s8_f16(uint16_t h) {
  float v = orc_f16_to_f32(h);
  if (isnan(v)) return 0;
  if (v >= 127.0f) return 127;
  if (v <= -128.0f) return -128;
  float r = nearbyintf(v); /* default rounding mode: to nearest even */
  return (int)r;
}

/* ------------------------------------------------------------ FP8 decode - */

/* fp8_e4m3_to_f32 (src/fp8imma/fp8imma_internal.cuh:54-70): bias 7,
 * subnormal m*2^-9, exponent 15 -> +-Inf (m==0) or NaN. */
static float ref_e4m3_to_f32(uint8_t v) {
  int sign = (v >> 7) & 1, ex = (v >> 3) & 0xF, mant = v & 7;
  float s = sign ? -1.0f : 1.0f;
  if (ex == 0) {
    if (mant == 0) return s * 0.0f;
    return s * ldexpf((float)mant, (1 - 7) - 3);
  }
  if (ex == 15) {
    if (mant == 0) return s * INFINITY;
    return NAN;
  }
  return s * ldexpf(1.0f + (float)mant / 8.0f, ex - 7);
}

/* init_fp8_e4m3_lut (src/fp8imma/fp8_lut.cu:11-23): table of fp16 bits. */
void orc_lut_e4m3_ref(uint16_t* out256) {
  for (int i = 0; i < 256; ++i) out256[i] = orc_f32_to_f16(ref_e4m3_to_f32((uint8_t)i));
}

/* E5M2 is not in the reference; its byte is exactly the high byte of the
 * fp16 encoding, so the table entry is b << 8 (IEEE Inf/NaN included). */
void orc_lut_e5m2(uint16_t* out256) {
  for (int i = 0; i < 256; ++i) out256[i] = (uint16_t)(i << 8);
}

/* OCP E4M3FN (hardware FP8): no Inf, 0x7F/0xFF NaN, max 448. */
float orc_e4m3fn_to_f32(uint8_t b) {
  int sign = b >> 7, ex = (b >> 3) & 0xF, mant = b & 7;
  float v;
  if ((b & 0x7F) == 0x7F) return NAN;
  if (ex == 0) v = ldexpf((float)mant, -9);
  else v = ldexpf(1.0f + (float)mant / 8.0f, ex - 7);
  return sign ? -v : v;
}

float orc_e5m2_to_f32(uint8_t b) { return orc_f16_to_f32((uint16_t)(b << 8)); }

/* Round-to-nearest-even encode with saturation to the largest finite value
 * (the semantics of cvt.rn.satfinite.{e4m3x2,e5m2x2}.f32). */
static uint8_t encode_fp8(float x, int mbits, int bias, float maxv, int is_e4m3) {
  if (isnan(x)) return is_e4m3 ? 0x7F : 0x7F;
  uint8_t sign = signbit(x) ? 0x80 : 0;
  double a = fabs((double)x);
  if (a >= maxv) a = maxv;
  int min_exp = 1 - bias;
  int e;
  if (a == 0.0) return sign;
  frexp(a, &e);
  e -= 1; /* a in [2^e, 2^(e+1)) */
  if (e < min_exp) e = min_exp;
  double quantum = ldexp(1.0, e - mbits);
  double r = nearbyint(a / quantum); /* ties to even */
  double v = r * quantum;
  if (v > maxv) v = maxv;
  if (v == 0.0) return sign;
  /* encode v */
  frexp(v, &e);
  e -= 1;
  uint8_t code;
  if (e < min_exp) {
    int m = (int)(v / ldexp(1.0, min_exp - mbits));
    code = (uint8_t)m;
  } else {
    int m = (int)((v / ldexp(1.0, e) - 1.0) * (1 << mbits) + 0.5);
    code = (uint8_t)(((e + bias) << mbits) | m);
  }
  return sign | code;
}

uint8_t orc_f32_to_e4m3fn_sat(float x) { return encode_fp8(x, 3, 7, 448.0f, 1); }
uint8_t orc_f32_to_e5m2_sat(float x) { return encode_fp8(x, 2, 15, 57344.0f, 0); }

/* ------------------------------------------------------- quant/transcode - */

/* Per-column inverse scale (src/fp8imma/impl/v4_kernels.inl:61-70):
 * s = float(scale_h); inv = |s| > 1e-8 ? 1/s : 0; stored as fp16 (RN). */
uint16_t orc_inv_scale_h(uint16_t scale_h) {
  float s = orc_f16_to_f32(scale_h);
  volatile float one = 1.0f;
  float inv = (fabsf(s) > 1e-8f) ? (one / s) : 0.0f;
  return orc_f32_to_f16(inv);
}

/* Activation quantisation (v4_kernels.inl:116-131, v3_kernels.inl:74-90):
 * q = sat_rni(fp16(to_half(a) * a_inv_h)). Elements of a trailing partial
 * group of `group` elements along K are zero (the reference only loads full
 * 16-byte / 16-element vectors: v4 `(gk+7)<K`, v3/v2 `(gk+15)<K`). */
void orc_quant_a(const void* A, int a_type, int M, int K, int group,
                 const uint16_t* a_inv_h_rows, uint16_t a_inv_h, int8_t* Aq) {
  int keff = K - K % group;
  for (int m = 0; m < M; ++m) {
    uint16_t inv = a_inv_h_rows ? a_inv_h_rows[m] : a_inv_h;
    for (int k = 0; k < K; ++k) {
      size_t i = (size_t)m * K + k;
      int8_t q = 0;
      if (k < keff) {
        if (a_type == ORC_A_S8) {
          q = ((const int8_t*)A)[i];
        } else {
          uint16_t h = ((const uint16_t*)A)[i];
          if (a_type == ORC_A_BF16) h = orc_bf16_to_f16(h);
          q = (int8_t)orc_cvt_rni_sat_s8_f16(orc_hmul(h, inv));
        }
      }
      Aq[i] = q;
    }
  }
}

/* Weight transcode (v4_kernels.inl:146-158, v2_kernels.inl:251-268):
 * w = sat_rni(fp16(lut[b] * inv_h[n])); trailing partial groups of 4 bytes
 * along K read as zero bytes (v4_kernels.inl:248-251). */
void orc_transcode_b(const uint8_t* B, const uint16_t* scale_u16, int N, int K,
                     int fmt, int8_t* Bq) {
  uint16_t lut[256];
  if (fmt == ORC_FMT_E5M2) orc_lut_e5m2(lut);
  else orc_lut_e4m3_ref(lut);
  int keff = K - K % 4;
  for (int n = 0; n < N; ++n) {
    uint16_t inv = orc_inv_scale_h(scale_u16[n]);
    int8_t tab[256];
    for (int b = 0; b < 256; ++b) tab[b] = (int8_t)orc_cvt_rni_sat_s8_f16(orc_hmul(lut[b], inv));
    for (int k = 0; k < K; ++k) {
      uint8_t b = k < keff ? B[(size_t)n * K + k] : 0;
      Bq[(size_t)n * K + k] = tab[b];
    }
  }
}

/* ---------------------------------------------------------------- GEMM --- */

typedef struct {
  const int8_t* Aq; const int8_t* Bq; int M, N, K, Keff; int32_t* acc; int n0, n1;
} gemm_job;

static void* gemm_worker(void* p) {
  gemm_job* j = (gemm_job*)p;
  for (int n = j->n0; n < j->n1; ++n) {
    const int8_t* b = j->Bq + (size_t)n * j->K;
    for (int m = 0; m < j->M; ++m) {
      const int8_t* a = j->Aq + (size_t)m * j->K;
      int32_t s = 0;
      for (int k = 0; k < j->Keff; ++k) s += (int32_t)a[k] * (int32_t)b[k];
      j->acc[(size_t)n * j->M + m] = s;
    }
  }
  return NULL;
}

/* int32 accumulation (WMMA s8 m16n16k16, v4_kernels.inl:192-201). Integer
 * addition is exact, so summation order is irrelevant. acc is [N][M]. */
void orc_gemm_s8(const int8_t* Aq, const int8_t* Bq, int M, int N, int K, int Keff,
                 int32_t* acc_nm, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  gemm_job jobs[256];
  int per = (N + nthreads - 1) / nthreads;
  int started = 0;
  for (int t = 0; t < nthreads; ++t) {
    int n0 = t * per, n1 = n0 + per > N ? N : n0 + per;
    if (n0 >= n1) break;
    gemm_job j = {Aq, Bq, M, N, K, Keff, acc_nm, n0, n1};
    jobs[t] = j;
    if (nthreads == 1) gemm_worker(&jobs[t]);
    else pthread_create(&th[t], NULL, gemm_worker, &jobs[t]);
    started++;
  }
  if (nthreads > 1)
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

/* Epilogue (v4_kernels.inl:280-285): v = float(acc) * (s_f32 * global_scale);
 * D = fp16_rn(v). Extensions (not in the reference): a per-row global scale
 * replaces global_scale, an fp32 per-column scale multiplies the combined
 * scale after it, bf16 output, and row-major [M,N] output. */
void orc_epilogue(const int32_t* acc_nm, const uint16_t* scale_u16,
                  const float* col_scale_f32, const float* row_gscale,
                  float global_scale, int M, int N, int out_bf16, int out_row_major,
                  uint16_t* D) {
  for (int n = 0; n < N; ++n) {
    float s = orc_f16_to_f32(scale_u16[n]);
    for (int m = 0; m < M; ++m) {
      volatile float g = row_gscale ? row_gscale[m] : global_scale;
      volatile float se = s * g;
      if (col_scale_f32) se = se * col_scale_f32[n];
      volatile float v = (float)acc_nm[(size_t)n * M + m] * se;
      uint16_t o = out_bf16 ? orc_f32_to_bf16(v) : orc_f32_to_f16(v);
      if (out_row_major) D[(size_t)m * N + n] = o;
      else D[(size_t)n * M + m] = o;
    }
  }
}

/* Per-row dynamic quantisation (extension; defined as the reference called
 * once per row): a_inv_m = 127 / absmax_m in fp32 (fp16 for the multiply, as
 * the reference launcher converts it, imma_fp8_v4.cu:38), and the row's
 * global scale g_m = 1 / a_inv_m. absmax is taken over to_half(a); a row
 * whose absmax is 0 or not finite gets a_inv = 0 and g = 0. */
void orc_row_scales(const void* A, int a_type, int M, int K, float* a_inv_f32,
                    uint16_t* a_inv_h, float* gscale) {
  for (int m = 0; m < M; ++m) {
    float amax = 0.0f;
    for (int k = 0; k < K; ++k) {
      uint16_t h = ((const uint16_t*)A)[(size_t)m * K + k];
      if (a_type == ORC_A_BF16) h = orc_bf16_to_f16(h);
      float v = fabsf(orc_f16_to_f32(h));
      if (v > amax) amax = v; /* NaN compares false: ignored */
    }
    volatile float inv = 0.0f, g = 0.0f;
    if (amax > 0.0f && isfinite(amax)) {
      volatile float c127 = 127.0f, one = 1.0f;
      inv = c127 / amax;
      g = one / inv;
    }
    if (a_inv_f32) a_inv_f32[m] = inv;
    if (a_inv_h) a_inv_h[m] = orc_f32_to_f16(inv);
    if (gscale) gscale[m] = g;
  }
}

/* Whole reference launch: variant 0 = v2 (int8 A), 1 = v2_i8lut, 2 = v3 f16,
 * 3 = v3 bf16, 4 = v4 f16, 5 = v4 bf16 (texscale variants equal v4).
 * Returns 0, or 1 (cudaErrorInvalidValue) for kChunk not in {32,64}
 * (imma_fp8_v4.cu:40-60). */
int orc_imma_fp8(int variant, int kChunk, const void* A, const uint8_t* B,
                 const uint16_t* scale_u16, uint16_t* D_col, int M, int N, int K,
                 float global_scale, float a_inv_scale, int32_t* acc_out, int nthreads) {
  if (kChunk != 32 && kChunk != 64) return 1;
  int a_type, group;
  switch (variant) {
    case 0: case 1: a_type = ORC_A_S8; group = 16; break;
    case 2: a_type = ORC_A_F16; group = 16; break;
    case 3: a_type = ORC_A_BF16; group = 16; break;
    case 4: a_type = ORC_A_F16; group = 8; break;
    case 5: a_type = ORC_A_BF16; group = 8; break;
    default: return 1;
  }
  int8_t* Aq = (int8_t*)malloc((size_t)M * K + 1);
  int8_t* Bq = (int8_t*)malloc((size_t)N * K + 1);
  int32_t* acc = acc_out ? acc_out : (int32_t*)malloc((size_t)M * N * 4 + 4);
  uint16_t a_inv_h = orc_f32_to_f16(a_inv_scale); /* imma_fp8_v4.cu:38 */
  orc_quant_a(A, a_type, M, K, group, NULL, a_inv_h, Aq);
  orc_transcode_b(B, scale_u16, N, K, ORC_FMT_E4M3_REF, Bq);
  orc_gemm_s8(Aq, Bq, M, N, K, K - K % group, acc, nthreads);
  orc_epilogue(acc, scale_u16, NULL, NULL, global_scale, M, N, 0, 0, D_col);
  free(Aq);
  free(Bq);
  if (!acc_out) free(acc);
  return 0;
}

/* Extended int8-exact GEMM (the library's fp8imma_gemm_ex int8 path). */
int orc_gemm_ex(int a_type, int b_fmt, int row_quant, const void* A, const uint8_t* B,
                const uint16_t* scale_u16, const float* col_scale_f32, uint16_t* D,
                int M, int N, int K, float global_scale, float a_inv_scale,
                int out_bf16, int out_row_major, int32_t* acc_out, int nthreads) {
  int group = (a_type == ORC_A_S8) ? 16 : 8;
  int8_t* Aq = (int8_t*)malloc((size_t)M * K + 1);
  int8_t* Bq = (int8_t*)malloc((size_t)N * K + 1);
  int32_t* acc = acc_out ? acc_out : (int32_t*)malloc((size_t)M * N * 4 + 4);
  uint16_t* inv_rows = NULL;
  float* g_rows = NULL;
  if (row_quant && a_type != ORC_A_S8) {
    inv_rows = (uint16_t*)malloc((size_t)M * 2 + 2);
    g_rows = (float*)malloc((size_t)M * 4 + 4);
    orc_row_scales(A, a_type, M, K, NULL, inv_rows, g_rows);
  }
  orc_quant_a(A, a_type, M, K, group, inv_rows, orc_f32_to_f16(a_inv_scale), Aq);
  orc_transcode_b(B, scale_u16, N, K, b_fmt == ORC_FMT_E5M2 ? ORC_FMT_E5M2 : ORC_FMT_E4M3_REF, Bq);
  orc_gemm_s8(Aq, Bq, M, N, K, K - K % group, acc, nthreads);
  orc_epilogue(acc, scale_u16, col_scale_f32, g_rows, global_scale, M, N, out_bf16,
               out_row_major, D);
  free(Aq);
  free(Bq);
  free(inv_rows);
  free(g_rows);
  if (!acc_out) free(acc);
  return 0;
}

/* fp8wgt_ext (torch_ext/fp8wgt/fp8wgt_ext_cuda.cu:20-122,195-198):
 * Bdec = fp16_rn(float(lut[b]) * scale_b); C[m,n] = sum_k A*Bdec, fp32
 * accumulation (summation order differs on tensor cores: compare with a
 * tolerance). The fp8wgt LUT equals the fp8imma one on every non-NaN code. */
typedef struct {
  const uint16_t* A; const uint16_t* Bd; int M, N, K; float* C; int m0, m1;
} wgt_job;

static void* wgt_worker(void* p) {
  wgt_job* j = (wgt_job*)p;
  for (int m = j->m0; m < j->m1; ++m)
    for (int n = 0; n < j->N; ++n) {
      double s = 0.0;
      for (int k = 0; k < j->K; ++k)
        s += (double)orc_f16_to_f32(j->A[(size_t)m * j->K + k]) *
             (double)orc_f16_to_f32(j->Bd[(size_t)n * j->K + k]);
      j->C[(size_t)m * j->N + n] = (float)s;
    }
  return NULL;
}

void orc_fp8wgt(const uint16_t* A, const uint8_t* B, float scale_b, int M, int N, int K,
                float* C, int nthreads) {
  uint16_t lut[256];
  orc_lut_e4m3_ref(lut);
  uint16_t* Bd = (uint16_t*)malloc((size_t)N * K * 2 + 2);
  for (size_t i = 0; i < (size_t)N * K; ++i) {
    volatile float v = orc_f16_to_f32(lut[B[i]]) * scale_b;
    Bd[i] = orc_f32_to_f16(v);
  }
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  wgt_job jobs[256];
  int per = (M + nthreads - 1) / nthreads, started = 0;
  for (int t = 0; t < nthreads; ++t) {
    int m0 = t * per, m1 = m0 + per > M ? M : m0 + per;
    if (m0 >= m1) break;
    wgt_job j = {A, Bd, M, N, K, C, m0, m1};
    jobs[t] = j;
    pthread_create(&th[t], NULL, wgt_worker, &jobs[t]);
    started++;
  }
  for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
  free(Bd);
}

/* Native FP8 path (extension, no reference counterpart): per-row
 * s_m = absmax(to_half(a_m)) / 448 (fp32), a8 = e4m3fn_rn_satfinite(a * (448 / absmax)),
 * D = fp16/bf16( sum_k a8*b8 * s_m * col_scale[n] ), b8 decoded as hardware
 * E4M3FN or E5M2. Rows with absmax 0 give s_m = 0. */
void orc_fp8_native(int b_fmt, const void* A, int a_type, const uint8_t* B,
                    const float* col_scale_f32, int M, int N, int K, int out_bf16,
                    int out_row_major, uint16_t* D, uint8_t* Aq_out, float* row_scale_out,
                    int nthreads) {
  (void)nthreads;
  uint8_t* Aq = Aq_out ? Aq_out : (uint8_t*)malloc((size_t)M * K + 1);
  float* rs = (float*)malloc((size_t)M * 4 + 4);
  for (int m = 0; m < M; ++m) {
    float amax = 0.0f;
    for (int k = 0; k < K; ++k) {
      uint16_t h = ((const uint16_t*)A)[(size_t)m * K + k];
      if (a_type == ORC_A_BF16) h = orc_bf16_to_f16(h);
      float v = fabsf(orc_f16_to_f32(h));
      if (v > amax) amax = v;
    }
    volatile float qs = 0.0f, s = 0.0f;
    if (amax > 0.0f && isfinite(amax)) {
      volatile float c = 448.0f;
      qs = c / amax;
      s = amax / c;
    }
    rs[m] = s;
    for (int k = 0; k < K; ++k) {
      uint16_t h = ((const uint16_t*)A)[(size_t)m * K + k];
      if (a_type == ORC_A_BF16) h = orc_bf16_to_f16(h);
      volatile float v = orc_f16_to_f32(h) * qs;
      Aq[(size_t)m * K + k] = orc_f32_to_e4m3fn_sat(v);
    }
  }
  float dec[256];
  for (int b = 0; b < 256; ++b)
    dec[b] = (b_fmt == ORC_FMT_E5M2) ? orc_e5m2_to_f32((uint8_t)b) : orc_e4m3fn_to_f32((uint8_t)b);
  float adec[256];
  for (int b = 0; b < 256; ++b) adec[b] = orc_e4m3fn_to_f32((uint8_t)b);
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int k = 0; k < K; ++k)
        acc += (double)adec[Aq[(size_t)m * K + k]] * (double)dec[B[(size_t)n * K + k]];
      float v = (float)acc * rs[m] * (col_scale_f32 ? col_scale_f32[n] : 1.0f);
      uint16_t o = out_bf16 ? orc_f32_to_bf16(v) : orc_f32_to_f16(v);
      if (out_row_major) D[(size_t)m * N + n] = o;
      else D[(size_t)n * M + m] = o;
    }
  if (row_scale_out) memcpy(row_scale_out, rs, (size_t)M * 4);
  if (!Aq_out) free(Aq);
  free(rs);
}
