// fp8imma C++ API and C ABI (include/fp8imma/imma_fp8.h, fp8imma_ext.h).
//
// Host-side dispatch: validate, pick a kernel family for the shape, launch on
// the caller's stream. Mirrors the reference launchers in
// src/fp8imma/imma_fp8_v{2,3,4,4_texscale}.cu and the C wrappers in
// src/fp8imma/impl/cabi_wrappers.inl (same names, argument order, return
// codes).
#include "fp8imma/fp8imma_ext.h"
#include "fp8imma/imma_fp8.h"
#include "fp8imma_kernels.h"
#include "nvtx_range.h"

#include <algorithm>
#include <atomic>
#include <mutex>
#include <set>
#include <utility>

namespace fp8imma_b200 {

namespace {
std::atomic<int> g_splitk{0};
std::atomic<int> g_small_m_max{64};
std::atomic<int> g_pdl{1};
thread_local int t_last_path = 0;
// fp8imma_gemm_host_io on the decode path: mapped host buffers used in place
thread_local const void* t_a_host = nullptr;
thread_local void* t_d_host = nullptr;
#ifdef FP8IMMA_TRACE
unsigned long long* g_trace = nullptr;  // trace builds only
int g_dbg = 0;
#endif

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }



enum { FMT_E4M3_REF = 0, FMT_E5M2 = 1 };
}  // namespace

int api_pdl() { return g_pdl.load(); }
int api_splitk() { return g_splitk.load(); }

cudaError_t ensure_smem_attr(const void* kernel, int bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_pair(kernel, dev);
  if (done.count(key)) return cudaSuccess;
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return e;
  // the opt-in limit counts static shared memory too
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - (int)fa.sharedSizeBytes);
  if (e == cudaSuccess) done.insert(key);
  return e;
}

int num_sms_current() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

// One reference-semantics int8 GEMM. `group` is the activation load group
// of the reference variant (8 for v4, 16 for v2/v3).
static cudaError_t run_int8(GemvParams p, int a_type, int fmt, int group, cudaStream_t stream) {
  t_last_path = 0;
  if (p.M <= 0 || p.N <= 0) return cudaErrorInvalidConfiguration;
  if (p.K < 0 || !p.A || !p.B || !p.D || (!p.scale_u16 && !p.scale_tex)) return cudaErrorInvalidValue;
  p.keff_a = p.K - p.K % group;
  p.pdl = g_pdl.load();
  p.a_host = t_a_host;
  p.d_host = t_d_host;
#ifdef FP8IMMA_TRACE
  p.trace = g_trace;
  p.dbg = g_dbg;
#endif
  const bool fast_shape = p.K > 0 && (p.K % 16) == 0 && aligned16(p.A) && aligned16(p.B);
  if (fast_shape && p.M > g_small_m_max.load()) {
    ScopedScratch sc;
    cudaError_t e = sc.get(gemm_tc_scratch_bytes(p.M, p.N, p.K, false), stream, kScratchTc);
    if (e != cudaSuccess) return e;
    t_last_path = 3;
    e = launch_gemm_tc_s8(p, a_type, fmt, sc.ptr, stream);
    cudaError_t e2 = sc.release(stream);
    return e != cudaSuccess ? e : e2;
  }
  if (fast_shape) {
    const cudaError_t e = launch_gemv_s8(p, a_type, fmt, g_splitk.load(), stream);
    t_last_path = gemv_last_used_decode() ? 6 : 1;
    return e;
  }
  t_last_path = 2;
  return launch_generic_s8(p, a_type, fmt, stream);
}

static GemvParams base_params(const void* A, const void* B, const void* scales, unsigned long long tex,
                              void* D, int M, int N, int K, float global_scale, float a_inv_scale) {
  GemvParams p = {};
  p.A = A;
  p.B = static_cast<const uint8_t*>(B);
  p.scale_u16 = static_cast<const uint16_t*>(scales);
  p.scale_tex = tex;
  p.D = D;
  p.M = M;
  p.N = N;
  p.K = K;
  p.global_scale = global_scale;
  // the reference converts a_inv_scale to fp16 once on the host (imma_fp8_v4.cu:38)
  p.a_inv_h = __half_as_ushort(__float2half(a_inv_scale));
  return p;
}

static int ref_launch(int kChunk, int a_type, int group, const void* A, const void* B, const void* scales,
                      unsigned long long tex, void* D, int M, int N, int K, float gs, float ainv,
                      void* stream) {
  FP8IMMA_RANGE("fp8imma reference launcher");
  if (kChunk != 32 && kChunk != 64) return (int)cudaErrorInvalidValue;
  GemvParams p = base_params(A, B, scales, tex, D, M, N, K, gs, ainv);
  return (int)run_int8(p, a_type, FMT_E4M3_REF, group, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------- extended GEMM ----

// Native FP8 path: activations quantised per row to E4M3, weights used as raw
// E4M3FN / E5M2 bytes, fp32 accumulation, D = acc * row_scale * col_scale.
// Fused epilogue of the current fp8imma_gemm_epilogue call on this thread.
thread_local const float* t_bias = nullptr;
thread_local int t_act = 0;

static cudaError_t gemm_native(const fp8imma_gemm_args* a, cudaStream_t stream) {
  if (a->M <= 0 || a->N <= 0) return cudaErrorInvalidConfiguration;
  if (a->K <= 0 || !a->A || !a->B || !a->D || !a->col_scales_f32) return cudaErrorInvalidValue;
  if (a->a_type != FP8IMMA_A_F16 && a->a_type != FP8IMMA_A_BF16) return cudaErrorInvalidValue;
  if (a->b_format < 0 || a->b_format > 1 || a->out_type < 0 || a->out_type > 1 || a->out_layout < 0 ||
      a->out_layout > 1)
    return cudaErrorInvalidValue;
  if ((a->K % 16) != 0 || !aligned16(a->A) || !aligned16(a->B)) return cudaErrorInvalidValue;
  ScopedScratch sc;
  cudaError_t e = sc.get(gemm_tc_scratch_bytes(a->M, a->N, a->K, true), stream, kScratchTc);
  if (e != cudaSuccess) return e;
  void* scratch = sc.ptr;
  if (a->M <= g_small_m_max.load()) {
    // small M: per-row E4M3 activations, then the split-K kernel with FP8 tensor-core MMAs
    uint8_t* Aq = static_cast<uint8_t*>(scratch);
    float* rs = reinterpret_cast<float*>(Aq + (((size_t)a->M * a->K + 255) & ~size_t(255)));
    e = launch_quant_a_e4m3(a->A, a->a_type, a->M, a->K, Aq, rs, stream);
    if (e == cudaSuccess) {
      GemvParams p = {};
      p.A = Aq;
      p.B = static_cast<const uint8_t*>(a->B);
      p.D = a->D;
      p.row_g = rs;
      p.col_scale_f32 = a->col_scales_f32;
      p.M = a->M;
      p.N = a->N;
      p.K = a->K;
      p.keff_a = a->K;
      p.out_bf16 = a->out_type;
      p.out_row_major = a->out_layout;
      p.bias = t_bias;
      p.act = t_act;
      t_last_path = 5;
      p.pdl = 1;  // weights stream while the quantisation kernel finishes; rows and scales are read after it
      e = launch_gemv_s8(p, A_S8, a->b_format == FP8IMMA_B_E5M2 ? 3 : 2, g_splitk.load(), stream);
    }
  } else {
    t_last_path = 4;
    e = launch_gemm_tc_fp8(a->A, a->a_type, static_cast<const uint8_t*>(a->B), a->b_format, a->col_scales_f32,
                           a->D, a->M, a->N, a->K, a->out_type, a->out_layout, scratch, stream, t_bias, t_act);
  }
  cudaError_t e2 = sc.release(stream);
  return e != cudaSuccess ? e : e2;
}

static cudaError_t gemm_ex(const fp8imma_gemm_args* a, cudaStream_t stream) {
  t_last_path = 0;
  if (!a) return cudaErrorInvalidValue;
  if (a->path == FP8IMMA_PATH_FP8_NATIVE) return gemm_native(a, stream);
  if (a->path != FP8IMMA_PATH_INT8_EXACT) return cudaErrorInvalidValue;
  if (a->a_type < 0 || a->a_type > 2 || a->b_format < 0 || a->b_format > 1) return cudaErrorInvalidValue;
  if (a->out_type < 0 || a->out_type > 1 || a->out_layout < 0 || a->out_layout > 1) return cudaErrorInvalidValue;
  if (a->act_quant < 0 || a->act_quant > 1) return cudaErrorInvalidValue;
  if (a->act_quant == FP8IMMA_AQ_ROW && a->a_type == FP8IMMA_A_S8) return cudaErrorInvalidValue;
  GemvParams p = base_params(a->A, a->B, a->col_scales_u16, 0ull, a->D, a->M, a->N, a->K,
                             a->global_scale, a->a_inv_scale);
  p.col_scale_f32 = a->col_scales_f32;
  p.acc_out = a->acc_out;
  p.out_bf16 = a->out_type;
  p.out_row_major = a->out_layout;
  p.bias = t_bias;
  p.act = t_act;
  const int group = a->a_type == FP8IMMA_A_S8 ? 16 : 8;
  if (a->act_quant == FP8IMMA_AQ_ROW) {
    if (a->M <= 0 || a->N <= 0) return cudaErrorInvalidConfiguration;
    if (!a->A || a->K < 0) return cudaErrorInvalidValue;
    // decode shapes: row scales and quantisation in one pre-pass before the decode kernel
    if (a->K > 0 && (a->K % 16) == 0 && aligned16(a->A) && aligned16(a->B) && a->M <= g_small_m_max.load() &&
        g_splitk.load() == 0) {
      GemvParams q = p;
      q.pdl = g_pdl.load();
      if (decode_applicable(q, a->a_type, a->b_format)) {
        const cudaError_t e = launch_decode_rowquant(q, a->a_type, a->b_format, stream);
        if (e != cudaErrorNotSupported) {
          t_last_path = 6;
          return e;
        }
      }
    }
    ScopedScratch sc;
    size_t bytes = (size_t)a->M * (sizeof(float) + sizeof(uint16_t)) + 16;
    cudaError_t e = sc.get(bytes, stream, kScratchRowScales);
    if (e != cudaSuccess) return e;
    float* g = static_cast<float*>(sc.ptr);
    uint16_t* inv = reinterpret_cast<uint16_t*>(g + a->M);
    e = launch_row_scales(a->A, a->a_type, a->M, a->K, inv, g, stream);
    if (e == cudaSuccess) {
      p.row_inv_h = inv;
      p.row_g = g;
      e = run_int8(p, a->a_type, a->b_format, group, stream);
    }
    cudaError_t e2 = sc.release(stream);
    return e != cudaSuccess ? e : e2;
  }
  return run_int8(p, a->a_type, a->b_format, group, stream);
}

// Small host<->device transfers for fp8imma_gemm_host_io. A kernel that
// reads (or writes) page-locked host memory through its mapped device
// address moves a few hundred KB in a couple of microseconds and keeps the
// whole step on the compute engine; a copy-engine transfer of the same size
// costs several microseconds of engine switch and DMA set-up on each side of
// the GEMM. Pageable host memory is not device-accessible and goes through
// cudaMemcpyAsync.
__global__ void __launch_bounds__(256) copy16_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                     size_t n16) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

static const void* mapped_host_ptr(const void* p) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) return p;
  if (attr.type == cudaMemoryTypeHost && attr.devicePointer) return attr.devicePointer;
  return nullptr;  // pageable host memory
}

static cudaError_t copy_via_sm(void* dst, const void* src, size_t bytes, cudaStream_t st) {
  const void* d = mapped_host_ptr(dst);
  const void* s = mapped_host_ptr(src);
  const bool vec = d && s && ((reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(s) | bytes) & 15u) == 0;
  if (!vec) return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, st);
  const size_t n16 = bytes >> 4;
  const int grid = (int)std::min<size_t>((n16 + 255) / 256, 296);
  if (grid > 0)
    copy16_kernel<<<grid, 256, 0, st>>>(static_cast<uint4*>(const_cast<void*>(d)), static_cast<const uint4*>(s), n16);
  return cudaGetLastError();
}

}  // namespace fp8imma_b200

using namespace fp8imma_b200;

// ------------------------------------------------------------ C++ API -----
namespace fp8imma {

void init_fp8_e4m3_lut() {}

cudaError_t launch_imma_fp8_jit_v2(int kChunk, const int8_t* A, const uint8_t* B, const uint16_t* s,
                                   half* D, int M, int N, int K, float gs, cudaStream_t st) {
  return (cudaError_t)ref_launch(kChunk, A_S8, 16, A, B, s, 0ull, D, M, N, K, gs, 1.0f, st);
}
cudaError_t launch_imma_fp8_jit_v2_i8lut(int kChunk, const int8_t* A, const uint8_t* B,
                                         const uint16_t* s, half* D, int M, int N, int K, float gs,
                                         cudaStream_t st) {
  return (cudaError_t)ref_launch(kChunk, A_S8, 16, A, B, s, 0ull, D, M, N, K, gs, 1.0f, st);
}
cudaError_t launch_imma_fp8_actquant_v3_f16(int kChunk, const half* A, const uint8_t* B,
                                            const uint16_t* s, half* D, int M, int N, int K,
                                            float gs, float ainv, cudaStream_t st) {
  return (cudaError_t)ref_launch(kChunk, A_F16, 16, A, B, s, 0ull, D, M, N, K, gs, ainv, st);
}
cudaError_t launch_imma_fp8_actquant_v3_bf16(int kChunk, const __nv_bfloat16* A, const uint8_t* B,
                                             const uint16_t* s, half* D, int M, int N, int K,
                                             float gs, float ainv, cudaStream_t st) {
  return (cudaError_t)ref_launch(kChunk, A_BF16, 16, A, B, s, 0ull, D, M, N, K, gs, ainv, st);
}
cudaError_t launch_imma_fp8_actquant_v4_f16(int kChunk, const half* A, const uint8_t* B,
                                            const uint16_t* s, half* D, int M, int N, int K,
                                            float gs, float ainv, cudaStream_t st) {
  return (cudaError_t)ref_launch(kChunk, A_F16, 8, A, B, s, 0ull, D, M, N, K, gs, ainv, st);
}
cudaError_t launch_imma_fp8_actquant_v4_bf16(int kChunk, const __nv_bfloat16* A, const uint8_t* B,
                                             const uint16_t* s, half* D, int M, int N, int K,
                                             float gs, float ainv, cudaStream_t st) {
  return (cudaError_t)ref_launch(kChunk, A_BF16, 8, A, B, s, 0ull, D, M, N, K, gs, ainv, st);
}
cudaError_t launch_imma_fp8_actquant_v4_texscale_f16(int kChunk, const half* A, const uint8_t* B,
                                                     cudaTextureObject_t tex, half* D, int M, int N,
                                                     int K, float gs, float ainv, cudaStream_t st) {
  if (tex == 0) return cudaErrorInvalidValue;
  return (cudaError_t)ref_launch(kChunk, A_F16, 8, A, B, nullptr, (unsigned long long)tex, D, M, N, K,
                                 gs, ainv, st);
}
cudaError_t launch_imma_fp8_actquant_v4_texscale_bf16(int kChunk, const __nv_bfloat16* A,
                                                      const uint8_t* B, cudaTextureObject_t tex,
                                                      half* D, int M, int N, int K, float gs,
                                                      float ainv, cudaStream_t st) {
  if (tex == 0) return cudaErrorInvalidValue;
  return (cudaError_t)ref_launch(kChunk, A_BF16, 8, A, B, nullptr, (unsigned long long)tex, D, M, N, K,
                                 gs, ainv, st);
}

}  // namespace fp8imma

// --------------------------------------------------------------- C ABI -----
extern "C" {

#ifdef FP8IMMA_TRACE
void fp8imma_debug_set_trace(void* buf) { g_trace = static_cast<unsigned long long*>(buf); }
void fp8imma_debug_set_mode(int m) { g_dbg = m; }
#endif

void fp8imma_init_fp8_e4m3_lut(void) { fp8imma::init_fp8_e4m3_lut(); }

int fp8imma_launch_imma_fp8_jit_v2(int kChunk, const void* A, const void* B, const void* s, void* D,
                                   int M, int N, int K, float gs, void* stream) {
  return ref_launch(kChunk, A_S8, 16, A, B, s, 0ull, D, M, N, K, gs, 1.0f, stream);
}
int fp8imma_launch_imma_fp8_jit_v2_i8lut(int kChunk, const void* A, const void* B, const void* s,
                                         void* D, int M, int N, int K, float gs, void* stream) {
  return ref_launch(kChunk, A_S8, 16, A, B, s, 0ull, D, M, N, K, gs, 1.0f, stream);
}
int fp8imma_launch_imma_fp8_actquant_v3_f16(int kChunk, const void* A, const void* B, const void* s,
                                            void* D, int M, int N, int K, float gs, float ainv,
                                            void* stream) {
  return ref_launch(kChunk, A_F16, 16, A, B, s, 0ull, D, M, N, K, gs, ainv, stream);
}
int fp8imma_launch_imma_fp8_actquant_v3_bf16(int kChunk, const void* A, const void* B, const void* s,
                                             void* D, int M, int N, int K, float gs, float ainv,
                                             void* stream) {
  return ref_launch(kChunk, A_BF16, 16, A, B, s, 0ull, D, M, N, K, gs, ainv, stream);
}
int fp8imma_launch_imma_fp8_actquant_v4_texscale_f16(int kChunk, const void* A, const void* B,
                                                     void* tex, void* D, int M, int N, int K,
                                                     float gs, float ainv, void* stream) {
  if (!tex) return (int)cudaErrorInvalidValue;
  return ref_launch(kChunk, A_F16, 8, A, B, nullptr, (unsigned long long)(uintptr_t)tex, D, M, N, K, gs,
                    ainv, stream);
}
int fp8imma_launch_imma_fp8_actquant_v4_texscale_bf16(int kChunk, const void* A, const void* B,
                                                      void* tex, void* D, int M, int N, int K,
                                                      float gs, float ainv, void* stream) {
  if (!tex) return (int)cudaErrorInvalidValue;
  return ref_launch(kChunk, A_BF16, 8, A, B, nullptr, (unsigned long long)(uintptr_t)tex, D, M, N, K, gs,
                    ainv, stream);
}
int fp8imma_launch_imma_fp8_actquant_v4_f16(int kChunk, const void* A, const void* B, const void* s,
                                            void* D, int M, int N, int K, float gs, float ainv,
                                            void* stream) {
  return ref_launch(kChunk, A_F16, 8, A, B, s, 0ull, D, M, N, K, gs, ainv, stream);
}
int fp8imma_launch_imma_fp8_actquant_v4_bf16(int kChunk, const void* A, const void* B, const void* s,
                                             void* D, int M, int N, int K, float gs, float ainv,
                                             void* stream) {
  return ref_launch(kChunk, A_BF16, 8, A, B, s, 0ull, D, M, N, K, gs, ainv, stream);
}

int fp8imma_gemm(const fp8imma_gemm_args* args, void* stream) {
  FP8IMMA_RANGE("fp8imma_gemm");
  return (int)gemm_ex(args, static_cast<cudaStream_t>(stream));
}

int fp8imma_gemm_epilogue(const fp8imma_gemm_args* args, const float* bias, int act, void* stream) {
  if (act < 0 || act > 3) return (int)cudaErrorInvalidValue;
  t_bias = bias;
  t_act = act;
  const int r = fp8imma_gemm(args, stream);
  t_bias = nullptr;
  t_act = 0;
  return r;
}

int fp8imma_gemm_host_io(const fp8imma_gemm_args* a, const void* A_host, void* D_host, void* stream) {
  FP8IMMA_RANGE("fp8imma_gemm_host_io");
  if (!a || !A_host || !D_host || !a->A || !a->D || a->M <= 0 || a->N <= 0 || a->K <= 0)
    return (int)cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t a_bytes = (size_t)a->M * a->K * (a->a_type == FP8IMMA_A_S8 ? 1 : 2);
  const size_t d_bytes = (size_t)a->M * a->N * 2;
  // decode shapes: the activation pre-pass reads the page-locked host rows
  // and the epilogue writes the host result directly (no copy kernels); the
  // device buffers a->A and a->D are then not both used as staging (a->D
  // still receives the result, a->A is not written)
  const void* ah = mapped_host_ptr(A_host);
  void* dh = const_cast<void*>(mapped_host_ptr(D_host));
  if (ah && dh && a->path == FP8IMMA_PATH_INT8_EXACT && a->act_quant == FP8IMMA_AQ_TENSOR &&
      (a->a_type == FP8IMMA_A_F16 || a->a_type == FP8IMMA_A_BF16) && (a->b_format == 0 || a->b_format == 1) &&
      a->out_type >= 0 && a->out_type <= 1 && a->out_layout >= 0 && a->out_layout <= 1 && (a->K % 16) == 0 &&
      aligned16(a->A) && aligned16(a->B) && aligned16(ah) && a->col_scales_u16 && a->M <= g_small_m_max.load()) {
    GemvParams p = base_params(a->A, a->B, a->col_scales_u16, 0ull, a->D, a->M, a->N, a->K, a->global_scale,
                               a->a_inv_scale);
    p.out_bf16 = a->out_type;
    p.out_row_major = a->out_layout;
    if (gemv_would_decode(p, a->a_type, a->b_format, g_splitk.load()) &&
        decode_host_direct_ok(p, a->a_type, a->b_format, st)) {
      t_a_host = ah;
      t_d_host = dh;
      const int r = fp8imma_gemm(a, stream);
      t_a_host = nullptr;
      t_d_host = nullptr;
      return r;
    }
  }
  cudaError_t e = copy_via_sm(const_cast<void*>(a->A), A_host, a_bytes, st);
  if (e != cudaSuccess) return (int)e;
  int r = fp8imma_gemm(a, stream);
  if (r != 0) return r;
  return (int)copy_via_sm(D_host, a->D, d_bytes, st);
}

int fp8imma_set_splitk(int splits) {
  if (splits != 0 && splits != 1 && splits != 2 && splits != 4 && splits != 8) return (int)cudaErrorInvalidValue;
  g_splitk.store(splits);
  return 0;
}

int fp8imma_set_stream_k(int enable) {
  if (enable < 0 || enable > 2) return (int)cudaErrorInvalidValue;
  gemv_set_stream_k(enable);
  return 0;
}

int fp8imma_set_small_m_max(int m) {
  if (m < 0) return (int)cudaErrorInvalidValue;
  g_small_m_max.store(m);
  return 0;
}

int fp8imma_last_path(void) { return t_last_path; }

int fp8imma_set_tc_splitk(int splits) {
  if (splits < -1 || splits == 0 || splits > 64) return (int)cudaErrorInvalidValue;
  tc_set_splitk(splits);
  return 0;
}

int fp8imma_set_tc_tile_x(int rows) {
  if (rows != 0 && rows != 128 && rows != 192 && rows != 256) return (int)cudaErrorInvalidValue;
  tc_set_tile_x(rows);
  return 0;
}

int fp8imma_set_tc_half_tail(int enable) {
  if (enable != 0 && enable != 1) return (int)cudaErrorInvalidValue;
  tc_set_half_tail(enable != 0);
  return 0;
}

int fp8imma_set_tc_pair(int enable) {
  tc_set_pair_mode(enable != 0);
  return 0;
}

int fp8imma_set_decode_kernel(int enable) {
  if (enable < 0 || enable > 2) return (int)cudaErrorInvalidValue;
  decode_set_mode(enable);
  return 0;
}

int fp8imma_set_pdl(int enable) {
  g_pdl.store(enable ? 1 : 0);
  return 0;
}

unsigned int fp8imma_device_error(int clear) {
  return gemv_device_error(clear != 0) | decode_device_error(clear != 0) | tc_device_error(clear != 0) |
         peer_device_error(clear != 0);
}

int fp8imma_set_wait_limit_ns(unsigned long long ns) {
  if (ns == 0) return (int)cudaErrorInvalidValue;
  cudaError_t e = gemv_set_wait_limit(ns);
  if (e == cudaSuccess) e = decode_set_wait_limit(ns);
  if (e == cudaSuccess) e = tc_set_wait_limit(ns);
  if (e == cudaSuccess) e = peer_set_wait_limit(ns);
  return (int)e;
}

const char* fp8imma_version(void) { return "fp8imma-b200 0.1 (sm_100a)"; }

}  // extern "C"
