// Allocation-free variant of the per-row-quantised int8-exact GEMM.
//
// fp8imma_gemm with act_quant = FP8IMMA_AQ_ROW needs a little device memory
// between its two kernels: the per-row activation multiplier (fp16) and the
// per-row output scale (fp32) that the row-scale kernel writes and the GEMM
// kernel reads. fp8imma_gemm takes it from the stream-ordered allocator.
// Some callers cannot allow that: runtimes that reserve nearly all of HBM for
// their own pool up front (a driver allocation may then fail), serving loops
// that forbid allocation on the request path (a driver allocation can block
// or synchronise), and plugin hosts whose contract hands the plugin only
// caller-owned input and output buffers. fp8imma_gemm_rowquant_noalloc serves
// them: the per-row values live in the fixed array below, which every GPU
// that loads this library holds until the process exits.
#include "fp8imma/fp8imma_ext.h"
#include "fp8imma_kernels.h"
#include "nvtx_range.h"

#include <mutex>

namespace fp8imma_b200 {
namespace {

constexpr int kMaxRows = FP8IMMA_NOALLOC_MAX_M;
// rows x (fp32 output scale + fp16 multiplier), rounded to 256-byte blocks
constexpr size_t kScratchBytes = ((size_t)kMaxRows * (sizeof(float) + sizeof(uint16_t)) + 255) & ~size_t(255);

static __device__ __align__(256) unsigned char g_rowquant_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device. The host-side
// name g_rowquant_scratch is only a stand-in, never a device address; the real
// address is looked up once per device (with that device current) and cached.
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rowquant_scratch);
    if (e != cudaSuccess) return e;
    if (!p) return cudaErrorInvalidSymbol;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace fp8imma_b200

using namespace fp8imma_b200;

extern "C" int fp8imma_gemm_rowquant_noalloc(const fp8imma_gemm_args* a, void* stream) {
  FP8IMMA_RANGE("fp8imma_gemm_rowquant_noalloc");
  if (!a) return (int)cudaErrorInvalidValue;
  if (a->path != FP8IMMA_PATH_INT8_EXACT || a->act_quant != FP8IMMA_AQ_ROW) return (int)cudaErrorInvalidValue;
  if (a->a_type != FP8IMMA_A_F16 && a->a_type != FP8IMMA_A_BF16) return (int)cudaErrorInvalidValue;
  if (a->b_format < 0 || a->b_format > 1 || a->out_type < 0 || a->out_type > 1 || a->out_layout < 0 ||
      a->out_layout > 1)
    return (int)cudaErrorInvalidValue;
  if (a->M <= 0 || a->N <= 0) return (int)cudaErrorInvalidConfiguration;
  if (a->M > FP8IMMA_NOALLOC_MAX_M) return (int)cudaErrorInvalidValue;  // more rows than the fixed array holds
  if (a->K < 0 || !a->A || !a->B || !a->D || !a->col_scales_u16) return (int)cudaErrorInvalidValue;

  void* base = nullptr;
  cudaError_t e = scratch_for_current_device(&base);
  if (e != cudaSuccess) return (int)e;
  float* g = static_cast<float*>(base);
  uint16_t* inv = reinterpret_cast<uint16_t*>(g + FP8IMMA_NOALLOC_MAX_M);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // Both kernels run on the caller's stream: the row-scale kernel overwrites
  // rows [0, M) of the array before the GEMM reads them, so nothing has to be
  // cleared between calls.
  e = launch_row_scales(a->A, a->a_type, a->M, a->K, inv, g, st);
  if (e != cudaSuccess) return (int)e;

  GemvParams p = {};
  p.A = a->A;
  p.B = static_cast<const uint8_t*>(a->B);
  p.scale_u16 = static_cast<const uint16_t*>(a->col_scales_u16);
  p.D = a->D;
  p.acc_out = a->acc_out;
  p.row_inv_h = inv;
  p.row_g = g;
  p.col_scale_f32 = a->col_scales_f32;
  p.M = a->M;
  p.N = a->N;
  p.K = a->K;
  p.keff_a = a->K - a->K % 8;
  p.global_scale = a->global_scale;
  p.out_bf16 = a->out_type;
  p.out_row_major = a->out_layout;
  const bool fast = a->K > 0 && (a->K % 16) == 0 && (reinterpret_cast<uintptr_t>(a->A) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(a->B) & 15u) == 0;
  p.no_alloc = 1;       // no pre-pass and no stream-K scratch (both allocate)
  p.pdl = api_pdl();    // the process-wide knobs apply here as in fp8imma_gemm
  if (fast) return (int)launch_gemv_s8(p, a->a_type, a->b_format, api_splitk(), st);
  return (int)launch_generic_s8(p, a->a_type, a->b_format, st);
}
