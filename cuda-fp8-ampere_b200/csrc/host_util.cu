// Host helpers: TMA tensor-map encoding through the driver entry point (no
// link-time dependency on libcuda), device-error readout.
#include "fp8imma_kernels.h"

#include <cuda.h>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

namespace fp8imma_b200 {

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
}
}  // namespace

// 2-D byte tensor [outer][inner] with row pitch `row_bytes`, box {box_inner, box_outer}.
cudaError_t make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                            uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (row_bytes & 15u)) return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Per-(device, stream, tag) scratch buffers, allocated on first use and grown
// when a larger one is asked for; a buffer is handed only to work on its own
// stream, so stream order keeps calls from overlapping on it. Buffers are
// never freed (a replaced one may still be referenced by a captured graph).
namespace {
std::mutex g_scratch_mu;
std::map<std::tuple<int, cudaStream_t, int>, std::pair<void*, size_t>> g_scratch;
std::vector<void*> g_scratch_retired;
}  // namespace

bool stream_scratch_ready(cudaStream_t stream, size_t bytes, int tag) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  auto it = g_scratch.find(std::make_tuple(dev, stream, tag));
  return it != g_scratch.end() && it->second.second >= bytes;
}

void* stream_scratch(cudaStream_t stream, size_t bytes, int tag, bool* fresh) {
  if (fresh) *fresh = false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  auto key = std::make_tuple(dev, stream, tag);
  auto it = g_scratch.find(key);
  if (it != g_scratch.end() && it->second.second >= bytes) return it->second.first;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;  // no allocation while a graph is being captured
  }
  size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
  void* p = nullptr;
  if (cudaMalloc(&p, want) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cudaMemset(p, 0, want) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    cudaGetLastError();
    return nullptr;
  }
  if (fresh) *fresh = true;
  if (it != g_scratch.end()) {
    g_scratch_retired.push_back(it->second.first);
    it->second = std::make_pair(p, want);
  } else {
    g_scratch.emplace(key, std::make_pair(p, want));
  }
  return p;
}

}  // namespace fp8imma_b200
