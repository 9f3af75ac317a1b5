// Column-parallel GEMM with the output gather done by this library over
// NVLink (no NCCL): entry point and gather kernel.
//
// fp8imma_gemm_allgather runs the small-M split-K GEMM for this rank's weight
// shard straight into its rows of its own full output buffer, then one gather
// kernel: every CTA copies a slice of those rows into every peer's buffer with
// 16-byte stores and publishes it with one system-scope release increment of
// a counter in that peer's signal pad; CTA 0 then waits until every peer's
// counter in this rank's pad has reached this call's target. Plain loads and
// stores to peer memory only (no multicast objects, no TMA on peer memory, no
// NCCL). Waits are bounded: on timeout a code is recorded and the kernel ends.
#include "fp8imma/fp8imma_ext.h"
#include "fp8imma_kernels.h"
#include "nvtx_range.h"

#include <cuda_fp16.h>

namespace fp8imma_b200 {
namespace {

static __device__ unsigned int g_peer_error;
bool g_fused_gather = false;  // gather in the GEMM epilogue (else, default, a separate gather kernel)
static __device__ unsigned long long g_peer_wait_ns = 2000000000ull;  // fp8imma_set_wait_limit_ns
constexpr int kEpochSlot = kPeerEpochSlot;  // per-rank call counter (device-side epoch) in each rank's own pad
constexpr int kGatherBlocks = 32;
constexpr int kGatherThreads = 256;

struct Ptrs8 {
  unsigned long long p[8];
};

// (__grid_constant__: the pointer tables are indexed at run time and read in
// place from parameter space instead of being copied to a local stack)
__global__ void __launch_bounds__(kGatherThreads) peer_gather_kernel(const __grid_constant__ Ptrs8 outs,
                                                                     const __grid_constant__ Ptrs8 pads, int world, int rank,
                                                                     unsigned long long byte0, unsigned long long nbytes,
                                                                     unsigned int epoch_arg) {
  // launched as a programmatic dependent of the GEMM: the next call's kernels
  // may start (they wait for this grid before touching its buffers), and this
  // grid waits for the GEMM's rows before copying them
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // 1. copy this rank's rows to every peer (grid-strided). byte0 = rank * N *
  //    M * 2 is only as aligned as N * M allows, so 16-byte granules are used
  //    only when both addresses are 16-byte aligned (all ranks' buffers share
  //    one alignment), else 4- or 2-byte ones.
  const uint8_t* src = reinterpret_cast<const uint8_t*>(outs.p[rank]) + byte0;
  const unsigned long long tid = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
  const unsigned long long nthr = (unsigned long long)gridDim.x * blockDim.x;
  for (int r = 1; r < world; ++r) {
    const int peer = (rank + r) % world;  // stagger destinations across ranks
    uint8_t* dst = reinterpret_cast<uint8_t*>(outs.p[peer]) + byte0;
    const uintptr_t al = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst);
    unsigned long long done = 0;
    if ((al & 15u) == 0) {
      const unsigned long long n16 = nbytes >> 4;
      for (unsigned long long i = tid; i < n16; i += nthr)
        reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
      done = n16 << 4;
    } else if ((al & 3u) == 0) {
      const unsigned long long n4 = nbytes >> 2;
      for (unsigned long long i = tid; i < n4; i += nthr)
        reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
      done = n4 << 2;
    }
    for (unsigned long long i = done + tid; i < nbytes; i += nthr) dst[i] = src[i];
  }
  __syncthreads();
  // 2. publish: one release increment per peer (cumulative over this CTA's
  //    stores, which the CTA barrier ordered before it)
  if (threadIdx.x < world && (int)threadIdx.x != rank) {
    unsigned int* slot = reinterpret_cast<unsigned int*>(pads.p[threadIdx.x]) + rank;
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(slot) : "memory");
  }
  if (blockIdx.x != 0) return;
  // 3. CTA 0 waits until every peer has published all of its CTAs for this call
  __shared__ unsigned int target_s;
  if (threadIdx.x == 0) {
    unsigned int e = epoch_arg;
    if (e == 0) {  // epoch counted on the device: advances on every launch, also on graph replays
      unsigned int* ctr = reinterpret_cast<unsigned int*>(pads.p[rank]) + kEpochSlot;
      e = *ctr + 1;
      *ctr = e;
    }
    target_s = e * gridDim.x;
  }
  __syncthreads();
  const unsigned int target = target_s;
  if (threadIdx.x < world && (int)threadIdx.x != rank) {
    const unsigned int* mine = reinterpret_cast<const unsigned int*>(pads.p[rank]) + threadIdx.x;
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int)(v - target) >= 0) break;
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (now - t0 > 1000000ull && now - t0 > *(volatile unsigned long long*)&g_peer_wait_ns) {  // read only after 1 ms
        atomicCAS(&g_peer_error, 0u, 5u);
        break;
      }
    }
  }
  __syncthreads();
}

}  // namespace

cudaError_t launch_peer_gather(const unsigned long long* outs, const unsigned long long* pads, int world, int rank,
                               size_t row0, size_t rows, int M, unsigned int epoch, bool pdl, cudaStream_t stream) {
  Ptrs8 o = {}, s = {};
  for (int i = 0; i < world; ++i) {
    o.p[i] = outs[i];
    s.p[i] = pads[i];
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(kGatherBlocks, 1, 1);
  lc.blockDim = dim3(kGatherThreads, 1, 1);
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&lc, peer_gather_kernel, o, s, world, rank, (unsigned long long)(row0 * M * 2),
                            (unsigned long long)(rows * M * 2), epoch);
}

cudaError_t peer_set_wait_limit(unsigned long long ns) { return cudaMemcpyToSymbol(g_peer_wait_ns, &ns, sizeof(ns)); }

unsigned int peer_device_error(bool clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_peer_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_peer_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace fp8imma_b200

using namespace fp8imma_b200;

extern "C" int fp8imma_set_fused_gather(int enable) {
  if (enable != 0 && enable != 1) return (int)cudaErrorInvalidValue;
  g_fused_gather = enable != 0;
  return 0;
}

extern "C" int fp8imma_gemm_allgather(const fp8imma_gemm_args* a, void* const* peer_out, void* const* peer_signal,
                                      int world, int rank, unsigned int epoch, void* stream) {
  FP8IMMA_RANGE("fp8imma_gemm_allgather");
  if (!a || !peer_out || !peer_signal || world < 1 || world > 8 || rank < 0 || rank >= world)
    return (int)cudaErrorInvalidValue;
  if (a->path != FP8IMMA_PATH_INT8_EXACT || a->act_quant != FP8IMMA_AQ_TENSOR || a->out_layout != FP8IMMA_OUT_COL)
    return (int)cudaErrorInvalidValue;
  if (a->a_type < 0 || a->a_type > 2 || a->b_format < 0 || a->b_format > 1 || a->out_type < 0 || a->out_type > 1)
    return (int)cudaErrorInvalidValue;
  if (a->M <= 0 || a->N <= 0) return (int)cudaErrorInvalidConfiguration;
  if (!a->A || !a->B || !a->col_scales_u16 || a->K <= 0 || (a->K % 16) != 0 ||
      (reinterpret_cast<uintptr_t>(a->A) & 15u) || (reinterpret_cast<uintptr_t>(a->B) & 15u))
    return (int)cudaErrorInvalidValue;
  unsigned long long outs[8], pads[8];
  for (int r = 0; r < world; ++r) {
    if (!peer_out[r] || !peer_signal[r]) return (int)cudaErrorInvalidValue;
    outs[r] = reinterpret_cast<unsigned long long>(peer_out[r]);
    pads[r] = reinterpret_cast<unsigned long long>(peer_signal[r]);
  }
  GemvParams p = {};
  p.A = a->A;
  p.B = static_cast<const uint8_t*>(a->B);
  p.scale_u16 = static_cast<const uint16_t*>(a->col_scales_u16);
  p.D = static_cast<uint16_t*>(peer_out[rank]) + (size_t)rank * a->N * a->M;  // this rank's rows
  p.acc_out = a->acc_out;
  p.col_scale_f32 = a->col_scales_f32;
  p.M = a->M;
  p.N = a->N;
  p.K = a->K;
  p.keff_a = a->K;
  p.global_scale = a->global_scale;
  p.a_inv_h = __half_as_ushort(__float2half(a->a_inv_scale));
  p.out_bf16 = a->out_type;
  p.pdl = api_pdl();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (world > 1 && g_fused_gather) {
    // the split-K kernel's epilogue writes into every peer's output and
    // signals; its first CTA waits for the peers (no separate gather kernel)
    p.world = world;
    p.rank = rank;
    p.epoch = epoch;
    for (int r = 0; r < world; ++r) {
      p.peer_rows[r] = outs[r] + (unsigned long long)rank * a->N * a->M * 2;
      p.peer_sig[r] = pads[r];
    }
    return (int)launch_gemv_s8(p, a->a_type, a->b_format, 0, st);
  }
  cudaError_t e = launch_gemv_s8(p, a->a_type, a->b_format, 0, st);
  if (e != cudaSuccess) return (int)e;
  if (world == 1) return 0;
  return (int)launch_peer_gather(outs, pads, world, rank, (size_t)rank * a->N, (size_t)a->N, a->M, epoch, p.pdl != 0,
                                 st);
}
