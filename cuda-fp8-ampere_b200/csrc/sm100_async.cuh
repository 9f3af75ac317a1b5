// sm_100a asynchronous-copy / barrier / tensor-memory primitives (inline PTX).
//
// Every wait here is bounded: after kWaitLimitNs a wait gives up, records
// an error code in the device-global error word (read back by
// fp8imma_device_error()) and returns false, so a broken pipeline ends the
// kernel instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace fp8imma_dev {

// Error word: one per translation unit and device; each kernel file exposes
// it to the host through a small accessor (see fp8imma_kernels.h).
static __device__ unsigned int g_fp8imma_device_error;

enum : unsigned int {
  ERR_WAIT_FULL = 1u,
  ERR_WAIT_EMPTY = 2u,
  ERR_WAIT_TMEM_FULL = 3u,
  ERR_WAIT_TMEM_EMPTY = 4u,
  ERR_WAIT_PEER = 5u,  // a peer GPU's gather signal did not arrive
};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any healthy wait
constexpr unsigned long long kWaitCheckNs = 1000000ull;     // 1 ms: waits shorter than this never read the limit

// The limit the waits use; kWaitLimitNs unless the host changed it
// (fp8imma_set_wait_limit_ns). One per translation unit and device, like the
// error word.
static __device__ unsigned long long g_fp8imma_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// kSuspend: let the hardware park the waiting thread until the phase
// completes (or a time hint passes) instead of returning at once; the
// tensor-core GEMMs, whose epilogue and producer warps wait through whole
// tiles, use it so that those waits do not spin.
template <bool kSuspend = false>
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if (kSuspend) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000000;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  }
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete: gives up
// after the wait limit (2 s unless changed) of wall time, records err_code and returns false.
template <bool kSuspend = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int err_code) {
  if (mbar_try_wait<kSuspend>(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned int i = 1;; ++i) {
    if (mbar_try_wait<kSuspend>(bar, parity)) return true;
    const unsigned long long dt = globaltimer_ns() - t0;
    // the limit (a global load) is read only once a wait has lasted 1 ms,
    // which no healthy wait does: limits below 1 ms act as 1 ms
    if (dt > kWaitCheckNs && dt > *(volatile unsigned long long*)&g_fp8imma_wait_limit_ns) break;
  }
  atomicCAS(&g_fp8imma_device_error, 0u, err_code);
  return false;
}

// 2-D tiled TMA load (no multicast) into this CTA's shared memory,
// completing transaction bytes on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// AND-reduction of `pred` over `count` threads at named barrier `id`
__device__ __forceinline__ bool named_bar_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %3, 0;\n\t"
      "barrier.red.and.pred q, %1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(count), "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

// Programmatic dependent launch: let the next grid in the stream start, and
// wait until the previous grid's memory operations are visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// named barrier among `count` threads (ids 1..15; 0 is __syncthreads)
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Host side, per translation unit (internal linkage: each kernel file reads
// and sets its own copies of the device words on the current device).
static inline unsigned int tu_device_error(bool clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fp8imma_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_fp8imma_device_error, &z, sizeof(z));
  }
  return v;
}
static inline cudaError_t tu_set_wait_limit(unsigned long long ns) {
  return cudaMemcpyToSymbol(g_fp8imma_wait_limit_ns, &ns, sizeof(ns));
}

}  // namespace fp8imma_dev
