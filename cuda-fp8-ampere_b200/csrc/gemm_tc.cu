// Large-M GEMM on the 5th-generation tensor cores (tcgen05, TMEM), sm_100a.
//
// Two paths share one persistent, warp-specialised kernel:
//   * int8-exact (kind::i8, s32 accumulators in TMEM): activations and
//     weights are first turned into int8 by two HBM-streaming prep kernels
//     using exactly the reference rounding chain (fp8imma_device.cuh), then
//     contracted. The int32 sums are exact, so the result equals the
//     reference (src/fp8imma/impl/v4_kernels.inl) bit for bit.
//   * native FP8 (kind::f8f6f4, f32 accumulators): weights are the raw
//     E4M3/E5M2 bytes (no transcode), activations are quantised per row to
//     E4M3 by the prep kernel.
// The GEMM computes D^T = W * X^T: the MMA's M side is 128 weight columns
// (TMEM lanes), its N side 256 activation rows (TMEM columns), so each
// epilogue thread owns one output column n and writes a contiguous run of
// D[n*M + m] (the reference's col-major output).
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2-5 epilogue. 4-stage smem ring of {16 KB weights, 32 KB
// activations} (128-byte swizzle, K-major UMMA descriptors), two 256-column
// TMEM accumulators so the epilogue of one tile overlaps the MMAs of the next.
// All waits are bounded (sm100_async.cuh).
#include "fp8imma_device.cuh"
#include "fp8imma_kernels.h"
#include "sm100_async.cuh"
#include "sm100_umma.cuh"

#include <algorithm>

using namespace fp8imma_dev;

// tensor-core GEMM waits park the thread (see mbar_try_wait)
#ifndef FP8IMMA_TC_SUSPEND
#define FP8IMMA_TC_SUSPEND 1
#endif
constexpr bool kTcSuspend = FP8IMMA_TC_SUSPEND != 0;

namespace fp8imma_b200 {
#ifdef FP8IMMA_TRACE
static unsigned long long* g_tc_trace = nullptr;  // trace builds only
#endif

namespace {

constexpr int kTileW = 128;  // weight columns per tile (MMA M)
constexpr int kTileX = 256;  // activation rows per tile (MMA N)
constexpr int kBK = 128;     // K bytes per stage
constexpr int kStages = 4;
constexpr int kBytesW = kTileW * kBK;
constexpr int kBytesX = kTileX * kBK;
constexpr int kStageBytes = kBytesW + kBytesX;
constexpr int kThreadsTC = 192;
constexpr int kTmemCols = 512;

enum { KIND_I8 = 0, KIND_F8 = 1, KIND_F16 = 2 };  // KIND_F16: fp8wgt (fp16 x fp16 -> fp32, CTA-pair kernel only)

// ---------------------------------------------------------------- tcgen05 --

template <int KIND>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  if (KIND == KIND_I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
  }
}

// Instruction descriptor: M=128, N=256, K-major A and B.
template <int KIND>
__host__ __device__ constexpr uint32_t make_idesc(int a_fmt) {
  // c_format [4,6): 1 = F32, 2 = S32; a_format [7,10); b_format [10,13);
  // n_dim [17,23) = N>>3; m_dim [24,29) = M>>4
  return (KIND == KIND_I8 ? (2u << 4) | (1u << 7) | (1u << 10) : (1u << 4) | ((uint32_t)a_fmt << 7) | (0u << 10)) |
         ((uint32_t)(kTileX >> 3) << 17) | ((uint32_t)(kTileW >> 4) << 24);
}

struct TcParams {
  int M, N, K;
  int tiles_w, tiles_x;
  uint32_t idesc;
  const uint16_t* scale_u16;       // int8 path: reference column scales (fp16 bits)
  unsigned long long scale_tex;    // or a texture over them
  const float* col_scale_f32;      // optional fp32 column multiplier (native path: weight scale)
  const float* row_g;              // per-row global scale (row quant / native row scale) or null
  float global_scale;
  void* D;
  int32_t* acc_out;
  int out_bf16, out_row_major;
  const float* bias;   // optional fused epilogue (bias_act)
  int act;
  int tile_x;          // CTA-pair kernel: activation rows per tile (256, 192 or 128; MMA N)
  int n_full;          // CTA-pair kernel: tiles run at full width; the rest run as two half-width items
  uint32_t idesc_half; // instruction descriptor of the half-width items (N = tile_x / 2)
  int splits;          // CTA-pair kernel: K splits per tile (1 = none)
  int kb_per_split;    // 128-byte K blocks per split
  uint32_t* ws;        // splits > 1: raw accumulators [split][n][m] (int32 or fp32 bits)
  int tma_out;         // CTA-pair kernel: col-major 16-bit output written by TMA stores (mapD)
  int pdl;             // CTA-pair kernel launched as a programmatic dependent of the prep kernels
  unsigned long long* trace;  // trace builds only: 64 words per CTA
};

// Epilogue of 32 accumulators (rows mbase .. mbase + 31 of weight column n):
// scale, optional bias and activation, round to fp16 / bf16 and pack pairs.
// Every decision (row scales, column scale, bias, activation, output type)
// is uniform over the kernel, so each is taken once per 32 values rather
// than per value: per-value branches, with the activations' tanhf / expf
// inlined 32 times, made this loop cost more than the matrix product.
// Arithmetic per value is unchanged: se = (cs * g) * cs2, v = acc * se
// (int8 path) or v = (acc * g) * cs2 (fp32 path); v + bias rounded; act.
template <int KIND>
__device__ __forceinline__ void tc_epi_pack(const uint32_t (&r)[32], int mbase, float cs, float cs2, const TcParams& p,
                                            int nb, uint32_t (&pk)[16]) {
  float v[32];
  const float c2 = p.col_scale_f32 ? cs2 : 1.0f;
  if (p.row_g) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int m = mbase + j;
      const float g = p.row_g[m < p.M ? m : 0];
      if (KIND == KIND_I8)
        v[j] = (float)(int32_t)r[j] * ((cs * g) * c2);
      else
        v[j] = __uint_as_float(r[j]) * g * cs2;
    }
  } else {
    const float se = (cs * p.global_scale) * c2;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = KIND == KIND_I8 ? (float)(int32_t)r[j] * se : __uint_as_float(r[j]) * cs2;
  }
  if (p.bias) {
    const float b = p.bias[nb];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], b);
  }
  if (p.act == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = bias_act(v[j], nullptr, 0, 1);
  } else if (p.act == 2) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = bias_act(v[j], nullptr, 0, 2);
  } else if (p.act == 3) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = bias_act(v[j], nullptr, 0, 3);
  }
  if (p.out_bf16) {
#pragma unroll
    for (int w = 0; w < 16; ++w) pk[w] = (uint32_t)store_val(v[2 * w], 1) | ((uint32_t)store_val(v[2 * w + 1], 1) << 16);
  } else {
#pragma unroll
    for (int w = 0; w < 16; ++w) pk[w] = (uint32_t)store_val(v[2 * w], 0) | ((uint32_t)store_val(v[2 * w + 1], 0) << 16);
  }
}

template <int KIND>
__global__ void __launch_bounds__(kThreadsTC, 1)
    gemm_tc_kernel(const __grid_constant__ TcParams p, const __grid_constant__ CUtensorMap mapW,
                   const __grid_constant__ CUtensorMap mapX) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.tiles_w * p.tiles_x;
  const int nkb = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&mapW);
      prefetch_tensormap(&mapX);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int tw = tile % p.tiles_w, tx = tile / p.tiles_w;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!(ok = mbar_wait<kTcSuspend>(&empty[stage], phase ^ 1u, ERR_WAIT_EMPTY))) break;
          uint8_t* sw = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(sw, &mapW, &full[stage], kb * kBK, tw * kTileW);
          tma_load_2d(sw + kBytesW, &mapX, &full[stage], kb * kBK, tx * kTileX);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // drain: every load issued must have landed before the CTA may exit
      for (int s = 0; s < kStages && ok; ++s) {
        // the last use of each stage is observed by the MMA issuer; waiting on
        // its release here guarantees the bytes arrived and were consumed
        ok = mbar_wait<kTcSuspend>(&empty[stage], phase ^ 1u, ERR_WAIT_EMPTY);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        if (!(ok = mbar_wait<kTcSuspend>(&tempty[buf], ((it >> 1) & 1) ^ 1u, ERR_WAIT_TMEM_EMPTY))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kTileX);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!(ok = mbar_wait<kTcSuspend>(&full[stage], phase, ERR_WAIT_FULL))) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint64_t adesc = sw128_desc(sa), bdesc = sw128_desc(sa + kBytesW);
#pragma unroll
          for (int j = 0; j < kBK / 32; ++j)
            umma<KIND>(d_tmem, adesc + 2 * j, bdesc + 2 * j, p.idesc, (kb | j) != 0);
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit(&tfull[buf]);
      }
      umma_commit(drain);
      mbar_wait<kTcSuspend>(drain, 0, ERR_WAIT_FULL);
    }
  } else {
    // ------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const int tw = tile % p.tiles_w, tx = tile / p.tiles_w;
      if (!mbar_wait<kTcSuspend>(&tfull[buf], (it >> 1) & 1, ERR_WAIT_TMEM_FULL)) break;
      tc_fence_after();
      const int n = tw * kTileW + q * 32 + lane;
      const bool nok = n < p.N;
      float cs = 1.0f;
      if (nok) {
        if (KIND == KIND_I8) {
          uint16_t sb = p.scale_tex ? tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n) : p.scale_u16[n];
          cs = __half2float(__ushort_as_half(sb));
        }
      }
      const float cs2 = (nok && p.col_scale_f32) ? p.col_scale_f32[n] : 1.0f;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kTileX);
      uint16_t* D = static_cast<uint16_t*>(p.D);
#pragma unroll 1
      for (int j0 = 0; j0 < kTileX; j0 += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + j0, r);
        const int mbase = tx * kTileX + j0;
        if (!nok || mbase >= p.M) continue;
        uint32_t pk[16];
        tc_epi_pack<KIND>(r, mbase, cs, cs2, p, n, pk);
        uint16_t o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = (uint16_t)(pk[j >> 1] >> (16 * (j & 1)));
        const int mcount = min(32, p.M - mbase);
        if (p.out_row_major) {
          _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mcount) D[(size_t)(mbase + j) * p.N + n] = o[j];
        } else {
          uint16_t* dst = D + (size_t)n * p.M + mbase;
          if (mcount == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              uint4 w;
              w.x = (uint32_t)o[8 * v4 + 0] | ((uint32_t)o[8 * v4 + 1] << 16);
              w.y = (uint32_t)o[8 * v4 + 2] | ((uint32_t)o[8 * v4 + 3] << 16);
              w.z = (uint32_t)o[8 * v4 + 4] | ((uint32_t)o[8 * v4 + 5] << 16);
              w.w = (uint32_t)o[8 * v4 + 6] | ((uint32_t)o[8 * v4 + 7] << 16);
              reinterpret_cast<uint4*>(dst)[v4] = w;
            }
          } else {
            _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mcount) dst[j] = o[j];
          }
        }
        if (KIND == KIND_I8 && p.acc_out) {
          _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mcount) p.acc_out[(size_t)n * p.M + mbase + j] = (int32_t)r[j];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------ prep kernels --

// Activations -> int8 with the reference rounding (per-tensor or per-row
// multiplier), 8 elements per thread-iteration. K % 8 == 0.
template <int AT>
__global__ void __launch_bounds__(256) quant_a_s8_kernel(const void* __restrict__ A, int M, int K, uint16_t a_inv_h,
                                                         const uint16_t* __restrict__ row_inv_h, int8_t* __restrict__ Aq,
                                                         int after_prev) {
  // the GEMM that consumes these rows may be launched as a programmatic
  // dependent: it sets itself up now and waits for this grid
  // (griddepcontrol.wait) before it reads the quantised rows
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const size_t total = (size_t)M * (K >> 3);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = i << 3;
    const int m = (int)(e / K);
    uint2 out;
    if (AT == A_S8) {
      out = reinterpret_cast<const uint2*>(A)[i];
    } else {
      uint4 v = reinterpret_cast<const uint4*>(A)[i];
      const uint16_t ainv = row_inv_h ? row_inv_h[m] : a_inv_h;
      const uint32_t ainv2 = (uint32_t)ainv | ((uint32_t)ainv << 16);
      if (AT == A_BF16) {
        v.x = bf16x2_to_f16x2(v.x);
        v.y = bf16x2_to_f16x2(v.y);
        v.z = bf16x2_to_f16x2(v.z);
        v.w = bf16x2_to_f16x2(v.w);
      }
      out.x = quant4_f16(v.x, v.y, ainv2);
      out.y = quant4_f16(v.z, v.w, ainv2);
    }
    reinterpret_cast<uint2*>(Aq)[i] = out;
  }
  // launched as a programmatic dependent of the weight transcode (which it
  // overlaps): finish only after that grid, so that a kernel waiting for this
  // one also waits for the transcode
  if (after_prev) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// FP8 weights -> int8 with the reference chain. One warp per weight row at a
// time (the column's inverse scale is formed once per row), each lane
// transcoding 16 contiguous bytes of every 512-byte step, two steps in
// flight. K % 16 == 0.
template <int FMT>
__global__ void __launch_bounds__(256) transcode_b_kernel(const uint8_t* __restrict__ B, int N, int K,
                                                          const uint16_t* __restrict__ scale_u16,
                                                          unsigned long long scale_tex, int8_t* __restrict__ Bq) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the activation quantisation may run alongside
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int k16 = K >> 4;  // 16-byte vectors per row
  for (int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
    const uint16_t sb = scale_tex ? tex1Dfetch<unsigned short>((cudaTextureObject_t)scale_tex, n) : scale_u16[n];
    const uint16_t inv = inv_scale_bits(sb);
    const bool fast = fast_ok<FMT>(inv);
    const uint32_t fs = fast_scale<FMT>(inv);
    const uint4* src = reinterpret_cast<const uint4*>(B + (size_t)n * K);
    uint4* dst = reinterpret_cast<uint4*>(Bq + (size_t)n * K);
    for (int v0 = lane; v0 < k16; v0 += 64) {
      uint4 v[2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
        if (v0 + 32 * j < k16) v[j] = ldg_stream_v4(src + v0 + 32 * j);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (v0 + 32 * j >= k16) continue;
        uint4 o;
        if (fast) {
          if (FMT == FMT_E5M2) {
            o.x = transcode4_fast_e5m2(v[j].x, fs);
            o.y = transcode4_fast_e5m2(v[j].y, fs);
            o.z = transcode4_fast_e5m2(v[j].z, fs);
            o.w = transcode4_fast_e5m2(v[j].w, fs);
          } else {
            o.x = transcode4_fast_e4m3(v[j].x, fs);
            o.y = transcode4_fast_e4m3(v[j].y, fs);
            o.z = transcode4_fast_e4m3(v[j].z, fs);
            o.w = transcode4_fast_e4m3(v[j].w, fs);
          }
        } else {
          o.x = transcode4_exact<FMT>(v[j].x, inv);
          o.y = transcode4_exact<FMT>(v[j].y, inv);
          o.z = transcode4_exact<FMT>(v[j].z, inv);
          o.w = transcode4_exact<FMT>(v[j].w, inv);
        }
        dst[v0 + 32 * j] = o;
      }
    }
  }
}

// Native path: per-row E4M3 quantisation. One CTA (256 threads) per row:
// absmax over to_half(a), row scale s = absmax/448, a8 = e4m3_rn_satfinite(a *
// (448/absmax)). K % 8 == 0.
// VPT > 0: the row is held in registers (VPT 16-byte vectors per thread,
// K <= VPT * 2048) between the absmax and the conversion, so it is read once;
// VPT == 0 reads it twice (any K).
template <int AT, int VPT>
__global__ void __launch_bounds__(256) quant_a_e4m3_kernel(const void* __restrict__ A, int M, int K,
                                                           uint8_t* __restrict__ Aq, float* __restrict__ row_scale) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // see quant_a_s8_kernel
  const int m = blockIdx.x;
  if (m >= M) return;
  const uint16_t* row = static_cast<const uint16_t*>(A) + (size_t)m * K;
  __shared__ float red[8];
  constexpr int kRegs = VPT > 0 ? VPT : 1;
  uint4 keep[kRegs];
  float amax = 0.0f;
  auto absmax8 = [&](const uint4& v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t h2 = AT == A_BF16 ? bf16x2_to_f16x2(w[j]) : w[j];
      float2 f = __half22float2(*reinterpret_cast<__half2*>(&h2));
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  };
  if (VPT > 0) {
#pragma unroll
    for (int i = 0; i < kRegs; ++i) {
      const int k = (threadIdx.x + 256 * i) * 8;
      keep[i] = k < K ? *reinterpret_cast<const uint4*>(row + k) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kRegs; ++i) absmax8(keep[i]);
  } else {
    for (int k = threadIdx.x * 8; k < K; k += 256 * 8) absmax8(*reinterpret_cast<const uint4*>(row + k));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  float qs = 0.0f, s = 0.0f;
  if (amax > 0.0f && amax <= 3.402823466e38f) {
    qs = __fdiv_rn(448.0f, amax);
    s = __fdiv_rn(amax, 448.0f);
  }
  if (threadIdx.x == 0) row_scale[m] = s;
  uint8_t* out = Aq + (size_t)m * K;
  auto convert8 = [&](const uint4& v, int k) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t h0 = AT == A_BF16 ? bf16x2_to_f16x2(w[2 * j]) : w[2 * j];
      uint32_t h1 = AT == A_BF16 ? bf16x2_to_f16x2(w[2 * j + 1]) : w[2 * j + 1];
      float2 f0 = __half22float2(*reinterpret_cast<__half2*>(&h0));
      float2 f1 = __half22float2(*reinterpret_cast<__half2*>(&h1));
      uint16_t lo, hi;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(__fmul_rn(f0.y, qs)), "f"(__fmul_rn(f0.x, qs)));
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(__fmul_rn(f1.y, qs)), "f"(__fmul_rn(f1.x, qs)));
      o[j] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint2*>(out + k) = make_uint2(o[0], o[1]);
  };
  if (VPT > 0) {
#pragma unroll
    for (int i = 0; i < kRegs; ++i) {
      const int k = (threadIdx.x + 256 * i) * 8;
      if (k < K) convert8(keep[i], k);
    }
  } else {
    for (int k = threadIdx.x * 8; k < K; k += 256 * 8) convert8(*reinterpret_cast<const uint4*>(row + k), k);
  }
}

template <int AT>
void launch_quant_e4m3_rows(const void* A, int M, int K, uint8_t* Aq, float* rs, cudaStream_t stream) {
  const int vpt = (K + 2047) / 2048;
  if (vpt <= 1) quant_a_e4m3_kernel<AT, 1><<<M, 256, 0, stream>>>(A, M, K, Aq, rs);
  else if (vpt <= 2) quant_a_e4m3_kernel<AT, 2><<<M, 256, 0, stream>>>(A, M, K, Aq, rs);
  else if (vpt <= 4) quant_a_e4m3_kernel<AT, 4><<<M, 256, 0, stream>>>(A, M, K, Aq, rs);
  else if (vpt <= 8) quant_a_e4m3_kernel<AT, 8><<<M, 256, 0, stream>>>(A, M, K, Aq, rs);
  else quant_a_e4m3_kernel<AT, 0><<<M, 256, 0, stream>>>(A, M, K, Aq, rs);
}

// ---------------------------------------------------------------- 2-SM ----
// cta_group::2 variant: a cluster of two CTAs computes a 256 (weight columns)
// x 256 (activation rows) tile with one M=256 MMA issued by the even CTA. Each
// CTA stages half of both operands (128 weight rows, 128 activation rows per
// 128-byte K step, 32 KB per stage, 6 stages), so every operand byte moved
// through L2 and shared memory feeds twice the MACs of the 1-CTA kernel. Both
// CTAs' TMA loads complete on the even CTA's `full` barrier; MMA completion is
// multicast to both CTAs' `empty` / `tfull` barriers; both CTAs' epilogue
// warps release the accumulator buffer on the even CTA's `tempty` barrier.
constexpr int kStages2 = 6;
constexpr int kHalfBytes = 128 * kBK;            // 16 KB: 128 rows x 128 K-bytes
constexpr int kStageBytes2 = 2 * kHalfBytes;     // weights half + activations half

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
template <int KIND>
__device__ __forceinline__ void umma2(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  if (KIND == KIND_I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
  } else if (KIND == KIND_F16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
  }
}
__device__ __forceinline__ void umma2_commit(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// Work item -> tile coordinates: tw (256-column weight tile), first activation
// row x0, width xw (tile_x or tile_x / 2), K split.
struct TcItem {
  int tw, x0, xw, split;
};
__device__ __forceinline__ TcItem tc_item(const TcParams& p, int wi) {
  TcItem it;
  int tile;
  if (p.splits > 1) {
    tile = wi / p.splits;
    it.split = wi - tile * p.splits;
    it.xw = p.tile_x;
    it.x0 = (tile / p.tiles_w) * p.tile_x;
  } else if (wi < p.n_full) {
    tile = wi;
    it.split = 0;
    it.xw = p.tile_x;
    it.x0 = (tile / p.tiles_w) * p.tile_x;
  } else {
    const int j = wi - p.n_full;
    tile = p.n_full + (j >> 1);
    it.split = 0;
    it.xw = p.tile_x >> 1;
    it.x0 = (tile / p.tiles_w) * p.tile_x + (j & 1) * it.xw;
  }
  it.tw = tile % p.tiles_w;
  return it;
}

template <int KIND>
__global__ void __launch_bounds__(kThreadsTC, 1)
    gemm_tc2_kernel(const __grid_constant__ TcParams p, const __grid_constant__ CUtensorMap mapW,
                    const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapXh,
                    const __grid_constant__ CUtensorMap mapD) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
#ifdef FP8IMMA_TRACE
  // per CTA 64 words, cycle counts since entry: [0] entry %globaltimer, [1] SM,
  // [3..4] producer empty-wait cycles / end, [5..7] MMA tempty-wait, full-wait,
  // end, [8..11] epilogue warp q=0: tfull-wait, tmem-load, work, end
  const long long tr0 = clock64();
  long long tr[16] = {0};
#define TC_T0() const long long _t = clock64()
#define TC_ACC(i) tr[i] += clock64() - _t
#else
#define TC_T0() do { } while (0)
#define TC_ACC(i) do { } while (0)
#endif
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages2 * kStageBytes2);
  uint64_t* empty = full + kStages2;
  uint64_t* tfull = empty + kStages2;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  // epilogue staging for TMA stores: 4 warps x 2 buffers x [32 columns][16 words]
  uint32_t* epi_stage = reinterpret_cast<uint32_t*>(smem + kStages2 * kStageBytes2 + 256);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader (issues the MMAs)
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int ntiles = p.tiles_w * p.tiles_x;  // tiles of 256 weight columns x tile_x activation rows
  // work items: (tile, K split); with splits == 1 the tiles past n_full (the
  // last, partly empty round) run as two half-width items each, so that round
  // spreads over twice as many CTA pairs
  const int nwork = p.splits > 1 ? ntiles * p.splits : p.n_full + 2 * (ntiles - p.n_full);
  const int nkb = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // 4 epilogue warps in each CTA of the pair
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_barrier();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
  const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);

  if (warp == 0) {
    // ---- TMA producer (both CTAs): this CTA's halves, completing on the leader's barrier
    if (lane == 0) {
      prefetch_tensormap(&mapW);
      prefetch_tensormap(&mapX);
      prefetch_tensormap(&mapXh);
      // as a programmatic dependent the CTA set itself up beside the prep
      // kernels; their operands are read only after they have finished
      if (p.pdl) pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int wi = pair; wi < nwork && ok; wi += npairs) {
        const TcItem it = tc_item(p, wi);
        const int kb0 = it.split * p.kb_per_split, kb1 = min(nkb, kb0 + p.kb_per_split);
        const CUtensorMap* mx = it.xw == p.tile_x ? &mapX : &mapXh;
        for (int kb = kb0; kb < kb1; ++kb) {
          {
            TC_T0();
            ok = mbar_wait<kTcSuspend>(&empty[stage], phase ^ 1u, ERR_WAIT_EMPTY);
            TC_ACC(3);
          }
          if (!ok) break;
          uint8_t* sw = smem + stage * kStageBytes2;
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (kHalfBytes + (it.xw >> 1) * kBK));
          const uint32_t fb = full_leader + stage * 8;
          tma_load_2d_pair(sw, &mapW, fb, kb * kBK, it.tw * 256 + 128 * (int)rank);
          tma_load_2d_pair(sw + kHalfBytes, mx, fb, kb * kBK, it.x0 + (it.xw >> 1) * (int)rank);
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < kStages2 && ok; ++s) {  // drain: all issued loads consumed
        ok = mbar_wait<kTcSuspend>(&empty[stage], phase ^ 1u, ERR_WAIT_EMPTY);
        if (++stage == kStages2) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (leader only)
    if (rank == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int wi = pair; wi < nwork && ok; wi += npairs, ++it) {
        const int buf = it & 1;
        const TcItem ti = tc_item(p, wi);
        const uint32_t idesc = ti.xw == p.tile_x ? p.idesc : p.idesc_half;
        const int kb0 = ti.split * p.kb_per_split, kb1 = min(nkb, kb0 + p.kb_per_split);
        {
          TC_T0();
          ok = mbar_wait<kTcSuspend>(&tempty[buf], ((it >> 1) & 1) ^ 1u, ERR_WAIT_TMEM_EMPTY);
          TC_ACC(5);
        }
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * 256);
        for (int kb = kb0; kb < kb1; ++kb) {
          {
            TC_T0();
            ok = mbar_wait<kTcSuspend>(&full[stage], phase, ERR_WAIT_FULL);
            TC_ACC(6);
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes2);
          const uint64_t adesc = sw128_desc(sa), bdesc = sw128_desc(sa + kHalfBytes);
#pragma unroll
          for (int j = 0; j < kBK / 32; ++j)
            umma2<KIND>(d_tmem, adesc + 2 * j, bdesc + 2 * j, idesc, (kb != kb0) || (j != 0));
          umma2_commit(&empty[stage], 0x3);
          if (++stage == kStages2) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma2_commit(&tfull[buf], 0x3);
      }
      umma2_commit(drain, 0x1);
      mbar_wait<kTcSuspend>(drain, 0, ERR_WAIT_FULL);
    }
  } else {
    // ---- epilogue (both CTAs): this CTA's 128 TMEM lanes = 128 weight columns
    const int q = warp & 3;
    int it = 0;
    int sbuf = 0;  // TMA-store staging buffer of this warp (two, alternating)
    for (int wi = pair; wi < nwork; wi += npairs, ++it) {
      const int buf = it & 1;
      const TcItem ti = tc_item(p, wi);
      const int tw = ti.tw, split = ti.split;
      bool okw;
      {
        TC_T0();
        okw = mbar_wait<kTcSuspend>(&tfull[buf], (it >> 1) & 1, ERR_WAIT_TMEM_FULL);
        TC_ACC(8);
      }
      if (!okw) break;
#ifdef FP8IMMA_TRACE
      const long long tw0 = clock64();
#endif
      tc_fence_after();
      const int n = tw * 256 + 128 * (int)rank + q * 32 + lane;
      const bool nok = n < p.N;
      float cs = 1.0f;
      if (nok && KIND == KIND_I8) {
        uint16_t sb = p.scale_tex ? tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n) : p.scale_u16[n];
        cs = __half2float(__ushort_as_half(sb));
      }
      const float cs2 = (nok && p.col_scale_f32) ? p.col_scale_f32[n] : 1.0f;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 256);
      uint16_t* D = static_cast<uint16_t*>(p.D);
#pragma unroll 1
      for (int j0 = 0; j0 < ti.xw; j0 += 32) {
        uint32_t r[32];
        {
          TC_T0();
          tmem_ld32(taddr + j0, r);
          TC_ACC(9);
        }
        const int mbase = ti.x0 + j0;
        // col-major 16-bit output: the warp stages its 32 columns x 32 rows in
        // shared memory and one lane writes the box with a TMA store (the
        // tensor map clips rows past M and columns past N). Per-lane 16-byte
        // stores, 32 columns 8 KB apart per instruction, ran at a fraction of
        // the GEMM's speed.
        if (p.tma_out) {
          uint32_t* st = epi_stage + (q * 2 + sbuf) * 512;  // [32 columns][16 words] dense, 2 KB
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");  // this buffer's last store read it
          __syncwarp();
          uint32_t pk[16];
          tc_epi_pack<KIND>(r, mbase, cs, cs2, p, nok ? n : 0, pk);
          uint4* row4 = reinterpret_cast<uint4*>(st + lane * 16);
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) row4[v4] = make_uint4(pk[4 * v4], pk[4 * v4 + 1], pk[4 * v4 + 2], pk[4 * v4 + 3]);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> async-proxy reads
          __syncwarp();
          if (lane == 0 && mbase < p.M) {
            asm volatile(
                "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                    reinterpret_cast<uint64_t>(&mapD)),
                "r"(mbase * 2), "r"(n - lane), "r"(smem_u32(st))
                : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          sbuf ^= 1;
          if (KIND == KIND_I8 && p.acc_out && nok) {
            const int mc = min(32, p.M - mbase);
            _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mc) p.acc_out[(size_t)n * p.M + mbase + j] = (int32_t)r[j];
          }
          continue;
        }
        if (!nok || mbase >= p.M) continue;
        if (p.splits > 1) {  // raw accumulators of this K split; tc_splitk_reduce_kernel finishes
          uint32_t* dst = p.ws + ((size_t)split * p.N + n) * p.M + mbase;
          const int mc = min(32, p.M - mbase);
          if (mc == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4)
              reinterpret_cast<uint4*>(dst)[v4] = make_uint4(r[4 * v4], r[4 * v4 + 1], r[4 * v4 + 2], r[4 * v4 + 3]);
          } else {
            _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mc) dst[j] = r[j];
          }
          continue;
        }
        if (KIND == KIND_F16) {  // fp8wgt: fp32 accumulators straight to row-major C[m, n]
          float* C = static_cast<float*>(p.D);
          const int mc = min(32, p.M - mbase);
          _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mc) C[(size_t)(mbase + j) * p.N + n] = __uint_as_float(r[j]);
          continue;
        }
        uint32_t pk[16];
        tc_epi_pack<KIND>(r, mbase, cs, cs2, p, n, pk);
        uint16_t o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = (uint16_t)(pk[j >> 1] >> (16 * (j & 1)));
        const int mcount = min(32, p.M - mbase);
        if (p.out_row_major) {
          _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mcount) D[(size_t)(mbase + j) * p.N + n] = o[j];
        } else {
          uint16_t* dst = D + (size_t)n * p.M + mbase;
          if (mcount == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              uint4 w;
              w.x = (uint32_t)o[8 * v4 + 0] | ((uint32_t)o[8 * v4 + 1] << 16);
              w.y = (uint32_t)o[8 * v4 + 2] | ((uint32_t)o[8 * v4 + 3] << 16);
              w.z = (uint32_t)o[8 * v4 + 4] | ((uint32_t)o[8 * v4 + 5] << 16);
              w.w = (uint32_t)o[8 * v4 + 6] | ((uint32_t)o[8 * v4 + 7] << 16);
              reinterpret_cast<uint4*>(dst)[v4] = w;
            }
          } else {
            _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mcount) dst[j] = o[j];
          }
        }
        if (KIND == KIND_I8 && p.acc_out) {
          _Pragma("unroll") for (int j = 0; j < 32; ++j) if (j < mcount) p.acc_out[(size_t)n * p.M + mbase + j] = (int32_t)r[j];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty_leader + buf * 8);
#ifdef FP8IMMA_TRACE
      tr[10] += clock64() - tw0;
#endif
    }
    if (p.tma_out && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // stores complete
  }
#ifdef FP8IMMA_TRACE
  if (p.trace && lane == 0) {
    unsigned long long* t = p.trace + (size_t)blockIdx.x * 64;
    if (warp == 0) {
      t[0] = globaltimer_ns();
      uint32_t smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      t[1] = smid;
      t[3] = tr[3];
      t[4] = clock64() - tr0;
    } else if (warp == 1) {
      t[5] = tr[5];
      t[6] = tr[6];
      t[7] = clock64() - tr0;
    } else if ((warp & 3) == 0) {
      t[8] = tr[8];
      t[9] = tr[9];
      t[10] = tr[10];
      t[11] = clock64() - tr0;
    }
  }
#endif

  tc_fence_before();
  cluster_barrier();  // no CTA leaves while its pair may still use its smem or TMEM
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
  }
}

// M=256 instruction descriptor for the pair MMA
template <int KIND>
__host__ __device__ constexpr uint32_t make_idesc2(int a_fmt, int n) {
  // kind::f16 (fp16 x fp16, fp32 accumulate): a/b format 0 = F16; M = 256, N = n
  return (KIND == KIND_I8 ? (2u << 4) | (1u << 7) | (1u << 10)
                          : (1u << 4) | (KIND == KIND_F16 ? 0u : ((uint32_t)a_fmt << 7))) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

bool g_use_pair = true;
int g_tc_splitk = -1;  // -1 automatic, else forced K splits of the CTA-pair kernel
int g_tc_tile_x = 0;   // 0 automatic, else forced activation rows per tile (256, 192, 128)
bool g_tc_half_tail = true;  // run the last partial round of tiles as half-width items

// Activation rows per CTA-pair tile (the MMA's N). 256 unless forced: 192 and
// 128 balance the rounds of tiles over the CTA pairs better (4096^2: 256
// tiles of 256 on 74 pairs = 3.46 rounds) but cost more operand traffic per
// MAC, and measured 5-60% slower on 4096^2, 2048x11008x4096, 8192^3 and
// 4096x28672x8192; the last partial round is handled by half-width items
// instead (n_full in launch_tc2).
int tc_pick_tile_x(int M, int N) {
  (void)M;
  (void)N;
  return g_tc_tile_x ? g_tc_tile_x : 256;
}

// Split-K finish: sum the raw accumulators of the K splits in a fixed order
// (exact for int32; deterministic for fp32) and apply the same epilogue as
// the tensor-core kernel. 32 x 32 (n, m) tiles through shared memory so that
// both the column-major reads and a row-major store are coalesced.
template <int KIND>
__global__ void __launch_bounds__(256) tc_splitk_reduce_kernel(const TcParams p) {
  __shared__ float tile[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  const int m0 = blockIdx.x * 32, n0 = blockIdx.y * 32;
  const size_t plane = (size_t)p.N * p.M;
  const bool row_out = KIND == KIND_F16 || p.out_row_major;
  // all four rows' partials of a split are loaded before any is added
  int32_t si4[4] = {0, 0, 0, 0};
  float sf4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const int m = m0 + tx;
  for (int s = 0; s < p.splits; ++s) {
    uint32_t x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = n0 + ty + 8 * i;
      x[i] = (n < p.N && m < p.M) ? __ldcs(p.ws + (size_t)s * plane + (size_t)n * p.M + m) : 0u;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (KIND == KIND_I8) si4[i] += (int32_t)x[i];
      else sf4[i] += __uint_as_float(x[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = n0 + ty + 8 * i;
    float v = 0.0f;
    if (n < p.N && m < p.M) {
      const size_t e = (size_t)n * p.M + m;
      const int32_t si = si4[i];
      const float sf = sf4[i];
      if (KIND == KIND_F16) {
        v = sf;
      } else if (KIND == KIND_I8) {
        uint16_t sb = p.scale_tex ? tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n) : p.scale_u16[n];
        float se = __half2float(__ushort_as_half(sb)) * (p.row_g ? p.row_g[m] : p.global_scale);
        if (p.col_scale_f32) se = se * p.col_scale_f32[n];
        v = (float)si * se;
        if (p.acc_out) p.acc_out[e] = si;
      } else {
        v = sf * (p.row_g ? p.row_g[m] : 1.0f) * (p.col_scale_f32 ? p.col_scale_f32[n] : 1.0f);
      }
      if (KIND != KIND_F16) v = bias_act(v, p.bias, n, p.act);
      if (!row_out) static_cast<uint16_t*>(p.D)[e] = store_val(v, p.out_bf16);
    }
    tile[ty + 8 * i][tx] = v;
  }
  if (!row_out) return;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 8 * i, n = n0 + tx;
    if (n >= p.N || m >= p.M) continue;
    const float v = tile[tx][ty + 8 * i];
    if (KIND == KIND_F16) static_cast<float*>(p.D)[(size_t)m * p.N + n] = v;
    else static_cast<uint16_t*>(p.D)[(size_t)m * p.N + n] = store_val(v, p.out_bf16);
  }
}

template <int KIND>
cudaError_t launch_tc2(TcParams p, const void* W, const void* X, int a_fmt, cudaStream_t stream) {
  CUtensorMap mw, mx;
  cudaError_t e;
  if ((e = make_tmap_2d_u8(&mw, W, p.K, p.N, p.K, kBK, 128, true)) != cudaSuccess) return e;
  CUtensorMap mxh;
  p.tile_x = tc_pick_tile_x(p.M, p.N);
  if ((e = make_tmap_2d_u8(&mx, X, p.K, p.M, p.K, kBK, p.tile_x / 2, true)) != cudaSuccess) return e;
  if ((e = make_tmap_2d_u8(&mxh, X, p.K, p.M, p.K, kBK, p.tile_x / 4, true)) != cudaSuccess) return e;
  p.tiles_w = (p.N + 255) / 256;
  p.tiles_x = (p.M + p.tile_x - 1) / p.tile_x;
  p.idesc = make_idesc2<KIND>(a_fmt, p.tile_x);
  p.idesc_half = make_idesc2<KIND>(a_fmt, p.tile_x / 2);
  // col-major fp16 / bf16 output through TMA stores: rows of M * 2 bytes must
  // be a multiple of 16 bytes and D 16-byte aligned
  CUtensorMap md = mw;
  p.tma_out = 0;
#ifdef FP8IMMA_TRACE
  p.trace = g_tc_trace;
#endif
  if (KIND != KIND_F16 && p.splits <= 1 && !p.out_row_major && (p.M % 8) == 0 &&
      (reinterpret_cast<uintptr_t>(p.D) & 15u) == 0 &&
      make_tmap_2d_u8(&md, p.D, (uint64_t)p.M * 2, p.N, (uint64_t)p.M * 2, 64, 32, false) == cudaSuccess)
    p.tma_out = 1;
  auto kern = gemm_tc2_kernel<KIND>;
  const int smem = kStages2 * kStageBytes2 + 1024 + 256 + 4 * 2 * 2048;
  if ((e = ensure_smem_attr((const void*)kern, smem)) != cudaSuccess) return e;
  const int ntiles = p.tiles_w * p.tiles_x;
  const int maxpairs = num_sms_current() / 2;
  const int nkb = (p.K + kBK - 1) / kBK;
  if (!p.ws) p.splits = 1;
  if (p.splits < 1) p.splits = 1;
  p.kb_per_split = (nkb + p.splits - 1) / p.splits;
  p.splits = (nkb + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  // last partial round of full tiles -> twice as many half-width items, when
  // they then fit in one round (4096^2: 256 = 3 x 74 + 34 tiles; 34 x 2 <= 74)
  const int rem = ntiles % maxpairs;
  p.n_full = ntiles;
  if (p.splits == 1 && g_tc_half_tail && ntiles > maxpairs && rem > 0 && 2 * rem <= maxpairs &&
      (p.tile_x / 2) % 32 == 0)
    p.n_full = ntiles - rem;
  const int nwork = p.splits > 1 ? ntiles * p.splits : p.n_full + 2 * (ntiles - p.n_full);
  const int pairs = nwork < maxpairs ? nwork : maxpairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreadsTC, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // (not with K splits: the finishing pass follows, and mid-M calls measured
  // slower as programmatic dependents, 44 vs 37 us at M = 128, N = K = 4096)
  if (p.splits > 1) p.pdl = 0;
  cfg.numAttrs = p.pdl ? 2 : 1;
  if ((e = cudaLaunchKernelEx(&cfg, kern, p, mw, mx, mxh, md)) != cudaSuccess || p.splits == 1) return e;
  const dim3 rgrid((p.M + 31) / 32, (p.N + 31) / 32);
  tc_splitk_reduce_kernel<KIND><<<rgrid, dim3(32, 8), 0, stream>>>(p);
  return cudaGetLastError();
}

int grid_for(size_t work_items) {
  const int sms = num_sms_current();
  size_t blocks = (work_items + 255) / 256;
  size_t cap = (size_t)sms * 8;
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

template <int KIND>
cudaError_t launch_tc(const TcParams& p, const CUtensorMap& mw, const CUtensorMap& mx, cudaStream_t stream) {
  auto kern = gemm_tc_kernel<KIND>;
  const int smem = kStages * kStageBytes + 1024 + 256;
  cudaError_t e = ensure_smem_attr((const void*)kern, smem);
  if (e != cudaSuccess) return e;
  const int ntiles = p.tiles_w * p.tiles_x;
  const int grid = ntiles < num_sms_current() ? ntiles : num_sms_current();
  kern<<<grid, kThreadsTC, smem, stream>>>(p, mw, mx);
  return cudaGetLastError();
}

}  // namespace

void tc_set_pair_mode(bool on) { g_use_pair = on; }

unsigned int tc_device_error(bool clear) { return tu_device_error(clear); }
cudaError_t tc_set_wait_limit(unsigned long long ns) { return tu_set_wait_limit(ns); }

void tc_set_splitk(int splits) { g_tc_splitk = splits; }
void tc_set_tile_x(int rows) { g_tc_tile_x = rows; }
void tc_set_half_tail(bool on) { g_tc_half_tail = on; }

// K splits for the CTA-pair kernel: enough (tile, split) work items to give
// most CTA pairs one, at least 4 K blocks (512 bytes of K) per split, and only
// where that is 3 or more splits.
int tc_pick_splits(int M, int N, int Kbytes) {
  if (!g_use_pair) return 1;
  const int nkb = (Kbytes + kBK - 1) / kBK;
  if (g_tc_splitk >= 1) return g_tc_splitk < nkb ? g_tc_splitk : nkb;
  const int t = tc_pick_tile_x(M, N);
  const int ntiles = ((N + 255) / 256) * ((M + t - 1) / t);
  const int pairs = num_sms_current() / 2;
  int s = pairs / ntiles;
  if (s > 8) s = 8;
  if (s > nkb / 4) s = nkb / 4;
  return s < 3 ? 1 : s;  // two splits measured no faster than none (the finishing pass costs ~4 us)
}

size_t tc_splitk_ws_bytes(int M, int N, int Kbytes) {
  const int s = tc_pick_splits(M, N, Kbytes);
  return s > 1 ? (((size_t)s * N * M * 4 + 255) & ~size_t(255)) : 0;
}

static size_t tc_ws_offset(int M, int N, int K, bool native) {
  size_t a = ((size_t)M * K + 255) & ~size_t(255);
  size_t b = native ? 0 : (((size_t)N * K + 255) & ~size_t(255));
  size_t r = native ? (((size_t)M * 4 + 255) & ~size_t(255)) : 0;
  return a + b + r;
}

size_t gemm_tc_scratch_bytes(int M, int N, int K, bool native) {
  return tc_ws_offset(M, N, K, native) + tc_splitk_ws_bytes(M, N, K);
}

// int8-exact large-M GEMM: prep (A quant, B transcode) into `scratch`, then tcgen05.
cudaError_t launch_gemm_tc_s8(const GemvParams& gp, int a_type, int fmt, void* scratch, cudaStream_t stream) {
  const int M = gp.M, N = gp.N, K = gp.K;
  int8_t* Aq = static_cast<int8_t*>(scratch);
  int8_t* Bq = Aq + (((size_t)M * K + 255) & ~size_t(255));
  const bool pdl = gp.pdl != 0;
  // 1. weights: one warp per row, at most 8 resident CTAs of 8 warps per SM.
  // An ordinary launch: it overwrites scratch that the previous call's GEMM
  // on this stream may still read.
  {
    const int sms = num_sms_current();
    const int grid = std::min((N + 7) / 8, sms * 8);
    if (fmt == FMT_E5M2)
      transcode_b_kernel<FMT_E5M2><<<grid, 256, 0, stream>>>(gp.B, N, K, gp.scale_u16, gp.scale_tex, Bq);
    else
      transcode_b_kernel<FMT_E4M3_REF><<<grid, 256, 0, stream>>>(gp.B, N, K, gp.scale_u16, gp.scale_tex, Bq);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // 2. activations, alongside the transcode when programmatic dependent
  // launch is on (the two touch disjoint memory; everything before the call
  // has finished once the transcode started)
  {
    const size_t items = (size_t)M * (K >> 3);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)grid_for(items), 1, 1);
    lc.blockDim = dim3(256, 1, 1);
    lc.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = pdl ? 1 : 0;
    const int after = pdl ? 1 : 0;
    switch (a_type) {
      case A_F16:
        e = cudaLaunchKernelEx(&lc, quant_a_s8_kernel<A_F16>, gp.A, M, K, gp.a_inv_h, gp.row_inv_h, Aq, after);
        break;
      case A_BF16:
        e = cudaLaunchKernelEx(&lc, quant_a_s8_kernel<A_BF16>, gp.A, M, K, gp.a_inv_h, gp.row_inv_h, Aq, after);
        break;
      default:
        e = cudaLaunchKernelEx(&lc, quant_a_s8_kernel<A_S8>, gp.A, M, K, gp.a_inv_h, gp.row_inv_h, Aq, after);
        break;
    }
    if (e != cudaSuccess) return e;
  }
  // 3. tensor-core GEMM
  CUtensorMap mw, mx;
  if ((e = make_tmap_2d_u8(&mw, Bq, K, N, K, kBK, kTileW, true)) != cudaSuccess) return e;
  if ((e = make_tmap_2d_u8(&mx, Aq, K, M, K, kBK, kTileX, true)) != cudaSuccess) return e;
  TcParams p = {};
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_w = (N + kTileW - 1) / kTileW;
  p.tiles_x = (M + kTileX - 1) / kTileX;
  p.idesc = make_idesc<KIND_I8>(0);
  p.scale_u16 = gp.scale_u16;
  p.scale_tex = gp.scale_tex;
  p.col_scale_f32 = gp.col_scale_f32;
  p.row_g = gp.row_g;
  p.global_scale = gp.global_scale;
  p.D = gp.D;
  p.acc_out = gp.acc_out;
  p.bias = gp.bias;
  p.act = gp.act;
  p.out_bf16 = gp.out_bf16;
  p.out_row_major = gp.out_row_major;
  if (g_use_pair) {
    p.splits = tc_pick_splits(M, N, K);
    p.ws = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(scratch) + tc_ws_offset(M, N, K, false));
    p.pdl = pdl ? 1 : 0;
    return launch_tc2<KIND_I8>(p, Bq, Aq, 0, stream);
  }
  return launch_tc<KIND_I8>(p, mw, mx, stream);
}

// Reference int8 activation quantisation alone (A_S8 copies). Used by the
// small-M kernel when the same activations would otherwise be re-quantised by
// many column tiles.
cudaError_t launch_quant_a_s8(const void* A, int a_type, int M, int K, uint16_t a_inv_h, const uint16_t* row_inv_h,
                              int8_t* Aq, cudaStream_t stream) {
  const int grid = grid_for((size_t)M * (K >> 3));
  switch (a_type) {
    case A_F16: quant_a_s8_kernel<A_F16><<<grid, 256, 0, stream>>>(A, M, K, a_inv_h, row_inv_h, Aq, 0); break;
    case A_BF16: quant_a_s8_kernel<A_BF16><<<grid, 256, 0, stream>>>(A, M, K, a_inv_h, row_inv_h, Aq, 0); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Per-row E4M3 activation quantisation alone (small-M native path).
cudaError_t launch_quant_a_e4m3(const void* A, int a_type, int M, int K, uint8_t* Aq, float* row_scale,
                                cudaStream_t stream) {
  if (a_type == A_BF16) launch_quant_e4m3_rows<A_BF16>(A, M, K, Aq, row_scale, stream);
  else launch_quant_e4m3_rows<A_F16>(A, M, K, Aq, row_scale, stream);
  return cudaGetLastError();
}

// Native FP8 large-M GEMM: per-row E4M3 activation quant, then kind::f8f6f4
// on the raw weight bytes. b_fmt: 0 = E4M3 (hardware E4M3FN), 1 = E5M2.
cudaError_t launch_gemm_tc_fp8(const void* A, int a_type, const uint8_t* B, int b_fmt, const float* col_scale,
                               void* D, int M, int N, int K, int out_bf16, int out_row_major, void* scratch,
                               cudaStream_t stream, const float* bias, int act) {
  uint8_t* Aq = static_cast<uint8_t*>(scratch);
  float* rs = reinterpret_cast<float*>(Aq + (((size_t)M * K + 255) & ~size_t(255)));
  if (a_type == A_BF16) launch_quant_e4m3_rows<A_BF16>(A, M, K, Aq, rs, stream);
  else launch_quant_e4m3_rows<A_F16>(A, M, K, Aq, rs, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  CUtensorMap mw, mx;
  if ((e = make_tmap_2d_u8(&mw, B, K, N, K, kBK, kTileW, true)) != cudaSuccess) return e;
  if ((e = make_tmap_2d_u8(&mx, Aq, K, M, K, kBK, kTileX, true)) != cudaSuccess) return e;
  TcParams p = {};
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_w = (N + kTileW - 1) / kTileW;
  p.tiles_x = (M + kTileX - 1) / kTileX;
  p.idesc = make_idesc<KIND_F8>(b_fmt == 1 ? 1 : 0);
  p.col_scale_f32 = col_scale;
  p.row_g = rs;
  p.global_scale = 1.0f;
  p.D = D;
  p.out_bf16 = out_bf16;
  p.out_row_major = out_row_major;
  p.bias = bias;
  p.act = act;
  if (g_use_pair) {
    p.splits = tc_pick_splits(M, N, K);
    p.ws = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(scratch) + tc_ws_offset(M, N, K, true));
    return launch_tc2<KIND_F8>(p, B, Aq, b_fmt == 1 ? 1 : 0, stream);
  }
  return launch_tc<KIND_F8>(p, mw, mx, stream);
}

namespace {
// fp8wgt weights -> fp16 (torch_ext/fp8wgt/fp8wgt_ext_cuda.cu:195-198):
// fp16_rn(float(lut_e4m3[b]) * scale_b), 16 bytes in, 32 bytes out per step;
// sb is scale_b / 256 for the packed decode (wgt_decode4_fast).
__global__ void __launch_bounds__(256) decode_b_f16_kernel(const uint8_t* __restrict__ B, size_t n16, float sb,
                                                           int fast, uint16_t* __restrict__ Bh) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 v = ldg_stream_v4(reinterpret_cast<const uint4*>(B) + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (fast) wgt_decode4_fast(w[j], sb, o[2 * j], o[2 * j + 1]);
      else wgt_decode4_exact(w[j], sb, o[2 * j], o[2 * j + 1]);
    }
    uint4* dst = reinterpret_cast<uint4*>(Bh) + 2 * i;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}
}  // namespace

// fp8wgt linear for large M: weights decoded once to fp16 (scratch, 2NK
// bytes), then the CTA-pair tcgen05 GEMM with kind::f16 and an fp32 row-major
// epilogue. K % 8 == 0 (16-byte TMA row pitch).
cudaError_t launch_gemm_tc_wgt(const void* A_f16, const uint8_t* B, float scale_b, float* C, int M, int N, int K,
                               void* scratch, cudaStream_t stream) {
  uint16_t* Bh = static_cast<uint16_t*>(scratch);
  const size_t n16 = (size_t)N * K / 16;
  const int sms = num_sms_current();
  // packed decode with scale/256 unless that is an fp32 subnormal (then the scalar one)
  const float mag = scale_b < 0.0f ? -scale_b : scale_b;
  const int fast = (mag == 0.0f || !(mag < 0x1p-117f)) ? 1 : 0;
  decode_b_f16_kernel<<<sms * 8, 256, 0, stream>>>(B, n16, fast ? scale_b * 0.00390625f : scale_b, fast, Bh);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  TcParams p = {};
  p.M = M;
  p.N = N;
  p.K = 2 * K;  // the pipeline works in bytes of K
  p.D = C;
  p.splits = tc_pick_splits(M, N, 2 * K);
  p.ws = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(scratch) + (((size_t)N * K * 2 + 255) & ~size_t(255)));
  return launch_tc2<KIND_F16>(p, Bh, A_f16, 0, stream);
}

}  // namespace fp8imma_b200

#ifdef FP8IMMA_TRACE
extern "C" void fp8imma_debug_set_tc_trace(void* buf) {
  fp8imma_b200::g_tc_trace = static_cast<unsigned long long*>(buf);
}
#endif
