// Split-K skinny GEMM for small M (decode shapes).
//
// Work split (B200):
//   * a CTA owns 128 weight columns and one K-slice; the K-slices of a column
//     tile form a thread-block cluster and reduce their int32 partials through
//     distributed shared memory (no global scratch);
//   * one producer warp streams the weight tile with 2-D TMA loads
//     (128 columns x 128 K-bytes = 16 KB per stage, 128-byte swizzle, 4-stage
//     mbarrier ring), so the HBM stream is deep and costs no registers;
//   * eight consumer warps each own 16 columns: 16-byte conflict-free shared
//     loads, FP8 -> int8 transcode in registers (fp8imma_device.cuh), and
//     mma.sync m16n8k32 s8 with the transcoded weights as the A operand and the
//     quantised activations (shared memory) as the B operand.
// Within each 64-byte K block the MMA's physical k index is a permutation of
// the logical k; both operands use the same permutation and int32 sums do not
// depend on order, so the result is exact. MMA rows map to tile columns
// through sigma(g) = (g>>1) + 4*(g&1), which puts the two rows read by one
// 8-lane shared-memory phase in different halves of the 128-byte swizzle
// pattern (conflict-free).
//
// Modes (FMT): reference-exact int8 (E4M3 table / E5M2 weights transcoded
// in registers, m16n8k32 s8), native FP8 (weight bytes and E4M3 activations
// straight into m16n8k32 e4m3/e5m2 with fp32 accumulation) and the fp8wgt
// fp16 mode (weights decoded to fp16(lut * scale), m16n8k16 f16, fp32 output).
// Two forms: the cluster form described above (default), and a stream-K kernel
// (persistent CTAs, an even share of 64-wide K halves each, partial tiles
// finished by the last arriving CTA) for large projections.
//
// Reference counterpart: imma_gemm_fp8_actquant_cpasync_int8_colscale_fp16_
// colmajor_kernel_v4 (src/fp8imma/impl/v4_kernels.inl:1-287), v3
// (impl/v3_kernels.inl) and v2 (impl/v2_kernels.inl): 64x64 tiles that waste
// 63/64 of their MMA rows at M=1.
#include "fp8imma_device.cuh"
#include "fp8imma_kernels.h"
#include "sm100_async.cuh"

#include <cooperative_groups.h>

#include <atomic>
#include <mutex>

// Opt-in phase tracing (compile with -DFP8IMMA_TRACE): thread 0 of each CTA
// records %globaltimer at fixed points into p.trace[cta * 16 + point].
#ifdef FP8IMMA_TRACE
#define TRACE_POINT(p, i)                                                                                 \
  do {                                                                                                     \
    if ((p).trace && (threadIdx.x & 31) == 0) {                                                           \
      unsigned long long t_;                                                                               \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                             \
      const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);                    \
      (p).trace[(size_t)cta_ * 16 + (i)] = t_;                                                             \
    }                                                                                                      \
  } while (0)
// slot 15 holds the SM the CTA ran on
#define TRACE_SMID(p)                                                                                      \
  do {                                                                                                     \
    if ((p).trace && threadIdx.x == 0) {                                                                   \
      unsigned int s_;                                                                                     \
      asm volatile("mov.u32 %0, %%smid;" : "=r"(s_));                                                     \
      const int cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);                    \
      (p).trace[(size_t)cta_ * 16 + 15] = s_;                                                              \
    }                                                                                                      \
  } while (0)
#else
#define TRACE_POINT(p, i) do { } while (0)
#define TRACE_SMID(p) do { } while (0)
#endif

namespace cg = cooperative_groups;
using namespace fp8imma_dev;

namespace fp8imma_b200 {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one TMA producer warp
constexpr int kTileN = 128;
constexpr int kBlockK = 128;
constexpr int kStages = 4;
constexpr int kStageBytes = kTileN * kBlockK;
constexpr int kBarOffset = kStages * kStageBytes;
constexpr int kScaleOffset = kBarOffset + 256;       // float[128] fp16 column scales
constexpr int kColScaleOffset = kBarOffset + 768;    // float[128] fp32 column multipliers
constexpr int kRowScaleOffset = kBarOffset + 1280;   // float[32] per-row / global scale
constexpr int kAqOffset = kBarOffset + 2048;

__device__ __forceinline__ void mma_s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// native FP8: weights (A operand) E4M3 or E5M2, activations E4M3, f32 accumulate
template <int FMT>
__device__ __forceinline__ void mma_f8_16832(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  if (FMT == FMT_NATIVE_E5M2) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.f32.e5m2.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <int FMT>
__host__ __device__ constexpr bool is_native() { return FMT == FMT_E4M3FN || FMT == FMT_NATIVE_E5M2; }
// fp32 accumulation (native FP8 and fp8wgt) instead of exact int32
template <int FMT>
__host__ __device__ constexpr bool is_float_acc() { return is_native<FMT>() || FMT == FMT_WGT; }

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(smem_u32(p)));
  return r;
}

__device__ __forceinline__ uint16_t load_col_scale_bits(const GemvParams& p, int n) {
  if (p.scale_tex) return tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n);
  return p.scale_u16[n];
}

template <int FMT, bool FAST>
__device__ __forceinline__ uint32_t tc4(uint32_t x, uint32_t fscale, uint16_t inv_h) {
  if (is_native<FMT>()) return x;  // FP8 bytes go to the tensor core as they are
  if (FAST) return FMT == FMT_E5M2 ? transcode4_fast_e5m2(x, fscale) : transcode4_fast_e4m3(x, fscale);
  return transcode4_exact<FMT>(x, inv_h);
}

// Quantise A[m0 : m0+MR, k0 : k0+len] into aq (row stride `stride`), zero-
// filling rows >= M and k >= kvalid. Consumer threads only.
template <int AT, int MR>
__device__ __forceinline__ void quant_chunk(const GemvParams& p, int8_t* aq, int stride, int m0, int k0, int len,
                                            int kvalid) {
  constexpr int kBatch = 4;  // loads in flight per thread before any is converted
  const int items_per_row = len >> 3;  // 8 elements per item
  const int total = MR * items_per_row;
  for (int base = threadIdx.x; base < total; base += kBatch * kConsumers) {
    uint4 v[kBatch];
    bool live[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int it = base + j * kConsumers;
      const int r = it / items_per_row, c = (it - r * items_per_row) << 3;
      const int m = m0 + r, k = k0 + c;
      live[j] = it < total && m < p.M && k < kvalid;
      v[j] = make_uint4(0u, 0u, 0u, 0u);
      if (live[j]) {
        if (AT == A_S8)
          *reinterpret_cast<uint2*>(&v[j]) =
              *reinterpret_cast<const uint2*>(static_cast<const int8_t*>(p.A) + (size_t)m * p.K + k);
        else
          v[j] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.A) + (size_t)m * p.K + k);
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int it = base + j * kConsumers;
      if (it >= total) break;
      const int r = it / items_per_row, c = (it - r * items_per_row) << 3;
      uint2 out = make_uint2(0u, 0u);
      if (live[j]) {
        if (AT == A_S8) {
          out = make_uint2(v[j].x, v[j].y);
        } else {
          const uint16_t ainv = p.row_inv_h ? p.row_inv_h[m0 + r] : p.a_inv_h;
          const uint32_t ainv2 = (uint32_t)ainv | ((uint32_t)ainv << 16);
          uint4 w = v[j];
          if (AT == A_BF16) {
            w.x = bf16x2_to_f16x2(w.x);
            w.y = bf16x2_to_f16x2(w.y);
            w.z = bf16x2_to_f16x2(w.z);
            w.w = bf16x2_to_f16x2(w.w);
          }
          out.x = quant4_f16(w.x, w.y, ainv2);
          out.y = quant4_f16(w.z, w.w, ainv2);
        }
      }
      *reinterpret_cast<uint2*>(aq + r * stride + c) = out;
    }
  }
}

// FMT_WGT: copy fp16 A[m0 : m0+MR, k0 : k0+len] into shared memory as it is
// (row stride `stride` bytes), zero-filling rows >= M and k >= kvalid.
template <int MR>
__device__ __forceinline__ void copy_chunk_f16(const GemvParams& p, uint8_t* a, int stride, int m0, int k0, int len,
                                               int kvalid) {
  constexpr int kBatch = 4;
  const int items_per_row = len >> 3;  // 8 halves per item
  const int total = MR * items_per_row;
  for (int base = threadIdx.x; base < total; base += kBatch * kConsumers) {
    uint4 v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int it = base + j * kConsumers;
      const int r = it / items_per_row, c = (it - r * items_per_row) << 3;
      const int m = m0 + r, k = k0 + c;
      v[j] = make_uint4(0u, 0u, 0u, 0u);
      if (it < total && m < p.M && k < kvalid)
        v[j] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.A) + (size_t)m * p.K + k);
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int it = base + j * kConsumers;
      if (it >= total) break;
      const int r = it / items_per_row, c = (it - r * items_per_row) << 3;
      *reinterpret_cast<uint4*>(a + r * stride + c * 2) = v[j];
    }
  }
}

template <int AT, int MR, int FMT>
__device__ __forceinline__ void stage_chunk(const GemvParams& p, int8_t* aq, int stride, int m0, int k0, int len,
                                            int kvalid) {
  // float-accumulating modes stage (zero-filled) up to the whole 128-wide
  // weight block: a half past K may still be multiplied (by zero weights),
  // and 0 * stale NaN bits would not be 0
  if (is_float_acc<FMT>()) len = (len + kBlockK - 1) & ~(kBlockK - 1);
  if (FMT == FMT_WGT)
    copy_chunk_f16<MR>(p, reinterpret_cast<uint8_t*>(aq), stride, m0, k0, len, kvalid);
  else
    quant_chunk<AT, MR>(p, aq, stride, m0, k0, len, kvalid);
}

// One 64-wide K half (h) of a staged 128-byte weight block: transcode (or
// decode) this lane's 2 x 16 weight bytes and run the MMAs against the staged
// activations at chunk offset koff.
template <int AT, int MB, int FMT, bool FAST>
__device__ __forceinline__ void mma_half(const GemvParams& p, int (&acc)[MB][4], const uint8_t* st, const int8_t* aq,
                                         int astride, int koff, int h, int rowA, int rowB, int swz, int g, int t,
                                         uint32_t fs0, uint32_t fs1, uint16_t inv0, uint16_t inv1) {
  const int c = (4 * h + t) ^ swz;
  uint4 w0 = lds128(st + rowA * kBlockK + (c << 4));
  uint4 w1 = lds128(st + rowB * kBlockK + (c << 4));
  if (FMT == FMT_WGT) {
    // lane holds logical k = 16t .. 16t+15 of this 64-wide half for rows
    // A/B; MMA j takes logical 16t+4j .. 16t+4j+3 as physical {2t, 2t+1,
    // 2t+8, 2t+9}, and the activations (raw fp16, 32 bytes per lane) the same
    const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w}, wb[4] = {w1.x, w1.y, w1.z, w1.w};
    uint32_t alo[4], ahi[4], blo[4], bhi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (FAST) {
        wgt_decode4_fast(wa[j], p.wgt_scale, alo[j], ahi[j]);
        wgt_decode4_fast(wb[j], p.wgt_scale, blo[j], bhi[j]);
      } else {
        wgt_decode4_exact(wa[j], p.wgt_scale, alo[j], ahi[j]);
        wgt_decode4_exact(wb[j], p.wgt_scale, blo[j], bhi[j]);
      }
    }
    const uint8_t* arow = reinterpret_cast<const uint8_t*>(aq) + (koff + 64 * h + 16 * t) * 2;
#pragma unroll
    for (int nb = 0; nb < MB; ++nb) {
      const uint8_t* ap = arow + (nb * 8 + g) * astride;
      uint4 q0 = lds128(ap), q1 = lds128(ap + 16);
      float(&fa)[4] = *reinterpret_cast<float(*)[4]>(&acc[nb][0]);
      mma_f16_16816(fa, alo[0], blo[0], ahi[0], bhi[0], q0.x, q0.y);
      mma_f16_16816(fa, alo[1], blo[1], ahi[1], bhi[1], q0.z, q0.w);
      mma_f16_16816(fa, alo[2], blo[2], ahi[2], bhi[2], q1.x, q1.y);
      mma_f16_16816(fa, alo[3], blo[3], ahi[3], bhi[3], q1.z, q1.w);
    }
    return;
  }
  uint32_t wa0 = tc4<FMT, FAST>(w0.x, fs0, inv0), wa1 = tc4<FMT, FAST>(w0.y, fs0, inv0);
  uint32_t wa2 = tc4<FMT, FAST>(w0.z, fs0, inv0), wa3 = tc4<FMT, FAST>(w0.w, fs0, inv0);
  uint32_t wb0 = tc4<FMT, FAST>(w1.x, fs1, inv1), wb1 = tc4<FMT, FAST>(w1.y, fs1, inv1);
  uint32_t wb2 = tc4<FMT, FAST>(w1.z, fs1, inv1), wb3 = tc4<FMT, FAST>(w1.w, fs1, inv1);
  const int8_t* arow = aq + koff + 64 * h + 16 * t;
#pragma unroll
  for (int nb = 0; nb < MB; ++nb) {
    uint4 q = lds128(arow + (nb * 8 + g) * astride);
    if (is_native<FMT>()) {
      float(&fa)[4] = *reinterpret_cast<float(*)[4]>(&acc[nb][0]);
      mma_f8_16832<FMT>(fa, wa0, wb0, wa1, wb1, q.x, q.y);
      mma_f8_16832<FMT>(fa, wa2, wb2, wa3, wb3, q.z, q.w);
    } else {
      mma_s8_16832(acc[nb], wa0, wb0, wa1, wb1, q.x, q.y);
      mma_s8_16832(acc[nb], wa2, wb2, wa3, wb3, q.z, q.w);
    }
  }
}

template <int AT, int MB, int FMT, bool FAST>
__device__ __forceinline__ void consumer_loop(const GemvParams& p, int (&acc)[MB][4], const uint8_t* stages,
                                              uint64_t* full, uint64_t* empty, int8_t* aq, int astride, int m0,
                                              int kbeg, int kend, int nkb, uint32_t fs0, uint32_t fs1, uint16_t inv0,
                                              uint16_t inv1, int warp, int lane) {
  constexpr int MR = MB * 8;
  const int g = lane >> 2, t = lane & 3;
  const int rowA = warp * 16 + (g >> 1) + 4 * (g & 1);
  const int rowB = rowA + 8;
  const int swz = rowA & 7;  // == rowB & 7
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int i = 0; i < nkb; ++i) {
    const int koff = (i * kBlockK) % p.kc;
    if (koff == 0 && i > 0) {
      named_bar_sync(1, kConsumers);
      int k0 = kbeg + i * kBlockK;
      int len = min(p.kc, kend - k0);
      len = (len + 63) & ~63;
      stage_chunk<AT, MR, FMT>(p, aq, astride, m0, k0, len, kend);
      named_bar_sync(1, kConsumers);
      if (i == 0 && threadIdx.x == 0) TRACE_POINT(p, 3);
    }
    if (ok) ok = mbar_wait(&full[stage], phase, ERR_WAIT_FULL);
    if (i == 0 && threadIdx.x == 0) TRACE_POINT(p, 4);
    const uint8_t* st = stages + stage * kStageBytes;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      mma_half<AT, MB, FMT, FAST>(p, acc, st, aq, astride, koff, h, rowA, rowB, swz, g, t, fs0, fs1, inv0, inv1);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == kStages) {
      stage = 0;
      phase ^= 1u;
    }
  }
}

// Epilogue of one output element from its reduced sum (int32 bits, or fp32
// bits for the float-accumulating modes): scales, cast, store.
template <int FMT>
__device__ __forceinline__ void store_out(const GemvParams& p, int n, int m, int32_t sum, float sc, float cs,
                                          float rg) {
  if (FMT == FMT_WGT) {  // fp32 row-major output C[m][n]
    static_cast<float*>(p.D)[(size_t)m * p.N + n] = __int_as_float(sum);
    return;
  }
  float v;
  if (is_native<FMT>()) {
    v = __int_as_float(sum) * rg * cs;
  } else {
    float se = sc * rg;
    if (p.col_scale_f32) se = se * cs;
    v = (float)sum * se;
    if (p.acc_out) p.acc_out[(size_t)n * p.M + m] = sum;
  }
  const uint16_t o = store_val(bias_act(v, p.bias, n, p.act), p.out_bf16);
  uint16_t* D = static_cast<uint16_t*>(p.D);
  if (p.out_row_major) {
    D[(size_t)m * p.N + n] = o;
  } else {
    D[(size_t)n * p.M + m] = o;
  }
}

// Column-parallel output gather fused into the epilogue (world > 1): the
// CTA's finished outputs (columns [n_lo, n_hi), rows [m0, m0+MR) of this
// rank's slice, already stored locally) are copied into the same place of
// every peer's full output with 16-byte stores over NVLink. Publication
// (peer_signal_and_wait): one system-scope release increment per cluster of
// this rank's counter in each peer's signal pad (slots kPeerFusedSlot +
// rank); the first CTA of the grid then advances this rank's call epoch (slot
// kPeerFusedEpochSlot of its own pad) and waits (bounded) until every peer's
// counter in its own pad has reached epoch x (clusters per grid).
__device__ __forceinline__ void peer_copy(const GemvParams& p, int n_lo, int n_hi, int m0, int MR) {
  __syncthreads();  // this CTA's local output stores are done
  const int m1 = min(p.M, m0 + MR);
  if (n_lo < n_hi && m0 < m1) {
    const uint8_t* src = static_cast<const uint8_t*>(p.D);
    if (m0 == 0 && m1 == p.M) {  // one contiguous run of the col-major slice
      const size_t b0 = (size_t)n_lo * p.M * 2, nb = (size_t)(n_hi - n_lo) * p.M * 2;
      for (int q = 0; q < p.world; ++q) {
        if (q == p.rank) continue;
        uint8_t* dst = reinterpret_cast<uint8_t*>(p.peer_rows[q]);
        if (((reinterpret_cast<uintptr_t>(src + b0) | reinterpret_cast<uintptr_t>(dst + b0) | nb) & 15u) == 0) {
          for (size_t i = threadIdx.x; i < (nb >> 4); i += blockDim.x)
            reinterpret_cast<uint4*>(dst + b0)[i] = reinterpret_cast<const uint4*>(src + b0)[i];
        } else {
          for (size_t i = threadIdx.x; i < (nb >> 1); i += blockDim.x)
            reinterpret_cast<uint16_t*>(dst + b0)[i] = reinterpret_cast<const uint16_t*>(src + b0)[i];
        }
      }
    } else {  // per-column runs of m1 - m0 rows
      const int rows = m1 - m0, cnt = (n_hi - n_lo) * rows;
      for (int q = 0; q < p.world; ++q) {
        if (q == p.rank) continue;
        uint16_t* dst = reinterpret_cast<uint16_t*>(p.peer_rows[q]);
        for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
          const int c = i / rows, r = i - c * rows;
          const size_t off = (size_t)(n_lo + c) * p.M + m0 + r;
          dst[off] = reinterpret_cast<const uint16_t*>(src)[off];
        }
      }
    }
  }
}

// After the cluster barrier that ends the kernel (which orders every CTA's
// peer stores of the cluster before it): the cluster's first CTA publishes
// them with one system-scope release per peer, and the grid's first CTA waits
// until every peer has published all of its clusters for this call. Every
// call adds exactly kPeerCallUnits to each counter whatever its grid (cluster
// i adds its share floor((i+1)U/n) - floor(iU/n) of U over n clusters), so
// calls of different shapes in a row keep the per-call targets e * U aligned.
constexpr unsigned int kPeerCallUnits = 1u << 20;

__device__ __forceinline__ void peer_signal_and_wait(const GemvParams& p, unsigned int cluster_rank,
                                                     unsigned int clusters, unsigned int cluster_id,
                                                     unsigned int* target_s) {
  if (cluster_rank != 0) return;
  if ((int)threadIdx.x < p.world && (int)threadIdx.x != p.rank) {
    const unsigned long long U = kPeerCallUnits;
    const unsigned int share = (unsigned int)(((cluster_id + 1ull) * U) / clusters - ((unsigned long long)cluster_id * U) / clusters);
    unsigned int* slot = reinterpret_cast<unsigned int*>(p.peer_sig[threadIdx.x]) + kPeerFusedSlot + p.rank;
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(slot), "r"(share) : "memory");
  }
  if (blockIdx.x != 0 || blockIdx.y != 0 || blockIdx.z != 0) return;
  if (threadIdx.x == 0) {
    unsigned int e = p.epoch;
    if (e == 0) {  // epoch counted on the device: advances on every launch, graph replays included
      unsigned int* ctr = reinterpret_cast<unsigned int*>(p.peer_sig[p.rank]) + kPeerFusedEpochSlot;
      e = *ctr + 1;
      *ctr = e;
    }
    *target_s = e * kPeerCallUnits;  // modulo 2^32; compared by signed difference below
  }
  __syncthreads();
  const unsigned int target = *target_s;
  if ((int)threadIdx.x < p.world && (int)threadIdx.x != p.rank) {
    const unsigned int* mine = reinterpret_cast<const unsigned int*>(p.peer_sig[p.rank]) + kPeerFusedSlot + threadIdx.x;
    const unsigned long long t0 = globaltimer_ns();
    for (;;) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int)(v - target) >= 0) break;
      const unsigned long long dt = globaltimer_ns() - t0;
      if (dt > kWaitCheckNs && dt > *(volatile unsigned long long*)&g_fp8imma_wait_limit_ns) {
        atomicCAS(&g_fp8imma_device_error, 0u, ERR_WAIT_PEER);
        break;
      }
    }
  }
  __syncthreads();
}

template <int AT, int MB, int FMT>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_s8_splitk_kernel(const __grid_constant__ GemvParams p, const __grid_constant__ CUtensorMap tmap) {
  constexpr int MR = MB * 8;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOffset);
  uint64_t* empty = full + kStages;
  int8_t* aq = reinterpret_cast<int8_t*>(smem + kAqOffset);
  int32_t* part = reinterpret_cast<int32_t*>(smem + kAqOffset);  // reused after the main loop

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile_n0 = blockIdx.x * kTileN;
  const int m0 = blockIdx.z * MR;
  const int kbeg = blockIdx.y * p.k_per_cta;
  const int kend = min(p.K, kbeg + p.k_per_cta);
  const int nkb = kend > kbeg ? (kend - kbeg + kBlockK - 1) / kBlockK : 0;
  // +64 B (int8) / +16 B (fp16): conflict-free 16-byte fragment loads
  const int astride = FMT == FMT_WGT ? 2 * p.kc + 16 : p.kc + 64;

  if (threadIdx.x == 0) TRACE_POINT(p, 0);
  TRACE_SMID(p);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  const int g = lane >> 2;
  const int lc0 = warp * 16 + (g >> 1) + 4 * (g & 1);  // MMA rows g / g+8 -> tile columns lc0 / lc0+8
  const bool consumer = warp < kConsumerWarps;
  int acc[MB][4];
#pragma unroll
  for (int i = 0; i < MB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0;

  if (!consumer) {
    // ---- TMA producer: weights are streamed from the first cycle (they do
    // not depend on the previous kernel in the stream)
    if (lane != 0) {
      // the other 31 lanes pull this CTA's first activation chunk and its
      // column scales towards L2 while the consumers start up
      const int esz = AT == A_S8 ? 1 : 2;
      const int rows = min(MR, p.M - m0);
      const int bytes = (min(kend, kbeg + p.kc) - kbeg) * esz;
      const int lines_per_row = (bytes + 127) >> 7;
      const char* abase = static_cast<const char*>(p.A) + ((size_t)m0 * p.K + kbeg) * esz;
      for (int i = lane - 1; i < rows * lines_per_row; i += 31) {
        const int r = i / lines_per_row, l = i - r * lines_per_row;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(abase + (size_t)r * p.K * esz + ((size_t)l << 7)));
      }
      if (!is_float_acc<FMT>() && !p.scale_tex && lane <= 2)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(p.scale_u16 + tile_n0) + (lane - 1) * 128));
    }
    if (lane == 0) {
      prefetch_tensormap(&tmap);
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&full[stage], kStageBytes);
        tma_load_2d(stages + stage * kStageBytes, &tmap, &full[stage], kbeg + i * kBlockK, tile_n0);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    const int col0 = tile_n0 + lc0, col1 = col0 + 8;
    const bool ok0 = col0 < p.N, ok1 = col1 < p.N;
    // column scales are requested first; their latency overlaps the first
    // activation chunk's loads below
    const uint16_t sb0 = (ok0 && !is_float_acc<FMT>()) ? load_col_scale_bits(p, col0) : (uint16_t)0;
    const uint16_t sb1 = (ok1 && !is_float_acc<FMT>()) ? load_col_scale_bits(p, col1) : (uint16_t)0;
    const float cs0 = (ok0 && p.col_scale_f32) ? p.col_scale_f32[col0] : 1.0f;
    const float cs1 = (ok1 && p.col_scale_f32) ? p.col_scale_f32[col1] : 1.0f;
    if (p.pdl) pdl_wait();  // activations may come from the previous kernel
    float rg = 0.0f;
    if (threadIdx.x < MR && m0 + (int)threadIdx.x < p.M) rg = p.row_g ? p.row_g[m0 + threadIdx.x] : p.global_scale;
    if (nkb > 0) {
      int len = min(p.kc, kend - kbeg);
      len = (len + 63) & ~63;
      stage_chunk<AT, MR, FMT>(p, aq, astride, m0, kbeg, len, kend);
    }
    // epilogue constants staged in shared memory (no global loads at the end)
    float* sc_s = reinterpret_cast<float*>(smem + kScaleOffset);
    float* cs_s = reinterpret_cast<float*>(smem + kColScaleOffset);
    if ((lane & 3) == 0) {
      sc_s[lc0] = __half2float(__ushort_as_half(sb0));
      sc_s[lc0 + 8] = __half2float(__ushort_as_half(sb1));
    } else if ((lane & 3) == 1) {
      cs_s[lc0] = cs0;
      cs_s[lc0 + 8] = cs1;
    }
    if (threadIdx.x < MR) reinterpret_cast<float*>(smem + kRowScaleOffset)[threadIdx.x] = rg;
    const uint16_t inv0 = (ok0 && !is_float_acc<FMT>()) ? inv_scale_bits(sb0) : (uint16_t)0x3C00u;
    const uint16_t inv1 = (ok1 && !is_float_acc<FMT>()) ? inv_scale_bits(sb1) : (uint16_t)0x3C00u;
    // CTA-uniform transcode choice; also the barrier that publishes chunk 0
    const bool lane_fast = FMT == FMT_WGT ? p.wgt_fast != 0 : (fast_ok<FMT>(inv0) && fast_ok<FMT>(inv1));
    const bool all_fast = named_bar_and(2, kConsumers, lane_fast);
    if (threadIdx.x == 0) TRACE_POINT(p, 2);
    const uint32_t fs0 = fast_scale<FMT>(inv0), fs1 = fast_scale<FMT>(inv1);
    if (all_fast)
      consumer_loop<AT, MB, FMT, true>(p, acc, stages, full, empty, aq, astride, m0, kbeg, kend, nkb, fs0, fs1,
                                       inv0, inv1, warp, lane);
    else
      consumer_loop<AT, MB, FMT, false>(p, acc, stages, full, empty, aq, astride, m0, kbeg, kend, nkb, fs0, fs1,
                                        inv0, inv1, warp, lane);
  }

  // ---- partials -> shared memory, [128 cols][MR] int32
  __syncthreads();
  if (p.pdl) pdl_launch_dependents();  // the next grid's prologue overlaps this epilogue
  if (consumer) {
    const int t = lane & 3;
#pragma unroll
    for (int nb = 0; nb < MB; ++nb) {
      *reinterpret_cast<int2*>(part + lc0 * MR + nb * 8 + 2 * t) = make_int2(acc[nb][0], acc[nb][1]);
      *reinterpret_cast<int2*>(part + (lc0 + 8) * MR + nb * 8 + 2 * t) = make_int2(acc[nb][2], acc[nb][3]);
    }
  }
  cg::cluster_group cluster = cg::this_cluster();
  if (threadIdx.x == 0) TRACE_POINT(p, 5);
  cluster.sync();
  if (threadIdx.x == 0) TRACE_POINT(p, 6);
  if (p.pdl) pdl_wait();  // outputs may still be read by the previous kernel

  // ---- cluster reduction + epilogue: CTA rank r finishes 128/S columns
  const int S = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int cols_per = kTileN / S;
  const int nelem = cols_per * MR;
  const float* sc_s = reinterpret_cast<const float*>(smem + kScaleOffset);
  const float* cs_s = reinterpret_cast<const float*>(smem + kColScaleOffset);
  const float* rg_s = reinterpret_cast<const float*>(smem + kRowScaleOffset);
  constexpr int kEpiBatch = 4;  // partial-sum reads in flight per thread
  const int32_t* peer_part[8];  // distributed shared memory address of each cluster rank's partials
#pragma unroll
  for (int q = 0; q < 8; ++q) peer_part[q] = q < S ? cluster.map_shared_rank(part, q) : part;
  for (int base = threadIdx.x; base < nelem; base += kEpiBatch * kThreads) {
    int32_t sum[kEpiBatch];
    int lcs[kEpiBatch], mrs[kEpiBatch];
#pragma unroll
    for (int j = 0; j < kEpiBatch; ++j) {
      const int e = base + j * kThreads;
      int lc = 0, mr = 0;
      if (p.out_row_major) {
        mr = e / cols_per;
        lc = rank * cols_per + (e - mr * cols_per);
      } else {
        lc = rank * cols_per + e / MR;
        mr = e % MR;
      }
      lcs[j] = lc;
      mrs[j] = mr;
      int32_t acc_s = 0;
      float acc_f = 0.0f;
      if (e < nelem) {
        // all S remote partials of the element in flight at once, summed in rank order
        int32_t v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = q < S ? peer_part[q][lc * MR + mr] : 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (q >= S) break;
          if (is_float_acc<FMT>()) acc_f += __int_as_float(v[q]);
          else acc_s += v[q];
        }
      }
      sum[j] = is_float_acc<FMT>() ? __float_as_int(acc_f) : acc_s;
    }
#pragma unroll
    for (int j = 0; j < kEpiBatch; ++j) {
      const int e = base + j * kThreads;
      const int lc = lcs[j], mr = mrs[j];
      const int n = tile_n0 + lc, m = m0 + mr;
      if (e >= nelem || n >= p.N || m >= p.M) continue;
      store_out<FMT>(p, n, m, sum[j], sc_s[lc], cs_s[lc], rg_s[mr]);
    }
  }
  if (threadIdx.x == 0) TRACE_POINT(p, 7);
  if (p.world > 1) peer_copy(p, tile_n0 + rank * cols_per, min(p.N, tile_n0 + (rank + 1) * cols_per), m0, MR);
  cluster.sync();  // keep shared memory alive until every peer has read it
  if (threadIdx.x == 0) TRACE_POINT(p, 8);
  if (p.world > 1)
    peer_signal_and_wait(p, (unsigned int)rank, (gridDim.x * gridDim.y * gridDim.z) / (unsigned int)S,
                         blockIdx.x + gridDim.x * blockIdx.z,  // clusters span y (the K slices)
                         reinterpret_cast<unsigned int*>(smem + kBarOffset + 128));
}

// ---------------------------------------------------------------------------
// Stream-K form (default). Persistent CTAs, two per SM, no clusters: the work
// (m-chunk, 128-column tile, 64-wide K half) units are laid out tile-major and
// CTA c takes units [c*U/G, (c+1)*U/G), so every SM gets the same number of
// weight bytes to within one 8 KB half-block whatever N and K are. A CTA's
// range is a run of segments, one per column tile it touches; only its first
// and last segment can be a part of a tile. Whole tiles are finished from
// registers; a part writes int32 (fp32 bits) partials to the CTA's global
// slot, and the CTA that brings the tile's arrival counter to its contributor
// count sums the slots (L2 reads) and stores the epilogue, then re-arms the
// counter. No CTA ever waits for another.

// (unit counts fit in int: the launcher keeps U below 2^31)
__device__ __forceinline__ int sk_begin(int c, int U, int G) { return (int)((long long)c * U / G); }
// the CTA whose range holds unit u
__device__ __forceinline__ int sk_owner(int u, int U, int G) { return (int)(((long long)(u + 1) * G - 1) / U); }

template <int AT, int MB, int FMT, bool FAST>
__device__ __forceinline__ bool segment_loop(const GemvParams& p, int (&acc)[MB][4], const uint8_t* stages,
                                             uint64_t* full, uint64_t* empty, int8_t* aq, int astride, int m0,
                                             int hs, int he, int kseg0, int kvalid, uint32_t fs0, uint32_t fs1,
                                             uint16_t inv0, uint16_t inv1, int warp, int lane, int& stage,
                                             uint32_t& phase, bool ok) {
  constexpr int MR = MB * 8;
  const int g = lane >> 2, t = lane & 3;
  const int rowA = warp * 16 + (g >> 1) + 4 * (g & 1);
  const int rowB = rowA + 8;
  const int swz = rowA & 7;
  const int b0 = hs >> 1, b1 = (he + 1) >> 1;
  for (int b = b0; b < b1; ++b) {
    const int rel = (b - b0) * kBlockK;
    const int koff = rel % p.kc;
    if (koff == 0 && rel > 0) {
      named_bar_sync(1, kConsumers);
      const int k0 = kseg0 + rel;
      int len = min(p.kc, kvalid - k0);
      len = (len + 63) & ~63;
      stage_chunk<AT, MR, FMT>(p, aq, astride, m0, k0, len, kvalid);
      named_bar_sync(1, kConsumers);
    }
    if (ok) ok = mbar_wait(&full[stage], phase, ERR_WAIT_FULL);
    const uint8_t* st = stages + stage * kStageBytes;
    if (2 * b >= hs && 2 * b + 2 <= he) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
        mma_half<AT, MB, FMT, FAST>(p, acc, st, aq, astride, koff, h, rowA, rowB, swz, g, t, fs0, fs1, inv0, inv1);
    } else {  // a segment that starts or ends on an odd half
      const int h = 2 * b < hs ? 1 : 0;
      mma_half<AT, MB, FMT, FAST>(p, acc, st, aq, astride, koff, h, rowA, rowB, swz, g, t, fs0, fs1, inv0, inv1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == kStages) {
      stage = 0;
      phase ^= 1u;
    }
  }
  return ok;
}

template <int AT, int MB, int FMT>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_streamk_kernel(const __grid_constant__ GemvParams p, const __grid_constant__ CUtensorMap tmap,
                        int32_t* __restrict__ partials, unsigned int* __restrict__ counters) {
  constexpr int MR = MB * 8;
  constexpr int kSlot = kTileN * MR;  // int32 words per partial slot
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOffset);
  uint64_t* empty = full + kStages;
  int8_t* aq = reinterpret_cast<int8_t*>(smem + kAqOffset);
  int32_t* part = reinterpret_cast<int32_t*>(smem + kAqOffset);  // whole-tile epilogue staging
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + kBarOffset + 2 * kStages * 8);
  float* sc_s = reinterpret_cast<float*>(smem + kScaleOffset);
  float* cs_s = reinterpret_cast<float*>(smem + kColScaleOffset);
  float* rg_s = reinterpret_cast<float*>(smem + kRowScaleOffset);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = gridDim.x;
  const int cta = blockIdx.x;
  const int tiles = (p.N + kTileN - 1) / kTileN;
  const int hpt = (p.K + 63) >> 6;  // 64-wide K halves per tile
  const int per_mc = (int)tiles * hpt;
  const int U = per_mc * ((p.M + MR - 1) / MR);
  const int ub = sk_begin(cta, U, G), ue = sk_begin(cta + 1, U, G);
  const int astride = FMT == FMT_WGT ? 2 * p.kc + 16 : p.kc + 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---- TMA producer: the same segment walk, one 16 KB block per stage
    if (lane == 0) {
      prefetch_tensormap(&tmap);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = ub; u < ue && ok;) {
        const int rem = u % per_mc;
        const int tile = (int)(rem / hpt), hs = (int)(rem % hpt);
        const int se = min(ue, u - hs + hpt);
        const int he = hs + (int)(se - u);
        for (int b = hs >> 1; b < (he + 1) >> 1; ++b) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, ERR_WAIT_EMPTY)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(stages + stage * kStageBytes, &tmap, &full[stage], b * kBlockK, tile * kTileN);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        u = se;
      }
    }
    return;
  }

  // ---- consumers
  if (threadIdx.x == 0) TRACE_POINT(p, 0);
  if (p.pdl) pdl_wait();
  const int g = lane >> 2, t = lane & 3;
  const int lc0 = warp * 16 + (g >> 1) + 4 * (g & 1);
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int u = ub; u < ue;) {
    const int mcl = u / per_mc;
    const int rem = u - mcl * per_mc;
    const int tile = (int)(rem / hpt), hs = (int)(rem % hpt);
    const int se = min(ue, u - hs + hpt);
    const int he = hs + (int)(se - u);
    const int tile_u0 = u - hs;
    const int m0 = (int)mcl * MR, tile_n0 = tile * kTileN;
    const int kseg0 = (hs >> 1) * kBlockK;
    const int kvalid = min(p.K, he * 64);
    const int col0 = tile_n0 + lc0, col1 = col0 + 8;
    const bool ok0 = col0 < p.N, ok1 = col1 < p.N;
    const uint16_t sb0 = (ok0 && !is_float_acc<FMT>()) ? load_col_scale_bits(p, col0) : (uint16_t)0;
    const uint16_t sb1 = (ok1 && !is_float_acc<FMT>()) ? load_col_scale_bits(p, col1) : (uint16_t)0;
    const float cs0 = (ok0 && p.col_scale_f32) ? p.col_scale_f32[col0] : 1.0f;
    const float cs1 = (ok1 && p.col_scale_f32) ? p.col_scale_f32[col1] : 1.0f;
    float rg = 0.0f;
    if (threadIdx.x < MR && m0 + (int)threadIdx.x < p.M) rg = p.row_g ? p.row_g[m0 + threadIdx.x] : p.global_scale;
    named_bar_sync(1, kConsumers);  // the previous segment is done with aq / part / the constants
    {
      int len = min(p.kc, kvalid - kseg0);
      len = (len + 63) & ~63;
      stage_chunk<AT, MR, FMT>(p, aq, astride, m0, kseg0, len, kvalid);
    }
    if ((lane & 3) == 0) {
      sc_s[lc0] = __half2float(__ushort_as_half(sb0));
      sc_s[lc0 + 8] = __half2float(__ushort_as_half(sb1));
    } else if ((lane & 3) == 1) {
      cs_s[lc0] = cs0;
      cs_s[lc0 + 8] = cs1;
    }
    if (threadIdx.x < MR) rg_s[threadIdx.x] = rg;
    const uint16_t inv0 = (ok0 && !is_float_acc<FMT>()) ? inv_scale_bits(sb0) : (uint16_t)0x3C00u;
    const uint16_t inv1 = (ok1 && !is_float_acc<FMT>()) ? inv_scale_bits(sb1) : (uint16_t)0x3C00u;
    const bool lane_fast = FMT == FMT_WGT ? p.wgt_fast != 0 : (fast_ok<FMT>(inv0) && fast_ok<FMT>(inv1));
    const bool all_fast = named_bar_and(2, kConsumers, lane_fast);  // also publishes chunk 0
    if (threadIdx.x == 0 && u == ub) TRACE_POINT(p, 2);
    const uint32_t fs0 = fast_scale<FMT>(inv0), fs1 = fast_scale<FMT>(inv1);
    int acc[MB][4];
#pragma unroll
    for (int i = 0; i < MB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0;
    if (all_fast)
      ok = segment_loop<AT, MB, FMT, true>(p, acc, stages, full, empty, aq, astride, m0, hs, he, kseg0, kvalid, fs0,
                                           fs1, inv0, inv1, warp, lane, stage, phase, ok);
    else
      ok = segment_loop<AT, MB, FMT, false>(p, acc, stages, full, empty, aq, astride, m0, hs, he, kseg0, kvalid, fs0,
                                            fs1, inv0, inv1, warp, lane, stage, phase, ok);

    if (threadIdx.x == 0 && u == ub) TRACE_POINT(p, 4);
    const int nelem = kTileN * MR;
    if (hs == 0 && he == hpt) {
      // whole tile: registers -> shared memory -> epilogue
      named_bar_sync(1, kConsumers);  // every warp is done reading aq
#pragma unroll
      for (int nb = 0; nb < MB; ++nb) {
        *reinterpret_cast<int2*>(part + lc0 * MR + nb * 8 + 2 * t) = make_int2(acc[nb][0], acc[nb][1]);
        *reinterpret_cast<int2*>(part + (lc0 + 8) * MR + nb * 8 + 2 * t) = make_int2(acc[nb][2], acc[nb][3]);
      }
      named_bar_sync(1, kConsumers);
      for (int e = threadIdx.x; e < nelem; e += kConsumers) {
        int lc, mr;
        if (p.out_row_major || FMT == FMT_WGT) {
          mr = e / kTileN;
          lc = e - mr * kTileN;
        } else {
          lc = e / MR;
          mr = e - lc * MR;
        }
        const int n = tile_n0 + lc, m = m0 + mr;
        if (n < p.N && m < p.M) store_out<FMT>(p, n, m, part[lc * MR + mr], sc_s[lc], cs_s[lc], rg_s[mr]);
      }
    } else {
      // part of a tile: partials -> this CTA's slot; the last arrival finishes
      const int slot = ub >= tile_u0 ? 0 : 1;  // the tile is this CTA's first (0) or last (1) segment
      int32_t* mine = partials + ((size_t)cta * 2 + slot) * kSlot;
#pragma unroll
      for (int nb = 0; nb < MB; ++nb) {
        *reinterpret_cast<int2*>(mine + lc0 * MR + nb * 8 + 2 * t) = make_int2(acc[nb][0], acc[nb][1]);
        *reinterpret_cast<int2*>(mine + (lc0 + 8) * MR + nb * 8 + 2 * t) = make_int2(acc[nb][2], acc[nb][3]);
      }
      named_bar_sync(1, kConsumers);
      const int cf = sk_owner(tile_u0, U, G), cl = sk_owner(tile_u0 + hpt - 1, U, G);
      if (threadIdx.x == 0) {
        // acq_rel: releases this CTA's partials (ordered before by the barrier)
        // and, for the last arrival, acquires every other contributor's
        unsigned int* ctr = counters + mcl * tiles + tile;
        unsigned int prev;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ctr) : "memory");
        const int last = prev == (unsigned int)(cl - cf);
        if (last) *ctr = 0u;  // re-armed for the next call
        *last_flag = last;
      }
      named_bar_sync(1, kConsumers);
      if (threadIdx.x == 0 && u == ub) TRACE_POINT(p, 5);
      if (*last_flag) {
        // 4 consecutive rows of one column per thread, up to 8 contributors'
        // 16-byte partials in flight at once
        const int ncontrib = (int)(cl - cf + 1);
        for (int qd = threadIdx.x; qd < kTileN * MR / 4; qd += kConsumers) {
          const int lc = qd / (MR / 4), mr0 = (qd - lc * (MR / 4)) * 4;
          int si[4] = {0, 0, 0, 0};
          float sf[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int j0 = 0; j0 < ncontrib; j0 += 4) {
            int4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (j0 + j < ncontrib) {
                const int q = cf + j0 + j;
                const int sl = sk_begin(q, U, G) >= tile_u0 ? 0 : 1;
                v[j] = __ldcg(reinterpret_cast<const int4*>(partials + ((size_t)q * 2 + sl) * kSlot + lc * MR + mr0));
              }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (j0 + j < ncontrib) {
                if (is_float_acc<FMT>()) {
                  sf[0] += __int_as_float(v[j].x);
                  sf[1] += __int_as_float(v[j].y);
                  sf[2] += __int_as_float(v[j].z);
                  sf[3] += __int_as_float(v[j].w);
                } else {
                  si[0] += v[j].x;
                  si[1] += v[j].y;
                  si[2] += v[j].z;
                  si[3] += v[j].w;
                }
              }
            }
          }
          const int n = tile_n0 + lc;
          if (n < p.N) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const int m = m0 + mr0 + r;
              if (m < p.M)
                store_out<FMT>(p, n, m, is_float_acc<FMT>() ? __float_as_int(sf[r]) : si[r], sc_s[lc], cs_s[lc],
                               rg_s[mr0 + r]);
            }
          }
        }
      }
    }
    if (threadIdx.x == 0 && u == ub) TRACE_POINT(p, 6);
    u = se;
  }
  if (threadIdx.x == 0) TRACE_POINT(p, 8);
}

struct LaunchShape {
  int S, mchunks;
  size_t smem;
  int sk_grid;  // > 0: stream-K kernel on this many CTAs
  int32_t* partials;
  unsigned int* counters;
};

template <int AT, int MB, int FMT>
cudaError_t launch_t(const GemvParams& p, const CUtensorMap& tmap, const LaunchShape& ls, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = ls.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  cfg.attrs = attr;
  if (ls.sk_grid > 0) {
    auto kern = gemv_streamk_kernel<AT, MB, FMT>;
    cudaError_t e = ensure_smem_attr((const void*)kern, (int)ls.smem);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(ls.sk_grid, 1, 1);
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p, tmap, ls.partials, ls.counters);
  }
  auto kern = gemv_s8_splitk_kernel<AT, MB, FMT>;
  cudaError_t e = ensure_smem_attr((const void*)kern, (int)ls.smem);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3((p.N + kTileN - 1) / kTileN, ls.S, ls.mchunks);
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = ls.S;
  attr[1].val.clusterDim.z = 1;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, p, tmap);
}

template <int AT, int FMT>
cudaError_t launch_mb(const GemvParams& p, const CUtensorMap& tmap, int MB, const LaunchShape& ls, cudaStream_t st) {
  switch (MB) {
    case 1: return launch_t<AT, 1, FMT>(p, tmap, ls, st);
    case 2: return launch_t<AT, 2, FMT>(p, tmap, ls, st);
    case 3: return launch_t<AT, 3, FMT>(p, tmap, ls, st);
    default: return launch_t<AT, 4, FMT>(p, tmap, ls, st);
  }
}

// Stream-K scratch (arrival counters + partial sums): one buffer per (device,
// stream), allocated on first use outside stream capture and never freed, so
// captured graphs keep valid pointers. Calls on one stream are ordered (also
// with programmatic dependent launch: every use of the scratch follows the
// kernel's griddepcontrol.wait), so they never share it concurrently.
constexpr int kSkMinUnits = 6;
constexpr int kSkAutoUnits = 48;
constexpr int kSkMaxCounters = 16384;  // m-chunks x column tiles per call
std::atomic<int> g_stream_k{1};

bool stream_k_scratch(cudaStream_t st, int grid_max, bool may_alloc, int32_t** part, unsigned int** ctr) {
  if (!may_alloc) return false;
  const size_t part_bytes = (size_t)grid_max * 2 * kTileN * 32 * sizeof(int32_t);
  char* s = static_cast<char*>(stream_scratch(st, (size_t)kSkMaxCounters * 4 + part_bytes, 0));
  if (!s) return false;
  *ctr = reinterpret_cast<unsigned int*>(s);
  *part = reinterpret_cast<int32_t*>(s + (size_t)kSkMaxCounters * 4);
  return true;
}

}  // namespace

int gemv_pick_splits(int N, int K, int mchunks, int num_sms) {
  int tiles = (N + kTileN - 1) / kTileN;
  int S = 1;
  while (S < 8 && tiles * mchunks * S < 2 * num_sms && K / (S * 2) >= 256) S *= 2;
  return S;
}

static cudaError_t launch_gemv_impl(GemvParams p, int a_type, int fmt, int splits, cudaStream_t stream);

thread_local bool t_used_decode = false;
bool gemv_last_used_decode() { return t_used_decode; }

bool gemv_would_decode(const GemvParams& p, int a_type, int fmt, int splits) {
  return splits == 0 && g_stream_k.load() != 2 && decode_applicable(p, a_type, fmt);
}

cudaError_t launch_gemv_s8(GemvParams p, int a_type, int fmt, int splits, cudaStream_t stream) {
  // shapes that fit one balanced wave (decode sizes) take the one-CTA-per-SM kernel
  t_used_decode = gemv_would_decode(p, a_type, fmt, splits);
  if (t_used_decode) {
    const cudaError_t e = launch_decode(p, a_type, fmt, stream);
    if (e != cudaErrorNotSupported) return e;
    t_used_decode = false;  // the shape needs the pre-pass, which had no scratch: split-K kernels instead
  }
  // host buffers in place are only ever handed to the decode kernel
  if (p.a_host || p.d_host) return cudaErrorNotSupported;
  // Every column tile stages and quantises its own copy of the activations;
  // when that repeated work is large (many tiles, M >= 16) the activations are
  // quantised once by a pre-pass and the kernel copies int8 rows instead.
  const long long tiles = (p.N + kTileN - 1) / kTileN;
  if (!p.no_alloc && (fmt == FMT_E4M3_REF || fmt == FMT_E5M2) && (a_type == A_F16 || a_type == A_BF16) &&
      p.M >= 16 && (long long)p.M * p.K * tiles >= (16LL << 20) && p.keff_a == p.K) {
    ScopedScratch sc;
    cudaError_t e = sc.get((size_t)p.M * p.K, stream, kScratchGemvRows);
    if (e != cudaSuccess) return e;
    void* aq = sc.ptr;
    e = launch_quant_a_s8(p.A, a_type, p.M, p.K, p.a_inv_h, p.row_inv_h, static_cast<int8_t*>(aq), stream);
    if (e == cudaSuccess) {
      GemvParams q = p;
      q.A = aq;
      q.pdl = 1;  // weights stream while the pre-pass finishes; activations are read after it
      e = launch_gemv_impl(q, A_S8, fmt, splits, stream);
    }
    cudaError_t e2 = sc.release(stream);
    return e != cudaSuccess ? e : e2;
  }
  return launch_gemv_impl(p, a_type, fmt, splits, stream);
}

static cudaError_t launch_gemv_impl(GemvParams p, int a_type, int fmt, int splits, cudaStream_t stream) {
  if (fmt == FMT_E4M3FN || fmt == FMT_NATIVE_E5M2) a_type = A_S8;  // pre-quantised E4M3 activations are copied
  const int MB = p.M >= 32 ? 4 : (p.M + 7) / 8;
  const int MR = MB * 8;
  const int mchunks = (p.M + MR - 1) / MR;
  const int tiles = (p.N + kTileN - 1) / kTileN;
  // activation chunk staged per refill: 1024 K (fp16 rows at 32 rows: 512, to
  // keep two CTAs' shared memory within an SM)
  const int kc_max = (MR > 16 && fmt == FMT_WGT) ? 512 : 1024;
  LaunchShape ls = {};
  ls.mchunks = mchunks;
  const int sms = num_sms_current();
  // stream-K only where every CTA gets at least kSkAutoUnits halves (its
  // partial-tile fix-up, about 2 us, is then amortised): the large
  // projections, where the cluster form's 2-per-SM waves are uneven
  const long long all_units = (long long)mchunks * tiles * ((p.K + 63) / 64);
  const bool big = all_units >= (long long)kSkAutoUnits * 2 * sms;
  if (splits == 0 && p.world <= 1 && g_stream_k.load() && (g_stream_k.load() == 2 || big) &&
      (long long)tiles * mchunks <= kSkMaxCounters) {
    const long long units = (long long)mchunks * tiles * ((p.K + 63) / 64);
    // at least kSkMinUnits halves (48 KB of weights) per CTA keeps tiles to a few contributors
    const long long want = (units + kSkMinUnits - 1) / kSkMinUnits;
    const int grid = (int)(want < 2LL * sms ? want : 2LL * sms);
    if (units < (1LL << 30) && stream_k_scratch(stream, 2 * sms, !p.no_alloc, &ls.partials, &ls.counters)) {
      ls.sk_grid = grid;
      const int kr = (p.K + kBlockK - 1) & ~(kBlockK - 1);
      p.kc = kr < kc_max ? kr : kc_max;
      p.k_per_cta = p.K;
    }
  }
  if (ls.sk_grid == 0) {
    int S = splits > 0 ? splits : gemv_pick_splits(p.N, p.K, mchunks, num_sms_current());
    if (S != 1 && S != 2 && S != 4 && S != 8) return cudaErrorInvalidValue;
    int kper = (p.K + S - 1) / S;
    kper = (kper + 255) & ~255;
    p.k_per_cta = kper;
    p.kc = kper < kc_max ? kper : kc_max;
    ls.S = S;
  }
  size_t smem_a = fmt == FMT_WGT ? (size_t)MR * (2 * p.kc + 16) : (size_t)MR * (p.kc + 64);
  size_t smem_p = (size_t)kTileN * MR * 4;
  ls.smem = (size_t)kAqOffset + (smem_a > smem_p ? smem_a : smem_p) + 1024;  // + alignment slack
  CUtensorMap tmap;
  cudaError_t e = make_tmap_2d_u8(&tmap, p.B, (uint64_t)p.K, (uint64_t)p.N, (uint64_t)p.K, kBlockK, kTileN,
                                  /*swizzle128=*/true);
  if (e != cudaSuccess) return e;
  switch (a_type * 8 + fmt) {
    case A_F16 * 8 + FMT_E4M3_REF: return launch_mb<A_F16, FMT_E4M3_REF>(p, tmap, MB, ls, stream);
    case A_F16 * 8 + FMT_E5M2: return launch_mb<A_F16, FMT_E5M2>(p, tmap, MB, ls, stream);
    case A_BF16 * 8 + FMT_E4M3_REF: return launch_mb<A_BF16, FMT_E4M3_REF>(p, tmap, MB, ls, stream);
    case A_BF16 * 8 + FMT_E5M2: return launch_mb<A_BF16, FMT_E5M2>(p, tmap, MB, ls, stream);
    case A_S8 * 8 + FMT_E4M3_REF: return launch_mb<A_S8, FMT_E4M3_REF>(p, tmap, MB, ls, stream);
    case A_S8 * 8 + FMT_E5M2: return launch_mb<A_S8, FMT_E5M2>(p, tmap, MB, ls, stream);
    case A_S8 * 8 + FMT_E4M3FN: return launch_mb<A_S8, FMT_E4M3FN>(p, tmap, MB, ls, stream);
    case A_S8 * 8 + FMT_NATIVE_E5M2: return launch_mb<A_S8, FMT_NATIVE_E5M2>(p, tmap, MB, ls, stream);
    case A_F16 * 8 + FMT_WGT: return launch_mb<A_F16, FMT_WGT>(p, tmap, MB, ls, stream);
    default: return cudaErrorInvalidValue;
  }
}

void gemv_set_stream_k(int mode) { g_stream_k.store(mode); }

unsigned int gemv_device_error(bool clear) { return tu_device_error(clear); }
cudaError_t gemv_set_wait_limit(unsigned long long ns) { return tu_set_wait_limit(ns); }

}  // namespace fp8imma_b200
