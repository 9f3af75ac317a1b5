// Balanced decode-shape GEMM (M <= 16, int8-exact path): one CTA per SM.
//
// The weight matrix is cut into 8-column groups. A cluster of S CTAs (S = 1,
// or a pair on one TPC, S = 2) owns a contiguous run of G groups (G differs by
// at most one between clusters, so every SM streams the same number of
// weight bytes to within one group); the S CTAs of the cluster split K. The
// grid is a single wave of at most one CTA per SM.
//
// Inside a CTA (2*G consumer warps + one TMA producer warp):
//   * the producer requests a few weight stages (8G rows x 128 K-bytes, one
//     2-D TMA box with 128-byte swizzle), then the CTA's activation rows (one
//     2-D TMA box of up to 16 rows x 128 bytes each, issued after the previous
//     kernel has finished when launched with programmatic dependent launch),
//     then the rest of the weight stages: at decode sizes the ring holds the
//     whole K-slice, so every byte of the call is requested at once;
//   * the consumers quantise the activation rows from shared memory into an
//     int8 copy (row stride = 64 mod 128 bytes: conflict-free fragment loads);
//   * consumer warp (c, q) owns group c and every stage i = q (mod 2): two
//     16-byte conflict-free shared loads of its column's 128 bytes, the FP8 ->
//     int8 transcode in registers, and four mma.sync m16n8k32 s8 with the
//     weights as the B operand (8 columns) and the activation rows as the A
//     operand (16 rows), into four independent accumulator sets;
//   * the two warps of a group add their fragments through shared memory;
//     with S = 2 each CTA owns the epilogue of half of the groups and pushes
//     the other half's sums into its peer's shared memory with st.async,
//     completing on the peer's mbarrier (no cluster-wide barrier at the end).
// K order inside each 64-byte half is permuted identically for both operands
// (int32 sums do not depend on order). Lane group g reads weight column
// sigma(g) = (g>>1) + 4(g&1) of its group, which makes each 8-lane shared
// memory phase conflict-free under the 128-byte swizzle.
//
// Semantics (every rounding step) are those of the reference v4 kernel,
// src/fp8imma/impl/v4_kernels.inl:61-70 (weight transcode), 116-131
// (activation quantisation) and 280-285 (epilogue); the arithmetic helpers
// live in fp8imma_device.cuh.
#include "fp8imma_device.cuh"
#include "fp8imma_kernels.h"
#include "sm100_async.cuh"

#include <atomic>

using namespace fp8imma_dev;

namespace fp8imma_b200 {

namespace {

#ifndef DEC_WPG
#define DEC_WPG 2
#endif
constexpr int kDecMaxG = 8;        // 8-column groups per CTA
constexpr int kDecWpg = DEC_WPG;   // consumer warps per group (stage i goes to warp i mod kDecWpg)
constexpr int kDecBoxK = 128;      // K bytes per weight stage
constexpr int kDecMaxStages = 16;
constexpr int kDecMaxThreads = kDecMaxG * kDecWpg * 32 + 32;
constexpr int kDecEarlyStages = 4;  // weight stages requested before the activations
constexpr int kDecRows = 16;        // activation rows (one m16 block)
constexpr int kDecABox = 128;       // fp16/bf16 activation bytes per row per TMA box
constexpr int kDecQBox = 64;        // int8 activation bytes per row per TMA box (direct layout)

struct DecodeCfg {
  int S;            // CTAs per cluster (K split)
  int P;            // clusters
  int NG;           // 8-column groups in N
  int gmax;         // groups of the widest cluster
  int D;            // stage ring depth
  int kper;         // K per CTA (multiple of kDecBoxK)
  int astride;      // int8 activation row stride in shared memory (kper + 64)
  int stage_bytes;  // gmax * 1024
  int arows;        // activation rows moved per box (min(M, 16))
  int pre;          // the ring holds the whole K-slice: weights transcoded before the activations arrive
  int off_bar, off_const, off_raw, off_aq, off_tot, off_recv;
};

#ifdef FP8IMMA_TRACE
// per CTA 64 words: [0] %globaltimer at entry, [1] SM id, [2, 16) clock64
// cycles since entry at point i
// (kept in thread 0's registers and written at the end: a global store before
// the barrier-initialisation fence would make the fence wait for it)
#define DEC_TRACE(i)                                      \
  do {                                                    \
    if (threadIdx.x == 0) trace_pt[i] = clock64() - trace_clk0; \
  } while (0)
#define DEC_DBG(bit) ((dbg & (bit)) != 0)
#else
#define DEC_TRACE(i) do { } while (0)
#define DEC_DBG(bit) false
#endif

__device__ __forceinline__ void dec_mma(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 dec_lds128(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}

__device__ __forceinline__ void dec_sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ uint16_t dec_scale_bits(const GemvParams& p, int n) {
  if (p.scale_tex) return tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n);
  return p.scale_u16[n];
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
// 8-byte store into another CTA's shared memory, counted on its mbarrier
__device__ __forceinline__ void st_async_v2(uint32_t remote_addr, int a, int b, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.s32 [%0], {%1, %2}, [%3];" ::"r"(remote_addr), "r"(a),
      "r"(b), "r"(remote_bar)
      : "memory");
}

// Bounded mbarrier wait with the first probe inline and the polling loop out
// of line (keeps the hot loop small).
__device__ __noinline__ bool dec_wait_slow(uint64_t* bar, uint32_t parity, unsigned int err) {
  return mbar_wait(bar, parity, err);
}
__device__ __forceinline__ bool dec_wait(uint64_t* bar, uint32_t parity, unsigned int err) {
  if (mbar_try_wait(bar, parity)) return true;
  return dec_wait_slow(bar, parity, err);
}

template <int FMT, bool FAST>
__device__ __forceinline__ uint32_t dec_tc4(uint32_t x, uint32_t fscale, uint16_t inv_h) {
  if (FAST) return FMT == FMT_E5M2 ? transcode4_fast_e5m2(x, fscale) : transcode4_fast_e4m3(x, fscale);
  return transcode4_exact<FMT>(x, inv_h);
}

// Activation rows (TMA-staged, `raw`: box j = [arows][128 bytes] at j * 2048)
// -> int8 rows of `aq` (row stride astride), reference rounding. One item is
// 16 raw bytes: 8 fp16/bf16 values or 16 int8 values.
template <int AT>
__device__ __forceinline__ void dec_quant_rows(const uint8_t* raw, int8_t* aq, int astride, int nbox, int arows,
                                               const uint16_t* rowinv_s, int tid, int nthr) {
  const int per_box = arows * 8;
  const int total = nbox * per_box;
  // item it = jb * per_box + rem, advanced without divisions; four items'
  // shared loads in flight before any is converted
  const int djb = nthr / per_box, drem = nthr - djb * per_box;
  int jb = tid / per_box, rem = tid - jb * per_box;
  constexpr int kB = 4;
  for (int base = tid; base < total; base += kB * nthr) {
    uint4 v[kB];
    int off[kB];
    uint16_t ainv[kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const int r = rem >> 3, c = rem & 7;
      off[j] = -1;
      if (base + j * nthr < total) {
        v[j] = *reinterpret_cast<const uint4*>(raw + (size_t)jb * (kDecRows * kDecABox) + rem * 16);
        off[j] = r * astride + (AT == A_S8 ? jb * kDecABox + c * 16 : jb * (kDecABox / 2) + c * 8);
        ainv[j] = rowinv_s[r];
      }
      jb += djb;
      rem += drem;
      if (rem >= per_box) {
        rem -= per_box;
        ++jb;
      }
    }
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      if (off[j] < 0) break;
      if (AT == A_S8) {
        *reinterpret_cast<uint4*>(aq + off[j]) = v[j];
      } else {
        const uint32_t ainv2 = (uint32_t)ainv[j] | ((uint32_t)ainv[j] << 16);
        uint4 w = v[j];
        if (AT == A_BF16) {
          w.x = bf16x2_to_f16x2(w.x);
          w.y = bf16x2_to_f16x2(w.y);
          w.z = bf16x2_to_f16x2(w.z);
          w.w = bf16x2_to_f16x2(w.w);
        }
        *reinterpret_cast<uint2*>(aq + off[j]) = make_uint2(quant4_f16(w.x, w.y, ainv2), quant4_f16(w.z, w.w, ainv2));
      }
    }
  }
}

// One element of the epilogue from its int32 sum: scales in the reference's
// order, optional bias/activation, cast, store (col-major or row-major).
__device__ __forceinline__ void dec_store(const GemvParams& p, int n, int m, int32_t sum, float sc, float cs,
                                          float rg) {
  float se = sc * rg;
  if (p.col_scale_f32) se = se * cs;
  const float v = (float)sum * se;
  if (p.acc_out) p.acc_out[(size_t)n * p.M + m] = sum;
  const uint16_t o = store_val(bias_act(v, p.bias, n, p.act), p.out_bf16);
  uint16_t* D = static_cast<uint16_t*>(p.D);
  const size_t idx = p.out_row_major ? (size_t)m * p.N + n : (size_t)n * p.M + m;
  D[idx] = o;
  if (p.d_host) static_cast<uint16_t*>(p.d_host)[idx] = o;  // the host-buffer entry's output, in place
}

// One stage of a consumer warp: this lane's 2 x 16 weight bytes, eight
// transcodes, four MMAs into four accumulator sets.
// Activation fragment layout: `a_half` bytes from K half 0 to half 1 of a
// stage, `a_hi` bytes from rows 0..7 to rows 8..15.
template <int FMT, bool FAST, bool PRE>
__device__ __forceinline__ void dec_stage(int (&acc)[2][2][4], uint32_t w_addr, uint32_t a_addr, int a_half, int a_hi,
                                          bool hi_rows, uint32_t fs, uint16_t inv, int sw0, int sw1, int dbg) {
  const uint4 w0 = dec_lds128(w_addr + sw0);
  const uint4 w1 = dec_lds128(w_addr + sw1);
  uint32_t b[2][4];
  if (PRE || DEC_DBG(4)) {  // weights transcoded ahead (or experiment: no transcode)
    b[0][0] = w0.x; b[0][1] = w0.y; b[0][2] = w0.z; b[0][3] = w0.w;
    b[1][0] = w1.x; b[1][1] = w1.y; b[1][2] = w1.z; b[1][3] = w1.w;
  } else {
  b[0][0] = dec_tc4<FMT, FAST>(w0.x, fs, inv);
  b[0][1] = dec_tc4<FMT, FAST>(w0.y, fs, inv);
  b[0][2] = dec_tc4<FMT, FAST>(w0.z, fs, inv);
  b[0][3] = dec_tc4<FMT, FAST>(w0.w, fs, inv);
  b[1][0] = dec_tc4<FMT, FAST>(w1.x, fs, inv);
  b[1][1] = dec_tc4<FMT, FAST>(w1.y, fs, inv);
  b[1][2] = dec_tc4<FMT, FAST>(w1.z, fs, inv);
  b[1][3] = dec_tc4<FMT, FAST>(w1.w, fs, inv);
  }
  if (DEC_DBG(2)) {  // experiment: no MMA
    acc[0][0][0] ^= b[0][0] ^ b[0][1] ^ b[0][2] ^ b[0][3] ^ b[1][0] ^ b[1][1] ^ b[1][2] ^ b[1][3];
    return;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 x = dec_lds128(a_addr + a_half * h);
    uint4 y = make_uint4(0u, 0u, 0u, 0u);
    if (hi_rows) y = dec_lds128(a_addr + a_hi + a_half * h);
    dec_mma(acc[h][0], x.x, y.x, x.y, y.y, b[h][0], b[h][1]);
    dec_mma(acc[h][1], x.z, y.z, x.w, y.w, b[h][2], b[h][3]);
  }
}

// Two stages of a consumer warp at once: sixteen independent transcodes in
// flight (the warp count per SM is low, so the latency is hidden inside the
// warp), their MMAs into a second set of accumulators.
template <int FMT, bool FAST, bool PRE>
__device__ __forceinline__ void dec_stage2(int (&accA)[2][2][4], int (&accB)[2][2][4], uint32_t wA, uint32_t wB,
                                           uint32_t aA, uint32_t aB, int a_half, int a_hi, bool hi_rows, uint32_t fs,
                                           uint16_t inv, int sw0, int sw1) {
  const uint4 x0 = dec_lds128(wA + sw0), x1 = dec_lds128(wA + sw1);
  const uint4 y0 = dec_lds128(wB + sw0), y1 = dec_lds128(wB + sw1);
  uint32_t bA[2][4], bB[2][4];
  if (PRE) {
    bA[0][0] = x0.x; bA[0][1] = x0.y; bA[0][2] = x0.z; bA[0][3] = x0.w;
    bA[1][0] = x1.x; bA[1][1] = x1.y; bA[1][2] = x1.z; bA[1][3] = x1.w;
    bB[0][0] = y0.x; bB[0][1] = y0.y; bB[0][2] = y0.z; bB[0][3] = y0.w;
    bB[1][0] = y1.x; bB[1][1] = y1.y; bB[1][2] = y1.z; bB[1][3] = y1.w;
  } else {
  bA[0][0] = dec_tc4<FMT, FAST>(x0.x, fs, inv);
  bB[0][0] = dec_tc4<FMT, FAST>(y0.x, fs, inv);
  bA[0][1] = dec_tc4<FMT, FAST>(x0.y, fs, inv);
  bB[0][1] = dec_tc4<FMT, FAST>(y0.y, fs, inv);
  bA[0][2] = dec_tc4<FMT, FAST>(x0.z, fs, inv);
  bB[0][2] = dec_tc4<FMT, FAST>(y0.z, fs, inv);
  bA[0][3] = dec_tc4<FMT, FAST>(x0.w, fs, inv);
  bB[0][3] = dec_tc4<FMT, FAST>(y0.w, fs, inv);
  bA[1][0] = dec_tc4<FMT, FAST>(x1.x, fs, inv);
  bB[1][0] = dec_tc4<FMT, FAST>(y1.x, fs, inv);
  bA[1][1] = dec_tc4<FMT, FAST>(x1.y, fs, inv);
  bB[1][1] = dec_tc4<FMT, FAST>(y1.y, fs, inv);
  bA[1][2] = dec_tc4<FMT, FAST>(x1.z, fs, inv);
  bB[1][2] = dec_tc4<FMT, FAST>(y1.z, fs, inv);
  bA[1][3] = dec_tc4<FMT, FAST>(x1.w, fs, inv);
  bB[1][3] = dec_tc4<FMT, FAST>(y1.w, fs, inv);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 u = dec_lds128(aA + a_half * h);
    const uint4 v = dec_lds128(aB + a_half * h);
    uint4 u8 = make_uint4(0u, 0u, 0u, 0u), v8 = make_uint4(0u, 0u, 0u, 0u);
    if (hi_rows) {
      u8 = dec_lds128(aA + a_hi + a_half * h);
      v8 = dec_lds128(aB + a_hi + a_half * h);
    }
    dec_mma(accA[h][0], u.x, u8.x, u.y, u8.y, bA[h][0], bA[h][1]);
    dec_mma(accA[h][1], u.z, u8.z, u.w, u8.w, bA[h][2], bA[h][3]);
    dec_mma(accB[h][0], v.x, v8.x, v.y, v8.y, bB[h][0], bB[h][1]);
    dec_mma(accB[h][1], v.z, v8.z, v.w, v8.w, bB[h][2], bB[h][3]);
  }
}

// Weights ahead of the activations: when the ring holds the whole K-slice,
// each consumer warp transcodes its stages (i = q mod W) in place, FP8 bytes
// -> int8 bytes at the same shared memory addresses, as they land. This runs
// while the activation rows are still to come (they follow the previous
// kernel), so the ALU-bound transcode overlaps the call's head instead of
// following it. Each lane rewrites exactly the 32 bytes it read, so no other
// thread's data is touched.
template <int FMT, bool FAST>
__device__ __forceinline__ bool dec_pretranscode(uint32_t stages_a, uint64_t* full, int stage_bytes, int nst, int c,
                                                 int q, int lane, uint32_t fs, uint16_t inv) {
  constexpr int W = kDecWpg;
  const int g = lane >> 2, t = lane & 3;
  const int sg = (g >> 1) + 4 * (g & 1);
  const uint32_t wrow = stages_a + (8 * c + sg) * kDecBoxK;
  const int sw0 = (t ^ sg) << 4, sw1 = ((4 + t) ^ sg) << 4;
  bool ok = true;
  int i = q;
  for (; i + W < nst; i += 2 * W) {
    if (ok) ok = dec_wait(&full[i], 0, ERR_WAIT_FULL);
    if (ok) ok = dec_wait(&full[i + W], 0, ERR_WAIT_FULL);
    const uint32_t a = wrow + i * stage_bytes, b = wrow + (i + W) * stage_bytes;
    const uint4 x0 = dec_lds128(a + sw0), x1 = dec_lds128(a + sw1);
    const uint4 y0 = dec_lds128(b + sw0), y1 = dec_lds128(b + sw1);
    uint4 u0, u1, v0, v1;
    u0.x = dec_tc4<FMT, FAST>(x0.x, fs, inv);
    v0.x = dec_tc4<FMT, FAST>(y0.x, fs, inv);
    u0.y = dec_tc4<FMT, FAST>(x0.y, fs, inv);
    v0.y = dec_tc4<FMT, FAST>(y0.y, fs, inv);
    u0.z = dec_tc4<FMT, FAST>(x0.z, fs, inv);
    v0.z = dec_tc4<FMT, FAST>(y0.z, fs, inv);
    u0.w = dec_tc4<FMT, FAST>(x0.w, fs, inv);
    v0.w = dec_tc4<FMT, FAST>(y0.w, fs, inv);
    u1.x = dec_tc4<FMT, FAST>(x1.x, fs, inv);
    v1.x = dec_tc4<FMT, FAST>(y1.x, fs, inv);
    u1.y = dec_tc4<FMT, FAST>(x1.y, fs, inv);
    v1.y = dec_tc4<FMT, FAST>(y1.y, fs, inv);
    u1.z = dec_tc4<FMT, FAST>(x1.z, fs, inv);
    v1.z = dec_tc4<FMT, FAST>(y1.z, fs, inv);
    u1.w = dec_tc4<FMT, FAST>(x1.w, fs, inv);
    v1.w = dec_tc4<FMT, FAST>(y1.w, fs, inv);
    dec_sts128(a + sw0, u0);
    dec_sts128(a + sw1, u1);
    dec_sts128(b + sw0, v0);
    dec_sts128(b + sw1, v1);
  }
  for (; i < nst; i += W) {
    if (ok) ok = dec_wait(&full[i], 0, ERR_WAIT_FULL);
    const uint32_t a = wrow + i * stage_bytes;
    const uint4 x0 = dec_lds128(a + sw0), x1 = dec_lds128(a + sw1);
    uint4 u0, u1;
    u0.x = dec_tc4<FMT, FAST>(x0.x, fs, inv);
    u0.y = dec_tc4<FMT, FAST>(x0.y, fs, inv);
    u0.z = dec_tc4<FMT, FAST>(x0.z, fs, inv);
    u0.w = dec_tc4<FMT, FAST>(x0.w, fs, inv);
    u1.x = dec_tc4<FMT, FAST>(x1.x, fs, inv);
    u1.y = dec_tc4<FMT, FAST>(x1.y, fs, inv);
    u1.z = dec_tc4<FMT, FAST>(x1.z, fs, inv);
    u1.w = dec_tc4<FMT, FAST>(x1.w, fs, inv);
    dec_sts128(a + sw0, u0);
    dec_sts128(a + sw1, u1);
  }
  __syncwarp();  // the warp's later fragment loads see every lane's int8 bytes
  return ok;
}

// Activation layouts: quantised in the kernel (direct = false: row stride
// astride, K contiguous) or copied by TMA as int8 boxes of 16 rows x 64 bytes
// (direct = true: box j = K bytes [64j, 64j + 64) at j * 1024, rows 64 bytes
// apart, so each 8-lane phase of a fragment load covers all 32 banks).
template <int FMT, bool FAST, int W, bool PRE>
__device__ __forceinline__ bool dec_loop(int (&acc)[2][2][4], uint32_t stages_a, uint64_t* full, uint64_t* empty,
                                         uint32_t aq_a, bool direct, int astride, int stage_bytes, int D, int nst,
                                         int c, int q, int lane, bool hi_rows, uint32_t fs, uint16_t inv, int dbg) {
  const int g = lane >> 2, t = lane & 3;
  const int sg = (g >> 1) + 4 * (g & 1);
  const uint32_t wrow = stages_a + (8 * c + sg) * kDecBoxK;
  const int sw0 = (t ^ sg) << 4, sw1 = ((4 + t) ^ sg) << 4;  // 16-byte chunks of halves 0 and 1 (swizzled)
  const int a_half = direct ? kDecRows * kDecQBox : 64;
  const int a_hi = direct ? 8 * kDecQBox : 8 * astride;
  const int a_stage = direct ? 2 * kDecRows * kDecQBox : kDecBoxK;  // bytes per 128-K stage
  uint32_t a_addr = aq_a + (direct ? g * kDecQBox : g * astride) + 16 * t + q * a_stage;
  bool ok = true;
  int s = q;
  uint32_t phase = 0;
  const bool recycle = nst > D;
  int acc2[2][2][4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int j = 0; j < 2; ++j) acc2[h][j][0] = acc2[h][j][1] = acc2[h][j][2] = acc2[h][j][3] = 0;
  auto advance = [&](int& slot, uint32_t& ph) {
    slot += W;
    if (slot >= D) {
      slot -= D;
      ph ^= 1u;
    }
  };
  int i = q;
  // two stages at a time, except when the ring recycles with fewer than 2W
  // slots: the second stage's slot could then still wait for the first's release
  const int pair_end = (recycle && D < 2 * W) ? q : nst;
  for (; i + W < pair_end; i += 2 * W) {
    int s2 = s;
    uint32_t phase2 = phase;
    advance(s2, phase2);
    if (!PRE && ok && !DEC_DBG(1)) ok = dec_wait(&full[s], phase, ERR_WAIT_FULL);
    if (!PRE && ok && !DEC_DBG(1)) ok = dec_wait(&full[s2], phase2, ERR_WAIT_FULL);
    dec_stage2<FMT, FAST, PRE>(acc, acc2, wrow + s * stage_bytes, wrow + s2 * stage_bytes, a_addr, a_addr + W * a_stage,
                          a_half, a_hi, hi_rows, fs, inv, sw0, sw1);
    if (recycle) {  // the producer refills these slots: release them once every lane has read them
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        mbar_arrive(&empty[s2]);
      }
    }
    a_addr += 2 * W * a_stage;
    s = s2;
    phase = phase2;
    advance(s, phase);
  }
  for (; i < nst; i += W) {
    if (!PRE && ok && !DEC_DBG(1)) ok = dec_wait(&full[s], phase, ERR_WAIT_FULL);
    dec_stage<FMT, FAST, PRE>(acc, wrow + s * stage_bytes, a_addr, a_half, a_hi, hi_rows, fs, inv, sw0, sw1, dbg);
    if (recycle) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    a_addr += W * a_stage;
    advance(s, phase);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int x = 0; x < 4; ++x) acc[h][j][x] += acc2[h][j][x];
  return ok;
}

// ---- column-parallel gather fused into the epilogue (world > 1, col-major)
// Every call adds exactly kDecPeerUnits to each peer counter whatever the
// grid (CTA i adds floor((i+1)U/n) - floor(iU/n)), the same per-call total
// and the same signal-pad slots as the split-K kernel's fused gather, so the
// two kernels may alternate between calls.
constexpr unsigned int kDecPeerUnits = 1u << 20;

// This CTA's finished columns [c0, c1) (a contiguous run of the col-major
// slice, already stored locally) into every peer's output, then one
// system-scope release increment per peer.
__device__ __forceinline__ void dec_peer_publish(const GemvParams& p, int c0, int c1) {
  __syncthreads();  // the CTA's local output stores are done
  if (c0 < c1) {
    const size_t b0 = (size_t)c0 * p.M * 2, nb = (size_t)(c1 - c0) * p.M * 2;
    const uint8_t* src = static_cast<const uint8_t*>(p.D) + b0;
    for (int q = 0; q < p.world; ++q) {
      if (q == p.rank) continue;
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.peer_rows[q]) + b0;
      if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | nb) & 15u) == 0) {
        for (size_t i = threadIdx.x; i < (nb >> 4); i += blockDim.x)
          reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
      } else {
        for (size_t i = threadIdx.x; i < (nb >> 1); i += blockDim.x)
          reinterpret_cast<uint16_t*>(dst)[i] = reinterpret_cast<const uint16_t*>(src)[i];
      }
    }
  }
  __syncthreads();  // (orders every thread's peer stores before the release below)
  if ((int)threadIdx.x < p.world && (int)threadIdx.x != p.rank) {
    const unsigned long long U = kDecPeerUnits, n = gridDim.x, i = blockIdx.x;
    const unsigned int share = (unsigned int)(((i + 1) * U) / n - (i * U) / n);
    unsigned int* slot = reinterpret_cast<unsigned int*>(p.peer_sig[threadIdx.x]) + kPeerFusedSlot + p.rank;
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(slot), "r"(share) : "memory");
  }
}

// One CTA, launched as a programmatic dependent of the decode kernel: advance
// this rank's call epoch and wait (bounded) until every peer has published
// this call's rows; finish only after the decode grid, so that whatever
// follows in the stream sees the whole gathered output.
__global__ void __launch_bounds__(32) dec_peer_wait_kernel(const __grid_constant__ GemvParams p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ unsigned int target_s;
  if (threadIdx.x == 0) {
    unsigned int e = p.epoch;
    if (e == 0) {  // counted on the device: advances on every launch, graph replays included
      unsigned int* ctr = reinterpret_cast<unsigned int*>(p.peer_sig[p.rank]) + kPeerFusedEpochSlot;
      e = *ctr + 1;
      *ctr = e;
    }
    target_s = e * kDecPeerUnits;  // modulo 2^32; compared by signed difference
  }
  __syncthreads();
  const unsigned int target = target_s;
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
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <int AT, int FMT>
__global__ void __launch_bounds__(kDecMaxThreads, 1)
    decode_kernel(const __grid_constant__ GemvParams p, const __grid_constant__ CUtensorMap tm_full,
                  const __grid_constant__ CUtensorMap tm_short, const __grid_constant__ CUtensorMap tm_act,
                  const __grid_constant__ DecodeCfg cfg) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
#ifdef FP8IMMA_TRACE
  const long long trace_clk0 = clock64();
  const unsigned long long trace_gt0 = globaltimer_ns();
  long long trace_pt[16] = {0};
#endif
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + cfg.off_bar);
  uint64_t* empty = full + kDecMaxStages;
  uint64_t* recv_bar = empty + kDecMaxStages;
  uint64_t* act_bar = recv_bar + 1;
  float* sc_s = reinterpret_cast<float*>(smem + cfg.off_const);  // [64] column int8 steps (fp32)
  float* cs_s = sc_s + 64;                                       // [64] fp32 column multipliers
  float* rg_s = cs_s + 64;                                       // [16] per-row global scales
  uint16_t* rowinv_s = reinterpret_cast<uint16_t*>(rg_s + 16);   // [16] per-row activation multipliers
  uint8_t* raw = smem + cfg.off_raw;
  int8_t* aq = reinterpret_cast<int8_t*>(smem + cfg.off_aq);
  int32_t* tot = reinterpret_cast<int32_t*>(smem + cfg.off_tot);    // [gmax][wpg][16][8] own sums, parking
  int32_t* recv = reinterpret_cast<int32_t*>(smem + cfg.off_recv);  // [gmax][16][8] the peer's sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nthr = blockDim.x - 32;  // consumer threads
  const int cwarps = nthr >> 5;
  const int S = cfg.S;
  const int rank = S > 1 ? (int)cluster_ctarank() : 0;
  const int pc = blockIdx.x / S;
  const int cg0 = pc * cfg.NG / cfg.P;  // (fits in 32 bits: pc < 148, NG < 2^24)
  const int G = (pc + 1) * cfg.NG / cfg.P - cg0;
  const int n0 = cg0 * 8;
  const int k0 = rank * cfg.kper;
  const int k1 = min(p.K, k0 + cfg.kper);
  const int nst = k1 > k0 ? (k1 - k0 + kDecBoxK - 1) / kDecBoxK : 0;
  constexpr bool kDirect = AT == A_S8;  // int8 rows: TMA straight into the fragment layout
  const int esz = AT == A_S8 ? 1 : 2;
  const int abox_k = kDirect ? kDecQBox : kDecABox / esz;  // activation K elements per box
  const int abox_bytes = kDirect ? kDecQBox : kDecABox;      // bytes per row per box
  const int abox_slot = kDecRows * abox_bytes;                // shared memory per box
  const int nbox = k1 > k0 ? (k1 - k0 + abox_k - 1) / abox_k : 0;
  const int gh = (G + 1) >> 1;  // groups [0, gh) finish on rank 0, [gh, G) on rank 1
  const int own_lo = rank == 0 ? 0 : gh, own_hi = (S == 1 || rank == 1) ? G : gh;

  // The producer thread initialises the barriers and issues the first weight
  // stages (and, without programmatic dependent launch, the activation rows)
  // before the CTA-wide barrier: nothing waits on them before it.
  const CUtensorMap* tm = G == cfg.gmax ? &tm_full : &tm_short;
  const uint32_t wbytes = (uint32_t)G * 8 * kDecBoxK;
  // with the whole K-slice resident every stage is requested at once (the
  // consumers transcode them while the activation rows are still to come)
  const int early = cfg.pre ? nst : min(nst, min(cfg.D, kDecEarlyStages));
  uint8_t* adst = kDirect ? reinterpret_cast<uint8_t*>(aq) : raw;
  const bool producer = warp == cwarps && lane == 0 && G > 0;
  DEC_TRACE(10);
  if (warp == cwarps && G > 0) {  // the producer warp's lanes initialise the barriers in parallel, then
    if (lane < cfg.D) {
      mbar_init(&full[lane], 1);
      mbar_init(&empty[lane], G);
    }
    if (lane == 31) {
      mbar_init(recv_bar, 1);
      mbar_init(act_bar, 1);
    }
    fence_barrier_init();
    if (lane == 0) prefetch_tensormap(tm);
    __syncwarp();
    // the first weight stages, requested by the lanes at once (with
    // programmatic dependent launch they stream while the previous kernel
    // finishes); the activation rows follow (measured faster than the rows
    // first), then the rest of a recycling ring
    for (int i = lane; i < early; i += 32) {  // the ring is empty: no waits
      mbar_arrive_expect_tx(&full[i], wbytes);
      tma_load_2d(stages + i * cfg.stage_bytes, tm, &full[i], k0 + i * kDecBoxK, n0);
    }
  }
  if (producer) {
    prefetch_tensormap(&tm_act);
    if (!p.pdl) {
      mbar_arrive_expect_tx(act_bar, (uint32_t)(nbox * cfg.arows * abox_bytes));
      for (int j = 0; j < nbox; ++j) tma_load_2d(adst + j * abox_slot, &tm_act, act_bar, (k0 + j * abox_k) * esz, 0);
    }
  }
  DEC_TRACE(11);
  __syncthreads();
  if (S > 1) {
    cluster_arrive_relaxed();  // the initialisation fence above publishes the barriers to the peer
    if (threadIdx.x == 0) mbar_arrive_expect_tx(recv_bar, (uint32_t)((own_hi - own_lo) * kDecRows * 8 * 4));
  }
  if (p.pdl) pdl_launch_dependents();  // the next grid may take SMs as this one's CTAs exit
  DEC_TRACE(2);

  const int c = warp / kDecWpg, q = warp - c * kDecWpg;
  int acc[2][2][4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int j = 0; j < 2; ++j) acc[h][j][0] = acc[h][j][1] = acc[h][j][2] = acc[h][j][3] = 0;

  if (warp == cwarps) {
    // ---- TMA producer warp: the activation rows (after the previous kernel
    // when launched as a programmatic dependent), then the remaining weight
    // stages of a recycling ring
    if (G > 0 && p.pdl) {  // the activation boxes, one per lane, after the previous kernel
      pdl_wait();  // activations may come from the previous kernel
      if (lane == 0) mbar_arrive_expect_tx(act_bar, (uint32_t)(nbox * cfg.arows * abox_bytes));
      __syncwarp();
      for (int j = lane; j < nbox; j += 32) tma_load_2d(adst + j * abox_slot, &tm_act, act_bar, (k0 + j * abox_k) * esz, 0);
    }
    if (producer) {
      const int D = cfg.D;
      for (int i = early; i < nst; ++i) {
        const int s = i % D;
        if (i >= D && !mbar_wait(&empty[s], ((i / D) & 1) ^ 1u, ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&full[s], wbytes);
        tma_load_2d(stages + s * cfg.stage_bytes, tm, &full[s], k0 + i * kDecBoxK, n0);
      }
    }
  } else {
    const int g = lane >> 2;
    const int sg = (g >> 1) + 4 * (g & 1);
    const bool active = c < G;
    const int col = n0 + 8 * c + sg;  // the weight column this lane transcodes
    const bool col_ok = active && col < p.N;
    const uint16_t sb = col_ok ? dec_scale_bits(p, col) : (uint16_t)0;
    const int tid = threadIdx.x;
    // the epilogue's column scale tables (weight metadata: read before the
    // dependency wait; stored now so the loads' latency hides behind the
    // weight stream)
    if (tid < 64) {
      float scv = 0.0f, csv = 1.0f;
      if (tid < 8 * G && n0 + tid < p.N) {
        scv = __half2float(__ushort_as_half(dec_scale_bits(p, n0 + tid)));
        if (p.col_scale_f32) csv = p.col_scale_f32[n0 + tid];
      }
      sc_s[tid] = scv;
      cs_s[tid] = csv;
    }
    const uint16_t inv = col_ok ? inv_scale_bits(sb) : (uint16_t)0x3C00u;
    const bool all_fast = named_bar_and(2, nthr, fast_ok<FMT>(inv));  // CTA-uniform transcode choice
    const uint32_t fs = fast_scale<FMT>(inv);
    bool pre_ok = true;
    if (cfg.pre && active) {
      if (all_fast)
        pre_ok = dec_pretranscode<FMT, true>(smem_u32(stages), full, cfg.stage_bytes, nst, c, q, lane, fs, inv);
      else
        pre_ok = dec_pretranscode<FMT, false>(smem_u32(stages), full, cfg.stage_bytes, nst, c, q, lane, fs, inv);
    }
    DEC_TRACE(12);
    // per-row scales may come from the previous kernel; without them the
    // consumers read nothing it writes (the activation rows arrive through the
    // producer, which waited for it, and the outputs are written after they land)
    if (p.pdl && (p.row_g || p.row_inv_h)) pdl_wait();
    if (tid < kDecRows) {
      const bool live = tid < p.M;
      rg_s[tid] = live ? (p.row_g ? p.row_g[tid] : p.global_scale) : 0.0f;
      rowinv_s[tid] = (live && p.row_inv_h) ? p.row_inv_h[tid] : p.a_inv_h;
    }
    if (!kDirect) named_bar_sync(1, nthr);  // rowinv_s
    DEC_TRACE(3);
    if (nbox > 0) dec_wait(act_bar, 0, ERR_WAIT_FULL);
    DEC_TRACE(9);
    if (!kDirect) {
      dec_quant_rows<AT>(raw, aq, cfg.astride, nbox, cfg.arows, rowinv_s, tid, nthr);
      named_bar_sync(1, nthr);  // publishes the int8 rows
    }
    DEC_TRACE(4);
    if (active && pre_ok) {
      const uint32_t st_a = smem_u32(stages), aq_a = smem_u32(aq);
      const bool hi_rows = p.M > 8;  // rows 8..15 of the m16 block hold data
#ifdef FP8IMMA_TRACE
      const int dbg = p.dbg;
#else
      const int dbg = 0;
#endif
      if (cfg.pre)
        dec_loop<FMT, true, kDecWpg, true>(acc, st_a, full, empty, aq_a, kDirect, cfg.astride, cfg.stage_bytes, cfg.D,
                                           nst, c, q, lane, hi_rows, fs, inv, dbg);
      else if (all_fast)
        dec_loop<FMT, true, kDecWpg, false>(acc, st_a, full, empty, aq_a, kDirect, cfg.astride, cfg.stage_bytes, cfg.D,
                                            nst, c, q, lane, hi_rows, fs, inv, dbg);
      else
        dec_loop<FMT, false, kDecWpg, false>(acc, st_a, full, empty, aq_a, kDirect, cfg.astride, cfg.stage_bytes,
                                             cfg.D, nst, c, q, lane, hi_rows, fs, inv, dbg);
    }
    DEC_TRACE(5);
  }

  // ---- reduction: the four accumulator sets, the two warps of a group,
  // then (S = 2) the two CTAs
  int a0 = (acc[0][0][0] + acc[0][1][0]) + (acc[1][0][0] + acc[1][1][0]);
  int a1 = (acc[0][0][1] + acc[0][1][1]) + (acc[1][0][1] + acc[1][1][1]);
  int a2 = (acc[0][0][2] + acc[0][1][2]) + (acc[1][0][2] + acc[1][1][2]);
  int a3 = (acc[0][0][3] + acc[0][1][3]) + (acc[1][0][3] + acc[1][1][3]);
  const int g = lane >> 2, t = lane & 3;
  __syncthreads();
  DEC_TRACE(6);
  const bool frag = warp < cwarps && c < G;
  // slot (c, 0) of tot receives group c's sums; the group's other warps park
  // their fragments in slots (c, q) first
  int32_t* fbase = tot + ((c * kDecWpg * kDecRows + g) * 8 + 2 * t);
  int32_t* park = fbase + q * kDecRows * 8;
  if (frag && q > 0) {
    *reinterpret_cast<int2*>(park) = make_int2(a0, a1);
    *reinterpret_cast<int2*>(park + 64) = make_int2(a2, a3);
  }
  __syncthreads();
  if (frag && q == 0) {
#pragma unroll
    for (int w = 1; w < kDecWpg; ++w) {
      const int32_t* pk = fbase + w * kDecRows * 8;
      const int2 u = *reinterpret_cast<const int2*>(pk);
      const int2 v = *reinterpret_cast<const int2*>(pk + 64);
      a0 += u.x;
      a1 += u.y;
      a2 += v.x;
      a3 += v.y;
    }
  }
  if (S > 1) cluster_wait_acquire();  // the peer's barrier is initialised
  if (frag && q == 0) {
    if (c >= own_lo && c < own_hi) {
      *reinterpret_cast<int2*>(fbase) = make_int2(a0, a1);
      *reinterpret_cast<int2*>(fbase + 64) = make_int2(a2, a3);
    } else {
      const uint32_t peer = (uint32_t)(rank ^ 1);
      const uint32_t rbar = map_to_rank(recv_bar, peer);
      const int32_t* rb = recv + ((c * kDecRows + g) * 8 + 2 * t);
      st_async_v2(map_to_rank(rb, peer), a0, a1, rbar);
      st_async_v2(map_to_rank(rb + 64, peer), a2, a3, rbar);
    }
  }
  __syncthreads();
  if (S > 1) dec_wait(recv_bar, 0, ERR_WAIT_PEER);
  DEC_TRACE(7);

  // ---- epilogue of the owned groups
  const int ncols = (own_hi - own_lo) * 8;
  const int nel = ncols * p.M;
  // e / d by multiply-high: exact for e < 2^28 and d <= 64
  const int dv = p.out_row_major ? ncols : p.M;
  const unsigned int magic = dv > 0 ? 0xFFFFFFFFu / (unsigned int)dv + 1u : 0u;
  for (int e = threadIdx.x; e < nel; e += blockDim.x) {
    const int qt = dv == 1 ? e : (int)__umulhi((unsigned int)e, magic);
    const int rm = e - qt * dv;
    const int lc = p.out_row_major ? rm : qt;
    const int m = p.out_row_major ? qt : rm;
    const int cc = own_lo + (lc >> 3), j = lc & 7;
    const int f = j < 4 ? 2 * j : 2 * (j - 4) + 1;  // MMA output column holding weight column j
    const int n = n0 + 8 * cc + j;
    if (n >= p.N) continue;
    int32_t sum = tot[(cc * kDecWpg * kDecRows + m) * 8 + f];
    if (S > 1) sum += recv[(cc * kDecRows + m) * 8 + f];
    dec_store(p, n, m, sum, sc_s[8 * cc + j], cs_s[8 * cc + j], rg_s[m]);
  }
  if (p.world > 1) dec_peer_publish(p, n0 + own_lo * 8, min(p.N, n0 + own_hi * 8));
  DEC_TRACE(8);
#ifdef FP8IMMA_TRACE
  if (p.trace && threadIdx.x == 0) {
    unsigned int sm_;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm_));
    p.trace[(size_t)blockIdx.x * 64 + 0] = trace_gt0;
    p.trace[(size_t)blockIdx.x * 64 + 1] = sm_;
#pragma unroll
    for (int i = 2; i < 16; ++i) p.trace[(size_t)blockIdx.x * 64 + i] = trace_pt[i];
  }
#endif
}

// Activation pre-pass: the rows quantised once, for every CTA of the decode
// grid to copy (without it each CTA pair quantises all of A for its K half).
// Launched as a programmatic dependent when PDL is on: its CTAs start next to
// the previous kernel's and wait for it (griddepcontrol.wait) before reading
// A or writing the rows that the previous call's kernel may still be reading.
template <int AT>
__global__ void __launch_bounds__(256) dec_quant_kernel(const void* __restrict__ A, int M, int K, uint16_t a_inv_h,
                                                        const uint16_t* __restrict__ row_inv_h,
                                                        int8_t* __restrict__ Aq) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int items = K >> 3;  // 8 values per item
  const size_t total = (size_t)M * items;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / items);
    uint4 v = reinterpret_cast<const uint4*>(A)[i];
    const uint16_t ainv = row_inv_h ? row_inv_h[m] : a_inv_h;
    const uint32_t ainv2 = (uint32_t)ainv | ((uint32_t)ainv << 16);
    if (AT == A_BF16) {
      v.x = bf16x2_to_f16x2(v.x);
      v.y = bf16x2_to_f16x2(v.y);
      v.z = bf16x2_to_f16x2(v.z);
      v.w = bf16x2_to_f16x2(v.w);
    }
    reinterpret_cast<uint2*>(Aq)[i] = make_uint2(quant4_f16(v.x, v.y, ainv2), quant4_f16(v.z, v.w, ainv2));
  }
}

// Per-row variant of the pre-pass: one CTA per row computes the row's absolute
// maximum (fp16 values; bf16 rounded to fp16 first), its multiplier
// fp16(127 / amax) and output scale 1 / (127 / amax) exactly as the row-scale
// kernel does (amax 0 or not finite: both 0), and quantises the row with it.
template <int AT>
__global__ void __launch_bounds__(256) dec_rowquant_kernel(const void* __restrict__ A, int K,
                                                           int8_t* __restrict__ Aq, uint16_t* __restrict__ a_inv_h,
                                                           float* __restrict__ g) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float red[8];
  __shared__ uint32_t inv_s;
  const int m = blockIdx.x;
  const uint4* row = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(A) + (size_t)m * K);
  uint2* out = reinterpret_cast<uint2*>(Aq + (size_t)m * K);
  const int items = K >> 3;
  float amax = 0.0f;
  auto absmax8 = [&](const uint4& v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t h2 = AT == A_BF16 ? bf16x2_to_f16x2(w[j]) : w[j];
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  };
  // the first kKeep vectors of each thread stay in registers for the
  // quantisation (one read of the row for K <= 8192), the rest is read again
  constexpr int kKeep = 4;
  uint4 keep[kKeep];
#pragma unroll
  for (int j = 0; j < kKeep; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < items) {
      keep[j] = row[i];
      absmax8(keep[j]);
    }
  }
  for (int i = threadIdx.x + kKeep * blockDim.x; i < items; i += blockDim.x) absmax8(row[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) a = fmaxf(a, red[w]);
    float inv = 0.0f, gg = 0.0f;
    if (a > 0.0f && a <= 3.402823466e38f) {
      inv = __fdiv_rn(127.0f, a);
      gg = __fdiv_rn(1.0f, inv);
    }
    const uint16_t ih = __half_as_ushort(__float2half_rn(inv));
    a_inv_h[m] = ih;
    g[m] = gg;
    inv_s = (uint32_t)ih | ((uint32_t)ih << 16);
  }
  __syncthreads();
  const uint32_t ainv2 = inv_s;
  auto quant8 = [&](uint4 v, int i) {
    if (AT == A_BF16) {
      v.x = bf16x2_to_f16x2(v.x);
      v.y = bf16x2_to_f16x2(v.y);
      v.z = bf16x2_to_f16x2(v.z);
      v.w = bf16x2_to_f16x2(v.w);
    }
    out[i] = make_uint2(quant4_f16(v.x, v.y, ainv2), quant4_f16(v.z, v.w, ainv2));
  };
#pragma unroll
  for (int j = 0; j < kKeep; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < items) quant8(keep[j], i);
  }
  for (int i = threadIdx.x + kKeep * blockDim.x; i < items; i += blockDim.x) quant8(row[i], i);  // L1 / L2 resident
}

std::atomic<int> g_decode_mode{1};
constexpr int kDecPrepassM = 1;  // rows from which the pre-pass beats per-CTA quantisation

template <int AT, int FMT>
cudaError_t dec_launch(const GemvParams& p, const CUtensorMap& tf, const CUtensorMap& ts, const CUtensorMap& ta,
                       const DecodeCfg& cfg, size_t smem, cudaStream_t stream) {
  auto kern = decode_kernel<AT, FMT>;
  cudaError_t e = ensure_smem_attr((const void*)kern, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(cfg.P * cfg.S, 1, 1);
  lc.blockDim = dim3(cfg.gmax * kDecWpg * 32 + 32, 1, 1);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cfg.S;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = cfg.S > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&lc, kern, p, tf, ts, ta, cfg);
}

}  // namespace

// Shape plan: S (1 or a CTA pair), groups per cluster, stage ring, shared
// memory layout. Returns false when the shape does not fit one wave of at most
// 8 groups per CTA with the CTA's whole activation slice in shared memory.
static bool decode_plan(int M, int N, int K, int a_bytes, int sms, DecodeCfg* out, size_t* smem_out) {
  if (M < 1 || M > kDecRows || N < 1 || K < 1) return false;
  const int NG = (N + 7) / 8;
  long long best = -1;
  DecodeCfg cfg = {};
  for (int S = 1; S <= 2; ++S) {
    int P = sms / S;
    if (P > NG) P = NG;
    if (P < 1) continue;
    const int gmax = (NG + P - 1) / P;
    if (gmax > kDecMaxG) continue;
    const int kper = ((K + S - 1) / S + kDecBoxK - 1) / kDecBoxK * kDecBoxK;
    if (S > 1 && kper >= K) continue;  // nothing for the second CTA
    const long long work = (long long)gmax * 8 * kper;
    if (best < 0 || work < best) {
      best = work;
      cfg.S = S;
      cfg.P = P;
      cfg.NG = NG;
      cfg.gmax = gmax;
      cfg.kper = kper;
    }
  }
  if (best < 0) return false;
  const int nst = cfg.kper / kDecBoxK;
  cfg.stage_bytes = cfg.gmax * 8 * kDecBoxK;
  cfg.arows = M < kDecRows ? M : kDecRows;
  cfg.astride = cfg.kper + 64;
  // int8 rows (a_bytes == 1) go straight into the fragment layout; 16-bit
  // rows are staged raw and quantised into a row-strided int8 copy
  const bool direct = a_bytes == 1;
  const size_t raw = direct ? 0 : (size_t)((cfg.kper + 63) / 64) * kDecRows * kDecABox;
  const size_t fixed = (2 * kDecMaxStages + 2) * 8 + (64 + 64 + 16) * 4 + 16 * 2 + 64;
  const size_t aqb = direct ? (size_t)((cfg.kper + kDecQBox - 1) / kDecQBox) * kDecRows * kDecQBox
                            : (size_t)kDecRows * cfg.astride;
  const size_t red = (size_t)(kDecWpg + 1) * cfg.gmax * kDecRows * 8 * 4;
  const size_t budget = 227 * 1024 - 1024;  // alignment slack
  if (fixed + raw + aqb + red + (size_t)4 * cfg.stage_bytes > budget) return false;
  int D = nst < kDecMaxStages ? nst : kDecMaxStages;
  while (D > 4 && fixed + raw + aqb + red + (size_t)D * cfg.stage_bytes > budget) --D;
  D -= D % kDecWpg;  // a multiple of the warps per group: warp q keeps ring slots s = q (mod kDecWpg)
  if (D < kDecWpg) D = kDecWpg;
  cfg.D = D;
  cfg.pre = nst <= D && g_decode_mode.load() != 2;
  size_t off = (size_t)D * cfg.stage_bytes;
  cfg.off_raw = (int)off;  // 1024-aligned (stages are multiples of 1 KB)
  off += raw;
  cfg.off_aq = (int)off;
  off += aqb;
  off = (off + 15) & ~size_t(15);
  cfg.off_tot = (int)off;
  off += (size_t)cfg.gmax * kDecWpg * kDecRows * 8 * 4;
  cfg.off_recv = (int)off;
  off += (size_t)cfg.gmax * kDecRows * 8 * 4;
  cfg.off_bar = (int)off;
  off += (2 * kDecMaxStages + 2) * 8;
  cfg.off_const = (int)off;
  off += (64 + 64 + 16) * 4 + 16 * 2;
  *out = cfg;
  *smem_out = off + 1024;
  return true;
}

bool decode_host_direct_ok(const GemvParams& p, int a_type, int fmt, cudaStream_t stream) {
  if (a_type == A_S8 || p.M < kDecPrepassM || p.no_alloc || p.world > 1 || !decode_applicable(p, a_type, fmt))
    return false;
  DecodeCfg cfg;
  size_t smem;
  return decode_plan(p.M, p.N, p.K, 1, num_sms_current(), &cfg, &smem) &&
         stream_scratch_ready(stream, (size_t)p.M * p.K, 1);
}

bool decode_applicable(const GemvParams& p, int a_type, int fmt) {
  if (g_decode_mode.load() == 0) return false;
  if (fmt != 0 && fmt != 1) return false;  // int8-exact formats (E4M3 table, E5M2)
  // several ranks: the fused gather needs the col-major layout
  if (p.world > 1 && (p.out_row_major || p.world > 8)) return false;
  DecodeCfg cfg;
  size_t smem;
  // rows quantised by the pre-pass arrive as int8 (half the shared memory)
  const bool prepass = a_type != A_S8 && p.M >= kDecPrepassM && !p.no_alloc;
  return decode_plan(p.M, p.N, p.K, (a_type == A_S8 || prepass) ? 1 : 2, num_sms_current(), &cfg, &smem);
}

cudaError_t launch_decode(const GemvParams& p_in, int a_type, int fmt, cudaStream_t stream) {
  GemvParams p = p_in;
  if (p.a_host && (a_type == A_S8 || p.M < kDecPrepassM || p.no_alloc)) return cudaErrorNotSupported;
  if (a_type != A_S8 && p.M >= kDecPrepassM && !p.no_alloc) {
    void* aq = stream_scratch(stream, (size_t)p.M * p.K, 1);
    if (!aq && p.a_host) return cudaErrorNotSupported;  // (the pre-pass is what reads the host rows)
    const void* a_src = p.a_host ? p.a_host : p.A;
    if (aq) {
      const size_t total = (size_t)p.M * (p.K >> 3);
      cudaLaunchConfig_t lc = {};
      lc.gridDim = dim3((unsigned)((total + 255) / 256), 1, 1);
      lc.blockDim = dim3(256, 1, 1);
      lc.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
      lc.attrs = attr;
      lc.numAttrs = 1;
      cudaError_t e = a_type == A_BF16
                          ? cudaLaunchKernelEx(&lc, dec_quant_kernel<A_BF16>, a_src, p.M, p.K, p.a_inv_h, p.row_inv_h,
                                               static_cast<int8_t*>(aq))
                          : cudaLaunchKernelEx(&lc, dec_quant_kernel<A_F16>, a_src, p.M, p.K, p.a_inv_h, p.row_inv_h,
                                               static_cast<int8_t*>(aq));
      if (e != cudaSuccess) return e;
      p.A = aq;
      p.row_inv_h = nullptr;
      p.pdl = 1;  // weights stream while the pre-pass runs; the rows are read after it
      a_type = A_S8;
    }
  }
  DecodeCfg cfg;
  size_t smem = 0;
  const int esz = a_type == A_S8 ? 1 : 2;
  // (only when the pre-pass could not get its scratch and 16-bit rows do not fit)
  if (!decode_plan(p.M, p.N, p.K, esz, num_sms_current(), &cfg, &smem)) return cudaErrorNotSupported;
  CUtensorMap tf, ts, ta;
  cudaError_t e = make_tmap_2d_u8(&tf, p.B, (uint64_t)p.K, (uint64_t)p.N, (uint64_t)p.K, kDecBoxK,
                                  (uint32_t)cfg.gmax * 8, /*swizzle128=*/true);
  if (e != cudaSuccess) return e;
  if (cfg.gmax > 1) {
    e = make_tmap_2d_u8(&ts, p.B, (uint64_t)p.K, (uint64_t)p.N, (uint64_t)p.K, kDecBoxK, (uint32_t)(cfg.gmax - 1) * 8,
                        true);
    if (e != cudaSuccess) return e;
  } else {
    ts = tf;
  }
  // activation rows as bytes: [M][K * esz], boxes of arows x 128 bytes
  // (16-bit rows) or arows x 64 bytes (int8 rows, the fragment layout)
  e = make_tmap_2d_u8(&ta, p.A, (uint64_t)p.K * esz, (uint64_t)p.M, (uint64_t)p.K * esz,
                      esz == 1 ? kDecQBox : kDecABox, (uint32_t)cfg.arows, false);
  if (e != cudaSuccess) return e;
  switch (a_type * 8 + fmt) {
    case A_F16 * 8 + 0: e = dec_launch<A_F16, FMT_E4M3_REF>(p, tf, ts, ta, cfg, smem, stream); break;
    case A_F16 * 8 + 1: e = dec_launch<A_F16, FMT_E5M2>(p, tf, ts, ta, cfg, smem, stream); break;
    case A_BF16 * 8 + 0: e = dec_launch<A_BF16, FMT_E4M3_REF>(p, tf, ts, ta, cfg, smem, stream); break;
    case A_BF16 * 8 + 1: e = dec_launch<A_BF16, FMT_E5M2>(p, tf, ts, ta, cfg, smem, stream); break;
    case A_S8 * 8 + 0: e = dec_launch<A_S8, FMT_E4M3_REF>(p, tf, ts, ta, cfg, smem, stream); break;
    case A_S8 * 8 + 1: e = dec_launch<A_S8, FMT_E5M2>(p, tf, ts, ta, cfg, smem, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess || p.world <= 1) return e;
  // gathered output: wait for the peers' rows (a programmatic dependent, so
  // it is resident while the decode kernel still runs)
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(1, 1, 1);
  lc.blockDim = dim3(32, 1, 1);
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, dec_peer_wait_kernel, p);
}

cudaError_t launch_decode_rowquant(const GemvParams& p_in, int a_type, int fmt, cudaStream_t stream) {
  if (a_type != A_F16 && a_type != A_BF16) return cudaErrorNotSupported;
  GemvParams p = p_in;
  p.row_quant = 0;
  DecodeCfg cfg;
  size_t smem;
  if (p.no_alloc || !decode_plan(p.M, p.N, p.K, 1, num_sms_current(), &cfg, &smem)) return cudaErrorNotSupported;
  const size_t rows_bytes = ((size_t)p.M * p.K + 255) & ~size_t(255);
  uint8_t* sc = static_cast<uint8_t*>(stream_scratch(stream, rows_bytes + (size_t)p.M * 8 + 256, 1));
  if (!sc) return cudaErrorNotSupported;
  int8_t* aq = reinterpret_cast<int8_t*>(sc);
  float* g = reinterpret_cast<float*>(sc + rows_bytes);
  uint16_t* inv = reinterpret_cast<uint16_t*>(g + p.M);
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)p.M, 1, 1);
  lc.blockDim = dim3(256, 1, 1);
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  lc.attrs = attr;
  lc.numAttrs = 1;
  cudaError_t e = a_type == A_BF16 ? cudaLaunchKernelEx(&lc, dec_rowquant_kernel<A_BF16>, p.A, p.K, aq, inv, g)
                                   : cudaLaunchKernelEx(&lc, dec_rowquant_kernel<A_F16>, p.A, p.K, aq, inv, g);
  if (e != cudaSuccess) return e;
  p.A = aq;
  p.row_inv_h = nullptr;
  p.row_g = g;
  p.pdl = 1;  // weights stream while the pre-pass runs; rows and row scales are read after it
  return launch_decode(p, A_S8, fmt, stream);
}

void decode_set_mode(int mode) { g_decode_mode.store(mode); }
unsigned int decode_device_error(bool clear) { return tu_device_error(clear); }
cudaError_t decode_set_wait_limit(unsigned long long ns) { return tu_set_wait_limit(ns); }

}  // namespace fp8imma_b200
