// Split-K "skinny" GEMM for small M (decode shapes), reference-exact int8 path.
//
// Work split (B200): a CTA owns 128 weight columns and one K-slice; the
// K-slices of one column tile form a thread-block cluster and reduce their
// int32 partials through distributed shared memory, so no global scratch is
// needed. Each warp owns 16 weight columns and streams them with 128-bit
// non-allocating loads (16 contiguous K bytes per lane), transcodes the FP8
// bytes to int8 in registers (fp8imma_device.cuh) and feeds them straight into
// mma.sync m16n8k32 s8 as the A operand, with the quantised activations (from
// shared memory) as the B operand. Within a 64-byte K block the physical MMA
// k index is a permutation of the logical k; the same permutation is applied
// to both operands, and int32 sums do not depend on order, so the result is
// exact.
//
// Reference counterpart: imma_gemm_fp8_actquant_cpasync_int8_colscale_fp16_
// colmajor_kernel_v4 (src/fp8imma/impl/v4_kernels.inl:1-287), v3
// (impl/v3_kernels.inl) and v2 (impl/v2_kernels.inl), which tile 64x64 and
// waste 63/64 of their MMA rows at M=1.
#include "fp8imma_kernels.h"
#include "fp8imma_device.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;
using namespace fp8imma_dev;

namespace fp8imma_b200 {

namespace {

constexpr int kThreads = 256;
constexpr int kTileN = 128;
constexpr int kUnroll = 4;  // 64-byte K blocks per register batch

__device__ __forceinline__ void mma_s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float load_col_scale(const GemvParams& p, int n) {
  uint16_t bits;
  if (p.scale_tex) bits = tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n);
  else bits = p.scale_u16[n];
  return __half2float(__ushort_as_half(bits));
}

__device__ __forceinline__ uint16_t load_col_scale_bits(const GemvParams& p, int n) {
  if (p.scale_tex) return tex1Dfetch<unsigned short>((cudaTextureObject_t)p.scale_tex, n);
  return p.scale_u16[n];
}

// Quantise A[m0 : m0+MR, k0 : k0+len] into aq (row stride `stride`), zero-
// filling rows >= M and k >= kvalid.
template <int AT, int MR>
__device__ __forceinline__ void quant_chunk(const GemvParams& p, int8_t* aq, int stride, int m0,
                                            int k0, int len, int kvalid) {
  const int items_per_row = len >> 3;  // 8 elements per item
  const int total = MR * items_per_row;
  for (int it = threadIdx.x; it < total; it += kThreads) {
    int r = it / items_per_row;
    int c = (it - r * items_per_row) << 3;
    int m = m0 + r, k = k0 + c;
    uint2 out = make_uint2(0u, 0u);
    if (m < p.M && k < kvalid) {
      if (AT == A_S8) {
        out = *reinterpret_cast<const uint2*>(static_cast<const int8_t*>(p.A) + (size_t)m * p.K + k);
      } else {
        uint4 v = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.A) + (size_t)m * p.K + k);
        uint16_t ainv = p.row_inv_h ? p.row_inv_h[m] : p.a_inv_h;
        uint32_t ainv2 = (uint32_t)ainv | ((uint32_t)ainv << 16);
        if (AT == A_BF16) {
          v.x = bf16x2_to_f16x2(v.x);
          v.y = bf16x2_to_f16x2(v.y);
          v.z = bf16x2_to_f16x2(v.z);
          v.w = bf16x2_to_f16x2(v.w);
        }
        out.x = quant4_f16(v.x, v.y, ainv2);
        out.y = quant4_f16(v.z, v.w, ainv2);
      }
    }
    *reinterpret_cast<uint2*>(aq + r * stride + c) = out;
  }
}

template <int AT, int MB, int FMT>
__global__ void __launch_bounds__(kThreads, 2) gemv_s8_splitk_kernel(const __grid_constant__ GemvParams p) {
  constexpr int MR = MB * 8;
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int tile_n0 = blockIdx.x * kTileN;
  const int m0 = blockIdx.z * MR;
  const int kbeg = blockIdx.y * p.k_per_cta;
  const int kend = min(p.K, kbeg + p.k_per_cta);
  const int astride = p.kc + 64;  // +64 B: conflict-free 16-byte fragment loads
  int8_t* aq = reinterpret_cast<int8_t*>(smem);
  int32_t* part = reinterpret_cast<int32_t*>(smem);  // reused after the main loop

  // ---- per-column constants (two columns per lane: rows g and g+8 of the MMA)
  const int col0 = tile_n0 + warp * 16 + g, col1 = col0 + 8;
  const bool ok0 = col0 < p.N, ok1 = col1 < p.N;
  uint16_t inv0 = ok0 ? inv_scale_bits(load_col_scale_bits(p, col0)) : (uint16_t)0x3C00u;
  uint16_t inv1 = ok1 ? inv_scale_bits(load_col_scale_bits(p, col1)) : (uint16_t)0x3C00u;
  const bool fast0 = fast_ok<FMT>(inv0), fast1 = fast_ok<FMT>(inv1);
  const uint32_t fs0 = fast_scale<FMT>(inv0), fs1 = fast_scale<FMT>(inv1);
  const uint8_t* b0 = p.B + (size_t)(ok0 ? col0 : 0) * p.K + 16 * t;
  const uint8_t* b1 = p.B + (size_t)(ok1 ? col1 : 0) * p.K + 16 * t;

  int acc[MB][4];
#pragma unroll
  for (int i = 0; i < MB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0;

  const int niter = kend > kbeg ? (kend - kbeg + 63) >> 6 : 0;
  uint4 cur0[kUnroll], cur1[kUnroll];

  auto load_batch = [&](uint4 (&d0)[kUnroll], uint4 (&d1)[kUnroll], int it0) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int k = kbeg + ((it0 + u) << 6) + 16 * t;
      bool kv = (it0 + u) < niter && k < kend;
      d0[u] = (kv && ok0) ? ldg_stream_v4(b0 + (k - 16 * t)) : make_uint4(0u, 0u, 0u, 0u);
      d1[u] = (kv && ok1) ? ldg_stream_v4(b1 + (k - 16 * t)) : make_uint4(0u, 0u, 0u, 0u);
    }
  };

  load_batch(cur0, cur1, 0);
  for (int it0 = 0; it0 < niter; it0 += kUnroll) {
    const int koff = (it0 << 6) % p.kc;  // offset inside the current A chunk
    if (koff == 0) {
      __syncthreads();
      int k0 = kbeg + (it0 << 6);
      int len = min(p.kc, kend - k0);
      len = (len + 63) & ~63;
      quant_chunk<AT, MR>(p, aq, astride, m0, k0, len, kend);
      __syncthreads();
    }
    uint4 nxt0[kUnroll], nxt1[kUnroll];
    load_batch(nxt0, nxt1, it0 + kUnroll);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (it0 + u < niter) {
        uint32_t wa[4], wb[4];
        wa[0] = transcode4<FMT>(cur0[u].x, fast0, fs0, inv0);
        wa[1] = transcode4<FMT>(cur0[u].y, fast0, fs0, inv0);
        wa[2] = transcode4<FMT>(cur0[u].z, fast0, fs0, inv0);
        wa[3] = transcode4<FMT>(cur0[u].w, fast0, fs0, inv0);
        wb[0] = transcode4<FMT>(cur1[u].x, fast1, fs1, inv1);
        wb[1] = transcode4<FMT>(cur1[u].y, fast1, fs1, inv1);
        wb[2] = transcode4<FMT>(cur1[u].z, fast1, fs1, inv1);
        wb[3] = transcode4<FMT>(cur1[u].w, fast1, fs1, inv1);
        const int8_t* arow = aq + koff + (u << 6) + 16 * t;
#pragma unroll
        for (int nb = 0; nb < MB; ++nb) {
          uint4 q = *reinterpret_cast<const uint4*>(arow + (nb * 8 + g) * astride);
          mma_s8_16832(acc[nb], wa[0], wb[0], wa[1], wb[1], q.x, q.y);
          mma_s8_16832(acc[nb], wa[2], wb[2], wa[3], wb[3], q.z, q.w);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      cur0[u] = nxt0[u];
      cur1[u] = nxt1[u];
    }
  }

  // ---- partials -> shared memory, [128 cols][MR] int32
  __syncthreads();
  {
    const int r0 = warp * 16 + g;
#pragma unroll
    for (int nb = 0; nb < MB; ++nb) {
      *reinterpret_cast<int2*>(part + r0 * MR + nb * 8 + 2 * t) = make_int2(acc[nb][0], acc[nb][1]);
      *reinterpret_cast<int2*>(part + (r0 + 8) * MR + nb * 8 + 2 * t) = make_int2(acc[nb][2], acc[nb][3]);
    }
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();

  // ---- cluster reduction + epilogue: CTA rank r finishes 128/S columns
  const int S = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int cols_per = kTileN / S;
  const int nelem = cols_per * MR;
  for (int e = threadIdx.x; e < nelem; e += kThreads) {
    int lc, mr;
    if (p.out_row_major) { mr = e / cols_per; lc = rank * cols_per + (e - mr * cols_per); }
    else { lc = rank * cols_per + e / MR; mr = e % MR; }
    int n = tile_n0 + lc, m = m0 + mr;
    int32_t s = 0;
    for (int q = 0; q < S; ++q) {
      const int32_t* rp = cluster.map_shared_rank(part, q);
      s += rp[lc * MR + mr];
    }
    if (n < p.N && m < p.M) {
      float se = load_col_scale(p, n) * (p.row_g ? p.row_g[m] : p.global_scale);
      if (p.col_scale_f32) se = se * p.col_scale_f32[n];
      float v = (float)s * se;
      uint16_t o = store_val(v, p.out_bf16);
      uint16_t* D = static_cast<uint16_t*>(p.D);
      if (p.out_row_major) D[(size_t)m * p.N + n] = o;
      else D[(size_t)n * p.M + m] = o;
      if (p.acc_out) p.acc_out[(size_t)n * p.M + m] = s;
    }
  }
  cluster.sync();  // keep shared memory alive until every peer has read it
}

template <int AT, int MB, int FMT>
cudaError_t launch_t(const GemvParams& p, int S, int mchunks, size_t smem, cudaStream_t stream) {
  auto kern = gemv_s8_splitk_kernel<AT, MB, FMT>;
  cudaError_t e = ensure_smem_attr((const void*)kern, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + kTileN - 1) / kTileN, S, mchunks);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = S;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int AT, int FMT>
cudaError_t launch_mb(const GemvParams& p, int MB, int S, int mchunks, size_t smem, cudaStream_t st) {
  switch (MB) {
    case 1: return launch_t<AT, 1, FMT>(p, S, mchunks, smem, st);
    case 2: return launch_t<AT, 2, FMT>(p, S, mchunks, smem, st);
    case 3: return launch_t<AT, 3, FMT>(p, S, mchunks, smem, st);
    default: return launch_t<AT, 4, FMT>(p, S, mchunks, smem, st);
  }
}

}  // namespace

int gemv_pick_splits(int N, int K, int mchunks, int num_sms) {
  int tiles = (N + kTileN - 1) / kTileN;
  int S = 1;
  while (S < 8 && tiles * mchunks * S < 2 * num_sms && K / (S * 2) >= 256) S *= 2;
  return S;
}

cudaError_t launch_gemv_s8(GemvParams p, int a_type, int fmt, int splits, cudaStream_t stream) {
  const int MB = p.M >= 32 ? 4 : (p.M + 7) / 8;
  const int MR = MB * 8;
  const int mchunks = (p.M + MR - 1) / MR;
  int S = splits > 0 ? splits : gemv_pick_splits(p.N, p.K, mchunks, num_sms_current());
  if (S != 1 && S != 2 && S != 4 && S != 8) return cudaErrorInvalidValue;
  int kper = (p.K + S - 1) / S;
  kper = (kper + 255) & ~255;
  p.k_per_cta = kper;
  const int kc_max = MR > 16 ? 1024 : 2048;
  p.kc = kper < kc_max ? kper : kc_max;
  size_t smem_a = (size_t)MR * (p.kc + 64);
  size_t smem_p = (size_t)kTileN * MR * 4;
  size_t smem = smem_a > smem_p ? smem_a : smem_p;
  switch (a_type * 3 + fmt) {
    case A_F16 * 3 + FMT_E4M3_REF: return launch_mb<A_F16, FMT_E4M3_REF>(p, MB, S, mchunks, smem, stream);
    case A_F16 * 3 + FMT_E5M2: return launch_mb<A_F16, FMT_E5M2>(p, MB, S, mchunks, smem, stream);
    case A_BF16 * 3 + FMT_E4M3_REF: return launch_mb<A_BF16, FMT_E4M3_REF>(p, MB, S, mchunks, smem, stream);
    case A_BF16 * 3 + FMT_E5M2: return launch_mb<A_BF16, FMT_E5M2>(p, MB, S, mchunks, smem, stream);
    case A_S8 * 3 + FMT_E4M3_REF: return launch_mb<A_S8, FMT_E4M3_REF>(p, MB, S, mchunks, smem, stream);
    case A_S8 * 3 + FMT_E5M2: return launch_mb<A_S8, FMT_E5M2>(p, MB, S, mchunks, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fp8imma_b200
