// Internal launch interface between the C ABI (api.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace fp8imma_b200 {

enum { A_F16 = 0, A_BF16 = 1, A_S8 = 2 };

// Arguments of one reference-exact int8 GEMM launch (small-M split-K path,
// generic path). Layouts as in the reference API: A [M,K] row-major,
// B [N,K] row-major ("col-major KxN"), D col-major [N,M] unless out_row_major.
struct GemvParams {
  const void* A;
  const uint8_t* B;
  const uint16_t* scale_u16;        // [N] fp16 bits (ignored when use_tex)
  unsigned long long scale_tex;     // cudaTextureObject_t over u16 scale bits (0: none)
  void* D;
  int32_t* acc_out;                 // optional [N,M] int32 accumulators
  const uint16_t* row_inv_h;        // optional per-row fp16 a_inv (row quant)
  const float* row_g;               // optional per-row global scale (row quant)
  const float* col_scale_f32;       // optional [N] fp32 extra column scale
  int M, N, K;
  int k_per_cta;                    // filled by the launcher
  int kc;                           // activation chunk staged in shared memory
  int keff_a;                       // generic path: A elements with k >= keff_a read 0
  float global_scale;
  uint16_t a_inv_h;                 // per-tensor activation multiplier (fp16 bits)
  int out_bf16;
  int out_row_major;
  int pdl;                          // launched with programmatic stream serialisation
  float wgt_scale;                  // FMT_WGT: scale_b (or scale_b / 256 when wgt_fast)
  int wgt_fast;                     // FMT_WGT: packed decode allowed for this scale
  int no_alloc;                     // the launcher may not allocate device memory
  int row_quant;                    // per-row scales still to be computed (decode pre-pass)
  const float* bias;                // optional fused epilogue: + bias[n] (fp32)
  int act;                          // then 0 none, 1 ReLU, 2 GELU (tanh), 3 SiLU
  // column-parallel gather fused into the split-K epilogue (world > 1)
  int world, rank;
  unsigned int epoch;                       // 0: counted on the device
  unsigned long long peer_rows[8];          // this rank's output slice inside each rank's full output
  unsigned long long peer_sig[8];           // each rank's signal pad (u32 counters, epoch at kPeerEpochSlot)
  // host-buffer entry on the decode path: device addresses of page-locked
  // host activations (read by the activation pre-pass) and host output
  // (written by the epilogue beside D); null otherwise
  const void* a_host;
  void* d_host;
  unsigned long long* trace;        // FP8IMMA_TRACE builds only: per-CTA phase timestamps
  int dbg;                          // FP8IMMA_TRACE builds only: decode kernel experiment switches
};

// Signal pad layout (u32 words): [0, 8) arrival counters of the separate
// gather kernel, [8, 16) arrival counters of the gather fused into the GEMM
// epilogue, 32 / 33 the two forms' call epochs. 64 words in all.
constexpr int kPeerEpochSlot = 32;
constexpr int kPeerFusedSlot = 8;
constexpr int kPeerFusedEpochSlot = 33;

cudaError_t ensure_smem_attr(const void* kernel, int bytes);

// process-wide settings of the C ABI (fp8imma_set_pdl, fp8imma_set_splitk)
int api_pdl();
int api_splitk();

// Scratch memory owned by (current device, stream, tag): allocated on first
// use (zero-filled) and grown on demand, never freed; nullptr while the
// stream is capturing a graph and no large enough buffer exists yet (callers
// then take a path without scratch). *fresh tells whether the buffer was just
// (re)allocated. Tags: 0 stream-K partials, 1 decode activation rows,
// 2 tensor-core prep operands, 3 per-row activation scales.
void* stream_scratch(cudaStream_t stream, size_t bytes, int tag, bool* fresh = nullptr);

// Temporary device memory of one call: the calling stream's own scratch buffer
// (allocated once per device and stream, outside graph capture, and reused by
// every later call on that stream), or, while a graph is being captured before
// that buffer exists, a stream-ordered allocation freed at the end of the call.
struct ScopedScratch {
  void* ptr = nullptr;
  bool owned = false;
  cudaError_t get(size_t bytes, cudaStream_t st, int tag) {
    ptr = stream_scratch(st, bytes, tag);
    if (ptr) return cudaSuccess;
    owned = true;
    return cudaMallocAsync(&ptr, bytes, st);
  }
  cudaError_t release(cudaStream_t st) { return owned && ptr ? cudaFreeAsync(ptr, st) : cudaSuccess; }
};
// Tags of the callers of ScopedScratch
enum { kScratchTc = 2, kScratchRowScales = 3, kScratchGemvRows = 4, kScratchWgt = 5 };

// TMA descriptor for a 2-D byte tensor [outer][inner] (row pitch row_bytes).
cudaError_t make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                            uint32_t box_inner, uint32_t box_outer, bool swizzle128);

// Device error words of the kernel files that wait on barriers (0 = none),
// and their wait limits (current device).
unsigned int gemv_device_error(bool clear);
unsigned int decode_device_error(bool clear);
cudaError_t gemv_set_wait_limit(unsigned long long ns);
cudaError_t decode_set_wait_limit(unsigned long long ns);
cudaError_t tc_set_wait_limit(unsigned long long ns);
cudaError_t peer_set_wait_limit(unsigned long long ns);
int num_sms_current();

// Small-M split-K kernel (requires K % 16 == 0, 16-byte aligned A/B rows).
// splits = 0 picks the K split from the shape.
cudaError_t launch_gemv_s8(GemvParams p, int a_type, int fmt, int splits, cudaStream_t stream);
// launch_gemv_s8 with these arguments would run the decode kernel
bool gemv_would_decode(const GemvParams& p, int a_type, int fmt, int splits);
// the decode kernel would read the activations through its pre-pass (whose
// scratch already exists on `stream`): host activations / outputs can be used
// in place (GemvParams::a_host, d_host)
bool decode_host_direct_ok(const GemvParams& p, int a_type, int fmt, cudaStream_t stream);
// a per-stream scratch buffer of at least `bytes` already exists (no allocation)
bool stream_scratch_ready(cudaStream_t stream, size_t bytes, int tag);
// whether the last launch_gemv_s8 on this thread ran the balanced decode kernel
bool gemv_last_used_decode();
int gemv_pick_splits(int N, int K, int mchunks, int num_sms);
// Small-M kernel form: 1 (default) = stream-K where the cluster form would
// need more than one wave, else clusters; 2 = always stream-K; 0 = never.
void gemv_set_stream_k(int mode);

// Balanced decode kernel (one CTA per SM, CTA pairs split K): int8-exact
// formats, M <= 16, shapes that fit one wave of at most 8 column groups of 8
// per CTA. decode_set_mode(0) turns it off (the split-K kernels run instead).
bool decode_applicable(const GemvParams& p, int a_type, int fmt);
cudaError_t launch_decode(const GemvParams& p, int a_type, int fmt, cudaStream_t stream);
// Per-row quantised decode in two launches: one pre-pass computes each row's
// scales (as launch_row_scales) and quantises the row, then the decode kernel.
// cudaErrorNotSupported when the shape or the stream's scratch does not allow
// it (the caller then takes the row-scale kernel + GEMM route).
cudaError_t launch_decode_rowquant(const GemvParams& p, int a_type, int fmt, cudaStream_t stream);
void decode_set_mode(int mode);

// Large-M tensor-core path (tcgen05). Scratch must hold
// gemm_tc_scratch_bytes() bytes (16-byte aligned).
size_t gemm_tc_scratch_bytes(int M, int N, int K, bool native);
cudaError_t launch_gemm_tc_s8(const GemvParams& p, int a_type, int fmt, void* scratch, cudaStream_t stream);
cudaError_t launch_gemm_tc_fp8(const void* A, int a_type, const uint8_t* B, int b_fmt, const float* col_scale,
                               void* D, int M, int N, int K, int out_bf16, int out_row_major, void* scratch,
                               cudaStream_t stream, const float* bias = nullptr, int act = 0);
unsigned int tc_device_error(bool clear);
cudaError_t launch_gemm_tc_wgt(const void* A_f16, const uint8_t* B, float scale_b, float* C, int M, int N, int K,
                               void* scratch, cudaStream_t stream);
void tc_set_pair_mode(bool on);
// CTA-pair kernel K splits: -1 automatic (default), else forced.
void tc_set_splitk(int splits);
// CTA-pair kernel activation rows per tile: 0 automatic (default), or 256 / 192 / 128.
void tc_set_tile_x(int rows);
// CTA-pair kernel: last partial round of tiles as half-width items (default on).
void tc_set_half_tail(bool on);
int tc_pick_splits(int M, int N, int Kbytes);
// split-K accumulator workspace the CTA-pair kernel needs for this shape
size_t tc_splitk_ws_bytes(int M, int N, int Kbytes);  // tcgen05 GEMM: CTA-pair (cta_group::2) kernel or 1-CTA kernel
cudaError_t launch_quant_a_s8(const void* A, int a_type, int M, int K, uint16_t a_inv_h, const uint16_t* row_inv_h,
                              int8_t* Aq, cudaStream_t stream);
cudaError_t launch_quant_a_e4m3(const void* A, int a_type, int M, int K, uint8_t* Aq, float* row_scale,
                                cudaStream_t stream);

// Push this rank's rows [row0, row0+rows) of a [*, M] fp16 buffer into every
// peer's buffer at the same rows, then wait until every peer has done the
// same (bounded wait; a timeout records a code and returns). pdl: launched as
// a programmatic dependent of the GEMM that wrote the rows.
cudaError_t launch_peer_gather(const unsigned long long* outs, const unsigned long long* pads, int world, int rank,
                               size_t row0, size_t rows, int M, unsigned int epoch, bool pdl, cudaStream_t stream);
unsigned int peer_device_error(bool clear);

// Exact fallback for shapes the fast kernels do not take (any K, any alignment).
cudaError_t launch_generic_s8(const GemvParams& p, int a_type, int fmt, cudaStream_t stream);

// Per-row dynamic activation scales: a_inv_h[m] (fp16 bits), g[m] (fp32).
cudaError_t launch_row_scales(const void* A, int a_type, int M, int K, uint16_t* a_inv_h,
                              float* g, cudaStream_t stream);

}  // namespace fp8imma_b200
