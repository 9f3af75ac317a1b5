// fp8imma extension C ABI — B200 (sm_100a).
//
// Entry points for features the reference API (imma_fp8.h) has no slot for:
// per-row dynamic activation quantisation, an fp32 per-column scale fused
// into the epilogue, bf16 output, row-major output, E5M2 weight storage, the
// native FP8 tensor-core path, an int32 accumulator export, and the fp8wgt
// torch extension's fp16-activation kernel as a C entry point.
// Same conventions as the reference C ABI: plain pointers, void* stream
// (cudaStream_t), int return = cudaError_t (0 = success); the library
// launches asynchronously on the caller's stream.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum fp8imma_a_type { FP8IMMA_A_F16 = 0, FP8IMMA_A_BF16 = 1, FP8IMMA_A_S8 = 2 };

// B byte format. On the int8-exact path E4M3 decodes through the reference
// table semantics (exponent 15: +-Inf for mantissa 0, NaN otherwise); on the
// native path E4M3 is the hardware E4M3FN format. E5M2 is IEEE-like on both.
enum fp8imma_b_format { FP8IMMA_B_E4M3 = 0, FP8IMMA_B_E5M2 = 1 };

enum fp8imma_path {
  FP8IMMA_PATH_INT8_EXACT = 0,  // reference arithmetic, bit-exact int32 accumulators
  FP8IMMA_PATH_FP8_NATIVE = 1   // activations -> E4M3 per row, FP8 tensor cores, fp32 accumulate
};

enum fp8imma_act_quant {
  FP8IMMA_AQ_TENSOR = 0,  // one a_inv_scale / global_scale for the tensor (reference behaviour)
  FP8IMMA_AQ_ROW = 1      // per-row absmax: a_inv_m = 127/absmax_m, g_m = 1/a_inv_m
};

enum fp8imma_out_type { FP8IMMA_OUT_F16 = 0, FP8IMMA_OUT_BF16 = 1 };
enum fp8imma_out_layout { FP8IMMA_OUT_COL = 0 /* D[n*M+m] */, FP8IMMA_OUT_ROW = 1 /* D[m*N+n] */ };

typedef struct fp8imma_gemm_args {
  int path;        // fp8imma_path
  int a_type;      // fp8imma_a_type (S8 only on the int8-exact path)
  int b_format;    // fp8imma_b_format
  int act_quant;   // fp8imma_act_quant (int8-exact path; the native path is always per row)
  int out_type;    // fp8imma_out_type
  int out_layout;  // fp8imma_out_layout
  int M, N, K;
  const void* A;               // [M,K] row-major
  const void* B;               // [N,K] row-major FP8 bytes
  const void* col_scales_u16;  // int8-exact path: [N] fp16 int8-step scales (required)
  const float* col_scales_f32; // optional [N] fp32 multiplier (sigma_c); native path: weight scale
  float global_scale;          // int8-exact path with FP8IMMA_AQ_TENSOR
  float a_inv_scale;           // int8-exact path with FP8IMMA_AQ_TENSOR
  void* D;                     // output, out_type / out_layout
  int32_t* acc_out;            // optional [N,M] int32 accumulators (int8-exact path)
} fp8imma_gemm_args;

// Extended GEMM. No reference counterpart (extends imma_fp8.h:230). On the
// int8-exact path with act_quant = TENSOR, out F16/COL, no col_scales_f32 it
// equals fp8imma_launch_imma_fp8_actquant_v4_{f16,bf16} bit for bit.
// Temporaries (per-row scales, int8 / E4M3 copies of the operands on the
// large-M paths, quantised activation rows) live in per-(device, stream)
// scratch buffers allocated on the first call that needs them and reused by
// later calls on that stream; a call captured in a CUDA graph before its
// buffer exists uses stream-ordered cudaMallocAsync / cudaFreeAsync instead.
int fp8imma_gemm(const fp8imma_gemm_args* args, void* stream);

// fp8imma_gemm with a fused epilogue after the scales, in fp32 before the
// final rounding: + bias[n] (device fp32 [N], or null), then `act`:
// 0 none, 1 ReLU, 2 GELU (tanh form), 3 SiLU. Both paths, every kernel.
int fp8imma_gemm_epilogue(const fp8imma_gemm_args* args, const float* bias, int act, void* stream);

// fp8imma_gemm with host-side activations and result: copies A_host (M x K
// elements of the activation type; page-locked memory for an asynchronous
// copy) into args->A, runs fp8imma_gemm, and copies args->D (M x N outputs)
// back into D_host, all queued on `stream` (the call returns before the
// copies finish; synchronise the stream before reading D_host). args->A and
// args->D are the caller's device staging buffers. On the decode shapes
// (int8-exact path, per-tensor quantisation, fp16 / bf16 activations, M small
// enough for the balanced decode kernel) with page-locked A_host and D_host,
// once the stream has run one such call, the kernels read A_host and write
// D_host in place instead (no copies): args->D still receives the result,
// args->A is then not written.
int fp8imma_gemm_host_io(const fp8imma_gemm_args* args, const void* A_host, void* D_host, void* stream);

// Weight quantiser (no reference counterpart beyond an approximate per-tensor
// benchmark encoder): W [N,K] (fp16 / bf16 / fp32, finite) -> FP8 bytes
// B_out [N,K] with a per-row (= per output column) scale:
//   sigma_n = max(absmax_k |W[n,k]|, 1e-30) / fmax, B = fp8_rne_satfinite(W / sigma_n),
// col_scale_out[n] = sigma_n (fp32, the native path's column scale; may be
// null), step_out[n] = fp16(max_k |decode(B[n,k])| / 127) (the int8 step the
// reference API takes as col_scales; may be null).
enum fp8imma_w_type { FP8IMMA_W_F16 = 0, FP8IMMA_W_BF16 = 1, FP8IMMA_W_F32 = 2 };
enum fp8imma_q_format {
  FP8IMMA_Q_E4M3FN = 0,   // fmax 448 (hardware E4M3FN range)
  FP8IMMA_Q_E5M2 = 1,     // fmax 57344
  FP8IMMA_Q_E4M3_REF = 2  // fmax 240: codes the reference decode table reads as finite
};
int fp8imma_quantize_weights(const void* W, int w_type, int N, int K, int fmt, void* B_out, float* col_scale_out,
                             uint16_t* step_out, void* stream);

// Largest M accepted by fp8imma_gemm_rowquant_noalloc.
#define FP8IMMA_NOALLOC_MAX_M 4096

// Allocation-free per-row-quantised GEMM. No counterpart in the reference (it
// has no per-row quantisation). Same arguments and results as fp8imma_gemm
// with path = FP8IMMA_PATH_INT8_EXACT and act_quant = FP8IMMA_AQ_ROW, for
// callers that may not allocate device memory: runtimes that reserve HBM for
// their own pool up front, serving loops that forbid allocation on the
// request path, and plugin hosts that pass the plugin only caller-owned
// buffers. The caller still passes A, B, scales and D; the per-row values the
// two internal kernels exchange live in a fixed device array of
// FP8IMMA_NOALLOC_MAX_M rows (24 KB) that every GPU loading the library keeps
// until exit. M > FP8IMMA_NOALLOC_MAX_M returns cudaErrorInvalidValue.
// It calls no cudaMalloc / cudaFree / cudaMallocAsync. The first call on each
// device looks up the array's device address (cudaGetSymbolAddress, with that
// device current); make that first call before any stream capture. Every call
// on a device shares the one array (each call overwrites the rows it uses
// before reading them), so calls that overlap on the GPU, e.g. on two streams
// at once, race and must not be issued. fp8imma_set_pdl and fp8imma_set_splitk
// apply as for fp8imma_gemm. Every M runs the small-M kernels (split-K /
// decode; the tensor-core path needs scratch), so M in the hundreds or
// thousands is correct but far slower than through fp8imma_gemm.
int fp8imma_gemm_rowquant_noalloc(const fp8imma_gemm_args* args, void* stream);

// fp8wgt linear: C[M,N] (fp32, row-major) = A[M,K] (fp16) x decode(B[N,K])^T,
// decode(b) = fp16_rn(float(lut_e4m3[b]) * scale_b). Replaces
// torch_ext/fp8wgt/fp8wgt_ext_cuda.cu:223 fp8_linear_forward (kernel :135),
// as a C entry point; runs on `stream` (the reference used the default stream).
int fp8imma_fp8wgt_linear_forward(const void* A_f16, const void* B_u8, float scale_b, void* C_f32,
                                  int M, int N, int K, void* stream);

// Column-parallel GEMM with the output gather fused in (no reference
// counterpart: the reference has no multi-GPU code). Rank `rank` of `world`
// (<= 8) passes its weight shard (args->B, [N_shard, K]) and shard scales;
// the GEMM writes this rank's [N_shard, M] slice of the col-major output into
// rows rank*N_shard.. of its own full buffer peer_out[rank] ([world*N_shard,
// M]) and into the same rows of every peer's buffer over NVLink (peer
// stores, from the GEMM's epilogue or a gather kernel, see
// fp8imma_set_fused_gather), then waits until every rank's slice has arrived
// here. peer_out / peer_signal hold device pointers to all ranks' buffers,
// valid in this process (e.g. a symmetric allocation); each signal pad needs
// 64 zero-initialised uint32 slots; `epoch` must grow by one per call
// (1, 2, ...), or be 0: the epoch is then counted on the device in the pad
// of this rank, so a captured CUDA graph can be replayed.
// Int8-exact path, per-tensor quantisation, col-major output, small M (the
// split-K kernel). The call returns when the launches are queued; the output
// is complete on every rank once this stream reaches the end of the call.
// The caller must not rewrite an output buffer that a peer may still be
// reading from the previous call (alternate two buffers).
int fp8imma_gemm_allgather(const fp8imma_gemm_args* args, void* const* peer_out, void* const* peer_signal, int world,
                           int rank, unsigned int epoch, void* stream);
// 1: the gather of fp8imma_gemm_allgather runs in the GEMM's own epilogue
// (peer stores + one system-scope release per CTA, first CTA waits for the
// peers); 0 (default, measured faster: 17.3 vs 19.4 us per decode step on 2
// GPUs): a separate gather kernel after the GEMM. Each form keeps its own
// counters and epoch in the signal pad, so the setting may change between
// calls.
int fp8imma_set_fused_gather(int enable);

// Tuning / introspection (no reference counterpart).
// Force the K split of the small-M kernel (0 = automatic; 1, 2, 4 or 8).
int fp8imma_set_splitk(int splits);
// Small-M kernel form when no split is forced. Stream-K: persistent CTAs
// with an even share of the weight bytes each, partial sums in a per-device
// scratch ring allocated on first use. Clusters: K slices of a column tile
// reducing in distributed shared memory. 1 (default) = stream-K where the
// cluster form would need more than one wave of CTAs, else clusters;
// 2 = always stream-K; 0 = always clusters.
int fp8imma_set_stream_k(int mode);
// Largest M routed to the small-M split-K kernel (default 64).
int fp8imma_set_small_m_max(int m);
// Large-M tensor-core kernel: 1 (default) = CTA-pair kernel (tcgen05
// cta_group::2, 256x256 tiles), 0 = single-CTA kernel (128x256 tiles).
int fp8imma_set_tc_pair(int enable);
// K splits of the CTA-pair tcgen05 kernel: -1 (default) = automatic (split
// when the 256 x 256 tiles would leave most CTA pairs idle, e.g. M <= 512 at
// N = 4096), 1 = never, n > 1 = forced. Partial accumulators go to
// stream-ordered scratch and a second kernel finishes the epilogue.
int fp8imma_set_tc_splitk(int splits);
// Activation rows per CTA-pair tile (the MMA's N): 0 (default) = chosen per
// shape to balance the rounds of tiles over the CTA pairs; 256, 192 or 128
// forced.
int fp8imma_set_tc_tile_x(int rows);
// 1 (default): when the CTA-pair kernel's last round of tiles would leave more
// than half of the CTA pairs idle, those tiles run as two half-width items
// each (4096 x 4096: 34 of 256 tiles); 0: all tiles at full width.
int fp8imma_set_tc_half_tail(int enable);
// 1 (default): small-M shapes that fit one wave of at most 64 weight columns
// per SM (e.g. N = K = 4096) run the balanced decode kernel (one CTA per SM,
// CTA pairs splitting K); 2: the decode kernel without the early weight
// transcode (it otherwise converts its weights to int8 in shared memory while
// the activations are still to come); 0: they run the split-K cluster kernel.
// Results are identical in every mode. No reference counterpart (tuning
// switch).
int fp8imma_set_decode_kernel(int enable);
// Programmatic dependent launch (default on). A small-M GEMM then starts
// streaming its weights and reading its column scales while the previous
// kernel in the stream is still running; activations are read, and outputs
// written, only after that kernel has finished (a kernel launched after the
// GEMM without the attribute is ordered as usual). Turn it off when weights or
// scales are written by the kernel launched just before the GEMM.
int fp8imma_set_pdl(int enable);
// Kernel family the last fp8imma call on this thread launched:
// 0 none, 1 small-M split-K, 2 generic fallback, 3 tcgen05 GEMM, 4 native FP8
// tcgen05 GEMM, 5 native FP8 small-M split-K, 6 balanced decode kernel.
int fp8imma_last_path(void);
const char* fp8imma_version(void);
// Error word of the current device: non-zero when a kernel gave up a bounded
// wait on its internal pipeline (the kernel then returned early and its output
// is not valid). Synchronises the device. clear != 0 resets it.
unsigned int fp8imma_device_error(int clear);
// Wall-time limit of every bounded wait in the kernels (mbarrier pipelines,
// the NVLink gather's peer flags) on the current device, in nanoseconds;
// default 2e9; values below 1e6 act as 1e6. A wait that runs out records a code in the error word above and
// lets its kernel finish. No reference counterpart (failure handling).
int fp8imma_set_wait_limit_ns(unsigned long long ns);

#ifdef __cplusplus
}  // extern "C"
#endif
