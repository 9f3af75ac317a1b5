// PyTorch binding of the fp8imma B200 library (module name fp8imma_ext).
//
// imma_fp8_v4_act mirrors the reference binding
// torch_ext/fp8imma/fp8imma_ext.cpp:41-126 (same arguments, checks, error
// messages and result layout) and calls the same C ABI entry points, which
// here run the sm_100a kernels of libfp8imma.so. imma_fp8_gemm exposes the
// extension entry point fp8imma_gemm (include/fp8imma/fp8imma_ext.h).
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdint>
#include <string>

#include "fp8imma/fp8imma_ext.h"
#include "fp8imma/imma_fp8.h"

static void check_launch(int err, const char* what) {
  TORCH_CHECK(err == 0, what, " failed, cudaError_t=", err);
}

static const void* scale_ptr(const torch::Tensor& s) {
  if (s.scalar_type() == at::kHalf) return (const void*)s.data_ptr<at::Half>();
  return (const void*)s.data_ptr<int16_t>();
}

torch::Tensor imma_fp8_v4_act(torch::Tensor A, torch::Tensor B_col_fp8, torch::Tensor col_scales_f16,
                              double global_scale, double a_inv_scale, int64_t kChunk) {
  TORCH_CHECK(A.is_cuda(), "A must be a CUDA tensor");
  TORCH_CHECK(B_col_fp8.is_cuda(), "B_col_fp8 must be a CUDA tensor");
  TORCH_CHECK(col_scales_f16.is_cuda(), "col_scales_f16 must be a CUDA tensor");
  TORCH_CHECK(A.is_contiguous(), "A must be contiguous");
  TORCH_CHECK(B_col_fp8.is_contiguous(), "B_col_fp8 must be contiguous");
  TORCH_CHECK(col_scales_f16.is_contiguous(), "col_scales_f16 must be contiguous");
  TORCH_CHECK(A.dim() == 2, "A must be 2D [M,K]");
  TORCH_CHECK(B_col_fp8.dim() == 2, "B_col_fp8 must be 2D [N,K]");
  TORCH_CHECK(col_scales_f16.dim() == 1, "col_scales_f16 must be 1D [N]");
  TORCH_CHECK(B_col_fp8.scalar_type() == at::kByte, "B_col_fp8 must be uint8");
  TORCH_CHECK(col_scales_f16.scalar_type() == at::kHalf || col_scales_f16.scalar_type() == at::kShort,
              "col_scales_f16 must be fp16 (scale bits) or uint16");
  TORCH_CHECK(kChunk == 32 || kChunk == 64, "kChunk must be 32 or 64");
  const int64_t M = A.size(0), K = A.size(1), N = B_col_fp8.size(0);
  TORCH_CHECK(B_col_fp8.size(1) == K, "B_col_fp8 must have shape [N,K]");
  TORCH_CHECK(col_scales_f16.size(0) == N, "col_scales_f16 must have shape [N]");
  TORCH_CHECK((M % 16) == 0 && (N % 16) == 0 && (K % 16) == 0, "M,N,K must be multiples of 16");

  const c10::cuda::CUDAGuard guard(A.device());
  fp8imma_init_fp8_e4m3_lut();
  auto out = torch::empty({N, M}, torch::TensorOptions().device(A.device()).dtype(torch::kFloat16));
  void* stream = (void*)at::cuda::getCurrentCUDAStream();
  if (A.scalar_type() == at::kHalf) {
    check_launch(fp8imma_launch_imma_fp8_actquant_v4_f16((int)kChunk, A.data_ptr(), B_col_fp8.data_ptr(),
                                                         scale_ptr(col_scales_f16), out.data_ptr(), (int)M,
                                                         (int)N, (int)K, (float)global_scale,
                                                         (float)a_inv_scale, stream),
                 "fp8imma_launch_imma_fp8_actquant_v4_f16");
  } else if (A.scalar_type() == at::kBFloat16) {
    check_launch(fp8imma_launch_imma_fp8_actquant_v4_bf16((int)kChunk, A.data_ptr(), B_col_fp8.data_ptr(),
                                                          scale_ptr(col_scales_f16), out.data_ptr(), (int)M,
                                                          (int)N, (int)K, (float)global_scale,
                                                          (float)a_inv_scale, stream),
                 "fp8imma_launch_imma_fp8_actquant_v4_bf16");
  } else {
    TORCH_CHECK(false, "A must be fp16 or bf16");
  }
  return out;
}

// General entry (no reference counterpart): any M >= 1, per-row quant, fp32
// column scale, bf16 / row-major output, E5M2 weights, native FP8 path,
// int32 accumulator export. Returns (D, acc or empty).
std::vector<torch::Tensor> imma_fp8_gemm(torch::Tensor A, torch::Tensor B, c10::optional<torch::Tensor> col_scales_f16,
                                         c10::optional<torch::Tensor> col_scales_f32, double global_scale,
                                         double a_inv_scale, std::string act_quant, std::string b_format,
                                         std::string path, std::string out_dtype, std::string out_layout,
                                         bool return_acc, c10::optional<torch::Tensor> out,
                                         c10::optional<torch::Tensor> a_host, c10::optional<torch::Tensor> out_host,
                                         c10::optional<torch::Tensor> bias, std::string act) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda(), "A and B must be CUDA tensors");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous(), "A and B must be contiguous");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "A must be [M,K] and B [N,K]");
  TORCH_CHECK(B.scalar_type() == at::kByte, "B must be uint8 FP8 bytes");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K, "B must have shape [N,K]");
  fp8imma_gemm_args a = {};
  if (path == "int8") a.path = FP8IMMA_PATH_INT8_EXACT;
  else if (path == "fp8") a.path = FP8IMMA_PATH_FP8_NATIVE;
  else TORCH_CHECK(false, "path must be 'int8' or 'fp8'");
  if (A.scalar_type() == at::kHalf) a.a_type = FP8IMMA_A_F16;
  else if (A.scalar_type() == at::kBFloat16) a.a_type = FP8IMMA_A_BF16;
  else if (A.scalar_type() == at::kChar) a.a_type = FP8IMMA_A_S8;
  else TORCH_CHECK(false, "A must be fp16, bf16 or int8");
  if (b_format == "e4m3") a.b_format = FP8IMMA_B_E4M3;
  else if (b_format == "e5m2") a.b_format = FP8IMMA_B_E5M2;
  else TORCH_CHECK(false, "b_format must be 'e4m3' or 'e5m2'");
  if (act_quant == "tensor") a.act_quant = FP8IMMA_AQ_TENSOR;
  else if (act_quant == "row") a.act_quant = FP8IMMA_AQ_ROW;
  else TORCH_CHECK(false, "act_quant must be 'tensor' or 'row'");
  at::ScalarType odt;
  if (out_dtype == "float16") { a.out_type = FP8IMMA_OUT_F16; odt = at::kHalf; }
  else if (out_dtype == "bfloat16") { a.out_type = FP8IMMA_OUT_BF16; odt = at::kBFloat16; }
  else TORCH_CHECK(false, "out_dtype must be 'float16' or 'bfloat16'");
  if (out_layout == "col") a.out_layout = FP8IMMA_OUT_COL;
  else if (out_layout == "row") a.out_layout = FP8IMMA_OUT_ROW;
  else TORCH_CHECK(false, "out_layout must be 'col' or 'row'");
  if (col_scales_f16.has_value()) {
    auto& s = *col_scales_f16;
    TORCH_CHECK(s.is_cuda() && s.is_contiguous() && s.dim() == 1 && s.size(0) == N, "col_scales_f16 must be [N] on CUDA");
    TORCH_CHECK(s.scalar_type() == at::kHalf || s.scalar_type() == at::kShort, "col_scales_f16 must be fp16 or int16 bits");
    a.col_scales_u16 = scale_ptr(s);
  }
  if (col_scales_f32.has_value()) {
    auto& s = *col_scales_f32;
    TORCH_CHECK(s.is_cuda() && s.is_contiguous() && s.dim() == 1 && s.size(0) == N && s.scalar_type() == at::kFloat,
                "col_scales_f32 must be float32 [N] on CUDA");
    a.col_scales_f32 = s.data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(A.device());
  std::vector<int64_t> shape = a.out_layout == FP8IMMA_OUT_COL ? std::vector<int64_t>{N, M} : std::vector<int64_t>{M, N};
  torch::Tensor D;
  if (out.has_value()) {
    D = *out;
    TORCH_CHECK(D.is_cuda() && D.is_contiguous() && D.scalar_type() == odt && D.sizes() == at::IntArrayRef(shape),
                "out has the wrong shape, dtype or layout");
  } else {
    D = torch::empty(shape, torch::TensorOptions().device(A.device()).dtype(odt));
  }
  torch::Tensor acc;
  if (return_acc) {
    acc = torch::empty({N, M}, torch::TensorOptions().device(A.device()).dtype(torch::kInt32));
    a.acc_out = acc.data_ptr<int32_t>();
  }
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.A = A.data_ptr();
  a.B = B.data_ptr();
  a.global_scale = (float)global_scale;
  a.a_inv_scale = (float)a_inv_scale;
  a.D = D.data_ptr();
  void* stream = (void*)at::cuda::getCurrentCUDAStream();
  int act_id = 0;
  if (act == "none") act_id = 0;
  else if (act == "relu") act_id = 1;
  else if (act == "gelu") act_id = 2;
  else if (act == "silu") act_id = 3;
  else TORCH_CHECK(false, "act must be 'none', 'relu', 'gelu' or 'silu'");
  if (bias.has_value() || act_id != 0) {
    // fused epilogue: + bias[n], activation (fp8imma_gemm_epilogue)
    TORCH_CHECK(!a_host.has_value() && !out_host.has_value(), "bias / act with host buffers is not supported");
    const float* bp = nullptr;
    if (bias.has_value()) {
      auto& b = *bias;
      TORCH_CHECK(b.is_cuda() && b.is_contiguous() && b.dim() == 1 && b.size(0) == N && b.scalar_type() == at::kFloat,
                  "bias must be float32 [N] on CUDA");
      bp = b.data_ptr<float>();
    }
    check_launch(fp8imma_gemm_epilogue(&a, bp, act_id, stream), "fp8imma_gemm_epilogue");
    return {D, acc.defined() ? acc : torch::Tensor()};
  }
  if (a_host.has_value() || out_host.has_value()) {
    // host-side activations in, host-side result out (fp8imma_gemm_host_io):
    // A is refreshed from a_host and D is copied to out_host on this stream
    TORCH_CHECK(a_host.has_value() && out_host.has_value(), "a_host and out_host go together");
    auto& ah = *a_host;
    auto& dh = *out_host;
    TORCH_CHECK(!ah.is_cuda() && ah.is_contiguous() && ah.scalar_type() == A.scalar_type() && ah.sizes() == A.sizes(),
                "a_host must be a contiguous host tensor shaped and typed like A");
    TORCH_CHECK(!dh.is_cuda() && dh.is_contiguous() && dh.scalar_type() == odt && dh.sizes() == at::IntArrayRef(shape),
                "out_host must be a contiguous host tensor shaped and typed like the output");
    check_launch(fp8imma_gemm_host_io(&a, ah.data_ptr(), dh.data_ptr(), stream), "fp8imma_gemm_host_io");
  } else {
    check_launch(fp8imma_gemm(&a, stream), "fp8imma_gemm");
  }
  return {D, acc.defined() ? acc : torch::Tensor()};
}

// Weight quantiser (fp8imma_quantize_weights): W [N,K] fp16/bf16/fp32 CUDA
// tensor -> (B [N,K] uint8, sigma [N] fp32, step [N] int16 fp16 bits).
std::vector<torch::Tensor> quantize_weights(torch::Tensor W, std::string fmt) {
  TORCH_CHECK(W.is_cuda() && W.is_contiguous() && W.dim() == 2, "W must be a contiguous 2-D CUDA tensor");
  int wt;
  if (W.scalar_type() == at::kHalf) wt = FP8IMMA_W_F16;
  else if (W.scalar_type() == at::kBFloat16) wt = FP8IMMA_W_BF16;
  else if (W.scalar_type() == at::kFloat) wt = FP8IMMA_W_F32;
  else TORCH_CHECK(false, "W must be fp16, bf16 or fp32");
  int f;
  if (fmt == "e4m3") f = FP8IMMA_Q_E4M3FN;
  else if (fmt == "e5m2") f = FP8IMMA_Q_E5M2;
  else if (fmt == "e4m3_ref") f = FP8IMMA_Q_E4M3_REF;
  else TORCH_CHECK(false, "fmt must be 'e4m3', 'e5m2' or 'e4m3_ref'");
  const int64_t N = W.size(0), K = W.size(1);
  const c10::cuda::CUDAGuard guard(W.device());
  auto B = torch::empty({N, K}, W.options().dtype(torch::kUInt8));
  auto sigma = torch::empty({N}, W.options().dtype(torch::kFloat));
  auto step = torch::empty({N}, W.options().dtype(torch::kShort));
  check_launch(fp8imma_quantize_weights(W.data_ptr(), wt, (int)N, (int)K, f, B.data_ptr(), sigma.data_ptr<float>(),
                                        reinterpret_cast<uint16_t*>(step.data_ptr<int16_t>()),
                                        (void*)at::cuda::getCurrentCUDAStream()),
               "fp8imma_quantize_weights");
  return {B, sigma, step};
}

int64_t last_path() { return fp8imma_last_path(); }
int64_t set_splitk(int64_t s) { return fp8imma_set_splitk((int)s); }
int64_t set_small_m_max(int64_t m) { return fp8imma_set_small_m_max((int)m); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("imma_fp8_v4_act", &imma_fp8_v4_act,
        "IMMA FP8-as-storage GEMM (v4 actquant), sm_100a\n"
        "A: [M,K] fp16/bf16 contiguous (row-major)\n"
        "B_col_fp8: [N,K] uint8 contiguous (represents col-major KxN)\n"
        "col_scales_f16: [N] fp16 contiguous (per-column scales)\n"
        "Returns D_col: [N,M] fp16 contiguous (represents col-major MxN)");
  m.def("imma_fp8_gemm", &imma_fp8_gemm, "extended fp8imma GEMM (see fp8imma_ext.h)", py::arg("A"), py::arg("B"),
        py::arg("col_scales_f16") = py::none(), py::arg("col_scales_f32") = py::none(), py::arg("global_scale") = 1.0,
        py::arg("a_inv_scale") = 1.0, py::arg("act_quant") = "tensor", py::arg("b_format") = "e4m3",
        py::arg("path") = "int8", py::arg("out_dtype") = "float16", py::arg("out_layout") = "col",
        py::arg("return_acc") = false, py::arg("out") = py::none(), py::arg("a_host") = py::none(),
        py::arg("out_host") = py::none(), py::arg("bias") = py::none(), py::arg("act") = "none");
  m.def("quantize_weights", &quantize_weights, "FP8 weight quantiser with per-column scales (see fp8imma_ext.h)",
        py::arg("W"), py::arg("fmt") = "e4m3");
  m.def("last_path", &last_path, "kernel family of the last call on this thread");
  m.def("set_splitk", &set_splitk, "force the small-M K split (0 = automatic)");
  m.def("set_small_m_max", &set_small_m_max, "largest M for the small-M kernel");
}
