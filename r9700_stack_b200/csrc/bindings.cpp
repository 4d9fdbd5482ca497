// torch.library registrations for the sm_100a kernel library (namespace torch.ops.r9k).
// Every op mutates preallocated outputs and returns nothing, so all of them are safe inside CUDA
// graph capture (no allocation, no host sync). Reference counterpart: the `r9700` op namespace
// registered in r9700_vllm/ops.py:125-136.
#include <torch/extension.h>
#include <torch/library.h>

namespace r9k {
// gemm_tc.cu
void gemm_mx(torch::Tensor w, torch::Tensor w_sf, bool w_fp4, torch::Tensor x, torch::Tensor x_sf, torch::Tensor out,
             c10::optional<torch::Tensor> residual, double alpha, torch::Tensor status);
void gemm_mx_swiglu(torch::Tensor wg, torch::Tensor wg_sf, torch::Tensor wu, torch::Tensor wu_sf, bool w_fp4,
                    torch::Tensor x, torch::Tensor x_sf, torch::Tensor out_q, torch::Tensor out_sf, torch::Tensor status);
void gemm_bf16(torch::Tensor w, torch::Tensor x, torch::Tensor out, c10::optional<torch::Tensor> residual, double alpha,
               torch::Tensor status);
// quant.cu
void rmsnorm_quant(torch::Tensor x, c10::optional<torch::Tensor> res_in, c10::optional<torch::Tensor> res_out,
                   torch::Tensor w, double eps, bool plus_one, c10::optional<torch::Tensor> y,
                   c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf);
void quant_act_mxfp8(torch::Tensor x, torch::Tensor q, torch::Tensor sf);
void quant_weight_mxfp4(torch::Tensor w, torch::Tensor packed, torch::Tensor sf, bool search);
void quant_weight_mxfp8(torch::Tensor w, torch::Tensor q, torch::Tensor sf);
void quant_weight_nvfp4(torch::Tensor w, double global_scale, torch::Tensor packed, torch::Tensor s16);
void nvfp4_to_mxfp4(torch::Tensor packed_in, torch::Tensor s16, double global_scale, torch::Tensor packed_out,
                    torch::Tensor sf, bool search);
void dequant_mx(torch::Tensor q, torch::Tensor sf, bool fp4, torch::Tensor out);
}  // namespace r9k

TORCH_LIBRARY(r9k, m) {
  m.def("gemm_mx(Tensor w, Tensor w_sf, bool w_fp4, Tensor x, Tensor x_sf, Tensor(a!) out, Tensor? residual, "
        "float alpha, Tensor(b!) status) -> ()");
  m.def("gemm_mx_swiglu(Tensor wg, Tensor wg_sf, Tensor wu, Tensor wu_sf, bool w_fp4, Tensor x, Tensor x_sf, "
        "Tensor(a!) out_q, Tensor(b!) out_sf, Tensor(c!) status) -> ()");
  m.def("gemm_bf16(Tensor w, Tensor x, Tensor(a!) out, Tensor? residual, float alpha, Tensor(b!) status) -> ()");
  m.def("rmsnorm_quant(Tensor x, Tensor? res_in, Tensor(a!)? res_out, Tensor w, float eps, bool plus_one, "
        "Tensor(b!)? y, Tensor(c!)? q, Tensor(d!)? sf) -> ()");
  m.def("quant_act_mxfp8(Tensor x, Tensor(a!) q, Tensor(b!) sf) -> ()");
  m.def("quant_weight_mxfp4(Tensor w, Tensor(a!) packed, Tensor(b!) sf, bool search) -> ()");
  m.def("quant_weight_mxfp8(Tensor w, Tensor(a!) q, Tensor(b!) sf) -> ()");
  m.def("quant_weight_nvfp4(Tensor w, float global_scale, Tensor(a!) packed, Tensor(b!) s16) -> ()");
  m.def("nvfp4_to_mxfp4(Tensor packed_in, Tensor s16, float global_scale, Tensor(a!) packed_out, Tensor(b!) sf, "
        "bool search) -> ()");
  m.def("dequant_mx(Tensor q, Tensor sf, bool fp4, Tensor(a!) out) -> ()");
}

TORCH_LIBRARY_IMPL(r9k, CUDA, m) {
  m.impl("gemm_mx", &r9k::gemm_mx);
  m.impl("gemm_mx_swiglu", &r9k::gemm_mx_swiglu);
  m.impl("gemm_bf16", &r9k::gemm_bf16);
  m.impl("rmsnorm_quant", &r9k::rmsnorm_quant);
  m.impl("quant_act_mxfp8", &r9k::quant_act_mxfp8);
  m.impl("quant_weight_mxfp4", &r9k::quant_weight_mxfp4);
  m.impl("quant_weight_mxfp8", &r9k::quant_weight_mxfp8);
  m.impl("quant_weight_nvfp4", &r9k::quant_weight_nvfp4);
  m.impl("nvfp4_to_mxfp4", &r9k::nvfp4_to_mxfp4);
  m.impl("dequant_mx", &r9k::dequant_mx);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) { m.doc() = "r9700_stack_b200 sm_100a kernel library"; }
