// Python bindings of the sm_100a extension (module h3_a100._C).
#include <torch/extension.h>

#include "attn/attention.h"
#include "comm/p2p.h"
#include "elementwise/elementwise.h"
#include "gemm/gemm.h"

namespace h3 {
at::Tensor pinned_empty(int64_t numel, c10::ScalarType dtype);
int64_t pinned_bytes();
}  // namespace h3

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "Hand-written sm_100a kernels of the H3 DMD trainer";
  m.def("gemm", &h3::gemm, "tcgen05 GEMM with fused epilogues");
  m.def("attention_fwd", &h3::attention_fwd, "tcgen05 attention forward", py::arg("qkv"), py::arg("heads"),
        py::arg("head_dim"), py::arg("status"), py::arg("limit_ns"), py::arg("trace") = py::none());
  m.def("attention_bwd", &h3::attention_bwd, "tcgen05 attention backward", py::arg("qkv"), py::arg("o"),
        py::arg("lse"), py::arg("dout"), py::arg("heads"), py::arg("head_dim"), py::arg("status"),
        py::arg("limit_ns"), py::arg("trace") = py::none());
  m.def("p2p_all_gather", &h3::p2p_all_gather, "pull all-gather over peer memory");
  m.def("p2p_all_gather_ce", &h3::p2p_all_gather_ce, "all-gather over peer memory on the copy engines");
  m.def("lora_rs_adamw", &h3::lora_rs_adamw, "fused LoRA reduce-scatter + clip + AdamW + all-gather");
  m.def("adaln_project_gather", &h3::adaln_project_gather, "row-sharded AdaLN GEMV with fused output all-gather");
  m.def("wait_flag_test", &h3::wait_flag_test, "bounded wait on a flag (failure-detection tests)");
  m.def("enable_peer_access", &h3::enable_peer_access, "let kernels on a device load from a peer GPU");
  m.def("launch_count", &h3::launch_count, "number of kernels launched by this extension");
  m.def("norm_modulate_fwd", &h3::norm_modulate_fwd);
  m.def("norm_modulate_bwd", &h3::norm_modulate_bwd);
  m.def("gate_mul", &h3::gate_mul);
  m.def("rope_inverse_", &h3::rope_inverse_);
  m.def("adaln_project", &h3::adaln_project);
  m.def("flow_step", &h3::flow_step);
  m.def("add_noise", &h3::add_noise);
  m.def("dmd_forward", &h3::dmd_forward);
  m.def("scale_copy", &h3::scale_copy);
  m.def("mse_forward", &h3::mse_forward);
  m.def("mse_backward", &h3::mse_backward);
  m.def("sum_squares", &h3::sum_squares);
  m.def("adamw_step", &h3::adamw_step);
  m.def("pinned_empty", &h3::pinned_empty);
  m.def("pinned_bytes", &h3::pinned_bytes);
  m.attr("EPI_BF16") = static_cast<int>(h3::kEpiBf16);
  m.attr("EPI_GELU") = static_cast<int>(h3::kEpiGelu);
  m.attr("EPI_ROPE") = static_cast<int>(h3::kEpiRope);
  m.attr("EPI_GATED_RES") = static_cast<int>(h3::kEpiGatedRes);
  m.attr("EPI_GELU_BWD") = static_cast<int>(h3::kEpiGeluBwd);
  m.attr("EPI_F32_ACC") = static_cast<int>(h3::kEpiF32Acc);
}
