// Host API of the bandwidth-bound kernels (see elementwise.cu).
#pragma once
#include <torch/extension.h>

#include <vector>

namespace h3 {

at::Tensor norm_modulate_fwd(const at::Tensor& x, const at::Tensor& shift, const at::Tensor& scale, int64_t split,
                             double eps);
std::vector<at::Tensor> norm_modulate_bwd(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& scale,
                                          int64_t split, double eps, const c10::optional<at::Tensor>& add,
                                          const c10::optional<at::Tensor>& gate);
at::Tensor gate_mul(const at::Tensor& g, const at::Tensor& gate, int64_t split);
void rope_inverse_(const at::Tensor& t, const at::Tensor& cos_t, const at::Tensor& sin_t, int64_t rope_cols,
                   int64_t head_dim);
at::Tensor adaln_project(const at::Tensor& temb, const at::Tensor& w, const c10::optional<at::Tensor>& b);
std::vector<at::Tensor> flow_step(const at::Tensor& xt, const at::Tensor& v, double s, double s_next, bool want_x0,
                                  bool want_next, c10::ScalarType next_dtype);
at::Tensor add_noise(const at::Tensor& x0, const at::Tensor& noise, double s);
std::vector<at::Tensor> dmd_forward(const at::Tensor& generated, const at::Tensor& x0_fake, const at::Tensor& x0_real);
at::Tensor scale_copy(const at::Tensor& g, double coef, const at::Tensor& upstream, c10::ScalarType out_dtype);
at::Tensor mse_forward(const at::Tensor& pred, const at::Tensor& target);
at::Tensor mse_backward(const at::Tensor& pred, const at::Tensor& target, const at::Tensor& upstream);
at::Tensor sum_squares(const at::Tensor& x);
void adamw_step(const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, const at::Tensor& grad,
                const at::Tensor& param, const at::Tensor& norm, double lr, double b1, double b2, double eps,
                double wd, int64_t step, double max_norm);

}  // namespace h3
