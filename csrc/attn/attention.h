// Host API of the tcgen05 attention kernels.
#pragma once
#include <torch/extension.h>

#include <vector>

namespace h3 {

// qkv [T, 3H] bf16 (RoPE applied) -> {o [T, H] bf16, lse [heads, T] fp32 (natural log)}
std::vector<at::Tensor> attention_fwd(const at::Tensor& qkv, int64_t heads, int64_t head_dim, const at::Tensor& status,
                                      int64_t limit_ns, const c10::optional<at::Tensor>& trace = c10::nullopt);

// dO [T, H] bf16 -> dqkv [T, 3H] bf16 (gradients w.r.t. the post-RoPE q, k and v)
at::Tensor attention_bwd(const at::Tensor& qkv, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dout,
                         int64_t heads, int64_t head_dim, const at::Tensor& status, int64_t limit_ns,
                         const c10::optional<at::Tensor>& trace = c10::nullopt);

}  // namespace h3
