// Host API of the peer-memory collectives (see p2p.cu).
#pragma once
#include <torch/extension.h>

#include <vector>

namespace h3 {

void p2p_all_gather(const std::vector<int64_t>& shard_ptrs, int64_t shard_bytes, const at::Tensor& out);
void p2p_all_gather_ce(const std::vector<int64_t>& shard_ptrs, int64_t shard_bytes, const at::Tensor& out);
void lora_rs_adamw(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& param_ptrs,
                   const std::vector<int64_t>& flag_ptrs, int64_t rank, int64_t epoch, const at::Tensor& master,
                   const at::Tensor& m, const at::Tensor& v, const at::Tensor& scratch, const at::Tensor& bar,
                   double lr, double b1, double b2, double eps, double wd, int64_t step, double max_norm,
                   const at::Tensor& status, int64_t limit_ns, int64_t mc_grad, int64_t mc_param);
void adaln_project_gather(const at::Tensor& temb, const at::Tensor& w, const c10::optional<at::Tensor>& b,
                          const std::vector<int64_t>& out_ptrs, const std::vector<int64_t>& flag_ptrs, int64_t rank,
                          int64_t epoch, int64_t slot, const at::Tensor& status, int64_t limit_ns);
void wait_flag_test(const at::Tensor& flag, int64_t epoch, const at::Tensor& status, int64_t limit_ns);
void enable_peer_access(int64_t device, int64_t peer);

}  // namespace h3
