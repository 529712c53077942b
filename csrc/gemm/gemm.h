// Host API of the tcgen05 GEMM (see gemm_tcgen05.cu).
#pragma once
#include <torch/extension.h>

#include <vector>

namespace h3 {

enum GemmEpilogue : int {
  kEpiBf16 = 0,      // out = bf16(alpha * acc + bias)
  kEpiGelu = 1,      // out = bf16(acc + bias) (pre-activation), out2 = bf16(gelu_tanh(out))
  kEpiRope = 2,      // out = bf16(rope(bf16(acc + bias))) on columns < rope_cols
  kEpiGatedRes = 3,  // out = bf16(res + gate[row] * bf16(acc + bias))
  kEpiGeluBwd = 4,   // out = bf16(bf16(acc) * gelu_tanh'(pre))
  kEpiF32Acc = 5,    // out_f32 += alpha * acc (atomic when split over K)
};

void gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t M, int64_t N, int64_t K,
          const std::vector<at::Tensor>& A2, const c10::optional<at::Tensor>& B2, int64_t K2, int64_t section_n,
          int64_t epi, const at::Tensor& out, const c10::optional<at::Tensor>& out2,
          const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& res,
          const c10::optional<at::Tensor>& gate, int64_t split_row, const c10::optional<at::Tensor>& cos_t,
          const c10::optional<at::Tensor>& sin_t, int64_t rope_cols, int64_t head_dim,
          const c10::optional<at::Tensor>& pre, double alpha, int64_t splits, int64_t block_n,
          const at::Tensor& status, int64_t limit_ns, const std::vector<int64_t>& gather_src,
          int64_t gather_rows, const c10::optional<at::Tensor>& gather_flags);

uint64_t launch_count();
void note_launch();

}  // namespace h3
