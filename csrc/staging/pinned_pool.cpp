// Exact-size pinned host buffers for checkpoint-boundary staging.
//
// torch's caching host allocator rounds every pinned block up to a power of
// two; a 405,672,960-byte boundary would take 512 MiB, i.e. 25.6 GB per rank
// for one grad forward and more than the host RAM of an 8-GPU box for eight
// ranks.  These buffers are allocated with cudaHostAlloc at their exact size
// (portable, so any device's stream can copy from them) and wrapped as CPU
// tensors whose deleter calls cudaFreeHost.  The pool in
// h3_a100/memory/boundary.py allocates them once and reuses them every cycle.
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <atomic>

namespace h3 {

static std::atomic<int64_t> g_pinned_bytes{0};

at::Tensor pinned_empty(int64_t numel, c10::ScalarType dtype) {
  TORCH_CHECK(numel >= 0, "negative size");
  const size_t bytes = static_cast<size_t>(numel) * c10::elementSize(dtype);
  void* ptr = nullptr;
  if (bytes > 0) {
    cudaError_t err = cudaHostAlloc(&ptr, bytes, cudaHostAllocPortable);
    TORCH_CHECK(err == cudaSuccess, "cudaHostAlloc(", bytes, ") failed: ", cudaGetErrorString(err));
    g_pinned_bytes.fetch_add(static_cast<int64_t>(bytes));
  }
  auto deleter = [bytes](void* p) {
    if (p != nullptr) {
      cudaFreeHost(p);
      g_pinned_bytes.fetch_sub(static_cast<int64_t>(bytes));
    }
  };
  return torch::from_blob(ptr, {numel}, deleter, at::TensorOptions().dtype(dtype).device(at::kCPU));
}

int64_t pinned_bytes() { return g_pinned_bytes.load(); }

}  // namespace h3
