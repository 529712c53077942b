// Allocation-free DMD generator loss (see dmd_loss_noalloc.h for the contract).
#include <cstdio>
#include <mutex>

#include "dmd_loss_noalloc.h"

namespace {

constexpr int kMaxDevices = 64;
constexpr int kThreads = 256;
constexpr int kMaxBlocksPerSample = 512;

// [0, samples): per-sample sum |generated - real|; [samples, 2*samples): per-sample sum grad^2.
static __device__ __align__(256) float g_dmd_scratch[2 * H3_DMD_NOALLOC_MAX_SAMPLES];

void* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

__device__ __forceinline__ float block_reduce(float v) {
  __shared__ float part[kThreads / 32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  float total = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < kThreads / 32; ++i) total += part[i];
  return total;
}

__global__ void clear_kernel(float* scratch, int count) {
  for (int i = threadIdx.x; i < count; i += blockDim.x) scratch[i] = 0.f;
}

__global__ void abs_diff_kernel(const float* gen, const float* real, long long per_sample, float* scratch) {
  const long long base = static_cast<long long>(blockIdx.y) * per_sample;
  float s = 0.f;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < per_sample;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    s += fabsf(gen[base + i] - real[base + i]);
  s = block_reduce(s);
  if (threadIdx.x == 0) atomicAdd(scratch + blockIdx.y, s);
}

__global__ void grad_kernel(const float* fake, const float* real, long long per_sample, int samples, float* grad,
                            float* scratch) {
  const long long base = static_cast<long long>(blockIdx.y) * per_sample;
  const float denom = fmaxf(scratch[blockIdx.y] / static_cast<float>(per_sample), 1e-12f);
  float s = 0.f;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < per_sample;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float g = (fake[base + i] - real[base + i]) / denom;
    if (!isfinite(g)) g = 0.f;
    grad[base + i] = g;
    s += g * g;
  }
  s = block_reduce(s);
  if (threadIdx.x == 0) atomicAdd(scratch + samples + blockIdx.y, s);
}

__global__ void finalize_kernel(const float* scratch, int samples, double count, float* loss) {
  if (threadIdx.x == 0) {
    double total = 0.0;
    for (int s = 0; s < samples; ++s) total += scratch[samples + s];
    *loss = static_cast<float>(0.5 * total / count);
  }
}

int fail(int code, const char* what) {
  std::fprintf(stderr, "h3_dmd_loss_noalloc: %s\n", what);
  return code;
}

}  // namespace

extern "C" int h3_dmd_loss_noalloc(const float* generated, const float* x0_fake, const float* x0_real,
                                   long long samples, long long per_sample, float* loss, float* grad,
                                   cudaStream_t stream) {
  if (generated == nullptr || x0_fake == nullptr || x0_real == nullptr || loss == nullptr || grad == nullptr)
    return fail(H3_NOALLOC_EINVAL, "null pointer argument");
  if (samples <= 0 || per_sample <= 0) return fail(H3_NOALLOC_EINVAL, "samples and per_sample must be positive");
  if (samples > H3_DMD_NOALLOC_MAX_SAMPLES)
    return fail(H3_NOALLOC_ETOOBIG, "samples exceeds H3_DMD_NOALLOC_MAX_SAMPLES (1024)");
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return fail(H3_NOALLOC_EDEVICE, "no usable current CUDA device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_addr[device] == nullptr) {
      void* addr = nullptr;
      const cudaError_t err = cudaGetSymbolAddress(&addr, g_dmd_scratch);
      if (err != cudaSuccess || addr == nullptr) return fail(H3_NOALLOC_ESYMBOL, cudaGetErrorString(err));
      g_scratch_addr[device] = addr;
    }
    scratch = g_scratch_addr[device];
  }
  float* acc = static_cast<float*>(scratch);
  const int n = static_cast<int>(samples);
  long long blocks = (per_sample + kThreads - 1) / kThreads;
  if (blocks > kMaxBlocksPerSample) blocks = kMaxBlocksPerSample;
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(n));
  clear_kernel<<<1, kThreads, 0, stream>>>(acc, 2 * n);
  abs_diff_kernel<<<grid, kThreads, 0, stream>>>(generated, x0_real, per_sample, acc);
  grad_kernel<<<grid, kThreads, 0, stream>>>(x0_fake, x0_real, per_sample, n, grad, acc);
  finalize_kernel<<<1, 32, 0, stream>>>(acc, n, static_cast<double>(samples) * static_cast<double>(per_sample), loss);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return fail(H3_NOALLOC_ELAUNCH, cudaGetErrorString(err));
  return H3_NOALLOC_OK;
}
