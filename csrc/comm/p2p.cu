// Collectives fused with compute over NVLink peer memory (symmetric buffers).
//
// Every rank passes the device addresses of all ranks' copies of a symmetric
// buffer (peer pointers, mapped through NVLink/NVSwitch).  Kernels read and
// write peers directly; cross-GPU ordering uses epoch flags in a symmetric
// int32 signal buffer: writer `fence.acq_rel.sys` then `st.release.sys` of
// the epoch into the reader's slot, reader `ld.acquire.sys` until it sees the
// epoch.  Every such wait is bounded (status code kStatusTimeoutPeer, then
// the kernel returns); no kernel traps.  Peer memory is only read with
// plain loads here; no TMA load reads another GPU's memory.
//
//   p2p_all_gather_ce    the same on the copy engines (one cudaMemcpyAsync per shard)
//   p2p_all_gather       pull every rank's shard of a (static) buffer into a
//                        local gathered copy; frozen weights need no flags
//   lora_rs_adamw        per LoRA role, one cooperative kernel:
//                          1. wait until every rank's gradients are final
//                          2. reduce-scatter: sum the peers' fp32 grads of this
//                             rank's chunk (NVLink loads), average, sum of squares
//                          3. exchange the sum-of-squares scalars -> global norm
//                          4. clip + AdamW on the chunk (fp32 master/m/v shard)
//                          5. all-gather: store the new bf16 params into every
//                             rank's replica (NVLink stores), then a done barrier
//   adaln_project_gather row-sharded AdaLN projection: each rank computes its
//                        rows of SiLU(temb) W^T + b and stores them straight
//                        into every rank's output buffer, then flags them
//   wait_flag_test       bounded wait on a flag nothing sets (failure tests)
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "../common/gemv.cuh"
#include "../common/ptx.cuh"
#include "../gemm/gemm.h"
#include "p2p.h"

namespace h3 {
namespace {

constexpr int kMaxRanks = 8;

struct PeerPtrs {
  uint64_t p[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(int* addr, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Bounded wait until *flag == epoch (or newer).  Returns false on timeout.
__device__ bool wait_flag(const int* flag, int epoch, uint64_t limit_ns) {
  if (ld_acquire_sys(flag) - epoch >= 0) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t it = 1; it != 0u; ++it) {   // also bounded by the iteration count
    if (ld_acquire_sys(flag) - epoch >= 0) return true;
    if ((it & 255u) == 0u && global_timer_ns() - start > limit_ns) return false;
  }
  return false;
}

// Signal slot layout: flags[slot * kMaxRanks + sender].
__device__ void signal_all(const PeerPtrs& flags, int world, int me, int slot, int epoch) {
  fence_sys();
  for (int r = 0; r < world; ++r)
    st_release_sys(reinterpret_cast<int*>(flags.p[r]) + slot * kMaxRanks + me, epoch);
}

__device__ bool wait_all(const int* my_flags, int world, int slot, int epoch, uint64_t limit_ns) {
  for (int r = 0; r < world; ++r)
    if (!wait_flag(my_flags + slot * kMaxRanks + r, epoch, limit_ns)) return false;
  return true;
}

// Grid-wide barrier for a cooperative launch (all CTAs co-resident), bounded.
// bar[0] = arrival count, bar[1] = generation.
__device__ bool grid_barrier(int* bar, uint64_t limit_ns) {
  __syncthreads();
  bool ok = true;
  if (threadIdx.x == 0) {
    volatile int* gen = bar + 1;
    const int g = *gen;
    __threadfence();
    if (atomicAdd(bar, 1) == static_cast<int>(gridDim.x) - 1) {
      bar[0] = 0;
      __threadfence();
      atomicAdd(bar + 1, 1);
    } else {
      const uint64_t start = global_timer_ns();
      for (uint32_t it = 1; *gen == g; ++it) {
        if (it == 0u || ((it & 255u) == 0u && global_timer_ns() - start > limit_ns)) {
          ok = false;
          break;
        }
      }
    }
    __threadfence();
  }
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = ok;
  __syncthreads();
  return s_ok != 0;
}

// NVLink SHARP (NVLS) through NVSwitch: a load from a multicast address returns
// the element-wise sum over every GPU bound to it; a store is written to all.
__device__ __forceinline__ float4 multimem_ld_add_v4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void multimem_st_v2_bf16x2(__nv_bfloat16* mc, uint32_t a, uint32_t b) {
  asm volatile("multimem.st.relaxed.sys.global.v2.bf16x2 [%0], {%1, %2};" ::"l"(mc), "r"(a), "r"(b) : "memory");
}

__device__ __forceinline__ float block_sum256(float v) {
  __shared__ float part[32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += part[i];
  return t;
}

// ------------------------------------------------------------------ all-gather (pull)
// Each thread keeps kUnroll 16-byte peer loads in flight before storing them
// (NVLink reads need many bytes outstanding to reach link bandwidth).
constexpr int kPullUnroll = 4;
__global__ void all_gather_pull_kernel(PeerPtrs src, int world, long shard_bytes, uint8_t* __restrict__ dst) {
  const long units_per_shard = shard_bytes >> 4;
  const long total = units_per_shard * world;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long base = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; base < total;
       base += stride * kPullUnroll) {
    uint4 v[kPullUnroll];
#pragma unroll
    for (int k = 0; k < kPullUnroll; ++k) {
      const long u = base + k * stride;
      if (u < total) {
        const int owner = static_cast<int>(u / units_per_shard);
        v[k] = reinterpret_cast<const uint4*>(src.p[owner])[u - owner * units_per_shard];
      }
    }
#pragma unroll
    for (int k = 0; k < kPullUnroll; ++k) {
      const long u = base + k * stride;
      if (u < total) reinterpret_cast<uint4*>(dst)[u] = v[k];
    }
  }
}

// ------------------------------------------------------------------ LoRA RS + clip + AdamW + AG
constexpr int kLoraScratchSlots = 16;   // scalar slots before the per-block partials
struct LoraParams {
  PeerPtrs grad;    // fp32 [n_pad] per rank
  PeerPtrs param;   // bf16 [n_pad] per rank (replicated compute copy)
  PeerPtrs flags;   // int32 signal buffers
  const int* my_flags;
  const float* mc_grad;       // multicast (NVLS) address of the gradient buffer, or null
  __nv_bfloat16* mc_param;    // multicast address of the parameter buffer, or null
  float* master;    // fp32 [chunk] (this rank's shard)
  float* m;
  float* v;
  float* scratch;   // [0] local sum of squares, [15] norm, [16 + b] block b's partial sum of squares
  int* bar;         // grid barrier words
  long chunk;
  int world, rank, epoch;
  float lr, b1, b2, eps, wd, bc1, bc2_sqrt, max_norm, inv_world;
  KernelStatus status;
};

__global__ void __launch_bounds__(256) lora_rs_adamw_kernel(LoraParams p) {
  const long lo = static_cast<long>(p.rank) * p.chunk;
  // 1. every rank's gradients are final (each rank signals at kernel start)
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    signal_all(p.flags, p.world, p.rank, 0, p.epoch);
    if (!wait_all(p.my_flags, p.world, 0, p.epoch, p.status.limit_ns)) report_status(p.status, kStatusTimeoutPeer, 0);
  }
  if (!grid_barrier(p.bar, p.status.limit_ns)) {
    if (threadIdx.x == 0) report_status(p.status, kStatusTimeoutPeer, 10);
    return;
  }
  if (p.status.word != nullptr && *reinterpret_cast<volatile int*>(p.status.word) != 0) return;
  // 2. reduce-scatter of this rank's chunk, in place into its own gradient buffer
  float* my_grad = reinterpret_cast<float*>(p.grad.p[p.rank]);
  float ss = 0.f;
  const long n4 = p.chunk >> 2;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  constexpr int kU = 4;   // float4 units in flight per thread
  for (long base = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; base < n4; base += stride * kU) {
    float4 acc[kU];
    if (p.mc_grad != nullptr) {
      // the switch sums the world's copies: one chunk crosses NVLink, not world-1
#pragma unroll
      for (int k = 0; k < kU; ++k)
        acc[k] = base + k * stride < n4 ? multimem_ld_add_v4(p.mc_grad + lo + 4 * (base + k * stride))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
#pragma unroll
      for (int k = 0; k < kU; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r < p.world) {
          const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.grad.p[r]) + lo);
          float4 g[kU];
#pragma unroll
          for (int k = 0; k < kU; ++k)
            g[k] = base + k * stride < n4 ? src[base + k * stride] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int k = 0; k < kU; ++k) {
            acc[k].x += g[k].x;
            acc[k].y += g[k].y;
            acc[k].z += g[k].z;
            acc[k].w += g[k].w;
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      const long i = base + k * stride;
      if (i < n4) {
        float4 a = acc[k];
        a.x *= p.inv_world;
        a.y *= p.inv_world;
        a.z *= p.inv_world;
        a.w *= p.inv_world;
        reinterpret_cast<float4*>(my_grad + lo)[i] = a;
        ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
      }
    }
  }
  // Each block's partial lands in its own slot and block 0 sums the slots in
  // a fixed order (a float atomicAdd would make the norm, and so every
  // parameter, depend on the order in which blocks arrive).
  ss = block_sum256(ss);
  if (threadIdx.x == 0) p.scratch[kLoraScratchSlots + blockIdx.x] = ss;
  if (!grid_barrier(p.bar, p.status.limit_ns)) {
    if (threadIdx.x == 0) report_status(p.status, kStatusTimeoutPeer, 11);
    return;
  }
  if (blockIdx.x == 0) {
    float part = 0.f;
    for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += blockDim.x)
      part += __ldcg(p.scratch + kLoraScratchSlots + b);
    part = block_sum256(part);
    if (threadIdx.x == 0) p.scratch[0] = part;
  }
  // 3. exchange partial sums of squares -> global norm
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const float mine = p.scratch[0];
    for (int r = 0; r < p.world; ++r) {
      float* peer_scratch_slot = reinterpret_cast<float*>(reinterpret_cast<int*>(p.flags.p[r]) + 4 * kMaxRanks) + p.rank;
      *peer_scratch_slot = mine;
    }
    signal_all(p.flags, p.world, p.rank, 1, p.epoch);
    float total = 0.f;
    if (wait_all(p.my_flags, p.world, 1, p.epoch, p.status.limit_ns)) {
      const float* slots = reinterpret_cast<const float*>(p.my_flags + 4 * kMaxRanks);
      for (int r = 0; r < p.world; ++r) total += reinterpret_cast<const volatile float*>(slots)[r];
    } else {
      report_status(p.status, kStatusTimeoutPeer, 1);
    }
    p.scratch[15] = sqrtf(total);
  }
  if (!grid_barrier(p.bar, p.status.limit_ns)) {
    if (threadIdx.x == 0) report_status(p.status, kStatusTimeoutPeer, 12);
    return;
  }
  if (p.status.word != nullptr && *reinterpret_cast<volatile int*>(p.status.word) != 0) return;
  // 4. clip + AdamW on the chunk; 5. store the new bf16 params into every replica
  const float norm = *reinterpret_cast<volatile float*>(p.scratch + 15);
  const float coef = p.max_norm > 0.f ? fminf(1.f, p.max_norm / (norm + 1e-6f)) : 1.f;
  const float step = p.lr / p.bc1, decay = 1.f - p.lr * p.wd;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float4 g4 = reinterpret_cast<const float4*>(my_grad + lo)[i];
    float4 w4 = reinterpret_cast<float4*>(p.master)[i];
    float4 m4 = reinterpret_cast<float4*>(p.m)[i];
    float4 v4 = reinterpret_cast<float4*>(p.v)[i];
    float g[4] = {g4.x * coef, g4.y * coef, g4.z * coef, g4.w * coef};
    float* w = &w4.x;
    float* mm = &m4.x;
    float* vv = &v4.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      mm[k] = p.b1 * mm[k] + (1.f - p.b1) * g[k];
      vv[k] = p.b2 * vv[k] + (1.f - p.b2) * g[k] * g[k];
      w[k] = w[k] * decay - step * mm[k] / (sqrtf(vv[k]) / p.bc2_sqrt + p.eps);
    }
    reinterpret_cast<float4*>(p.master)[i] = w4;
    reinterpret_cast<float4*>(p.m)[i] = m4;
    reinterpret_cast<float4*>(p.v)[i] = v4;
    uint2 packed;
    packed.x = pack_bf16x2(w[0], w[1]);
    packed.y = pack_bf16x2(w[2], w[3]);
    if (p.mc_param != nullptr) {
      multimem_st_v2_bf16x2(p.mc_param + lo + 4 * i, packed.x, packed.y);   // one store reaches every replica
    } else {
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < p.world) reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.param.p[r]) + lo)[i] = packed;
    }
  }
  if (!grid_barrier(p.bar, p.status.limit_ns)) {
    if (threadIdx.x == 0) report_status(p.status, kStatusTimeoutPeer, 13);
    return;
  }
  // done barrier: every replica is complete, and no rank still reads a peer's gradients
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    signal_all(p.flags, p.world, p.rank, 2, p.epoch);
    if (!wait_all(p.my_flags, p.world, 2, p.epoch, p.status.limit_ns)) report_status(p.status, kStatusTimeoutPeer, 2);
  }
}

// ------------------------------------------------------------------ AdaLN GEMV + output all-gather
struct AdalnParams {
  const __nv_bfloat16* temb;  // [R, K]
  const __nv_bfloat16* w;     // [rows, K] this rank's rows
  const __nv_bfloat16* b;     // [rows]
  PeerPtrs out;               // fp32 [R, world*rows] per rank
  PeerPtrs flags;
  const int* my_flags;
  int R, K, rows, world, rank, epoch, slot;
  KernelStatus status;
};

template <int R>
__global__ void adaln_gather_kernel(AdalnParams p) {
  extern __shared__ float st[];
  silu_to_smem<R>(p.temb, p.K, st);
  constexpr int kRows = 4;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int ncols = p.world * p.rows;
  const int groups = (p.rows + kRows - 1) / kRows;
  for (int g = blockIdx.x * warps + (threadIdx.x >> 5); g < groups; g += gridDim.x * warps) {
    const int n0 = g * kRows;
    float acc[kRows][R];
    if (n0 + kRows <= p.rows) {
      warp_rows_dot<R, kRows>(p.w + static_cast<long>(n0) * p.K, st, p.K, acc);
    } else {
      for (int q = 0; q < kRows; ++q) {   // ragged last group: one row at a time
        float one[1][R];
        warp_rows_dot<R, 1>(p.w + static_cast<long>(min(n0 + q, p.rows - 1)) * p.K, st, p.K, one);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[q][r] = one[0][r];
      }
    }
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      const int n = n0 + q;
      if (n >= p.rows) break;
      const float bias = p.b != nullptr ? __bfloat162float(p.b[n]) : 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (lane < p.world)  // lane `peer` stores the value into that rank's output
          reinterpret_cast<float*>(p.out.p[lane])[static_cast<long>(r) * ncols + p.rank * p.rows + n] =
              acc[q][r] + bias;
      }
    }
  }
}

__global__ void adaln_signal_kernel(AdalnParams p) {
  // runs after the GEMV kernel on the same stream: all of this rank's stores are issued
  if (threadIdx.x == 0) {
    signal_all(p.flags, p.world, p.rank, p.slot, p.epoch);
    if (!wait_all(p.my_flags, p.world, p.slot, p.epoch, p.status.limit_ns))
      report_status(p.status, kStatusTimeoutPeer, 3);
  }
}

__global__ void wait_flag_test_kernel(const int* flag, int epoch, KernelStatus st) {
  if (threadIdx.x == 0 && !wait_flag(flag, epoch, st.limit_ns)) report_status(st, kStatusTimeoutPeer, 99);
}

PeerPtrs peers_of(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK(!ptrs.empty() && ptrs.size() <= kMaxRanks, "1..8 peer pointers expected");
  PeerPtrs out{};
  for (size_t i = 0; i < ptrs.size(); ++i) {
    TORCH_CHECK((ptrs[i] & 15) == 0, "peer buffers must be 16-byte aligned");
    out.p[i] = static_cast<uint64_t>(ptrs[i]);
  }
  return out;
}

KernelStatus status_of(const at::Tensor& status, int64_t limit_ns) {
  return KernelStatus{status.data_ptr<int>(), static_cast<uint64_t>(limit_ns)};
}

}  // namespace

// The same all-gather on the copy engines: one cudaMemcpyAsync per owner's
// shard (a peer address mapped into this process), in rank order on the
// current stream.  No SM runs it, so a gather prefetched on a side stream
// leaves every SM to the compute kernels it overlaps.
void p2p_all_gather_ce(const std::vector<int64_t>& shard_ptrs, int64_t shard_bytes, const at::Tensor& out) {
  TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "out must be contiguous CUDA");
  const int world = static_cast<int>(shard_ptrs.size());
  TORCH_CHECK(out.numel() * out.element_size() >= shard_bytes * world, "out too small");
  c10::cuda::CUDAGuard guard(out.get_device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(out.get_device()).stream();
  auto* dst = static_cast<uint8_t*>(out.data_ptr());
  for (int r = 0; r < world; ++r) {
    C10_CUDA_CHECK(cudaMemcpyAsync(dst + static_cast<long>(r) * shard_bytes,
                                   reinterpret_cast<const void*>(shard_ptrs[r]), static_cast<size_t>(shard_bytes),
                                   cudaMemcpyDeviceToDevice, stream));
  }
}

void p2p_all_gather(const std::vector<int64_t>& shard_ptrs, int64_t shard_bytes, const at::Tensor& out) {
  TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "out must be contiguous CUDA");
  TORCH_CHECK(shard_bytes % 16 == 0, "shard size must be a multiple of 16 bytes");
  const int world = static_cast<int>(shard_ptrs.size());
  TORCH_CHECK(out.numel() * out.element_size() >= shard_bytes * world, "out too small");
  c10::cuda::CUDAGuard guard(out.get_device());
  const long units = shard_bytes / 16 * world;
  const int grid = static_cast<int>(std::min<long>((units + 255) / 256, 148L * 8));
  all_gather_pull_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream(out.get_device()).stream()>>>(
      peers_of(shard_ptrs), world, shard_bytes, reinterpret_cast<uint8_t*>(out.data_ptr()));
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lora_rs_adamw(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& param_ptrs,
                   const std::vector<int64_t>& flag_ptrs, int64_t rank, int64_t epoch, const at::Tensor& master,
                   const at::Tensor& m, const at::Tensor& v, const at::Tensor& scratch, const at::Tensor& bar,
                   double lr, double b1, double b2, double eps, double wd, int64_t step, double max_norm,
                   const at::Tensor& status, int64_t limit_ns, int64_t mc_grad, int64_t mc_param) {
  const int world = static_cast<int>(grad_ptrs.size());
  TORCH_CHECK(param_ptrs.size() == grad_ptrs.size() && flag_ptrs.size() == grad_ptrs.size(), "peer lists");
  TORCH_CHECK(master.scalar_type() == at::kFloat && m.sizes() == master.sizes() && v.sizes() == master.sizes(),
              "optimizer shard");
  TORCH_CHECK(master.numel() % 4 == 0, "chunk must be a multiple of 4 elements");
  const int device = master.get_device();
  c10::cuda::CUDAGuard guard(device);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(device).stream();
  LoraParams p{};
  p.grad = peers_of(grad_ptrs);
  p.param = peers_of(param_ptrs);
  p.flags = peers_of(flag_ptrs);
  p.my_flags = reinterpret_cast<const int*>(flag_ptrs[rank]);
  TORCH_CHECK(mc_grad % 16 == 0 && mc_param % 16 == 0, "multicast addresses must be 16-byte aligned");
  p.mc_grad = reinterpret_cast<const float*>(mc_grad);
  p.mc_param = reinterpret_cast<__nv_bfloat16*>(mc_param);
  p.master = master.data_ptr<float>();
  p.m = m.data_ptr<float>();
  p.v = v.data_ptr<float>();
  TORCH_CHECK(scratch.scalar_type() == at::kFloat && scratch.is_contiguous(), "scratch must be contiguous fp32");
  p.scratch = scratch.data_ptr<float>();
  p.bar = bar.data_ptr<int>();
  p.chunk = master.numel();
  p.world = world;
  p.rank = static_cast<int>(rank);
  p.epoch = static_cast<int>(epoch);
  p.lr = static_cast<float>(lr);
  p.b1 = static_cast<float>(b1);
  p.b2 = static_cast<float>(b2);
  p.eps = static_cast<float>(eps);
  p.wd = static_cast<float>(wd);
  p.bc1 = static_cast<float>(1.0 - std::pow(b1, static_cast<double>(step)));
  p.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(b2, static_cast<double>(step))));
  p.max_norm = static_cast<float>(max_norm);
  p.inv_world = 1.f / static_cast<float>(world);
  p.status = status_of(status, limit_ns);
  cudaMemsetAsync(p.scratch, 0, sizeof(float), stream);
  static int grid_for_device[64] = {0};
  if (grid_for_device[device] == 0) {
    int per_sm = 0, sms = 0;
    C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lora_rs_adamw_kernel, 256, 0));
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    grid_for_device[device] = std::max(1, std::min(per_sm, 4)) * sms;
  }
  const int grid = grid_for_device[device];
  TORCH_CHECK(scratch.numel() >= kLoraScratchSlots + grid, "scratch needs ", kLoraScratchSlots + grid,
              " floats (16 scalar slots + one partial per block)");
  void* args[] = {&p};
  const cudaError_t err = cudaLaunchCooperativeKernel(reinterpret_cast<void*>(lora_rs_adamw_kernel), grid, 256,
                                                      args, 0, stream);
  TORCH_CHECK(err == cudaSuccess, "cooperative launch failed: ", cudaGetErrorString(err));
  note_launch();
}

void adaln_project_gather(const at::Tensor& temb, const at::Tensor& w, const c10::optional<at::Tensor>& b,
                          const std::vector<int64_t>& out_ptrs, const std::vector<int64_t>& flag_ptrs, int64_t rank,
                          int64_t epoch, int64_t slot, const at::Tensor& status, int64_t limit_ns) {
  TORCH_CHECK(temb.scalar_type() == at::kBFloat16 && temb.is_contiguous() && w.is_contiguous(), "operands");
  const int R = static_cast<int>(temb.size(0)), K = static_cast<int>(temb.size(1));
  TORCH_CHECK(R >= 1 && R <= 2 && K % 8 == 0 && w.size(1) == K, "adaln_project_gather shapes");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(w.data_ptr()) & 15u) == 0, "weight rows must be 16-byte aligned");
  TORCH_CHECK(slot >= 3 && slot < 4, "signal slot 3 is reserved for the AdaLN gather");
  const int device = w.get_device();
  c10::cuda::CUDAGuard guard(device);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(device).stream();
  AdalnParams p{};
  p.temb = reinterpret_cast<const __nv_bfloat16*>(temb.data_ptr());
  p.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  p.b = b.has_value() ? reinterpret_cast<const __nv_bfloat16*>(b->data_ptr()) : nullptr;
  p.out = peers_of(out_ptrs);
  p.flags = peers_of(flag_ptrs);
  p.my_flags = reinterpret_cast<const int*>(flag_ptrs[rank]);
  p.R = R;
  p.K = K;
  p.rows = static_cast<int>(w.size(0));
  p.world = static_cast<int>(out_ptrs.size());
  p.rank = static_cast<int>(rank);
  p.epoch = static_cast<int>(epoch);
  p.slot = static_cast<int>(slot);
  p.status = status_of(status, limit_ns);
  const size_t smem = static_cast<size_t>(R) * K * sizeof(float);
  auto go = [&](auto kernel) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int per_sm = 1;   // persistent grid: as many blocks as fit at once
    C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, smem));
    const int grid = std::max(1, std::min((p.rows + 31) / 32, std::max(1, per_sm) * 148));
    kernel<<<grid, 256, smem, stream>>>(p);
  };
  if (R == 1) {
    go(adaln_gather_kernel<1>);
  } else {
    go(adaln_gather_kernel<2>);
  }
  adaln_signal_kernel<<<1, 32, 0, stream>>>(p);
  note_launch();
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// The wait runs on the device that holds `status`; `flag` may live on a peer
// GPU (read with plain peer loads once peer access is enabled).
void wait_flag_test(const at::Tensor& flag, int64_t epoch, const at::Tensor& status, int64_t limit_ns) {
  TORCH_CHECK(flag.is_cuda() && status.is_cuda() && flag.scalar_type() == at::kInt && status.numel() >= 4,
              "wait_flag_test operands");
  c10::cuda::CUDAGuard guard(status.get_device());
  wait_flag_test_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream(status.get_device()).stream()>>>(
      flag.data_ptr<int>(), static_cast<int>(epoch), status_of(status, limit_ns));
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Lets kernels on `device` load from `peer`'s memory directly (idempotent).
void enable_peer_access(int64_t device, int64_t peer) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  int can = 0;
  C10_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, static_cast<int>(device), static_cast<int>(peer)));
  TORCH_CHECK(can, "device ", device, " cannot access device ", peer, " directly");
  const cudaError_t err = cudaDeviceEnablePeerAccess(static_cast<int>(peer), 0);
  if (err == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    return;
  }
  C10_CUDA_CHECK(err);
}

}  // namespace h3
