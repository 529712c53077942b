// Bandwidth-bound kernels of the DiT block, the DMD math and the optimizer.
//
// * norm_modulate_fwd : y = rmsnorm(x) * (1 + scale[row]) + shift[row]   (bf16 out)
// * norm_modulate_bwd : dx = add + rmsnorm'(x)^T (dy * (1 + scale[row])), optionally
//                       also gated = gate[row] * dx (the next residual branch's gradient)
// * gate_mul          : out = gate[row] * g
// * rope_inverse      : rotate q/k sections of dqkv back by -theta (in place)
// * adaln_project     : [R, N] = SiLU(temb) @ W^T + b, fp32 out (GEMV, R <= 4)
// * flow / DMD passes : x0 = xt + s*v and the Euler step in one pass, renoise,
//                       DMD direction + loss partial sums, MSE partial sums
// * sum_squares, adamw: global-norm partials and the fused clip + AdamW update
//
// A "row" of a modulation table is chosen per token: tokens < split use row 0.
// One CTA handles one token row for the row-wise kernels; everything else is
// a grid-stride loop with 16-byte vector accesses where alignment allows.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/gemv.cuh"
#include "../common/ptx.cuh"
#include "../gemm/gemm.h"
#include "elementwise.h"

namespace h3 {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float total = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) total += scratch[i];
  return total;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(b[j]);
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

__global__ void norm_modulate_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ shift,
                                         const float* __restrict__ scale, long ld_mod, int split, int H, float eps,
                                         __nv_bfloat16* __restrict__ y) {
  __shared__ float scratch[32];
  const long row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  const int nvec = H >> 3;
  float ss = 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    load8(xr + i * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  }
  const float r = rsqrtf(block_sum(ss, scratch) / H + eps);
  const long mrow = (row >= split) ? ld_mod : 0;
  const float* sh = shift + mrow;
  const float* sc = scale + mrow;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    load8(xr + i * 8, v);
    const float4 s0 = *reinterpret_cast<const float4*>(sh + i * 8);
    const float4 s1 = *reinterpret_cast<const float4*>(sh + i * 8 + 4);
    const float4 c0 = *reinterpret_cast<const float4*>(sc + i * 8);
    const float4 c1 = *reinterpret_cast<const float4*>(sc + i * 8 + 4);
    const float shv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const float scv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = v[j] * r * (1.f + scv[j]) + shv[j];
    store8(y + row * H + i * 8, v);
  }
}

__global__ void norm_modulate_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                                         const float* __restrict__ scale, long ld_mod, int split, int H, float eps,
                                         const __nv_bfloat16* __restrict__ add, const float* __restrict__ gate,
                                         long ld_gate, __nv_bfloat16* __restrict__ dx,
                                         __nv_bfloat16* __restrict__ gated) {
  __shared__ float scratch[32];
  const long row = blockIdx.x;
  const int nvec = H >> 3;
  const __nv_bfloat16* xr = x + row * H;
  const __nv_bfloat16* gr = dy + row * H;
  const float* sc = scale + ((row >= split) ? ld_mod : 0);
  float ss = 0.f, gx = 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float xv[8], gv[8];
    load8(xr + i * 8, xv);
    load8(gr + i * 8, gv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g = gv[j] * (1.f + sc[i * 8 + j]);
      ss += xv[j] * xv[j];
      gx += g * xv[j];
    }
  }
  const float sum_sq = block_sum(ss, scratch);
  const float sum_gx = block_sum(gx, scratch);
  const float r = rsqrtf(sum_sq / H + eps);
  // dx = r * (g - n * mean(g*n)), n = x*r  =>  dx = r*g - x * r^3 * mean(g*x)
  const float coef = r * r * r * (sum_gx / H);
  const float* gt = gate != nullptr ? gate + ((row >= split) ? ld_gate : 0) : nullptr;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float xv[8], gv[8], out[8];
    load8(xr + i * 8, xv);
    load8(gr + i * 8, gv);
    float av[8];
    if (add != nullptr) {
      load8(add + row * H + i * 8, av);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) av[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = av[j] + r * gv[j] * (1.f + sc[i * 8 + j]) - xv[j] * coef;
    store8(dx + row * H + i * 8, out);
    if (gt != nullptr) {
      float gd[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) gd[j] = gt[i * 8 + j] * bf16_round(out[j]);
      store8(gated + row * H + i * 8, gd);
    }
  }
}

__global__ void gate_mul_kernel(const __nv_bfloat16* __restrict__ g, const float* __restrict__ gate, long ld_gate,
                                int split, int H, long rows, __nv_bfloat16* __restrict__ out) {
  const long nvec_row = H >> 3;
  const long total = rows * nvec_row;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / nvec_row;
    const int c = static_cast<int>(i % nvec_row) * 8;
    const float* gt = gate + ((row >= split) ? ld_gate : 0) + c;
    float v[8];
    load8(g + row * H + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= gt[j];
    store8(out + row * H + c, v);
  }
}

// Inverse rotation of interleaved pairs in columns [0, rope_cols) of a [T, ld] bf16 matrix.
__global__ void rope_inverse_kernel(__nv_bfloat16* __restrict__ t, long ld, long rows, int rope_cols, int head_dim,
                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t) {
  const int half = head_dim >> 1;
  const long pairs_row = rope_cols >> 1;
  const long total = rows * pairs_row;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / pairs_row;
    const int pr = static_cast<int>(i % pairs_row);
    const int col = pr * 2;
    const int pi = (col % head_dim) >> 1;
    const float c = cos_t[row * half + pi], s = sin_t[row * half + pi];
    __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(t + row * ld + col);
    const float2 v = __bfloat1622float2(*p);
    *p = __floats2bfloat162_rn(v.x * c + v.y * s, -v.x * s + v.y * c);
  }
}

// out[r, n] = sum_k silu(temb[r, k]) * W[n, k] + b[n]; one warp per output
// column n at a time, persistent grid (rows strided over all warps).
template <int R>
__global__ void adaln_project_kernel(const __nv_bfloat16* __restrict__ temb, const __nv_bfloat16* __restrict__ w,
                                     const __nv_bfloat16* __restrict__ b, int N, int K, float* __restrict__ out) {
  extern __shared__ float st[];  // [R, K] silu(temb)
  silu_to_smem<R>(temb, K, st);
  constexpr int kRows = 4;
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int groups = (N + kRows - 1) / kRows;
  for (int g = blockIdx.x * warps + (threadIdx.x >> 5); g < groups; g += gridDim.x * warps) {
    const int n0 = g * kRows;
    float acc[kRows][R];
    if (n0 + kRows <= N) {
      warp_rows_dot<R, kRows>(w + static_cast<long>(n0) * K, st, K, acc);
    } else {
      for (int q = 0; q < kRows; ++q) {   // ragged last group: one row at a time
        float one[1][R];
        warp_rows_dot<R, 1>(w + static_cast<long>(min(n0 + q, N - 1)) * K, st, K, one);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[q][r] = one[0][r];
      }
    }
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      const int n = n0 + q;
      if (n < N && lane < R) {
        float v = acc[q][0];
#pragma unroll
        for (int r = 1; r < R; ++r) v = lane == r ? acc[q][r] : v;
        out[static_cast<long>(lane) * N + n] = v + (b != nullptr ? __bfloat162float(b[n]) : 0.f);
      }
    }
  }
}

// ------------------------------------------------------------------ flow / DMD
template <typename T>
__device__ __forceinline__ float ld_any(const T* p, long i) {
  if constexpr (std::is_same_v<T, float>) return p[i];
  else return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ void st_any(T* p, long i, float v) {
  if constexpr (std::is_same_v<T, float>) p[i] = v;
  else p[i] = __float2bfloat16(v);
}

// x0 = xt + s*v (fp32) and xt' = xt + (s - s_next)*v (dtype of xt') in one pass.
template <typename TX, typename TV, typename TO>
__global__ void flow_step_kernel(const TX* __restrict__ xt, const TV* __restrict__ v, long n, float s, float s_next,
                                 float* __restrict__ x0, TO* __restrict__ xnext) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float a = ld_any(xt, i), b = ld_any(v, i);
    if (x0 != nullptr) x0[i] = a + s * b;
    if (xnext != nullptr) st_any(xnext, i, a + (s - s_next) * b);
  }
}

// out = (1 - s) * x0 + s * noise
template <typename TX, typename TO>
__global__ void add_noise_kernel(const TX* __restrict__ x0, const float* __restrict__ noise, long n, float s,
                                 TO* __restrict__ out) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    st_any(out, i, (1.f - s) * ld_any(x0, i) + s * noise[i]);
}

// partial sums: acc[0] += sum |g - real|
template <typename TG>
__global__ void abs_diff_sum_kernel(const TG* __restrict__ g, const float* __restrict__ real, long n,
                                    float* __restrict__ acc) {
  __shared__ float scratch[32];
  float s = 0.f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    s += fabsf(ld_any(g, i) - real[i]);
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) atomicAdd(acc, s);
}

// grad = (fake - real) / max(norm_sum / n, 1e-12) (non-finite -> 0); acc[0] += sum grad^2
__global__ void dmd_grad_kernel(const float* __restrict__ fake, const float* __restrict__ real, long n,
                                const float* __restrict__ norm_sum, float* __restrict__ grad, float* __restrict__ acc) {
  __shared__ float scratch[32];
  const float denom = fmaxf(norm_sum[0] / static_cast<float>(n), 1e-12f);
  float s = 0.f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float gv = (fake[i] - real[i]) / denom;
    if (!isfinite(gv)) gv = 0.f;
    grad[i] = gv;
    s += gv * gv;
  }
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) atomicAdd(acc, s);
}

// acc[0] += sum (p - t)^2
template <typename TP, typename TT>
__global__ void sq_diff_sum_kernel(const TP* __restrict__ p, const TT* __restrict__ t, long n,
                                   float* __restrict__ acc) {
  __shared__ float scratch[32];
  float s = 0.f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float d = ld_any(p, i) - ld_any(t, i);
    s += d * d;
  }
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) atomicAdd(acc, s);
}

// out = scale_ptr[0] * coef * (p - t)   (MSE backward), dtype of p
template <typename TP, typename TT>
__global__ void scaled_diff_kernel(const TP* __restrict__ p, const TT* __restrict__ t, long n, float coef,
                                   const float* __restrict__ upstream, TP* __restrict__ out) {
  const float u = upstream[0] * coef;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    st_any(out, i, u * (ld_any(p, i) - ld_any(t, i)));
}

// out = upstream * coef * grad
template <typename TO>
__global__ void scale_copy_kernel(const float* __restrict__ g, long n, float coef, const float* __restrict__ upstream,
                                  TO* __restrict__ out) {
  const float u = upstream[0] * coef;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    st_any(out, i, u * g[i]);
}

// ------------------------------------------------------------------ optimizer
__global__ void sum_squares_kernel(const float* __restrict__ x, long n, float* __restrict__ acc) {
  __shared__ float scratch[32];
  float s = 0.f;
  const long n4 = n >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const float4 v = x4[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long i = n4 * 4 + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    s += x[i] * x[i];
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) atomicAdd(acc, s);
}

// Clip by the device-side global norm, then decoupled-weight-decay AdamW on fp32
// master weights; writes the bf16 compute copy.  `norm` is sqrt(sum g^2).
__global__ void adamw_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                             const float* __restrict__ grad, __nv_bfloat16* __restrict__ param, long n, long n_param,
                             const float* __restrict__ norm, float lr, float b1, float b2, float eps, float wd,
                             float bc1, float bc2_sqrt, float max_norm) {
  float coef = 1.f;
  if (max_norm > 0.f) coef = fminf(1.f, max_norm / (norm[0] + 1e-6f));
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float g = grad[i] * coef;
    const float mi = b1 * m[i] + (1.f - b1) * g;
    const float vi = b2 * v[i] + (1.f - b2) * g * g;
    m[i] = mi;
    v[i] = vi;
    const float w = master[i] * decay - step * mi / (sqrtf(vi) / bc2_sqrt + eps);
    master[i] = w;
    if (i < n_param) param[i] = __float2bfloat16(w);
  }
}

int grid_for(long n, int threads = 256) {
  long blocks = (n + threads - 1) / threads;
  return static_cast<int>(std::max<long>(1, std::min<long>(blocks, 148L * 16)));
}

cudaStream_t cur_stream(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

void check_bf16_rows(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.is_contiguous(), what,
              " must be a contiguous 2-D CUDA bf16 tensor");
  TORCH_CHECK(t.size(1) % 8 == 0, what, ": row length must be a multiple of 8");
}

void check_table(const at::Tensor& t, int64_t H, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.dim() == 2 && t.stride(1) == 1 && t.size(1) == H,
              what, " must be an fp32 [R, H] table with unit column stride");
  TORCH_CHECK(t.size(0) == 1 || t.size(0) == 2, what, " must have 1 or 2 rows");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && (t.stride(0) * 4) % 16 == 0, what,
              " rows must be 16-byte aligned");
}

}  // namespace

at::Tensor norm_modulate_fwd(const at::Tensor& x, const at::Tensor& shift, const at::Tensor& scale, int64_t split,
                             double eps) {
  check_bf16_rows(x, "x");
  const int64_t H = x.size(1);
  check_table(shift, H, "shift");
  check_table(scale, H, "scale");
  TORCH_CHECK(shift.stride(0) == scale.stride(0), "shift/scale must share a row stride");
  c10::cuda::CUDAGuard g(x.get_device());
  auto y = at::empty_like(x);
  const long ld = shift.size(0) > 1 ? shift.stride(0) : 0;
  if (x.size(0) > 0) {
    norm_modulate_fwd_kernel<<<x.size(0), kRowThreads, 0, cur_stream(x)>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), shift.data_ptr<float>(), scale.data_ptr<float>(), ld,
        static_cast<int>(split), static_cast<int>(H), static_cast<float>(eps),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
    note_launch();
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return y;
}

std::vector<at::Tensor> norm_modulate_bwd(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& scale,
                                          int64_t split, double eps, const c10::optional<at::Tensor>& add,
                                          const c10::optional<at::Tensor>& gate) {
  check_bf16_rows(x, "x");
  check_bf16_rows(dy, "dy");
  const int64_t H = x.size(1);
  check_table(scale, H, "scale");
  if (add.has_value()) check_bf16_rows(*add, "add");
  if (gate.has_value()) check_table(*gate, H, "gate");
  c10::cuda::CUDAGuard g(x.get_device());
  auto dx = at::empty_like(x);
  at::Tensor gated;
  if (gate.has_value()) gated = at::empty_like(x);
  if (x.size(0) > 0) {
    norm_modulate_bwd_kernel<<<x.size(0), kRowThreads, 0, cur_stream(x)>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
        scale.data_ptr<float>(), scale.size(0) > 1 ? scale.stride(0) : 0, static_cast<int>(split),
        static_cast<int>(H), static_cast<float>(eps),
        add.has_value() ? reinterpret_cast<const __nv_bfloat16*>(add->data_ptr()) : nullptr,
        gate.has_value() ? gate->data_ptr<float>() : nullptr,
        gate.has_value() && gate->size(0) > 1 ? gate->stride(0) : 0, reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()),
        gate.has_value() ? reinterpret_cast<__nv_bfloat16*>(gated.data_ptr()) : nullptr);
    note_launch();
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (gate.has_value()) return {dx, gated};
  return {dx};
}

at::Tensor gate_mul(const at::Tensor& g, const at::Tensor& gate, int64_t split) {
  check_bf16_rows(g, "g");
  check_table(gate, g.size(1), "gate");
  c10::cuda::CUDAGuard guard(g.get_device());
  auto out = at::empty_like(g);
  const long total = g.size(0) * (g.size(1) / 8);
  if (total > 0) {
    gate_mul_kernel<<<grid_for(total), 256, 0, cur_stream(g)>>>(
        reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), gate.data_ptr<float>(),
        gate.size(0) > 1 ? gate.stride(0) : 0, static_cast<int>(split), static_cast<int>(g.size(1)), g.size(0),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
    note_launch();
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return out;
}

void rope_inverse_(const at::Tensor& t, const at::Tensor& cos_t, const at::Tensor& sin_t, int64_t rope_cols,
                   int64_t head_dim) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1, "dqkv layout");
  TORCH_CHECK(cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.size(0) == t.size(0), "rope tables");
  TORCH_CHECK(rope_cols % 2 == 0 && head_dim % 2 == 0, "rope sizes");
  c10::cuda::CUDAGuard guard(t.get_device());
  const long total = t.size(0) * (rope_cols / 2);
  if (total > 0) {
    rope_inverse_kernel<<<grid_for(total), 256, 0, cur_stream(t)>>>(
        reinterpret_cast<__nv_bfloat16*>(t.data_ptr()), t.stride(0), t.size(0), static_cast<int>(rope_cols),
        static_cast<int>(head_dim), cos_t.data_ptr<float>(), sin_t.data_ptr<float>());
    note_launch();
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

at::Tensor adaln_project(const at::Tensor& temb, const at::Tensor& w, const c10::optional<at::Tensor>& b) {
  TORCH_CHECK(temb.is_cuda() && temb.scalar_type() == at::kBFloat16 && temb.is_contiguous() && temb.dim() == 2,
              "temb must be contiguous bf16 [R, K]");
  check_bf16_rows(w, "w");
  const int R = static_cast<int>(temb.size(0));
  const int K = static_cast<int>(temb.size(1));
  TORCH_CHECK(w.size(1) == K && K % 8 == 0, "w must be [N, K]");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(w.data_ptr()) & 15u) == 0 && w.stride(0) == K,
              "w rows must be contiguous and 16-byte aligned");
  TORCH_CHECK(R >= 1 && R <= 4, "adaln_project supports 1..4 timestep rows");
  c10::cuda::CUDAGuard guard(w.get_device());
  const int N = static_cast<int>(w.size(0));
  auto out = at::empty({R, N}, temb.options().dtype(at::kFloat));
  const size_t smem = static_cast<size_t>(R) * K * sizeof(float);
  const int threads = 256, warps = threads / 32;
  const __nv_bfloat16* bp = b.has_value() ? reinterpret_cast<const __nv_bfloat16*>(b->data_ptr()) : nullptr;
  auto go = [&](auto kernel) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    // persistent: as many blocks as fit on the SMs at once (shared memory bounds it)
    int per_sm = 1;
    C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem));
    const int grid = std::max(1, std::min((N + 4 * warps - 1) / (4 * warps), std::max(1, per_sm) * 148));
    kernel<<<grid, threads, smem, cur_stream(w)>>>(reinterpret_cast<const __nv_bfloat16*>(temb.data_ptr()),
                                                   reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), bp, N, K,
                                                   out.data_ptr<float>());
  };
  switch (R) {
    case 1: go(adaln_project_kernel<1>); break;
    case 2: go(adaln_project_kernel<2>); break;
    case 3: go(adaln_project_kernel<3>); break;
    default: go(adaln_project_kernel<4>); break;
  }
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// ---------------------------------------------------------------- DMD / flow
#define H3_DISPATCH_FB(t, NAME, ...)                                            \
  if ((t).scalar_type() == at::kFloat) {                                        \
    using NAME = float;                                                         \
    __VA_ARGS__                                                                 \
  } else {                                                                      \
    TORCH_CHECK((t).scalar_type() == at::kBFloat16, "expected fp32 or bf16");   \
    using NAME = __nv_bfloat16;                                                 \
    __VA_ARGS__                                                                 \
  }

std::vector<at::Tensor> flow_step(const at::Tensor& xt, const at::Tensor& v, double s, double s_next,
                                  bool want_x0, bool want_next, c10::ScalarType next_dtype) {
  TORCH_CHECK(xt.is_contiguous() && v.is_contiguous() && xt.numel() == v.numel(), "flow_step operands");
  c10::cuda::CUDAGuard guard(xt.get_device());
  at::Tensor x0 = want_x0 ? at::empty(xt.sizes(), xt.options().dtype(at::kFloat)) : at::Tensor();
  at::Tensor nxt = want_next ? at::empty(xt.sizes(), xt.options().dtype(next_dtype)) : at::Tensor();
  const long n = xt.numel();
  H3_DISPATCH_FB(xt, TX, H3_DISPATCH_FB(v, TV, {
    auto launch = [&](auto* out_ptr) {
      using TO = std::remove_pointer_t<decltype(out_ptr)>;
      flow_step_kernel<TX, TV, TO><<<grid_for(n), 256, 0, cur_stream(xt)>>>(
          reinterpret_cast<const TX*>(xt.data_ptr()), reinterpret_cast<const TV*>(v.data_ptr()), n,
          static_cast<float>(s), static_cast<float>(s_next), want_x0 ? x0.data_ptr<float>() : nullptr, out_ptr);
    };
    if (!want_next || next_dtype == at::kFloat) launch(want_next ? nxt.data_ptr<float>() : (float*)nullptr);
    else launch(reinterpret_cast<__nv_bfloat16*>(nxt.data_ptr()));
  }))
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {x0, nxt};
}

at::Tensor add_noise(const at::Tensor& x0, const at::Tensor& noise, double s) {
  TORCH_CHECK(x0.is_contiguous() && noise.is_contiguous() && noise.scalar_type() == at::kFloat &&
                  x0.numel() == noise.numel(), "add_noise operands");
  c10::cuda::CUDAGuard guard(x0.get_device());
  auto out = at::empty_like(x0);
  const long n = x0.numel();
  H3_DISPATCH_FB(x0, TX, {
    add_noise_kernel<TX, TX><<<grid_for(n), 256, 0, cur_stream(x0)>>>(
        reinterpret_cast<const TX*>(x0.data_ptr()), noise.data_ptr<float>(), n, static_cast<float>(s),
        reinterpret_cast<TX*>(out.data_ptr()));
  })
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Returns (loss [1] fp32, grad fp32 like generated).  grad = DMD direction; the
// loss is 0.5 * mean(grad^2), its gradient w.r.t. generated is grad / n.
std::vector<at::Tensor> dmd_forward(const at::Tensor& generated, const at::Tensor& x0_fake, const at::Tensor& x0_real) {
  TORCH_CHECK(x0_fake.scalar_type() == at::kFloat && x0_real.scalar_type() == at::kFloat, "x0 tensors must be fp32");
  TORCH_CHECK(generated.is_contiguous() && x0_fake.is_contiguous() && x0_real.is_contiguous(), "dmd operands");
  TORCH_CHECK(generated.size(0) == 1, "dmd_forward expects batch 1 per rank");
  c10::cuda::CUDAGuard guard(generated.get_device());
  const long n = generated.numel();
  auto acc = at::zeros({2}, generated.options().dtype(at::kFloat));
  auto grad = at::empty(generated.sizes(), generated.options().dtype(at::kFloat));
  H3_DISPATCH_FB(generated, TG, {
    abs_diff_sum_kernel<TG><<<grid_for(n), 256, 0, cur_stream(generated)>>>(
        reinterpret_cast<const TG*>(generated.data_ptr()), x0_real.data_ptr<float>(), n, acc.data_ptr<float>());
  })
  dmd_grad_kernel<<<grid_for(n), 256, 0, cur_stream(generated)>>>(x0_fake.data_ptr<float>(), x0_real.data_ptr<float>(),
                                                                   n, acc.data_ptr<float>(), grad.data_ptr<float>(),
                                                                   acc.data_ptr<float>() + 1);
  note_launch();
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  auto loss = acc.narrow(0, 1, 1).mul(0.5 / static_cast<double>(n));
  return {loss, grad};
}

at::Tensor scale_copy(const at::Tensor& g, double coef, const at::Tensor& upstream, c10::ScalarType out_dtype) {
  c10::cuda::CUDAGuard guard(g.get_device());
  auto out = at::empty(g.sizes(), g.options().dtype(out_dtype));
  const long n = g.numel();
  if (out_dtype == at::kFloat)
    scale_copy_kernel<float><<<grid_for(n), 256, 0, cur_stream(g)>>>(g.data_ptr<float>(), n, static_cast<float>(coef),
                                                                      upstream.data_ptr<float>(), out.data_ptr<float>());
  else
    scale_copy_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, cur_stream(g)>>>(
        g.data_ptr<float>(), n, static_cast<float>(coef), upstream.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

at::Tensor mse_forward(const at::Tensor& pred, const at::Tensor& target) {
  TORCH_CHECK(pred.is_contiguous() && target.is_contiguous() && pred.numel() == target.numel(), "mse operands");
  c10::cuda::CUDAGuard guard(pred.get_device());
  const long n = pred.numel();
  auto acc = at::zeros({1}, pred.options().dtype(at::kFloat));
  H3_DISPATCH_FB(pred, TP, H3_DISPATCH_FB(target, TT, {
    sq_diff_sum_kernel<TP, TT><<<grid_for(n), 256, 0, cur_stream(pred)>>>(
        reinterpret_cast<const TP*>(pred.data_ptr()), reinterpret_cast<const TT*>(target.data_ptr()), n,
        acc.data_ptr<float>());
  }))
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return acc.div_(static_cast<double>(n));
}

at::Tensor mse_backward(const at::Tensor& pred, const at::Tensor& target, const at::Tensor& upstream) {
  c10::cuda::CUDAGuard guard(pred.get_device());
  const long n = pred.numel();
  auto out = at::empty_like(pred);
  H3_DISPATCH_FB(pred, TP, H3_DISPATCH_FB(target, TT, {
    scaled_diff_kernel<TP, TT><<<grid_for(n), 256, 0, cur_stream(pred)>>>(
        reinterpret_cast<const TP*>(pred.data_ptr()), reinterpret_cast<const TT*>(target.data_ptr()), n,
        2.f / static_cast<float>(n), upstream.data_ptr<float>(), reinterpret_cast<TP*>(out.data_ptr()));
  }))
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// ---------------------------------------------------------------- optimizer
at::Tensor sum_squares(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous(), "sum_squares needs contiguous fp32");
  c10::cuda::CUDAGuard guard(x.get_device());
  auto acc = at::zeros({1}, x.options());
  const long n = x.numel();
  if (n > 0) {
    sum_squares_kernel<<<grid_for(n / 4 + 1), 256, 0, cur_stream(x)>>>(x.data_ptr<float>(), n, acc.data_ptr<float>());
    note_launch();
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return acc;
}

void adamw_step(const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, const at::Tensor& grad,
                const at::Tensor& param, const at::Tensor& norm, double lr, double b1, double b2, double eps,
                double wd, int64_t step, double max_norm) {
  for (const auto* t : {&master, &m, &v, &grad}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous(), "adamw fp32 state");
  }
  TORCH_CHECK(param.scalar_type() == at::kBFloat16 && param.is_contiguous(), "adamw param must be bf16");
  TORCH_CHECK(grad.numel() >= master.numel() && param.numel() <= master.numel(), "adamw sizes");
  c10::cuda::CUDAGuard guard(master.get_device());
  const long n = master.numel();
  const double bc1 = 1.0 - std::pow(b1, static_cast<double>(step));
  const double bc2 = 1.0 - std::pow(b2, static_cast<double>(step));
  adamw_kernel<<<grid_for(n), 256, 0, cur_stream(master)>>>(
      master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), grad.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(param.data_ptr()), n, param.numel(), norm.data_ptr<float>(),
      static_cast<float>(lr), static_cast<float>(b1), static_cast<float>(b2), static_cast<float>(eps),
      static_cast<float>(wd), static_cast<float>(bc1), static_cast<float>(std::sqrt(bc2)),
      static_cast<float>(max_norm));
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace h3
