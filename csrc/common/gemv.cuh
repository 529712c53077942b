// Weight-streaming GEMV helpers for the AdaLN projection: out[r, n] =
// sum_k SiLU(temb[r, k]) * W[n, k].  Memory-bound (the weight is read once),
// so each lane keeps four 16-byte weight loads in flight and the loads bypass
// L1 (every weight byte is used exactly once).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace h3 {

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// SiLU of the [R, K] bf16 time embedding into shared memory (fp32).
template <int R>
__device__ __forceinline__ void silu_to_smem(const __nv_bfloat16* __restrict__ temb, int K, float* st) {
  for (int i = threadIdx.x; i < R * K; i += blockDim.x) {
    const float v = __bfloat162float(temb[i]);
    st[i] = v / (1.f + __expf(-v));
  }
  __syncthreads();
}

template <int R>
__device__ __forceinline__ void fma8(const uint4& u, const float* st, int K, int k, float (&acc)[R]) {
  const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&u);
  float w[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(w2[j]);
    w[2 * j] = f.x;
    w[2 * j + 1] = f.y;
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float4 a = *reinterpret_cast<const float4*>(st + r * K + k);
    const float4 b = *reinterpret_cast<const float4*>(st + r * K + k + 4);
    acc[r] += w[0] * a.x + w[1] * a.y + w[2] * a.z + w[3] * a.w + w[4] * b.x + w[5] * b.y + w[6] * b.z + w[7] * b.w;
  }
}

// One warp: the R dot products of weight row `wr` (K bf16, 16-byte aligned)
// with the SiLU'd embedding in smem; every lane returns the full sums.
template <int R>
__device__ __forceinline__ void warp_row_dot(const __nv_bfloat16* __restrict__ wr, const float* st, int K,
                                             float (&acc)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  const int lane = threadIdx.x & 31;
  int k = lane * 8;
  constexpr int kStep = 32 * 8;   // elements one warp-wide 16-byte load covers
  for (; k + 3 * kStep < K; k += 4 * kStep) {
    uint4 u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) u[i] = ld_stream16(wr + k + i * kStep);
#pragma unroll
    for (int i = 0; i < 4; ++i) fma8<R>(u[i], st, K, k + i * kStep, acc);
  }
  for (; k < K; k += kStep) fma8<R>(ld_stream16(wr + k), st, K, k, acc);
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
}

}  // namespace h3
