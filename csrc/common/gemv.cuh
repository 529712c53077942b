// Weight-streaming GEMV helpers for the AdaLN projection: out[r, n] =
// sum_k SiLU(temb[r, k]) * W[n, k].  Memory-bound (the weight is read once):
// a warp works on four rows at a time, so each lane keeps four 16-byte weight
// loads in flight and reads each slice of the embedding from shared memory
// once for all four rows; the loads bypass L1 (every weight byte is used
// exactly once).
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

// One warp: the R dot products of ROWS consecutive weight rows starting at
// `wr` (each K bf16, 16-byte aligned, row stride K) with the SiLU'd embedding
// in smem; every lane returns the full sums.  Each 8-element slice of the
// embedding is read from smem once and used for all ROWS rows.
template <int R, int ROWS>
__device__ __forceinline__ void warp_rows_dot(const __nv_bfloat16* __restrict__ wr, const float* st, int K,
                                              float (&acc)[ROWS][R]) {
#pragma unroll
  for (int q = 0; q < ROWS; ++q)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[q][r] = 0.f;
  const int lane = threadIdx.x & 31;
  constexpr int kStep = 32 * 8;   // elements one warp-wide 16-byte load covers
  for (int k = lane * 8; k < K; k += kStep) {
    uint4 u[ROWS];
#pragma unroll
    for (int q = 0; q < ROWS; ++q) u[q] = ld_stream16(wr + static_cast<long>(q) * K + k);
    float4 a[R][2];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      a[r][0] = *reinterpret_cast<const float4*>(st + r * K + k);
      a[r][1] = *reinterpret_cast<const float4*>(st + r * K + k + 4);
    }
#pragma unroll
    for (int q = 0; q < ROWS; ++q) {
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&u[q]);
      const float2 w01 = __bfloat1622float2(w2[0]), w23 = __bfloat1622float2(w2[1]);
      const float2 w45 = __bfloat1622float2(w2[2]), w67 = __bfloat1622float2(w2[3]);
#pragma unroll
      for (int r = 0; r < R; ++r)
        acc[q][r] += w01.x * a[r][0].x + w01.y * a[r][0].y + w23.x * a[r][0].z + w23.y * a[r][0].w +
                     w45.x * a[r][1].x + w45.y * a[r][1].y + w67.x * a[r][1].z + w67.y * a[r][1].w;
    }
  }
#pragma unroll
  for (int q = 0; q < ROWS; ++q)
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[q][r] += __shfl_xor_sync(0xffffffffu, acc[q][r], o);
}

}  // namespace h3
