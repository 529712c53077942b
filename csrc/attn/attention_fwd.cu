// Bidirectional multi-head attention forward on tcgen05 (sm_100a).
//
//   o[t, h*D:(h+1)*D] = softmax(q_h k_h^T / sqrt(D)) v_h,  lse[h, t] = log-sum-exp of the row
//
// q, k, v are read in place from the fused QKV output [T, 3H] (bf16, RoPE
// already applied by the QKV GEMM epilogue); o is [T, H] bf16, lse fp32.
// Head dim D = 128.  One CTA per (128-query tile, head), 192 threads:
//   warp 0      TMA: Q once, then K_j / V_j into a 2-stage ring
//   warp 1      tcgen05.mma issuer (one thread):
//                 S_j  = Q K_j^T   (128 x 128, into TMEM S[j % 2])
//                 O   += P_j V_j   (128 x 128, TMEM accumulator; P_j from smem)
//               S_{j+1} is issued before waiting for P_j, so the next QK^T
//               overlaps the current softmax.
//   warps 2..5  softmax, one query row per thread: tcgen05.ld of S_j,
//               running max / sum in base 2, P_j (bf16) written to smem in the
//               128-byte-swizzled K-major layout the MMA reads.  The O
//               accumulator is rescaled in TMEM only when some row's max grew
//               by more than 2^8 (the exponent base is allowed to lag the true
//               max by that much); the decision is warp-uniform because
//               tcgen05.ld/st are warp-collective.
// Keys past T are masked to -inf; queries past T are computed and not stored.
// Every wait is bounded (see ptx.cuh).  No TMA load uses cluster multicast.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "../common/ptx.cuh"
#include "../gemm/gemm.h"
#include "attention.h"

namespace h3 {
CUtensorMap attn_map_2d(const void* base, long rows, long cols, long ld);
int attn_num_sms(int device);

namespace {

constexpr int kBQ = 128;
constexpr int kBKV = 128;
constexpr int kD = 128;
constexpr int kThreads = 192;
constexpr int kChunk = 128 * 64 * 2;  // 128 rows x 64 bf16 (one 128B-swizzled column chunk)
constexpr int kTileBytes = 2 * kChunk;  // 128 rows x 128 bf16
constexpr int kSmem = 1024 + kTileBytes * 6 + 512;  // Q, K[2], V[2], P
constexpr float kRescaleThreshold = 8.0f;          // log2 units

struct FwdParams {
  int T, H;
  int n_kv;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* o;
  float* lse;
  KernelStatus status;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1) attn_fwd_kernel(const __grid_constant__ CUtensorMap tm, FwdParams p) {
  constexpr uint32_t kIdescS = umma_idesc_bf16(kBQ, kBKV, false, false);
  constexpr uint32_t kIdescPV = umma_idesc_bf16(kBQ, kD, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTileBytes;        // 2 stages
  uint8_t* sV = sK + 2 * kTileBytes;    // 2 stages
  uint8_t* sP = sV + 2 * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;    // [2]
  uint64_t* kv_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;     // [2]
  uint64_t* s_empty = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* o_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int q_tile = blockIdx.x, head = blockIdx.y;
  const int q0 = q_tile * kBQ;
  const int n_kv = p.n_kv;
  const uint64_t limit = p.status.limit_ns;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    if (elect_one()) {
      const int xq = head * kD, xk = p.H + head * kD, xv = 2 * p.H + head * kD;
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_2d(sQ, &tm, q_full, xq, q0);
      tma_load_2d(sQ + kChunk, &tm, q_full, xq + 64, q0);
      int issued_stage_phase[2] = {-1, -1};
      for (int j = 0; j < n_kv && !*abort_flag; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, limit, abort_flag)) {
          report_status(p.status, kStatusTimeoutEmpty, j);
          *abort_flag = 1;
          break;
        }
        const int y = j * kBKV;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
        tma_load_2d(sK + st * kTileBytes, &tm, &kv_full[st], xk, y);
        tma_load_2d(sK + st * kTileBytes + kChunk, &tm, &kv_full[st], xk + 64, y);
        tma_load_2d(sV + st * kTileBytes, &tm, &kv_full[st], xv, y);
        tma_load_2d(sV + st * kTileBytes + kChunk, &tm, &kv_full[st], xv + 64, y);
        issued_stage_phase[st] = static_cast<int>(ph);
      }
      volatile int never = 0;
      mbar_wait(q_full, 0, limit, &never);
      for (int st = 0; st < 2; ++st)
        if (issued_stage_phase[st] >= 0) mbar_wait(&kv_full[st], issued_stage_phase[st], limit, &never);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      bool any = false;
      bool ok = mbar_wait(q_full, 0, limit, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_full[st], ph, limit, abort_flag)) return false;
        if (!mbar_wait(&s_empty[st], ph ^ 1u, limit, abort_flag)) return false;
        tc_fence_after();
        const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK + st * kTileBytes);
#pragma unroll
        for (int ds = 0; ds < kD / 16; ++ds) {
          const uint32_t off = (ds >> 2) * kChunk + (ds & 3) * 32;
          umma_f16_ss(tS[st], umma_smem_desc(q_base + off, 16, 1024), umma_smem_desc(k_base + off, 16, 1024), kIdescS,
                      ds > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        any = true;
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(p_full, j & 1, limit, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = j & 1;
        const uint32_t p_base = smem_u32(sP), v_base = smem_u32(sV + st * kTileBytes);
#pragma unroll
        for (int ks = 0; ks < kBKV / 16; ++ks) {
          const uint64_t a = umma_smem_desc(p_base + (ks >> 2) * kChunk + (ks & 3) * 32, 16, 1024);
          const uint64_t b = umma_smem_desc(v_base + ks * 2048, kChunk, 1024);
          umma_f16_ss(tO, a, b, kIdescPV, (j > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(o_done);
        umma_commit(&kv_empty[st]);
      }
      if (!ok) {
        report_status(p.status, kStatusTimeoutFull, blockIdx.x);
        *abort_flag = 1;
      }
      if (any) {
        umma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, limit, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, limit, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kBKV];
#pragma unroll
      for (int c = 0; c < kBKV / 16; ++c) {
        uint32_t r[16];
        tmem_ld16(tS[sb] + lane_off + c * 16, r);
#pragma unroll
        for (int i = 0; i < 16; ++i) s[c * 16 + i] = __uint_as_float(r[i]);
      }
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      const int kv_valid = p.T - j * kBKV;
      float m_tile = -INFINITY;
#pragma unroll
      for (int i = 0; i < kBKV; ++i) {
        s[i] = (i < kv_valid) ? s[i] * p.scale_log2 : -INFINITY;
        m_tile = fmaxf(m_tile, s[i]);
      }
      const float m_new = fmaxf(m_used, m_tile);
      const bool need = (j == 0) || (m_new > m_used + kRescaleThreshold);
      const bool warp_need = __any_sync(0xffffffffu, need);
      const float alpha = need ? ex2(m_used - m_new) : 1.f;
      if (need) {
        l *= alpha;
        m_used = m_new;
      }
      // P_j = 2^(s - m_used), computed while PV_{j-1} may still be running.
      float rowsum = 0.f;
#pragma unroll
      for (int i = 0; i < kBKV; ++i) {
        s[i] = ex2(s[i] - m_used);
        rowsum += s[i];
      }
      // The P buffer and the O accumulator are free once PV_{j-1} completed.
      if (j > 0 && !mbar_wait(o_done, (j - 1) & 1, limit, abort_flag)) {
        ok = false;
        break;
      }
      if (warp_need && j > 0) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kD / 16; ++c) {
          uint32_t r[16];
          tmem_ld16(tO + lane_off + c * 16, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st16(tO + lane_off + c * 16, r);
        }
        tmem_st_wait();
      }
      // bf16 P rows into the 128B-swizzled K-major tile the PV MMA reads.
#pragma unroll
      for (int u = 0; u < kBKV / 8; ++u) {
        uint4 packed;
        packed.x = pack_bf16x2(s[u * 8 + 0], s[u * 8 + 1]);
        packed.y = pack_bf16x2(s[u * 8 + 2], s[u * 8 + 3]);
        packed.z = pack_bf16x2(s[u * 8 + 4], s[u * 8 + 5]);
        packed.w = pack_bf16x2(s[u * 8 + 6], s[u * 8 + 7]);
        const int chunk = u >> 3, unit = u & 7;
        uint8_t* dst = sP + chunk * kChunk + row * 128 + ((unit ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = packed;
      }
      l += rowsum;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && n_kv > 0 && mbar_wait(o_done, (n_kv - 1) & 1, limit, abort_flag)) {
      tc_fence_after();
      const int q = q0 + row;
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < kD / 16; ++c) {
        uint32_t r[16];
        tmem_ld16(tO + lane_off + c * 16, r);
        tmem_ld_wait();
        if (q < p.T) {
          uint4 a, b;
          a.x = pack_bf16x2(__uint_as_float(r[0]) * inv_l, __uint_as_float(r[1]) * inv_l);
          a.y = pack_bf16x2(__uint_as_float(r[2]) * inv_l, __uint_as_float(r[3]) * inv_l);
          a.z = pack_bf16x2(__uint_as_float(r[4]) * inv_l, __uint_as_float(r[5]) * inv_l);
          a.w = pack_bf16x2(__uint_as_float(r[6]) * inv_l, __uint_as_float(r[7]) * inv_l);
          b.x = pack_bf16x2(__uint_as_float(r[8]) * inv_l, __uint_as_float(r[9]) * inv_l);
          b.y = pack_bf16x2(__uint_as_float(r[10]) * inv_l, __uint_as_float(r[11]) * inv_l);
          b.z = pack_bf16x2(__uint_as_float(r[12]) * inv_l, __uint_as_float(r[13]) * inv_l);
          b.w = pack_bf16x2(__uint_as_float(r[14]) * inv_l, __uint_as_float(r[15]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(p.o + static_cast<long>(q) * p.H + head * kD + c * 16);
          dst[0] = a;
          dst[1] = b;
        }
      }
      if (q < p.T) p.lse[static_cast<long>(head) * p.T + q] = (m_used + __log2f(l)) * 0.6931471805599453f;
    } else if (!ok || n_kv > 0) {
      if (lane == 0) report_status(p.status, kStatusTimeoutAccFull, blockIdx.x);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

std::vector<at::Tensor> attention_fwd(const at::Tensor& qkv, int64_t heads, int64_t head_dim, const at::Tensor& status,
                                      int64_t limit_ns) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1,
              "qkv must be a 2-D CUDA bf16 tensor with unit column stride");
  TORCH_CHECK(head_dim == kD, "attention_fwd supports head_dim 128");
  const int64_t T = qkv.size(0);
  const int64_t H = heads * head_dim;
  TORCH_CHECK(qkv.size(1) == 3 * H, "qkv must be [T, 3*heads*head_dim]");
  c10::cuda::CUDAGuard guard(qkv.get_device());
  auto o = at::empty({T, H}, qkv.options());
  auto lse = at::empty({heads, T}, qkv.options().dtype(at::kFloat));
  if (T == 0) return {o, lse};
  CUtensorMap tm = attn_map_2d(qkv.data_ptr(), T, 3 * H, qkv.stride(0));
  FwdParams p{};
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.n_kv = static_cast<int>((T + kBKV - 1) / kBKV);
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(head_dim)));
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.status.word = status.data_ptr<int>();
  p.status.limit_ns = static_cast<uint64_t>(limit_ns);
  static bool configured[64] = {false};
  const int device = qkv.get_device();
  if (!configured[device]) {
    cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    configured[device] = true;
  }
  dim3 grid(static_cast<unsigned>((T + kBQ - 1) / kBQ), static_cast<unsigned>(heads));
  attn_fwd_kernel<<<grid, kThreads, kSmem, at::cuda::getCurrentCUDAStream(device).stream()>>>(tm, p);
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, lse};
}

}  // namespace h3
