// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
//   D[M, N] = epilogue( op(A)[M, K] * op(B)[N, K]^T  (+ A2[M, K2] * B2[N, K2]^T) )
//
// * A, B are bf16, each K-major (row = one M/N index, K contiguous) or
//   MN-major (row = one K index, M/N contiguous); accumulation is fp32 in
//   tensor memory (TMEM).
// * The optional second K-phase is how LoRA is fused: forward
//   y = x W^T + (s x A^T) B^T runs as one accumulation over K = in + r, with
//   the r-phase reading U = s x A^T and B.  For the fused QKV the second
//   phase is sectioned: output columns of section s read U[:, s*r:(s+1)*r].
// * Warp roles (192 threads, one CTA per SM, persistent over tiles):
//     warp 0      TMA producer (one elected thread), STAGES-deep smem ring
//     warp 1      MMA issuer (one elected thread), tcgen05.mma 128 x BN x 16
//     warps 2..5  epilogue: tcgen05.ld from TMEM -> registers -> global
//   TMEM holds two BN-column accumulators so the epilogue of tile i overlaps
//   the MMAs of tile i+1.
// * Tiles are rastered in groups of `group_m` M-tiles so the CTAs in flight
//   share both operand panels in L2.
// * All waits are bounded (see ptx.cuh); on a timeout the kernel records an
//   error code, drains its own TMA loads / MMAs, frees TMEM and returns.
// * Pair mode (PAIR, the 256-column bf16 epilogues): a 2-CTA cluster computes
//   one 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256).  Each CTA
//   TMA-loads its own 128 rows of A and its own 128-row half of B into its
//   own shared memory (plain loads, completing on the leader CTA's barrier),
//   holds its 128 x 256 accumulator in its own TMEM and runs its own
//   epilogue; the leader's single thread issues the MMAs for both, and its
//   commits arrive on both CTAs' barriers.  Each SM thereby stages half of B
//   per k-block (32 KB instead of 48 KB a stage).
// * Every TMA load in this file targets one CTA only.
#include <ATen/cuda/CUDAContext.h>
#include <cstdlib>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <atomic>
#include <mutex>

#include "../common/extent.h"
#include "../common/ptx.cuh"
#include "gemm.h"

namespace h3 {

std::atomic<uint64_t> g_launches{0};

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 256;   // TMA, MMA, 4 epilogue warps, 2 gather warps
constexpr int kGatherThreads = 64;
constexpr int kMaxPeers = 8;

struct GemmParams {
  int M, N;
  int tiles_m, tiles_n, splits;
  int kb_main, kb_second, kb_per_split;
  int section_n;
  int group_m;
  void* out;
  long ldo;
  void* out2;
  long ldo2;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* res;
  long ldr;
  const float* gate;
  long ldg;
  int split_row;
  const float* cos_t;
  const float* sin_t;
  int rope_cols;
  int head_dim;
  const __nv_bfloat16* pre;
  long ldp;
  float alpha;
  int tma_store;  // bf16 outputs leave through smem + TMA tensor stores (full 128-byte lines)
  // Fused all-gather of B (K-major): rank r owns rows [r*g_rows, (r+1)*g_rows) of
  // the [N, K] weight in its own memory (g_src[r], a peer pointer).  Every
  // CTA's gather warps copy a 1/gridDim slice of each N-tile (in tile order)
  // into the local B buffer (the tmB base, g_dst) and count it in
  // g_flags[tile] (zeroed before the launch); a producer waits until all
  // gridDim slices of its tile have landed before TMA-loading it, so the
  // transfer overlaps the GEMM tile by tile.
  int gather;
  int g_world;
  long g_rows;
  long g_row_bytes;
  const uint8_t* g_src[kMaxPeers];
  uint8_t* g_dst;
  int* g_flags;
  int ablate;     // diagnostic only (H3_GEMM_ABLATE): 1 = skip the epilogue's global stores
  // allocation extents (elements; 16-byte units for g_dst / each g_src shard),
  // checked in the bounds-checked build only
  long out_extent, out2_extent, g_dst_units, g_src_units;
  KernelStatus status;
};

template <int BN, bool PAIR = false>
struct Cfg {
  static constexpr int kBRows = PAIR ? BN / 2 : BN;   // rows of B this CTA stages per k-block
  static constexpr int kStages = PAIR ? 6 : ((BN == 256) ? 4 : 6);
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = kBRows * BK * 2;
  static constexpr int kTmemCols = 2 * BN;
  // epilogue staging: 4 warps x 2 slots x (32 rows x 64 bf16 columns)
  static constexpr int kEpiSlotBytes = 32 * 64 * 2;
  static constexpr int kEpiBytes = 4 * 2 * kEpiSlotBytes;
  static constexpr int kSmem = 1024 + kStages * (kABytes + kBBytes) + kEpiBytes + 256;
};

__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float inner = k0 * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}

__device__ __forceinline__ float gelu_tanh_grad_f(float x) {
  const float k0 = 0.7978845608028654f;
  const float inner = k0 * (x + 0.044715f * x * x * x);
  const float th = tanhf(inner);
  return 0.5f * (1.0f + th) + 0.5f * x * (1.0f - th * th) * k0 * (1.0f + 3.0f * 0.044715f * x * x);
}

__device__ __forceinline__ void tile_coords(const GemmParams& p, int work, int& m_blk, int& n_blk, int& ks) {
  ks = work % p.splits;
  const int tile = work / p.splits;
  const int group_size = p.group_m * p.tiles_n;
  const int g = tile / group_size;
  const int first_m = g * p.group_m;
  const int gm = min(p.tiles_m - first_m, p.group_m);
  const int in_group = tile % group_size;
  m_blk = first_m + in_group % gm;
  n_blk = in_group / gm;
}

// Store 16 consecutive bf16 values of one row, with an N bound.
__device__ __forceinline__ void store_row16_bf16(__nv_bfloat16* dst, const float (&v)[16], int valid) {
  if (valid >= 16 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    uint4 a, b;
    a.x = pack_bf16x2(v[0], v[1]);
    a.y = pack_bf16x2(v[2], v[3]);
    a.z = pack_bf16x2(v[4], v[5]);
    a.w = pack_bf16x2(v[6], v[7]);
    b.x = pack_bf16x2(v[8], v[9]);
    b.y = pack_bf16x2(v[10], v[11]);
    b.z = pack_bf16x2(v[12], v[13]);
    b.w = pack_bf16x2(v[14], v[15]);
    reinterpret_cast<uint4*>(dst)[0] = a;
    reinterpret_cast<uint4*>(dst)[1] = b;
  } else {
    for (int j = 0; j < 16 && j < valid; ++j) dst[j] = __float2bfloat16(v[j]);
  }
}

__device__ __forceinline__ void load_row16_bf16(const __nv_bfloat16* src, float (&v)[16], int valid) {
  if (valid >= 16 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    const uint4 a = reinterpret_cast<const uint4*>(src)[0];
    const uint4 b = reinterpret_cast<const uint4*>(src)[1];
    const __nv_bfloat16* pa = reinterpret_cast<const __nv_bfloat16*>(&a);
    const __nv_bfloat16* pb = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = __bfloat162float(pa[j]);
      v[8 + j] = __bfloat162float(pb[j]);
    }
  } else {
    for (int j = 0; j < 16; ++j) v[j] = (j < valid) ? __bfloat162float(src[j]) : 0.0f;
  }
}

// Output values of 16 consecutive columns of row m for the bf16 epilogues
// (v -> out; g -> out2 for GELU).  Columns past N come out as 0.
template <int EPI>
__device__ __forceinline__ void epilogue_vals(const GemmParams& p, int m, int n, const uint32_t (&r)[16],
                                              float (&v)[16], float (&g)[16], const float* aux = nullptr) {
  const int valid = min(16, p.N - n);
  if (valid <= 0) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = g[j] = 0.0f;
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
  float bias[16];
  if (p.bias != nullptr) {
    load_row16_bf16(p.bias + n, bias, valid);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) bias[j] = 0.0f;
  }
  if constexpr (EPI == kEpiBf16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = p.alpha * v[j] + bias[j];
  } else if constexpr (EPI == kEpiGelu) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = bf16_round(v[j] + bias[j]);
      g[j] = gelu_tanh_f(v[j]);
    }
  } else if constexpr (EPI == kEpiRope) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = bf16_round(v[j] + bias[j]);
    if (n < p.rope_cols) {
      // the 16 columns sit inside one head (n and head_dim are multiples of 16):
      // their 8 rotation pairs use 8 consecutive table entries (two float4 loads)
      const int half = p.head_dim >> 1;
      const int base = (n % p.head_dim) >> 1;
      const float4* cs = reinterpret_cast<const float4*>(p.cos_t + static_cast<long>(m) * half + base);
      const float4* sn = reinterpret_cast<const float4*>(p.sin_t + static_cast<long>(m) * half + base);
      const float4 c0 = cs[0], c1 = cs[1], s0 = sn[0], s1 = sn[1];
      const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float a = v[2 * j], b = v[2 * j + 1];
        v[2 * j] = a * cv[j] - b * sv[j];
        v[2 * j + 1] = a * sv[j] + b * cv[j];
      }
    }
  } else if constexpr (EPI == kEpiGatedRes) {
    float res[16];
    if (aux != nullptr) {
#pragma unroll
      for (int j = 0; j < 16; ++j) res[j] = aux[j];
    } else {
      load_row16_bf16(p.res + static_cast<long>(m) * p.ldr + n, res, valid);
    }
    const float* gate = p.gate + (m >= p.split_row ? p.ldg : 0) + n;
    float gt[16];
    if (valid == 16 && (reinterpret_cast<uintptr_t>(gate) & 15u) == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 g4 = reinterpret_cast<const float4*>(gate)[q];
        gt[4 * q] = g4.x;
        gt[4 * q + 1] = g4.y;
        gt[4 * q + 2] = g4.z;
        gt[4 * q + 3] = g4.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) gt[j] = j < valid ? gate[j] : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float y = bf16_round(v[j] + bias[j]);
      v[j] = res[j] + gt[j] * y;
    }
  } else if constexpr (EPI == kEpiGeluBwd) {
    float pre[16];
    if (aux != nullptr) {
#pragma unroll
      for (int j = 0; j < 16; ++j) pre[j] = aux[j];
    } else {
      load_row16_bf16(p.pre + static_cast<long>(m) * p.ldp + n, pre, valid);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = bf16_round(v[j]) * gelu_tanh_grad_f(pre[j]);
  }
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add_gpu(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Generic-proxy global writes (the gather warps' stores) become visible to the
// async proxy (TMA loads) issued after this.
__device__ __forceinline__ void fence_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Bounded wait until `target` slices of a gathered N-tile have landed.
__device__ __forceinline__ bool wait_tile_flag(const int* flag, int target, uint64_t limit_ns, volatile int* abort) {
  if (ld_acquire_gpu(flag) >= target) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t it = 1; it != 0u; ++it) {
    if (ld_acquire_gpu(flag) >= target) return true;
    if ((it & 63u) == 0u && (*abort || global_timer_ns() - start > limit_ns)) return false;
  }
  return false;
}

__device__ __forceinline__ void fence_async_smem_cta() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 bf16 values of `row` (columns 16*group ..) from a 128B-swizzled 32 x 64 staging tile.
__device__ __forceinline__ void unstage16(const uint8_t* slot, int row, int group, float (&v)[16]) {
  const int u0 = 2 * group, u1 = 2 * group + 1;
  const uint4 a = *reinterpret_cast<const uint4*>(slot + row * 128 + ((u0 ^ (row & 7)) << 4));
  const uint4 b = *reinterpret_cast<const uint4*>(slot + row * 128 + ((u1 ^ (row & 7)) << 4));
  const __nv_bfloat16* pa = reinterpret_cast<const __nv_bfloat16*>(&a);
  const __nv_bfloat16* pb = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = __bfloat162float(pa[j]);
    v[8 + j] = __bfloat162float(pb[j]);
  }
}

// 16 bf16 values as two 16-byte units of a 128B-swizzled 32 x 64 staging tile.
__device__ __forceinline__ void stage16(uint8_t* slot, int row, int group, const float (&v)[16]) {
  uint4 a, b;
  a.x = pack_bf16x2(v[0], v[1]);
  a.y = pack_bf16x2(v[2], v[3]);
  a.z = pack_bf16x2(v[4], v[5]);
  a.w = pack_bf16x2(v[6], v[7]);
  b.x = pack_bf16x2(v[8], v[9]);
  b.y = pack_bf16x2(v[10], v[11]);
  b.z = pack_bf16x2(v[12], v[13]);
  b.w = pack_bf16x2(v[14], v[15]);
  const int u0 = 2 * group, u1 = 2 * group + 1;
  *reinterpret_cast<uint4*>(slot + row * 128 + ((u0 ^ (row & 7)) << 4)) = a;
  *reinterpret_cast<uint4*>(slot + row * 128 + ((u1 ^ (row & 7)) << 4)) = b;
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------- 2-CTA pair helpers
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Tiled 2-D load into this CTA's shared memory whose completed bytes count on
// the leader CTA's barrier (`bar_cluster`, a shared::cluster address).  Not a
// multicast: the tile lands in this CTA only.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive on the barrier at this offset in both CTAs of the pair once all
// previously issued MMAs of this thread complete.
__device__ __forceinline__ void umma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair_own(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

template <int EPI>
__device__ __forceinline__ void epilogue16(const GemmParams& p, int m, int n, const uint32_t (&r)[16]) {
  const int valid = min(16, p.N - n);
  if (valid <= 0 || p.ablate) return;
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);

  if constexpr (EPI == kEpiF32Acc) {
    const long off = static_cast<long>(m) * p.ldo + n;
    if (!H3_IN_BOUNDS(off, off + valid - 1, p.out_extent, p.status)) return;
    float* dst = reinterpret_cast<float*>(p.out) + off;
    if (p.splits > 1) {
      for (int j = 0; j < valid; ++j) atomicAdd(dst + j, p.alpha * v[j]);
    } else {
      for (int j = 0; j < valid; ++j) dst[j] += p.alpha * v[j];
    }
    return;
  } else {
    float bias[16];
    if (p.bias != nullptr) {
      load_row16_bf16(p.bias + n, bias, valid);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) bias[j] = 0.0f;
    }
    const long off = static_cast<long>(m) * p.ldo + n;
    if (!H3_IN_BOUNDS(off, off + valid - 1, p.out_extent, p.status)) return;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + off;
    if constexpr (EPI == kEpiBf16) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = p.alpha * v[j] + bias[j];
      store_row16_bf16(dst, v, valid);
    } else if constexpr (EPI == kEpiGelu) {
      float g[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        v[j] = bf16_round(v[j] + bias[j]);
        g[j] = gelu_tanh_f(v[j]);
      }
      store_row16_bf16(dst, v, valid);
      const long off2 = static_cast<long>(m) * p.ldo2 + n;
      if (H3_IN_BOUNDS(off2, off2 + valid - 1, p.out2_extent, p.status))
        store_row16_bf16(reinterpret_cast<__nv_bfloat16*>(p.out2) + off2, g, valid);
    } else if constexpr (EPI == kEpiRope) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = bf16_round(v[j] + bias[j]);
      if (n < p.rope_cols) {
        const int half = p.head_dim >> 1;
        const float* cs = p.cos_t + static_cast<long>(m) * half;
        const float* sn = p.sin_t + static_cast<long>(m) * half;
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const int pi = ((n + j) % p.head_dim) >> 1;
          const float c = cs[pi], s = sn[pi];
          const float a = v[j], b = v[j + 1];
          v[j] = a * c - b * s;
          v[j + 1] = a * s + b * c;
        }
      }
      store_row16_bf16(dst, v, valid);
    } else if constexpr (EPI == kEpiGatedRes) {
      float res[16];
      load_row16_bf16(p.res + static_cast<long>(m) * p.ldr + n, res, valid);
      const float* gate = p.gate + (m >= p.split_row ? p.ldg : 0) + n;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float y = bf16_round(v[j] + bias[j]);
        v[j] = res[j] + (j < valid ? gate[j] : 0.0f) * y;
      }
      store_row16_bf16(dst, v, valid);
    } else if constexpr (EPI == kEpiGeluBwd) {
      float pre[16];
      load_row16_bf16(p.pre + static_cast<long>(m) * p.ldp + n, pre, valid);
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = bf16_round(v[j]) * gelu_tanh_grad_f(pre[j]);
      store_row16_bf16(dst, v, valid);
    }
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmA2a, const __grid_constant__ CUtensorMap tmA2b,
                const __grid_constant__ CUtensorMap tmA2c, const __grid_constant__ CUtensorMap tmB2,
                const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmOut2,
                const __grid_constant__ CUtensorMap tmAux, const GemmParams p) {
  using C = Cfg<BN, PAIR>;
  constexpr int S = C::kStages;
  constexpr uint32_t kIdesc = umma_idesc_bf16(PAIR ? 2 * BM : BM, BN, A_MN, B_MN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::kABytes;
  uint8_t* sEpi = sB + S * C::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + C::kEpiBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* aux_full = drain + 1;   // [4 warps][2 slots]: TMA load of the epilogue's second operand
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_full + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], PAIR ? 8 : 128);   // pair: one arrive per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&aux_full[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.kb_second > 0) {
      tma_prefetch_desc(&tmA2a);
      tma_prefetch_desc(&tmB2);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync_all();   // both CTAs' barriers initialised before any load or commit reaches them
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t limit = p.status.limit_ns;
  const int total_work = p.tiles_m * p.tiles_n * p.splits;
  const int total_kb = p.kb_main + p.kb_second;
  // Pair mode: work units are 256-row tiles shared by the two CTAs of a
  // cluster; rank 0 (the leader) issues the MMAs.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int m_mult = PAIR ? 2 : 1;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[S];
      bool issued[S];
      for (int s = 0; s < S; ++s) issued[s] = false;
      for (int work = unit0; work < total_work && !*abort_flag; work += units) {
        int m_blk, n_blk, ks;
        tile_coords(p, work, m_blk, n_blk, ks);
        const int m0 = (m_blk * m_mult + static_cast<int>(rank)) * BM;
        const int n0 = n_blk * BN + static_cast<int>(rank) * C::kBRows;   // this CTA's rows of B
        const int kb_lo = ks * p.kb_per_split;
        const int kb_hi = min(total_kb, kb_lo + p.kb_per_split);
        const CUtensorMap* a2 = &tmA2a;
        if (p.section_n > 0) {
          const int sec = n0 / p.section_n;
          a2 = sec == 0 ? &tmA2a : (sec == 1 ? &tmA2b : &tmA2c);
        }
        if (p.gather) {
          if (!wait_tile_flag(p.g_flags + n_blk, static_cast<int>(gridDim.x), limit, abort_flag)) {
            report_status(p.status, kStatusTimeoutPeer, n_blk);
            *abort_flag = 1;
            break;
          }
          fence_async_global();
        }
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, limit, abort_flag)) {
            report_status(p.status, kStatusTimeoutEmpty, kb);
            *abort_flag = 1;
            break;
          }
          uint8_t* a_dst = sA + stage * C::kABytes;
          uint8_t* b_dst = sB + stage * C::kBBytes;
          if constexpr (PAIR) {
            // Both CTAs' bytes count on the leader's barrier; only the leader arms it.
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (C::kABytes + C::kBBytes));
            const uint32_t bar = map_to_rank(&full[stage], 0);
            const int k0 = (kb < p.kb_main ? kb : kb - p.kb_main) * BK;
            const CUtensorMap* ma_ = kb < p.kb_main ? &tmA : a2;
            const CUtensorMap* mb_ = kb < p.kb_main ? &tmB : &tmB2;
            tma_load_2d_pair(a_dst, ma_, bar, k0, m0);
            if constexpr (!B_MN) {
              tma_load_2d_pair(b_dst, mb_, bar, k0, n0);
            } else {
#pragma unroll
              for (int c = 0; c < C::kBRows / 64; ++c) tma_load_2d_pair(b_dst + c * 8192, mb_, bar, n0 + c * 64, k0);
            }
            if (rank == 0) {
              issued[stage] = true;
              issued_phase[stage] = phase;
            }
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], C::kABytes + C::kBBytes);
          if (kb < p.kb_main) {
            const int k0 = kb * BK;
            if constexpr (!A_MN) {
              tma_load_2d(a_dst, &tmA, &full[stage], k0, m0);
            } else {
#pragma unroll
              for (int c = 0; c < BM / 64; ++c) tma_load_2d(a_dst + c * 8192, &tmA, &full[stage], m0 + c * 64, k0);
            }
            if constexpr (!B_MN) {
              tma_load_2d(b_dst, &tmB, &full[stage], k0, n0);
            } else {
#pragma unroll
              for (int c = 0; c < BN / 64; ++c) tma_load_2d(b_dst + c * 8192, &tmB, &full[stage], n0 + c * 64, k0);
            }
          } else {
            const int k0 = (kb - p.kb_main) * BK;
            tma_load_2d(a_dst, a2, &full[stage], k0, m0);
            if constexpr (!B_MN) {
              tma_load_2d(b_dst, &tmB2, &full[stage], k0, n0);
            } else {
#pragma unroll
              for (int c = 0; c < BN / 64; ++c) tma_load_2d(b_dst + c * 8192, &tmB2, &full[stage], n0 + c * 64, k0);
            }
          }
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Never leave a TMA write in flight into this CTA's shared memory.
      for (int s = 0; s < S; ++s) {
        if (issued[s] && !mbar_wait(&full[s], issued_phase[s], limit, abort_flag)) {
          // Abort path: wait again without the abort short-cut, still bounded.
          volatile int never = 0;
          mbar_wait(&full[s], issued_phase[s], limit, &never);
        }
      }
    }
  } else if (warp >= 6) {
    // ------------------------------------------------------------ gather warps
    if (p.gather) {
      const int gt = threadIdx.x - 6 * 32;   // 0 .. kGatherThreads-1
      const long units_per_row = p.g_row_bytes >> 4;
      // Tiles in order (the producers need the low N-tiles first); every CTA
      // copies its slice of each tile, so all SMs' bandwidth goes to tile 0 first.
      for (int nt = 0; nt < p.tiles_n && !*abort_flag; ++nt) {
        const long r0 = static_cast<long>(nt) * BN;
        const long r1 = min(static_cast<long>(p.N), r0 + BN);
        const long units = (r1 - r0) * units_per_row;
        const long per_cta = (units + gridDim.x - 1) / gridDim.x;
        const long u_lo = min(units, blockIdx.x * per_cta), u_hi = min(units, u_lo + per_cta);
        constexpr int kU = 8;   // 8 KB of loads in flight per CTA (NVLink latency needs depth)
        for (long base = u_lo + gt; base < u_hi; base += kGatherThreads * kU) {
          uint4 v[kU];
#pragma unroll
          for (int k = 0; k < kU; ++k) {
            const long u = base + k * kGatherThreads;
            if (u < u_hi) {
              const long row = r0 + u / units_per_row;
              const int owner = static_cast<int>(row / p.g_rows);
              const long local = (row - owner * p.g_rows) * units_per_row + u % units_per_row;
              v[k] = H3_IN_BOUNDS(local, local, p.g_src_units, p.status)
                         ? reinterpret_cast<const uint4*>(p.g_src[owner])[local]
                         : make_uint4(0u, 0u, 0u, 0u);
            }
          }
#pragma unroll
          for (int k = 0; k < kU; ++k) {
            const long u = base + k * kGatherThreads;
            if (u < u_hi && H3_IN_BOUNDS(r0 * units_per_row + u, r0 * units_per_row + u, p.g_dst_units, p.status))
              reinterpret_cast<uint4*>(p.g_dst)[r0 * units_per_row + u] = v[k];
          }
        }
        // The tile is read by TMA (async proxy) in other CTAs: order this
        // thread's generic-proxy stores before the async proxy on the writer
        // side too, then publish the slice with a release add.
        fence_async_global();
        asm volatile("bar.sync 1, %0;" ::"n"(kGatherThreads) : "memory");
        if (gt == 0) {
          __threadfence();
          red_release_add_gpu(p.g_flags + nt, 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (the leader's, in pair mode)
    if (elect_one() && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool any = false;
      for (int work = unit0; work < total_work && !*abort_flag; work += units) {
        int m_blk, n_blk, ks;
        tile_coords(p, work, m_blk, n_blk, ks);
        const int kb_lo = ks * p.kb_per_split;
        const int kb_hi = min(total_kb, kb_lo + p.kb_per_split);
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, limit, abort_flag)) {
          report_status(p.status, kStatusTimeoutAccEmpty, work);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[stage], phase, limit, abort_flag)) {
            report_status(p.status, kStatusTimeoutFull, kb);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * C::kABytes);
          const uint32_t b_base = smem_u32(sB + stage * C::kBBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? umma_smem_desc(a_base + kk * 2048, 8192, 1024)
                                     : umma_smem_desc(a_base + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? umma_smem_desc(b_base + kk * 2048, 8192, 1024)
                                     : umma_smem_desc(b_base + kk * 32, 16, 1024);
            if constexpr (PAIR) {
              umma_f16_ss_pair(d_tmem, ad, bd, kIdesc, (kb > kb_lo || kk > 0) ? 1u : 0u);
            } else {
              umma_f16_ss(d_tmem, ad, bd, kIdesc, (kb > kb_lo || kk > 0) ? 1u : 0u);
            }
          }
          any = true;
          if constexpr (PAIR) {
            umma_commit_pair_both(&empty[stage]);
          } else {
            umma_commit(&empty[stage]);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          umma_commit_pair_both(&acc_full[acc]);
        } else {
          umma_commit(&acc_full[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (any) {
        // Wait for every issued MMA before TMEM can be released.
        if constexpr (PAIR) {
          umma_commit_pair_own(drain);
        } else {
          umma_commit(drain);
        }
        volatile int never = 0;
        mbar_wait(drain, 0, limit, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    int store_idx = 0;
    uint32_t aux_phase[2] = {0u, 0u};
    // pair mode: the leader's accumulator-empty barrier, arrived on by one lane per warp of both CTAs
    const uint32_t acc_empty_leader[2] = {PAIR ? map_to_rank(&acc_empty[0], 0) : 0u,
                                          PAIR ? map_to_rank(&acc_empty[1], 0) : 0u};
    for (int work = unit0; work < total_work; work += units) {
      int m_blk, n_blk, ks;
      tile_coords(p, work, m_blk, n_blk, ks);
      m_blk = m_blk * m_mult + static_cast<int>(rank);   // this CTA's 128-row block
      if (!mbar_wait(&acc_full[acc], acc_phase, limit, abort_flag)) {
        if (lane == 0) report_status(p.status, kStatusTimeoutAccFull, work);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m = m_blk * BM + row;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if constexpr (EPI != kEpiF32Acc) {
        if (p.tma_store) {
          // Each warp stages its 32 rows x 64 columns in smem and stores them
          // with one TMA tensor store (full 128-byte lines; the per-row 16-byte
          // stores of the fallback cost up to a third of the GEMM time).
          uint8_t* wbuf = sEpi + quarter * (2 * C::kEpiSlotBytes);
#pragma unroll 1
          for (int c = 0; c < BN; c += 64) {
            uint32_t r[4][16];
#pragma unroll
            for (int g = 0; g < 4; ++g) tmem_ld16(t_row + c + 16 * g, r[g]);
            tmem_ld_wait();
            // the slot(s) written below must no longer be read by an earlier store
            if (lane == 0) {
              if (EPI == kEpiGelu) {
                bulk_wait_read<0>();
              } else if (store_idx >= 2) {
                bulk_wait_read<1>();
              }
            }
            __syncwarp();
            const int si = EPI == kEpiGelu ? 0 : (store_idx & 1);
            uint8_t* slot = wbuf + si * C::kEpiSlotBytes;
            uint8_t* slot2 = wbuf + C::kEpiSlotBytes;
            const int n = n_blk * BN + c;
            constexpr bool kAux = EPI == kEpiGatedRes || EPI == kEpiGeluBwd;
            if constexpr (kAux) {
              // the residual / GELU input tile arrives by TMA into the slot the
              // output then overwrites (coalesced 128-byte lines both ways)
              uint64_t* bar = &aux_full[quarter * 2 + si];
              if (lane == 0) {
                mbar_arrive_expect_tx(bar, C::kEpiSlotBytes);
                tma_load_2d(slot, &tmAux, bar, n, m_blk * BM + quarter * 32);
              }
              if (!mbar_wait(bar, aux_phase[si], limit, abort_flag)) {
                if (lane == 0) report_status(p.status, kStatusTimeoutAccFull, work);
                *abort_flag = 1;
              }
              aux_phase[si] ^= 1u;
            }
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              float v[16], gv[16];
              if (m < p.M && !p.ablate) {
                if constexpr (kAux) {
                  float a[16];
                  unstage16(slot, lane, g, a);
                  epilogue_vals<EPI>(p, m, n + 16 * g, r[g], v, gv, a);
                } else {
                  epilogue_vals<EPI>(p, m, n + 16 * g, r[g], v, gv);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = gv[j] = 0.0f;
              }
              stage16(slot, lane, g, v);
              if (EPI == kEpiGelu) stage16(slot2, lane, g, gv);
            }
            fence_async_smem_cta();
            __syncwarp();
            if (lane == 0 && !p.ablate) {
              const int y = m_blk * BM + quarter * 32;
              tma_store_2d(&tmOut, slot, n, y);
              if (EPI == kEpiGelu) tma_store_2d(&tmOut2, slot2, n, y);
            }
            store_idx += EPI == kEpiGelu ? 2 : 1;
          }
          tc_fence_before();
          if constexpr (PAIR) {
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(acc_empty_leader[acc]);
          } else {
            mbar_arrive(&acc_empty[acc]);
          }
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1u;
          continue;
        }
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r0[16], r1[16];
        tmem_ld16(t_row + c, r0);
        tmem_ld16(t_row + c + 16, r1);
        tmem_ld_wait();
        if (m < p.M) {
          const int n = n_blk * BN + c;
          epilogue16<EPI>(p, m, n, r0);
          epilogue16<EPI>(p, m, n + 16, r1);
        }
      }
      tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc_empty_leader[acc]);
      } else {
        mbar_arrive(&acc_empty[acc]);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0 && store_idx > 0) bulk_wait_all();   // the TMA stores are complete before exit
  }

  tc_fence_before();
  if constexpr (PAIR) {
    // Neither CTA leaves while the other may still touch its barriers or TMEM.
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem_base, C::kTmemCols);
    } else {
      tmem_dealloc(tmem_base, C::kTmemCols);
    }
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(ptr != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Row-major bf16 matrix [rows, cols] with row stride `ld` elements; box = {64, box_rows}.
CUtensorMap make_map(const void* base, long rows, long cols, long ld, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15u) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes (ld=", ld, ")");
  TORCH_CHECK(rows >= 1 && cols >= 1, "empty TMA operand");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(r));
  return map;
}

int num_sms(int device) {
  static int cached[64] = {0};
  if (cached[device] == 0) {
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, device);
    cached[device] = prop.multiProcessorCount;
  }
  return cached[device];
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool PAIR = false>
void launch_variant(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& a2a, const CUtensorMap& a2b,
                    const CUtensorMap& a2c, const CUtensorMap& b2, const CUtensorMap& o1, const CUtensorMap& o2,
                    const CUtensorMap& aux, const GemmParams& p, int device, cudaStream_t stream) {
  auto kernel = gemm_kernel<BN, A_MN, B_MN, EPI, PAIR>;
  constexpr int smem = Cfg<BN, PAIR>::kSmem;
  static_assert(smem <= 232448, "GEMM shared memory");
  static bool configured[64] = {false};
  if (!configured[device]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[device] = true;
  }
  const int work = p.tiles_m * p.tiles_n * p.splits;
  if constexpr (PAIR) {
    // One 2-CTA cluster per 256-row tile in flight, persistent over tiles.
    const int pairs = std::min(work, num_sms(device) / 2);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, a, b, a2a, a2b, a2c, b2, o1, o2, aux, p));
  } else {
    const int grid = std::min(work, num_sms(device));
    kernel<<<grid, kThreads, smem, stream>>>(a, b, a2a, a2b, a2c, b2, o1, o2, aux, p);
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

uint64_t launch_count() { return g_launches.load(); }

// 2-D bf16 tensor map with a {64, 128} box and 128-byte swizzle (used by attention).
CUtensorMap attn_map_2d(const void* base, long rows, long cols, long ld) { return make_map(base, rows, cols, ld, 128); }

// 2-D fp32 tensor map [rows, cols] (row stride `ld` elements), box {32, box_rows}, 128-byte swizzle.
CUtensorMap make_map_f32(const void* base, long rows, long cols, long ld, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15u) == 0 && (ld * 4) % 16 == 0, "fp32 TMA operand alignment");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 4)};
  cuuint32_t box[2] = {32u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (fp32) failed: ", static_cast<int>(r));
  return map;
}
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Operand view: base pointer, logical rows x cols of the *stored* row-major matrix, row stride.
struct Operand {
  const void* ptr;
  long rows, cols, ld;
};

static Operand operand_of(const at::Tensor& t) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, "GEMM operands must be CUDA bf16");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "GEMM operands must be 2-D with unit column stride");
  return {t.data_ptr(), t.size(0), t.size(1), t.stride(0)};
}

void gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t M, int64_t N, int64_t K,
          const std::vector<at::Tensor>& A2, const c10::optional<at::Tensor>& B2, int64_t K2, int64_t section_n,
          int64_t epi, const at::Tensor& out, const c10::optional<at::Tensor>& out2,
          const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& res,
          const c10::optional<at::Tensor>& gate, int64_t split_row, const c10::optional<at::Tensor>& cos_t,
          const c10::optional<at::Tensor>& sin_t, int64_t rope_cols, int64_t head_dim,
          const c10::optional<at::Tensor>& pre, double alpha, int64_t splits, int64_t block_n,
          const at::Tensor& status, int64_t limit_ns, const std::vector<int64_t>& gather_src,
          int64_t gather_rows, const c10::optional<at::Tensor>& gather_flags) {
  const int device = A.get_device();
  c10::cuda::CUDAGuard guard(device);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(device).stream();
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "GEMM sizes must be positive");
  const int bn = static_cast<int>(block_n);
  TORCH_CHECK(bn == 128 || bn == 256, "block_n must be 128 or 256");
  TORCH_CHECK(!(a_mn && K2 > 0), "the second K-phase needs a K-major A");
  // The compiled variants (checked here, before any tensor map is built):
  // K-major A with K-major B: every bf16 epilogue at block_n 256, plain bf16 at
  // 128; K-major A with MN-major B: bf16 / GELU-backward at 256, bf16 at 128;
  // MN-major A and B: the fp32 accumulate at either width.
  const bool bf16_epi = epi == kEpiBf16 || epi == kEpiRope || epi == kEpiGelu || epi == kEpiGatedRes;
  const bool variant_exists =
      (!a_mn && !b_mn && ((bn == 256 && bf16_epi) || (bn == 128 && epi == kEpiBf16))) ||
      (!a_mn && b_mn && ((bn == 256 && (epi == kEpiBf16 || epi == kEpiGeluBwd)) || (bn == 128 && epi == kEpiBf16))) ||
      (a_mn && b_mn && epi == kEpiF32Acc);
  TORCH_CHECK(variant_exists, "no GEMM variant for block_n=", bn, " a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);

  Operand oa = operand_of(A), ob = operand_of(B);
  // 2-CTA pair mode for the 256-column bf16 epilogues on K-major A (no
  // split-K); with the fused gather every CTA still copies its 1/gridDim slice
  // of each N-tile and each producer waits for the whole tile before loading
  // its half.  H3_GEMM_PAIR=0 turns it off for measurements.
  static const bool pair_enabled = [] {
    const char* v = std::getenv("H3_GEMM_PAIR");
    return v == nullptr || std::atoi(v) != 0;
  }();
  const bool pair = pair_enabled && bn == 256 && !a_mn && epi != kEpiF32Acc && splits <= 1 &&
                    (b_mn ? (epi == kEpiBf16 || epi == kEpiGeluBwd) : true);
  const int b_rows = pair ? bn / 2 : bn;   // rows of B one CTA stages (K-major B)
  // Stored shapes: K-major A = [M, K]; MN-major A = [K, M]; same for B with N.
  CUtensorMap ma = a_mn ? make_map(oa.ptr, oa.rows, oa.cols, oa.ld, 64) : make_map(oa.ptr, oa.rows, oa.cols, oa.ld, BM);
  CUtensorMap mb = b_mn ? make_map(ob.ptr, ob.rows, ob.cols, ob.ld, 64) : make_map(ob.ptr, ob.rows, ob.cols, ob.ld, b_rows);
  CUtensorMap ma2[3] = {ma, ma, ma};
  CUtensorMap mb2 = mb;
  int kb_second = 0;
  if (K2 > 0) {
    TORCH_CHECK(!A2.empty() && A2.size() <= 3 && B2.has_value(), "second K-phase needs A2 (1..3 sections) and B2");
    for (size_t i = 0; i < A2.size(); ++i) {
      Operand o = operand_of(A2[i]);
      ma2[i] = make_map(o.ptr, o.rows, o.cols, o.ld, BM);
    }
    for (size_t i = A2.size(); i < 3; ++i) ma2[i] = ma2[0];
    Operand o2 = operand_of(*B2);
    mb2 = b_mn ? make_map(o2.ptr, o2.rows, o2.cols, o2.ld, 64) : make_map(o2.ptr, o2.rows, o2.cols, o2.ld, b_rows);
    kb_second = static_cast<int>((K2 + BK - 1) / BK);
  }
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.tiles_m = static_cast<int>((M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM));
  p.tiles_n = static_cast<int>((N + bn - 1) / bn);
  p.kb_main = static_cast<int>((K + BK - 1) / BK);
  p.kb_second = kb_second;
  const int total_kb = p.kb_main + p.kb_second;
  int sp = std::max<int64_t>(1, std::min<int64_t>(splits, total_kb));
  p.kb_per_split = (total_kb + sp - 1) / sp;
  p.splits = (total_kb + p.kb_per_split - 1) / p.kb_per_split;
  TORCH_CHECK(p.splits == 1 || epi == kEpiF32Acc, "split-K needs the fp32 accumulate epilogue");
  TORCH_CHECK(section_n == 0 || section_n % bn == 0, "a LoRA section (", section_n,
              " columns) must be a multiple of block_n=", bn);
  p.section_n = static_cast<int>(section_n);
  p.group_m = 16;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.out_extent = extent_of(out);
  p.out2_extent = out2.has_value() ? extent_of(*out2) : 0;
#ifdef H3_BOUNDS_CHECK
  // Test hook of the checked build: H3_BOUNDS_SHRINK=n pretends the output
  // allocation is n elements shorter, so the checks must catch (and skip)
  // the stores into its last n elements.
  if (const char* shrink = std::getenv("H3_BOUNDS_SHRINK")) p.out_extent -= std::atol(shrink);
#endif
  p.out2 = out2.has_value() ? out2->data_ptr() : nullptr;
  p.ldo2 = out2.has_value() ? out2->stride(0) : 0;
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.res = res.has_value() ? reinterpret_cast<const __nv_bfloat16*>(res->data_ptr()) : nullptr;
  p.ldr = res.has_value() ? res->stride(0) : 0;
  p.gate = gate.has_value() ? gate->data_ptr<float>() : nullptr;
  p.ldg = gate.has_value() ? gate->stride(0) : 0;
  p.split_row = static_cast<int>(split_row);
  p.cos_t = cos_t.has_value() ? cos_t->data_ptr<float>() : nullptr;
  p.sin_t = sin_t.has_value() ? sin_t->data_ptr<float>() : nullptr;
  p.rope_cols = static_cast<int>(rope_cols);
  p.head_dim = static_cast<int>(head_dim);
  p.pre = pre.has_value() ? reinterpret_cast<const __nv_bfloat16*>(pre->data_ptr()) : nullptr;
  p.ldp = pre.has_value() ? pre->stride(0) : 0;
  p.alpha = static_cast<float>(alpha);
  static const int ablate = [] {
    const char* v = std::getenv("H3_GEMM_ABLATE");
    return v != nullptr ? std::atoi(v) : 0;
  }();
  p.ablate = ablate;
  p.status.word = status.data_ptr<int>();
  p.status.limit_ns = static_cast<uint64_t>(limit_ns);
  p.gather = 0;
  if (!gather_src.empty()) {
    // B is this rank's local gathered buffer; the rows come from the peers.
    TORCH_CHECK(!b_mn && ob.ld == K && (K * 2) % 16 == 0, "fused all-gather needs a contiguous K-major B");
    TORCH_CHECK(gather_src.size() <= static_cast<size_t>(kMaxPeers), "at most 8 peers");
    TORCH_CHECK(gather_rows > 0 && gather_rows * static_cast<int64_t>(gather_src.size()) >= N, "row shards");
    TORCH_CHECK(gather_flags.has_value() && gather_flags->scalar_type() == at::kInt &&
                    gather_flags->numel() >= p.tiles_n, "one int32 flag per N-tile");
    TORCH_CHECK(K2 == 0 && p.splits == 1, "fused all-gather supports the plain K-phase only");
    p.gather = 1;
    p.g_world = static_cast<int>(gather_src.size());
    p.g_rows = gather_rows;
    p.g_row_bytes = K * 2;
    for (size_t i = 0; i < gather_src.size(); ++i) {
      TORCH_CHECK((gather_src[i] & 15) == 0, "peer shards must be 16-byte aligned");
      p.g_src[i] = reinterpret_cast<const uint8_t*>(gather_src[i]);
    }
    p.g_dst = reinterpret_cast<uint8_t*>(const_cast<void*>(ob.ptr));
    p.g_dst_units = extent_of(B) * 2 / 16;
    p.g_src_units = gather_rows * K * 2 / 16;
    p.g_flags = gather_flags->data_ptr<int>();
    // slice counters start at zero every call (same stream, before the launch)
    C10_CUDA_CHECK(cudaMemsetAsync(p.g_flags, 0, sizeof(int) * p.tiles_n, stream));
  }

  if (epi == kEpiF32Acc) {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "fp32 accumulate epilogue needs an fp32 out");
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 epilogues need a bf16 out");
  }
  if (epi == kEpiGatedRes) TORCH_CHECK(res.has_value() && gate.has_value(), "gated residual needs res and gate");
  if (epi == kEpiRope) {
    TORCH_CHECK(cos_t.has_value() && sin_t.has_value() && head_dim % 16 == 0, "rope tables");
    // the epilogue reads 8 consecutive entries of a row with float4 loads
    TORCH_CHECK(cos_t->is_contiguous() && sin_t->is_contiguous() && cos_t->size(-1) == head_dim / 2 &&
                    (reinterpret_cast<uintptr_t>(cos_t->data_ptr()) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(sin_t->data_ptr()) & 15u) == 0,
                "rope tables must be contiguous [T, head_dim/2] fp32 with 16-byte aligned rows");
  }
  if (epi == kEpiGelu) TORCH_CHECK(out2.has_value(), "gelu epilogue needs out2");
  if (epi == kEpiGeluBwd) TORCH_CHECK(pre.has_value(), "gelu backward epilogue needs pre");
  // bf16 outputs go out by TMA tensor stores when their layout allows a tensor map
  CUtensorMap mo = ma, mo2 = ma;
  auto storable = [&](const at::Tensor& t) {
    return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) == 0 && (t.stride(0) * 2) % 16 == 0 && N >= 8 &&
           t.stride(1) == 1;
  };
  p.tma_store = 0;
  CUtensorMap maux = ma;
  const at::Tensor* aux_t = epi == kEpiGatedRes ? &*res : (epi == kEpiGeluBwd ? &*pre : nullptr);
  if (epi != kEpiF32Acc && storable(out) && (!out2.has_value() || storable(*out2)) &&
      (aux_t == nullptr || (aux_t->scalar_type() == at::kBFloat16 && storable(*aux_t)))) {
    mo = make_map(out.data_ptr(), M, N, out.stride(0), 32);
    if (out2.has_value()) mo2 = make_map(out2->data_ptr(), M, N, out2->stride(0), 32);
    if (aux_t != nullptr) maux = make_map(aux_t->data_ptr(), M, N, aux_t->stride(0), 32);
    p.tma_store = 1;
  }

#define H3_GEMM_PAIR_CASE(AMN_, BMN_, EPI_)                                                   \
  if (pair && a_mn == AMN_ && b_mn == BMN_ && epi == EPI_) {                                    \
    launch_variant<256, AMN_, BMN_, EPI_, true>(ma, mb, ma2[0], ma2[1], ma2[2], mb2, mo, mo2, maux, p, device, stream); \
    return;                                                                                     \
  }
  H3_GEMM_PAIR_CASE(false, false, kEpiBf16)
  H3_GEMM_PAIR_CASE(false, false, kEpiRope)
  H3_GEMM_PAIR_CASE(false, false, kEpiGelu)
  H3_GEMM_PAIR_CASE(false, false, kEpiGatedRes)
  H3_GEMM_PAIR_CASE(false, true, kEpiBf16)
  H3_GEMM_PAIR_CASE(false, true, kEpiGeluBwd)
#undef H3_GEMM_PAIR_CASE
  TORCH_CHECK(!pair, "no pair-mode GEMM variant for b_mn=", b_mn, " epi=", epi);
#define H3_GEMM_CASE(BN_, AMN_, BMN_, EPI_)                                                   \
  if (bn == BN_ && a_mn == AMN_ && b_mn == BMN_ && epi == EPI_) {                             \
    launch_variant<BN_, AMN_, BMN_, EPI_>(ma, mb, ma2[0], ma2[1], ma2[2], mb2, mo, mo2, maux, p, device, stream); \
    return;                                                                                   \
  }
  H3_GEMM_CASE(256, false, false, kEpiBf16)
  H3_GEMM_CASE(256, false, false, kEpiRope)
  H3_GEMM_CASE(256, false, false, kEpiGelu)
  H3_GEMM_CASE(256, false, false, kEpiGatedRes)
  H3_GEMM_CASE(128, false, false, kEpiBf16)
  H3_GEMM_CASE(256, false, true, kEpiBf16)
  H3_GEMM_CASE(256, false, true, kEpiGeluBwd)
  H3_GEMM_CASE(128, false, true, kEpiBf16)
  H3_GEMM_CASE(128, true, true, kEpiF32Acc)
  H3_GEMM_CASE(256, true, true, kEpiF32Acc)
#undef H3_GEMM_CASE
  TORCH_CHECK(false, "no GEMM variant for block_n=", bn, " a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

}  // namespace h3
