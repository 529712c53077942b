// Bidirectional multi-head attention backward on tcgen05 (sm_100a).
//
// Inputs: qkv [T, 3H] (post-RoPE q, k and v), o [T, H], do [T, H] (bf16), lse [heads, T]
// (natural log, from attention_fwd).  Output: dqkv [T, 3H] bf16 (dq, dk, dv in the
// same layout as qkv; RoPE is undone afterwards by the caller).  Head dim 128.
//
// Three kernels:
//   prep    delta[h, t] = sum_d do * o, lse2 = lse * log2(e), both padded to a
//           multiple of 128 rows (padding rows: lse2 = +inf, delta = 0)
//   main    one CTA per (128-key tile, head), 320 threads, looping over 128-query
//           tiles i:
//             S^T  = K Q_i^T,  dP^T = V dO_i^T          (tcgen05, smem operands)
//             P^T  = 2^(S^T*scale*log2e - lse2),  dS^T = scale * P^T (dP^T - delta)
//                    (warps 2..9: one key row per thread, the two warpgroups
//                    split the query columns; written back into TMEM as packed
//                    bf16 and dS^T also into smem; a quarter of the
//                    exponentials run on the FMA pipe)
//             dQ_i = dS K                               (smem A, MN-major), two
//                    N = 64 halves in the TMEM columns S^T / dP^T leave free
//             dV  += P^T dO_i,  dK += dS^T Q_i          (A from TMEM, .ts form)
//           the same warps then read dQ_i out of TMEM into registers (half of
//           it each) and release those TMEM columns to the next step's S^T /
//           dP^T at once, then stage dQ_i in the stage buffer whose Q_i / dO_i
//           the dV/dK MMAs just finished reading, and add it into an fp32
//           accumulator with TMA bulk tensor reduce-adds (whole 128-byte
//           lines; 16-byte red.add was slower).  The
//           wait for the reduces' smem reads is deferred by one step (until
//           after the next softmax), then the stage is handed back to the loader:
//           waiting right away put the reduce latency on the critical path
//           (121.7 ms -> 100.6 ms at T = 37,730, 42 heads);
//           warp 0 streams Q_i, dO_i, lse2_i, delta_i (2 stages), warp 1 issues
//           the MMAs.  dV/dK are written once at the end.
//   finish  dq = bf16(dQ accumulator)
// TMEM: dV [0,128) dK [128,256) S^T/P^T [256,384) dP^T/dS^T [384,512); dQ_i halves
// in [320,384) and [448,512).  Keys past T give zero P / dS; queries past T are
// neutralised by lse2 = +inf.  All waits are bounded; every TMA load targets one
// CTA only.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <cstdlib>

#include "../common/extent.h"
#include "../common/ptx.cuh"
#include "../gemm/gemm.h"
#include "attention.h"

namespace h3 {
CUtensorMap attn_map_2d(const void* base, long rows, long cols, long ld);
CUtensorMap make_map_f32(const void* base, long rows, long cols, long ld, int box_rows);

namespace {

constexpr int kB = 128;  // keys per CTA and queries per step
constexpr int kD = 128;
constexpr int kThreads = 320;  // TMA, MMA, 2 x 4 softmax / dQ-reducer warps
constexpr int kChunk = 128 * 64 * 2;
constexpr int kTile = 2 * kChunk;                       // 128 x 128 bf16
constexpr int kVecBytes = kB * 4;                       // 128 floats
constexpr int kStageBytes = 2 * kTile + 2 * kVecBytes;  // Q_i, dO_i, lse2_i, delta_i
constexpr int kSmem = 2 * kTile + 2 * kStageBytes + kTile + 256;  // K, V, stages, dS^T, barriers

struct BwdParams {
  int T, H, T_pad, n_q;
  float scale;       // softmax scale
  float scale_log2;  // softmax scale * log2(e)
  const float* lse2;
  const float* delta;
  float* dq_acc;           // [T, H] fp32
  __nv_bfloat16* dqkv;     // [T, 3H]
  int ablate;              // diagnostic only (H3_ATTN_BWD_ABLATE): 1 skip dQ adds, 2 skip exponentials
  // Diagnostic phase trace (null in normal runs): CTA (0, 0) records clock64
  // at each phase of query step i of warpgroup 0's first lane band and of the
  // MMA issuer, kBwdTraceSlots values per step.
  long long* trace;
  long dqkv_extent;         // allocation extent, checked in the bounds-checked build only
  KernelStatus status;
};
constexpr int kBwdTraceSlots = 12;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Bulk tensor reduce-add of one smem box into global memory (whole 128-byte lines).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2^x on the FMA pipe (round-to-nearest split, cubic least-squares fit of 2^f on
// [-1/2, 1/2] at Chebyshev nodes, max relative error 1.0e-4); x >= -126.
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -126.0f);
  const float magic = 12582912.0f;
  const float t = x + magic;
  const int n = __float_as_int(t) - 0x4B400000;
  const float f = x - (t - magic);
  float q = fmaf(0.05592203512787819f, f, 0.24264007806777954f);
  q = fmaf(q, f, 0.6931210160255432f);
  q = fmaf(q, f, 0.9999244809150696f);
  return __int_as_float(__float_as_int(q) + (n << 23));
}

__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                     const float* __restrict__ lse, int T, int T_pad, int H, int heads,
                                     float* __restrict__ lse2, float* __restrict__ delta) {
  // one warp per (head, t)
  const long warp_global = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long total = static_cast<long>(heads) * T_pad;
  if (warp_global >= total) return;
  const int h = static_cast<int>(warp_global / T_pad);
  const int t = static_cast<int>(warp_global % T_pad);
  float s = 0.f;
  if (t < T) {
    const __nv_bfloat16* orow = o + static_cast<long>(t) * H + h * kD + lane * 4;
    const __nv_bfloat16* drow = dout + static_cast<long>(t) * H + h * kD + lane * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) s += __bfloat162float(orow[i]) * __bfloat162float(drow[i]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    delta[warp_global] = t < T ? s : 0.f;
    lse2[warp_global] = t < T ? lse[static_cast<long>(h) * T + t] * 1.4426950408889634f : INFINITY;
  }
}

__global__ void attn_bwd_finish_kernel(const float* __restrict__ dq_acc, int T, int H, __nv_bfloat16* __restrict__ dqkv) {
  const long n4 = static_cast<long>(T) * H / 4;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(dq_acc)[i];
    const long e = i * 4;
    const long t = e / H, c = e % H;
    __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(dqkv + t * 3 * H + c);
    dst[0] = __floats2bfloat162_rn(v.x, v.y);
    dst[1] = __floats2bfloat162_rn(v.z, v.w);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq, BwdParams p) {
  constexpr uint32_t kIdescSS = umma_idesc_bf16(kB, kB, false, false);     // S^T, dP^T
  constexpr uint32_t kIdescQ = umma_idesc_bf16(kB, 64, true, true);        // dQ halves
  constexpr uint32_t kIdescTS = umma_idesc_bf16(kB, kD, false, true);      // dV, dK (A in TMEM)
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTile;
  uint8_t* sStage = sV + kTile;  // 2 x [Q_i | dO_i | lse2_i | delta_i]
  uint8_t* sDS = sStage + 2 * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + kTile);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;   // [2]
  uint64_t* qd_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* dq_full = bars + 7;
  uint64_t* dq_empty = bars + 8;
  uint64_t* acc_done = bars + 9;
  uint64_t* drain = bars + 10;
  uint64_t* stage_read = bars + 11;  // [2] the MMAs finished reading Q_i / dO_i of a stage
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int kv_tile = blockIdx.x, head = blockIdx.y;
  const int k0 = kv_tile * kB;
  const int n_q = p.n_q;
  const uint64_t limit = p.status.limit_ns;

  if ((smem_u32(smem) & 1023u) != 0u) {  // the swizzled layouts need a 1024-byte aligned base
    if (threadIdx.x == 0) report_status(p.status, kStatusBadArgument, 1);
    return;
  }
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 2);    // each warpgroup, once its dQ reduces have read the stage
      mbar_init(&stage_read[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 256);
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tDV = tmem, tDK = tmem + 128, tS = tmem + 256, tDP = tmem + 384;

  if (warp == 0) {
    // ------------------------------------------------------------ loads
    if (elect_one()) {
      const int xq = head * kD, xk = p.H + head * kD, xv = 2 * p.H + head * kD;
      mbar_arrive_expect_tx(kv_full, 2 * kTile);
      tma_load_2d(sK, &tm_qkv, kv_full, xk, k0);
      tma_load_2d(sK + kChunk, &tm_qkv, kv_full, xk + 64, k0);
      tma_load_2d(sV, &tm_qkv, kv_full, xv, k0);
      tma_load_2d(sV + kChunk, &tm_qkv, kv_full, xv + 64, k0);
      int issued_phase[2] = {-1, -1};
      for (int i = 0; i < n_q && !*abort_flag; ++i) {
        const int st = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&qd_empty[st], ph ^ 1u, limit, abort_flag)) {
          report_status(p.status, kStatusTimeoutEmpty, i);
          *abort_flag = 1;
          break;
        }
        uint8_t* base = sStage + st * kStageBytes;
        const int y = i * kB;
        mbar_arrive_expect_tx(&qd_full[st], 2 * kTile + 2 * kVecBytes);
        tma_load_2d(base, &tm_qkv, &qd_full[st], xq, y);
        tma_load_2d(base + kChunk, &tm_qkv, &qd_full[st], xq + 64, y);
        tma_load_2d(base + kTile, &tm_do, &qd_full[st], head * kD, y);
        tma_load_2d(base + kTile + kChunk, &tm_do, &qd_full[st], head * kD + 64, y);
        const long vec = static_cast<long>(head) * p.T_pad + y;
        bulk_load(base + 2 * kTile, p.lse2 + vec, kVecBytes, &qd_full[st]);
        bulk_load(base + 2 * kTile + kVecBytes, p.delta + vec, kVecBytes, &qd_full[st]);
        issued_phase[st] = static_cast<int>(ph);
      }
      volatile int never = 0;
      mbar_wait(kv_full, 0, limit, &never);
      for (int st = 0; st < 2; ++st)
        if (issued_phase[st] >= 0) mbar_wait(&qd_full[st], issued_phase[st], limit, &never);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      long long* mtrace = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0) ? p.trace : nullptr;
      bool ok = mbar_wait(kv_full, 0, limit, abort_flag);
      bool any = false;
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV), ds_base = smem_u32(sDS);
      for (int i = 0; ok && i < n_q; ++i) {
        const int st = i & 1;
        if (!mbar_wait(&qd_full[st], (i >> 1) & 1, limit, abort_flag)) { ok = false; break; }
        if (i > 0 && !mbar_wait(dq_empty, (i - 1) & 1, limit, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t q_base = smem_u32(sStage + st * kStageBytes);
        const uint32_t do_base = q_base + kTile;
#pragma unroll
        for (int ds = 0; ds < kD / 16; ++ds) {
          const uint32_t off = (ds >> 2) * kChunk + (ds & 3) * 32;
          umma_f16_ss(tS, umma_smem_desc(k_base + off, 16, 1024), umma_smem_desc(q_base + off, 16, 1024), kIdescSS,
                      ds > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int ds = 0; ds < kD / 16; ++ds) {
          const uint32_t off = (ds >> 2) * kChunk + (ds & 3) * 32;
          umma_f16_ss(tDP, umma_smem_desc(v_base + off, 16, 1024), umma_smem_desc(do_base + off, 16, 1024),
                      kIdescSS, ds > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        any = true;
        if (mtrace) mtrace[i * kBwdTraceSlots + 10] = clock64();
        if (!mbar_wait(p_full, i & 1, limit, abort_flag)) { ok = false; break; }
        if (mtrace) mtrace[i * kBwdTraceSlots + 11] = clock64();
        tc_fence_after();
        // dQ_i = dS K: A = dS (smem, rows = keys, queries contiguous: MN-major), B = K (MN-major), N = 64 halves.
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t d_tmem = (half == 0 ? tS : tDP) + 64;
#pragma unroll
          for (int ks = 0; ks < kB / 16; ++ks) {
            umma_f16_ss(d_tmem, umma_smem_desc(ds_base + ks * 2048, kChunk, 1024),
                        umma_smem_desc(k_base + half * kChunk + ks * 2048, kChunk, 1024), kIdescQ, ks > 0 ? 1u : 0u);
          }
        }
        umma_commit(dq_full);
        // dV += P^T dO_i ; dK += dS^T Q_i   (A from TMEM)
#pragma unroll
        for (int ks = 0; ks < kB / 16; ++ks)
          umma_f16_ts(tDV, tS + ks * 8, umma_smem_desc(do_base + ks * 2048, kChunk, 1024), kIdescTS,
                      (i > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < kB / 16; ++ks)
          umma_f16_ts(tDK, tDP + ks * 8, umma_smem_desc(q_base + ks * 2048, kChunk, 1024), kIdescTS,
                      (i > 0 || ks > 0) ? 1u : 0u);
        umma_commit(&stage_read[st]);
      }
      if (ok) umma_commit(acc_done);
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
    // ------------------------------------------------------------ P^T / dS^T and the dQ reduction
    // Warpgroup `half` (warps 2..5 -> 0, 6..9 -> 1) owns query columns
    // [64*half, 64*half + 64) of every step: it loads all of its S^T / dP^T
    // columns first, then writes P^T / dS^T as packed bf16 into columns
    // [32*half, 32*half + 32) of the same regions.  Warpgroup 1's writes land
    // on columns warpgroup 0 reads, so it waits on named barrier 1 until
    // warpgroup 0's loads completed.  Afterwards each warpgroup adds half of
    // dQ_i (d in [64*half, 64*half + 64)) into the fp32 accumulator.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;  // key (softmax) or query (dQ) row within the tile
    const bool key_valid = k0 + row < p.T;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    const bool reducer = quarter == 0 && lane == 0;   // issues this warpgroup's dQ reduces
    long long* trace = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && half == 0 && reducer)
                           ? p.trace : nullptr;
    for (int i = 0; i < n_q; ++i) {
      const int st = i & 1;
      if (trace) trace[i * kBwdTraceSlots + 0] = clock64();
      if (!mbar_wait(s_full, i & 1, limit, abort_flag)) { ok = false; break; }
      if (trace) trace[i * kBwdTraceSlots + 1] = clock64();
      tc_fence_after();
      const float* lse2 = reinterpret_cast<const float*>(sStage + st * kStageBytes + 2 * kTile);
      const float* delta = lse2 + kB;
      uint32_t rs[2][32], rd[2][32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        tmem_ld32(tS + lane_off + (half * 2 + cc) * 32, rs[cc]);
        tmem_ld32(tDP + lane_off + (half * 2 + cc) * 32, rd[cc]);
      }
      tmem_ld_wait();
      if (trace) trace[i * kBwdTraceSlots + 2] = clock64();
      if (half == 0) {
        asm volatile("bar.arrive 1, 256;" ::: "memory");
      } else {
        asm volatile("bar.sync 1, 256;" ::: "memory");
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;  // 32-query chunk of the step
        uint32_t pp[16], dd[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int q = c * 32 + 2 * j;
          const float xa = fmaf(__uint_as_float(rs[cc][2 * j]), p.scale_log2, -lse2[q]);
          const float xb = fmaf(__uint_as_float(rs[cc][2 * j + 1]), p.scale_log2, -lse2[q + 1]);
          float pa, pb;
          if (p.ablate & 2) {
            pa = xa;
            pb = xb;
          } else {
            pa = (j & 3) == 3 ? exp2_fma(xa) : ex2(xa);
            pb = (j & 3) == 3 ? exp2_fma(xb) : ex2(xb);
          }
          if (!key_valid) pa = pb = 0.f;
          const float da = p.scale * pa * (__uint_as_float(rd[cc][2 * j]) - delta[q]);
          const float db = p.scale * pb * (__uint_as_float(rd[cc][2 * j + 1]) - delta[q + 1]);
          pp[j] = pack_bf16x2(pa, pb);
          dd[j] = pack_bf16x2(da, db);
        }
        tmem_st16(tS + lane_off + c * 16, pp);
        tmem_st16(tDP + lane_off + c * 16, dd);
        // dS^T row into smem: chunk = 64 queries, 16-byte units swizzled by row.
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit_global = c * 4 + u;
          const int chunk = unit_global >> 3, unit = unit_global & 7;
          uint4 v;
          v.x = dd[u * 4 + 0];
          v.y = dd[u * 4 + 1];
          v.z = dd[u * 4 + 2];
          v.w = dd[u * 4 + 3];
          *reinterpret_cast<uint4*>(sDS + chunk * kChunk + row * 128 + ((unit ^ (row & 7)) << 4)) = v;
        }
      }
      tmem_st_wait();
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
      if (trace) trace[i * kBwdTraceSlots + 4] = clock64();
      // dQ_i (rows = queries): this warpgroup's 64 columns as two 32-column fp32
      // boxes, staged in the 128B-swizzled layout in the stage that held Q_i
      // (warpgroup 0) or dO_i (warpgroup 1) -- free once the dV / dK MMAs read
      // it -- and added into the accumulator by TMA bulk reduces whose smem
      // reads are waited for only one step later, after that step's softmax.
      if (reducer && i > 0) {
        // The previous step's reduces read their stage while this step's
        // MMAs and softmax ran; once read, the loader may refill that stage.
        bulk_wait_read_all();
        mbar_arrive(&qd_empty[(i - 1) & 1]);
      }
      if (trace) trace[i * kBwdTraceSlots + 5] = clock64();
      if (!mbar_wait(dq_full, i & 1, limit, abort_flag)) { ok = false; break; }
      if (trace) trace[i * kBwdTraceSlots + 6] = clock64();
      tc_fence_after();
      // Read this warpgroup's 64 dQ columns into registers and hand the TMEM
      // columns back at once: the next step's S^T / dP^T MMAs overwrite them,
      // and must not wait for the staging buffer below (that wait put ~1,800
      // cycles on every step's critical path).
      uint32_t rq[2][32];
      {
        const uint32_t src = (half == 0 ? tS : tDP) + 64 + lane_off;
        tmem_ld32(src, rq[0]);
        tmem_ld32(src + 32, rq[1]);
        tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(dq_empty);
      if (trace) trace[i * kBwdTraceSlots + 9] = clock64();
      if (!mbar_wait(&stage_read[st], (i >> 1) & 1, limit, abort_flag)) { ok = false; break; }
      if (trace) trace[i * kBwdTraceSlots + 7] = clock64();
      if (!(p.ablate & 1)) {
        uint8_t* stage = sStage + st * kStageBytes + half * kTile;
#pragma unroll
        for (int box = 0; box < 2; ++box) {
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            uint4 v;
            v.x = rq[box][u * 4];
            v.y = rq[box][u * 4 + 1];
            v.z = rq[box][u * 4 + 2];
            v.w = rq[box][u * 4 + 3];
            *reinterpret_cast<uint4*>(stage + box * (kTile / 2) + row * 128 + ((u ^ (row & 7)) << 4)) = v;
          }
        }
        fence_async_smem();
        named_sync(2 + half, 128);
        if (trace) trace[i * kBwdTraceSlots + 8] = clock64();
        if (reducer) {
          tma_reduce_add_2d(&tm_dq, stage, head * kD + half * 64, i * kB);
          tma_reduce_add_2d(&tm_dq, stage + kTile / 2, head * kD + half * 64 + 32, i * kB);
        }
      }
    }
    if (reducer) {
      bulk_wait_read_all();   // no reduce still reads this CTA's smem at exit
      if (ok && n_q > 0) mbar_arrive(&qd_empty[(n_q - 1) & 1]);
    }
    // final dV (warpgroup 0) / dK (warpgroup 1) rows -> dqkv
    if (ok && n_q > 0 && mbar_wait(acc_done, 0, limit, abort_flag)) {
      tc_fence_after();
      const long key = k0 + row;
      const uint32_t src = (half == 0 ? tDV : tDK) + lane_off;
      const long dst_off = key * 3 * p.H + (half == 0 ? 2 : 1) * p.H + head * kD;
      __nv_bfloat16* dst = p.dqkv + dst_off;
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(src + c * 32, r);
        tmem_ld_wait();
        if (key_valid && H3_IN_BOUNDS(dst_off + c * 32, dst_off + c * 32 + 31, p.dqkv_extent, p.status)) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(r[u * 8 + 0]), __uint_as_float(r[u * 8 + 1]));
            v.y = pack_bf16x2(__uint_as_float(r[u * 8 + 2]), __uint_as_float(r[u * 8 + 3]));
            v.z = pack_bf16x2(__uint_as_float(r[u * 8 + 4]), __uint_as_float(r[u * 8 + 5]));
            v.w = pack_bf16x2(__uint_as_float(r[u * 8 + 6]), __uint_as_float(r[u * 8 + 7]));
            reinterpret_cast<uint4*>(dst + c * 32)[u] = v;
          }
        }
      }
    } else if (n_q > 0) {
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

at::Tensor attention_bwd(const at::Tensor& qkv, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dout,
                         int64_t heads, int64_t head_dim, const at::Tensor& status, int64_t limit_ns,
                         const c10::optional<at::Tensor>& trace) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous(), "qkv must be contiguous bf16");
  TORCH_CHECK(o.is_contiguous() && dout.is_contiguous() && o.scalar_type() == at::kBFloat16 &&
                  dout.scalar_type() == at::kBFloat16, "o and do must be contiguous bf16");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous(), "lse must be contiguous fp32");
  TORCH_CHECK(head_dim == kD, "attention_bwd supports head_dim 128");
  const int64_t T = qkv.size(0), H = heads * head_dim;
  TORCH_CHECK(qkv.size(1) == 3 * H && o.size(0) == T && o.size(1) == H && dout.sizes() == o.sizes(), "shapes");
  TORCH_CHECK(lse.size(0) == heads && lse.size(1) == T, "lse must be [heads, T]");
  const int device = qkv.get_device();
  c10::cuda::CUDAGuard guard(device);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(device).stream();
  auto dqkv = at::empty_like(qkv);
  if (T == 0) return dqkv;
  const int64_t T_pad = (T + kB - 1) / kB * kB;
  auto lse2 = at::empty({heads, T_pad}, lse.options());
  auto delta = at::empty({heads, T_pad}, lse.options());
  auto dq_acc = at::zeros({T, H}, lse.options());
  {
    const long warps = heads * T_pad;
    const int threads = 256;
    attn_bwd_prep_kernel<<<static_cast<unsigned>((warps * 32 + threads - 1) / threads), threads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        lse.data_ptr<float>(), static_cast<int>(T), static_cast<int>(T_pad), static_cast<int>(H),
        static_cast<int>(heads), lse2.data_ptr<float>(), delta.data_ptr<float>());
    note_launch();
  }
  CUtensorMap tm_qkv = attn_map_2d(qkv.data_ptr(), T, 3 * H, qkv.stride(0));
  CUtensorMap tm_do = attn_map_2d(dout.data_ptr(), T, H, dout.stride(0));
  BwdParams p{};
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.T_pad = static_cast<int>(T_pad);
  p.n_q = static_cast<int>(T_pad / kB);
  p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)));
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(head_dim)));
  p.lse2 = lse2.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.dqkv_extent = extent_of(dqkv);
  if (const char* ab = std::getenv("H3_ATTN_BWD_ABLATE")) p.ablate = std::atoi(ab);
  p.status.word = status.data_ptr<int>();
  p.status.limit_ns = static_cast<uint64_t>(limit_ns);
  p.trace = nullptr;
  if (trace.has_value()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong &&
                    trace->numel() >= static_cast<int64_t>(p.n_q) * kBwdTraceSlots,
                "trace must be a CUDA int64 tensor of n_q * ", kBwdTraceSlots, " entries");
    p.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  static bool configured[64] = {false};
  if (!configured[device]) {
    cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    configured[device] = true;
  }
  dim3 grid(static_cast<unsigned>(T_pad / kB), static_cast<unsigned>(heads));
  CUtensorMap tm_dq = make_map_f32(dq_acc.data_ptr(), T, H, H, kB);
  attn_bwd_kernel<<<grid, kThreads, kSmem, stream>>>(tm_qkv, tm_do, tm_dq, p);
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  {
    const long n4 = T * H / 4;
    attn_bwd_finish_kernel<<<static_cast<unsigned>(std::min<long>((n4 + 255) / 256, 148L * 16)), 256, 0, stream>>>(
        dq_acc.data_ptr<float>(), static_cast<int>(T), static_cast<int>(H),
        reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()));
    note_launch();
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

}  // namespace h3
