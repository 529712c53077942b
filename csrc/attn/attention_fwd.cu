// Bidirectional multi-head attention forward on tcgen05 (sm_100a).
//
//   o[t, h*D:(h+1)*D] = softmax(q_h k_h^T / sqrt(D)) v_h,  lse[h, t] = log-sum-exp of the row
//
// q, k, v are read in place from the fused QKV output [T, 3H] (bf16, RoPE
// already applied by the QKV GEMM epilogue); o is [T, H] bf16, lse fp32.
// Head dim D = 128.
//
// One CTA per (pair of 128-query tiles, head), 384 threads:
//   warp 0      TMA: Q_0, Q_1 once, then K_0 V_0 K_1 V_1 ... through a ring of
//               five 32 KB slots; a K slot is released as soon as both S MMAs
//               that read it are done, a V slot once both PV MMAs are, so the
//               next tiles' loads start ~1.5 KV steps before they are needed
//   warp 1      tcgen05.mma issuer (one thread), per KV tile j:
//                 S_t = Q_t K_j^T         into TMEM S_t (t = 0, 1)
//                 O_t += P_t V_j          P_t read from TMEM (the .ts form),
//                                         O_t accumulates in TMEM
//               issue order S_0 S_1 | PV_0 S_0' PV_1 S_1' | ..., so the tensor
//               core works on one query tile while the other tile's softmax runs.
//   warps 2..5  softmax of query tile 0, warps 6..9 of query tile 1; one query
//               row per thread.  The row of S_t is read from TMEM once into
//               128 registers; the row max and the row sum each run as eight
//               independent chains (a single accumulator is a 128-deep
//               dependency chain that dominated the softmax time); P = 2^(s - m)
//               is written as packed bf16 pairs back into the first 64 TMEM
//               columns of S_t, where the PV MMA reads it.  O_t is rescaled in TMEM only when some row's max
//               grew by more than 2^8 (warp-uniform decision: tcgen05.ld/st
//               are warp-collective).
// TMEM: S_0 [0,128) S_1 [128,256) O_0 [256,384) O_1 [384,512) fp32 columns.
// Keys past T are masked to -inf; queries past T are computed and not stored.
// Every wait is bounded (see ptx.cuh).  Every TMA load targets one CTA only.
#include <ATen/cuda/CUDAContext.h>
#include <cstdlib>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "../common/extent.h"
#include "../common/ptx.cuh"
#include "../gemm/gemm.h"
#include "attention.h"

namespace h3 {
CUtensorMap attn_map_2d(const void* base, long rows, long cols, long ld);

namespace {

constexpr int kBQ = 128;
constexpr int kBKV = 128;
constexpr int kD = 128;
constexpr int kQTiles = 2;
constexpr int kThreads = 128 + kQTiles * 128;   // producer warpgroup + one softmax warpgroup per tile
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 = 64512),
// the producer warpgroup drops to 72 and each softmax warpgroup rises to 216:
// 128 x 72 + 256 x 216 = 64512, exactly the launch total (checked on the host).
constexpr int kLaunchRegs = 168;
constexpr int kRegsLow = 72;
constexpr int kRegsHigh = 216;
static_assert(128 * kRegsLow + kQTiles * 128 * kRegsHigh == kThreads * kLaunchRegs, "register split");
constexpr int kChunk = 128 * 64 * 2;    // 128 rows x 64 bf16 (one 128B-swizzled column chunk)
constexpr int kTileBytes = 2 * kChunk;  // 128 rows x 128 bf16
constexpr int kSlots = 5;               // K/V ring: K_j in slot 2j % 5, V_j in slot (2j+1) % 5
constexpr int kSmem = 1024 + kTileBytes * (kQTiles + kSlots) + 512;  // Q x2, ring
static_assert(kSmem <= 232448, "attention forward shared memory");
constexpr float kRescaleThreshold = 8.0f;                      // log2 units

struct FwdParams {
  int T, H;
  int n_kv;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* o;
  float* lse;
  // Diagnostic phase trace (null in normal runs): CTA (0, 0) records clock64
  // at each phase of its MMA issuer and of the first lane band's softmax warp
  // of each query tile, plus every softmax warp's P hand-off; kTraceSlots
  // values per (tile, KV step).
  long long* trace;
  long o_extent, lse_extent;   // allocation extents, checked in the bounds-checked build only
  KernelStatus status;
};
constexpr int kTraceSlots = 12;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed f32x2 arithmetic (sm_100): one instruction for two lanes of a pair.
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x on the FMA pipe, to take part of the exponentials off the MUFU unit:
// x = n + f with n = round(x) (magic-number add, no conversion instruction)
// and f in [-1/2, 1/2]; 2^f is a cubic least-squares fit at Chebyshev nodes
// (max relative error 1.0e-4, below bf16 resolution); 2^n is added to the
// exponent field.  Valid for x >= -126 (inputs are clamped).
// Applied to a pair with packed f32x2 arithmetic (one FADD2 / FFMA2 per step
// for both lanes), which halves the issue slots of the FMA-pipe share.
__device__ __forceinline__ void exp2_fma2(float xa, float xb, float& ra, float& rb) {
  const uint64_t x2 = pack2(fmaxf(xa, -126.0f), fmaxf(xb, -126.0f));
  const uint64_t t2 = add2(x2, pack2(12582912.0f, 12582912.0f));     // round to nearest: n in the low bits
  const uint64_t n2 = add2(t2, pack2(-12582912.0f, -12582912.0f));   // n as a float
  const uint64_t f2 = fma2(n2, pack2(-1.0f, -1.0f), x2);              // f = x - n in [-1/2, 1/2]
  uint64_t q2 = fma2(pack2(0.05592203512787819f, 0.05592203512787819f), f2,
                     pack2(0.24264007806777954f, 0.24264007806777954f));
  q2 = fma2(q2, f2, pack2(0.6931210160255432f, 0.6931210160255432f));
  q2 = fma2(q2, f2, pack2(0.9999244809150696f, 0.9999244809150696f));
  float qa, qb, ta, tb;
  unpack2(q2, qa, qb);
  unpack2(t2, ta, tb);
  ra = __int_as_float(__float_as_int(qa) + (__float_as_int(ta) << 23));
  rb = __int_as_float(__float_as_int(qb) + (__float_as_int(tb) << 23));
}

// 32 lanes x 32 bit, 32 consecutive columns per thread.
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

template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Three-input max (sm_100 PTX): halves the max instructions per element.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// One 128-key S row of this thread, loaded from TMEM once (four loads, one wait).
__device__ __forceinline__ void load_row(uint32_t tS, uint32_t (&r)[kBKV / 32][32]) {
#pragma unroll
  for (int c = 0; c < kBKV / 32; ++c) tmem_ld32(tS + c * 32, r[c]);
  tmem_ld_wait();
}

// Keys at or past `valid` get -inf (last KV tile only).
__device__ __forceinline__ void mask_row(uint32_t (&r)[kBKV / 32][32], int valid) {
#pragma unroll
  for (int c = 0; c < kBKV / 32; ++c)
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (c * 32 + i >= valid) r[c][i] = __float_as_uint(-INFINITY);
}

// Row max: eight independent chains of three-input maxes (a single running
// max is a 128-deep dependency chain on the critical path of every KV tile).
__device__ __forceinline__ float row_max(const uint32_t (&r)[kBKV / 32][32]) {
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) m[k] = fmaxf(__uint_as_float(r[0][2 * k]), __uint_as_float(r[0][2 * k + 1]));
#pragma unroll
  for (int c = 0; c < kBKV / 32; ++c)
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (c > 0 || i >= 8)
        m[i & 7] = fmax3(m[i & 7], __uint_as_float(r[c][2 * i]), __uint_as_float(r[c][2 * i + 1]));
  return fmaxf(fmax3(m[0], m[1], m[2]), fmax3(fmax3(m[3], m[4], m[5]), m[6], m[7]));
}

// P = 2^(s*scale - m) from the registers, stored as packed bf16 pairs over the
// first 64 S columns; returns the row sum.  The scale/offset and the sum use
// packed f32x2 instructions (four independent pair accumulators).  POLY of
// every 8 pairs go through the FMA-pipe exponential, the rest to MUFU: MUFU
// takes 8 cycles per warp instruction, so at POLY = 0 the exponentials alone
// are ~1,024 cycles per KV tile and warp, on the softmax's critical path.
template <bool MASKED, int POLY>
__device__ __forceinline__ float row_exp_pack(uint32_t tS, const uint32_t (&r)[kBKV / 32][32], int valid, float scale,
                                              float m) {
  const uint64_t scale2 = pack2(scale, scale), negm2 = pack2(-m, -m);
  uint64_t acc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) acc[k] = 0ull;   // (0.f, 0.f)
#pragma unroll
  for (int c = 0; c < kBKV / 32; ++c) {
    uint32_t packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float xa, xb;
      unpack2(fma2(pack2(__uint_as_float(r[c][2 * i]), __uint_as_float(r[c][2 * i + 1])), scale2, negm2), xa, xb);
      float a, b;
      if ((i & 7) < POLY) {
        exp2_fma2(xa, xb, a, b);
      } else {
        a = ex2(xa);
        b = ex2(xb);
      }
      if (MASKED) {
        const int k0 = c * 32 + 2 * i;
        a = k0 < valid ? a : 0.f;
        b = k0 + 1 < valid ? b : 0.f;
      }
      acc[i & 3] = add2(acc[i & 3], pack2(a, b));
      packed[i] = pack_bf16x2(a, b);
    }
    tmem_st16(tS + c * 16, packed);
  }
  const uint64_t s2 = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
  float sa, sb;
  unpack2(s2, sa, sb);
  return sa + sb;
}

__device__ __forceinline__ int ring_slot(int n) { return n % kSlots; }
__device__ __forceinline__ uint32_t ring_phase(int n) { return static_cast<uint32_t>((n / kSlots) & 1); }

// Producer warpgroup roles: warp 0 issues the TMA loads, warp 1 the MMAs.
// Load sequence n = 0, 1, 2, ...: K_{n/2} for even n, V_{n/2} for odd n.
__device__ __forceinline__ void producer_warps(const CUtensorMap& tm, const FwdParams& p, int warp, uint8_t* sQ,
                                               uint8_t* ring, uint64_t* q_full, uint64_t* slot_full,
                                               uint64_t* slot_empty, uint64_t* s_full, uint64_t* p_full,
                                               uint64_t* o_done, uint64_t* drain, volatile int* abort_flag,
                                               uint32_t tmem, int head, int q0, int n_kv, uint64_t limit) {
  constexpr uint32_t kIdescS = umma_idesc_bf16(kBQ, kBKV, false, false);
  constexpr uint32_t kIdescPV = umma_idesc_bf16(kBQ, kD, false, true);
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      const int xq = head * kD, xk = p.H + head * kD, xv = 2 * p.H + head * kD;
      mbar_arrive_expect_tx(q_full, kQTiles * kTileBytes);
      for (int t = 0; t < kQTiles; ++t) {
        tma_load_2d(sQ + t * kTileBytes, &tm, q_full, xq, q0 + t * kBQ);
        tma_load_2d(sQ + t * kTileBytes + kChunk, &tm, q_full, xq + 64, q0 + t * kBQ);
      }
      int issued_phase[kSlots];
#pragma unroll
      for (int s = 0; s < kSlots; ++s) issued_phase[s] = -1;
      for (int n = 0; n < 2 * n_kv && !*abort_flag; ++n) {
        const int slot = ring_slot(n);
        const uint32_t ph = ring_phase(n);
        if (!mbar_wait(&slot_empty[slot], ph ^ 1u, limit, abort_flag)) {
          report_status(p.status, kStatusTimeoutEmpty, n);
          *abort_flag = 1;
          break;
        }
        const int x = (n & 1) ? xv : xk, y = (n >> 1) * kBKV;
        mbar_arrive_expect_tx(&slot_full[slot], kTileBytes);
        tma_load_2d(ring + slot * kTileBytes, &tm, &slot_full[slot], x, y);
        tma_load_2d(ring + slot * kTileBytes + kChunk, &tm, &slot_full[slot], x + 64, y);
        issued_phase[slot] = static_cast<int>(ph);
      }
      // Never leave a TMA write in flight into this CTA's shared memory.
      volatile int never = 0;
      mbar_wait(q_full, 0, limit, &never);
      for (int s = 0; s < kSlots; ++s)
        if (issued_phase[s] >= 0) mbar_wait(&slot_full[s], issued_phase[s], limit, &never);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      long long* mtrace = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0) ? p.trace : nullptr;
      bool any = false;
      bool ok = mbar_wait(q_full, 0, limit, abort_flag);
      auto wait_slot = [&](int n) { return mbar_wait(&slot_full[ring_slot(n)], ring_phase(n), limit, abort_flag); };
      auto issue_s = [&](int t, int j) {
        const uint32_t q_base = smem_u32(sQ + t * kTileBytes);
        const uint32_t k_base = smem_u32(ring + ring_slot(2 * j) * kTileBytes);
#pragma unroll
        for (int ds = 0; ds < kD / 16; ++ds) {
          const uint32_t off = (ds >> 2) * kChunk + (ds & 3) * 32;
          umma_f16_ss(tmem + t * 128, umma_smem_desc(q_base + off, 16, 1024), umma_smem_desc(k_base + off, 16, 1024),
                      kIdescS, ds > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
        any = true;
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t v_base = smem_u32(ring + ring_slot(2 * j + 1) * kTileBytes);
        const uint32_t p_tmem = tmem + t * 128;          // packed bf16 P in the first 64 S columns
        const uint32_t o_tmem = tmem + 256 + t * 128;
#pragma unroll
        for (int ks = 0; ks < kBKV / 16; ++ks) {
          umma_f16_ts(o_tmem, p_tmem + ks * 8, umma_smem_desc(v_base + ks * 2048, kChunk, 1024), kIdescPV,
                      (j > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[t]);
      };
      if (ok && n_kv > 0) {
        ok = wait_slot(0);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < kQTiles; ++t) issue_s(t, 0);
          umma_commit(&slot_empty[ring_slot(0)]);        // K_0 read by both S MMAs
        }
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const bool more = j + 1 < n_kv;
        for (int t = 0; t < kQTiles && ok; ++t) {
          if (!mbar_wait(&p_full[t], j & 1, limit, abort_flag) || (t == 0 && !wait_slot(2 * j + 1))) {
            ok = false;
            break;
          }
          if (mtrace) mtrace[(static_cast<long>(t) * n_kv + j) * kTraceSlots + 6] = clock64();
          tc_fence_after();
          issue_pv(t, j);
          if (t == kQTiles - 1) umma_commit(&slot_empty[ring_slot(2 * j + 1)]);   // V_j consumed
          if (more) {
            if (t == 0 && !wait_slot(2 * j + 2)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(t, j + 1);
            if (mtrace) mtrace[(static_cast<long>(t) * n_kv + j) * kTraceSlots + 7] = clock64();
            if (t == kQTiles - 1) umma_commit(&slot_empty[ring_slot(2 * j + 2)]);  // K_{j+1} consumed
          }
        }
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
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int POLY>
__global__ void __launch_bounds__(kThreads, 1) attn_fwd_kernel(const __grid_constant__ CUtensorMap tm, FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                        // kQTiles tiles
  uint8_t* ring = sQ + kQTiles * kTileBytes; // kSlots K/V slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kSlots * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* slot_full = bars + 1;                // [kSlots]
  uint64_t* slot_empty = slot_full + kSlots;     // [kSlots]
  uint64_t* s_full = slot_empty + kSlots;        // [kQTiles]
  uint64_t* p_full = s_full + kQTiles;           // [kQTiles]
  uint64_t* o_done = p_full + kQTiles;           // [kQTiles]
  uint64_t* drain = o_done + kQTiles;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int head = blockIdx.y;
  const int q0 = blockIdx.x * (kQTiles * kBQ);
  const int n_kv = p.n_kv;
  const uint64_t limit = p.status.limit_ns;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&slot_full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    for (int t = 0; t < kQTiles; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
    }
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
  if (warp < 4) {
    // Producer warpgroup: warp 0 TMA, warp 1 MMA issuer, warps 2-3 idle.
    setmaxnreg_dec<kRegsLow>();
    producer_warps(tm, p, warp, sQ, ring, q_full, slot_full, slot_empty, s_full, p_full, o_done, drain, abort_flag,
                   tmem, head, q0, n_kv, limit);
    tc_fence_before();
    named_bar_sync(1, kThreads);
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, 512);
    }
    return;
  }
  setmaxnreg_inc<kRegsHigh>();
  // ------------------------------------------------------------ softmax (two warpgroups)
  const int t = (warp - 4) >> 2;           // query tile handled by this warpgroup
  const int quarter = warp & 3;            // TMEM lane quarter this warp may access
  const int row = quarter * 32 + lane;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const uint32_t tS = tmem + t * 128 + lane_off;
  const uint32_t tO = tmem + 256 + t * 128 + lane_off;
  float m_used = -INFINITY, l = 0.f;
  bool ok = true;
  long long* trace_band = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && lane == 0)
                             ? p.trace + static_cast<long>(t) * n_kv * kTraceSlots
                             : nullptr;
  long long* trace = quarter == 0 ? trace_band : nullptr;
  for (int j = 0; j < n_kv; ++j) {
    if (trace) trace[j * kTraceSlots + 0] = clock64();
    // O_t may be rescaled once PV_t of the previous tile completed (the
    // commit order already implies it: S_t(j) was issued after PV_t(j-1)).
    // Warp-uniform outcome: tcgen05.ld/st below are warp-collective.
    ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, limit, abort_flag) &&
                                     (j == 0 || mbar_wait(&o_done[t], (j - 1) & 1, limit, abort_flag)));
    if (!ok) break;
    if (trace) trace[j * kTraceSlots + 1] = clock64();
    tc_fence_after();
    const int kv_valid = p.T - j * kBKV;
    // One TMEM read of the row; the max uses raw scores (the scale is positive).
    uint32_t r[kBKV / 32][32];
    load_row(tS, r);
    if (kv_valid < kBKV) mask_row(r, kv_valid);
    if (trace) trace[j * kTraceSlots + 2] = clock64();
    const float m_tile = row_max(r) * p.scale_log2;
    const float m_new = fmaxf(m_used, m_tile);
    const bool need = (j == 0) || (m_new > m_used + kRescaleThreshold);
    const bool warp_need = __any_sync(0xffffffffu, need);
    const float alpha = need ? ex2(m_used - m_new) : 1.f;
    if (need) {
      l *= alpha;
      m_used = m_new;
    }
    if (trace) trace[j * kTraceSlots + 3] = clock64();
    tc_fence_after();
    // P = 2^(s*scale - m) as packed bf16 pairs over the consumed S columns.
    const float rowsum = kv_valid >= kBKV ? row_exp_pack<false, POLY>(tS, r, kv_valid, p.scale_log2, m_used)
                                          : row_exp_pack<true, POLY>(tS, r, kv_valid, p.scale_log2, m_used);
    l += rowsum;
    if (trace) trace[j * kTraceSlots + 4] = clock64();
    // Rescale O_t after P is written (the S registers are dead by then, so
    // the O chunk does not push the row past the register budget); PV_t(j)
    // is issued only after p_full, i.e. after this.
    if (warp_need && j > 0) {
#pragma unroll
      for (int c = 0; c < kD / 16; ++c) {
        uint32_t o[16];
        tmem_ld16(tO + c * 16, o);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
        tmem_st16(tO + c * 16, o);
      }
    }
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive(&p_full[t]);
    if (trace_band) trace_band[j * kTraceSlots + (quarter == 0 ? 5 : 7 + quarter)] = clock64();
  }
  const int q = q0 + t * kBQ + row;
  const bool done = __all_sync(0xffffffffu, ok && n_kv > 0 && mbar_wait(&o_done[t], (n_kv - 1) & 1, limit, abort_flag));
  if (done) {
    tc_fence_after();
    const float inv_l = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int c = 0; c < kD / 16; ++c) {
      uint32_t r[16];
      tmem_ld16(tO + c * 16, r);
      tmem_ld_wait();
      const long o_off = static_cast<long>(q) * p.H + head * kD + c * 16;
      if (q < p.T && H3_IN_BOUNDS(o_off, o_off + 15, p.o_extent, p.status)) {
        uint4 a, b;
        a.x = pack_bf16x2(__uint_as_float(r[0]) * inv_l, __uint_as_float(r[1]) * inv_l);
        a.y = pack_bf16x2(__uint_as_float(r[2]) * inv_l, __uint_as_float(r[3]) * inv_l);
        a.z = pack_bf16x2(__uint_as_float(r[4]) * inv_l, __uint_as_float(r[5]) * inv_l);
        a.w = pack_bf16x2(__uint_as_float(r[6]) * inv_l, __uint_as_float(r[7]) * inv_l);
        b.x = pack_bf16x2(__uint_as_float(r[8]) * inv_l, __uint_as_float(r[9]) * inv_l);
        b.y = pack_bf16x2(__uint_as_float(r[10]) * inv_l, __uint_as_float(r[11]) * inv_l);
        b.z = pack_bf16x2(__uint_as_float(r[12]) * inv_l, __uint_as_float(r[13]) * inv_l);
        b.w = pack_bf16x2(__uint_as_float(r[14]) * inv_l, __uint_as_float(r[15]) * inv_l);
        uint4* dst = reinterpret_cast<uint4*>(p.o + o_off);
        dst[0] = a;
        dst[1] = b;
      }
    }
    const long lse_off = static_cast<long>(head) * p.T + q;
    if (q < p.T && H3_IN_BOUNDS(lse_off, lse_off, p.lse_extent, p.status))
      p.lse[lse_off] = (m_used + __log2f(l)) * 0.6931471805599453f;
  } else if (n_kv > 0) {
    if (lane == 0) report_status(p.status, kStatusTimeoutAccFull, blockIdx.x);
    *abort_flag = 1;
  }

  tc_fence_before();
  named_bar_sync(1, kThreads);
}

}  // namespace

std::vector<at::Tensor> attention_fwd(const at::Tensor& qkv, int64_t heads, int64_t head_dim, const at::Tensor& status,
                                      int64_t limit_ns, const c10::optional<at::Tensor>& trace) {
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
  p.o_extent = extent_of(o);
  p.lse_extent = extent_of(lse);
  p.status.word = status.data_ptr<int>();
  p.status.limit_ns = static_cast<uint64_t>(limit_ns);
  p.trace = nullptr;
  if (trace.has_value()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong &&
                    trace->numel() >= static_cast<int64_t>(kQTiles) * p.n_kv * kTraceSlots,
                "trace must be a CUDA int64 tensor of 2 * n_kv * ", kTraceSlots, " entries");
    p.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  static bool configured[64] = {false};
  const int device = qkv.get_device();
  if (!configured[device]) {
    for (auto fn : {attn_fwd_kernel<0>, attn_fwd_kernel<4>}) {
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      // setmaxnreg.inc waits until the producer warpgroup has released enough
      // registers; that only balances if the launch count is the assumed one.
      cudaFuncAttributes attr{};
      C10_CUDA_CHECK(cudaFuncGetAttributes(&attr, fn));
      TORCH_CHECK(attr.numRegs == kLaunchRegs, "attention forward compiled with ", attr.numRegs,
                  " registers per thread; the register split assumes ", kLaunchRegs);
    }
    configured[device] = true;
  }
  // Exponentials: 0 = MUFU only, 4 = four of every 8 pairs on the FMA pipe
  // (measured slower at this issue rate; so was a packed bf16x2 MUFU form).
  // H3_ATTN_FWD_POLY selects it for measurements only.
  static const int poly = [] {
    const char* v = std::getenv("H3_ATTN_FWD_POLY");
    return v != nullptr ? std::atoi(v) : 0;
  }();
  dim3 grid(static_cast<unsigned>((T + kQTiles * kBQ - 1) / (kQTiles * kBQ)), static_cast<unsigned>(heads));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(device).stream();
  switch (poly) {
    case 4: attn_fwd_kernel<4><<<grid, kThreads, kSmem, stream>>>(tm, p); break;
    default: attn_fwd_kernel<0><<<grid, kThreads, kSmem, stream>>>(tm, p); break;
  }
  note_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, lse};
}

}  // namespace h3
