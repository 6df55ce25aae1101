// Flash-attention forward for sm_100a: out = softmax(scale * Q K^T) V per head, bf16 in / bf16 out, head_dim 128,
// fp32 accumulation in TMEM. Q [Tq, H, 128], K and V [Tk, H, 128] (token rows of any 16-byte-multiple stride,
// heads contiguous within a row); out [Tq, H, 128] contiguous.
//
// One CTA per (256 queries, head, key range), 384 threads. The CTA holds two query tiles Q_0, Q_1 of 128 rows,
// so every K / V block it loads feeds both (half the operand traffic per query of a 128-query CTA):
//   warps 0..3  softmax of tile 0, warps 4..7 of tile 1 (one thread per query row; TMEM lane = row).
//               Per block: load S (128 fp32 columns), row maximum, *lazy rescaling* (the running maximum
//               only moves when the block maximum exceeds it by more than 8 in log2 units, i.e. p <= 256;
//               then the row of O is rescaled in TMEM), P = exp2(scale * log2(e) * s - m) packed to bf16
//               pairs and stored back into TMEM over the first 64 columns of S, where the P V MMA reads
//               it as its A operand (tcgen05.mma with A in TMEM): P never touches shared memory.
//               The two warpgroups take turns on their exponential phases (named barriers).
//   warp 8      TMA producer: lane 0 loads Q_0 and Q_1 once and the K_j blocks of 128 keys into a 3-stage
//               ring, lane 1 the V_j blocks into a 2-stage ring.
//   warp 9      TMEM owner; lane 0 issues the MMAs. Per block j, in this order:
//                 O_0 += P_0(j-1) V_(j-1),  S_0 = Q_0 K_j^T,  O_1 += P_1(j-1) V_(j-1),  S_1 = Q_1 K_j^T
//               so the tensor core computes one tile's products while the other tile's softmax runs.
//               The next S MMA into the columns of P is issued after that P V MMA; tcgen05.mma operations
//               issued by one thread execute in issue order, so P is read before S is overwritten.
//   warps 10-11 idle (they complete the third warpgroup, which hands registers to the softmax warpgroups
//               with setmaxnreg: 88 per thread there, 208 in the softmax warpgroups).
// TMEM (512 columns): S_g at 128 g (P_g in its first 64 columns), O_g at 256 + 128 g.
//
// Key ranges (blockIdx.z): when one CTA per (256 queries, head) would leave the last wave of SMs mostly
// idle, the host splits the keys into ranges; each range writes its normalized partial output and
// log2-sum-exp in FP32 and a merge kernel combines them (the standard split-softmax combination).
//
// V is transposed once per call into V^T [H, 128, Tk_pad] so both GEMMs read K-major operands.
// Every wait is bounded (2 s): on expiry a status code is recorded, the loops stop, the MMA thread drains
// its MMAs (bounded) and TMEM is freed.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace rc {
namespace attn {

constexpr int kD = 128;
constexpr int kBM = 128;        // rows of one query tile
constexpr int kTilesPerCta = 2; // query tiles sharing each K / V block
constexpr int kBN = 128;        // keys per block
constexpr int kThreads = 384;   // two softmax warpgroups, then producer, MMA and two idle warps
// Register split: the kernel launches at kLaunchRegs per thread (checked on the host against the compiled count);
// the producer / MMA warpgroup drops to kRoleRegs and each softmax warpgroup rises to kSoftmaxRegs, enough for a
// whole row of 128 scores and its 64 bf16 pairs. The shares add up to exactly what the launch holds.
constexpr int kLaunchRegs = 168;
constexpr int kSoftmaxRegs = 208;
constexpr int kRoleRegs = 88;
static_assert(2 * kSoftmaxRegs + kRoleRegs == 3 * kLaunchRegs, "register split must equal the launch's registers");
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kBox = 128 * 64 * 2;     // one [128 rows x 64 cols] bf16 box: 16 KB
constexpr int kTileBytes = 2 * kBox;   // a 128 x 128 operand tile: 32 KB
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kTilesPerCta * kTileBytes;
constexpr int kVOff = kKOff + kKStages * kTileBytes;
constexpr int kBarOff = kVOff + kVStages * kTileBytes;
constexpr int kSmemBytes = kBarOff + 256 + 1024;  // + barriers + alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// option bits of a launch
constexpr int kOptSplitMask = 15;  // key ranges per (query pair, head); 0 = chosen by the host
constexpr int kOptPoly = 16;       // an eighth of the exponentials on the FMA pipe (exp2_fma)
constexpr int kOptTrace = 32;      // clock64 timeline of CTA (0, 0, 0) into `trace` (measurement only)
constexpr int kTraceBlocks = 32;   // blocks traced
constexpr int kTraceEvents = 16;   // events per block
constexpr int kOptNoTurns = 128;   // softmax warpgroups run their exponentials without taking turns
constexpr int kBarTurn = 1;        // named barriers 1 and 2: the softmax warpgroups' turns

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void named_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int kRegs>
__device__ __forceinline__ void regs_raise() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}

template <int kRegs>
__device__ __forceinline__ void regs_lower() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}

static_assert(kSmemBytes <= 227 * 1024, "shared memory of one CTA");

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for x <= 0 on the FMA/ALU pipes: x = n + f with n = rint(x) taken from the low mantissa bits of
// x + 1.5 * 2^23 (Cody-Waite style reduction), f in [-0.5, 0.5], 2^f by a cubic least-squares fit at Chebyshev
// nodes (relative error < 8e-5, far below the bfloat16 rounding of P), and 2^n added to the exponent field.
// x is clamped at -125 (the result stays normal).
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -125.0f);
  const float t = __fadd_rn(x, 12582912.0f);
  const float n = __fsub_rn(t, 12582912.0f);
  const float f = __fsub_rn(x, n);
  const float p = fmaf(fmaf(fmaf(0.05508868f, f, 0.24260405f), f, 0.69327623f), f, 0.99992895f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

// Online-softmax step of one 128-key block for this thread's row: r holds the block's raw scores (fp32 bits, keys
// past Tk already -inf), m_run the running maximum (log2 domain, already scaled). Writes the 64 bf16 pairs of P
// into pk and returns their sum. Every kPolyEvery-th pair takes its exponentials from the FMA pipe.
template <int kPolyEvery>
__device__ __forceinline__ float softmax_row(const uint32_t (&r)[2][64], float scale_log2, float m_run,
                                             uint32_t (&pk)[2][32]) {
  const float neg_m = -m_run;
  float ps[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int c = 0; c < 64; ++c) {
    const int e0 = 2 * c, e1 = 2 * c + 1;
    const float x0 = fmaf(__uint_as_float(r[e0 >> 6][e0 & 63]), scale_log2, neg_m);
    const float x1 = fmaf(__uint_as_float(r[e1 >> 6][e1 & 63]), scale_log2, neg_m);
    float p0, p1;
    if (kPolyEvery > 0 && (c % (kPolyEvery > 0 ? kPolyEvery : 1)) == kPolyEvery - 1) {
      p0 = exp2_fma(x0);
      p1 = exp2_fma(x1);
    } else {
      p0 = fast_exp2(x0);
      p1 = fast_exp2(x1);
    }
    ps[(2 * c) & 7] += p0;
    ps[(2 * c + 1) & 7] += p1;
    pk[c >> 5][c & 31] = pack_bf16x2(p0, p1);
  }
  return ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
}

template <int kPolyEvery>
__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmVt, int Tq, int Tk, int H, float scale_log2,
                         int blocks_per_range, __nv_bfloat16* __restrict__ out, int64_t out_row,
                         float* __restrict__ part_o, float* __restrict__ part_lse, int* status, int options,
                         long long* __restrict__ trace) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                 // [kKStages]
  uint64_t* k_empty = k_full + kKStages;       // [kKStages]
  uint64_t* v_full = k_empty + kKStages;       // [kVStages]
  uint64_t* v_empty = v_full + kVStages;       // [kVStages]
  uint64_t* s_full = v_empty + kVStages;       // [2] per query tile
  uint64_t* p_full = s_full + 2;               // [2]
  uint64_t* o_done = p_full + 2;               // [2]
  uint64_t* drained = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * (kTilesPerCta * kBM);
  const int h = blockIdx.y;
  const int range = blockIdx.z;
  const int blocks_total = (Tk + kBN - 1) / kBN;
  const int jb = range * blocks_per_range;
  const int nblk = min(blocks_total, jb + blocks_per_range) - jb;  // >= 1 (the host leaves no empty range)
  const bool tracing = trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
  auto stamp = [&](int i, int e) {
    if (tracing && i < kTraceBlocks) trace[i * kTraceEvents + e] = clock64();
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int b = 0; b < kKStages; ++b) {
      mbar_init(&k_full[b], 1);
      mbar_init(&k_empty[b], 1);
    }
    for (int b = 0; b < kVStages; ++b) {
      mbar_init(&v_full[b], 1);
      mbar_init(&v_empty[b], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 4);
      mbar_init(&o_done[g], 1);
    }
    mbar_init(drained, 1);
    fence_barrier_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmVt);
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= 8) {
   // ---------------- warpgroup 2: producer, MMA issuer, two idle warps ----------------
   regs_lower<kRoleRegs>();
   if (warp == kProducerWarp) {
    // ---------------- TMA producer: lane 0 streams Q and K, lane 1 streams V^T ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kTilesPerCta * kTileBytes);
      for (int g = 0; g < kTilesPerCta; ++g) {
        tma_load_3d(smem + kQOff + g * kTileBytes, &tmQ, q_full, 0, h, q0 + g * kBM);
        tma_load_3d(smem + kQOff + g * kTileBytes + kBox, &tmQ, q_full, 64, h, q0 + g * kBM);
      }
      for (int i = 0; i < nblk; ++i) {
        const int s = i % kKStages;
        if (!mbar_wait_park(&k_empty[s], ((i / kKStages) & 1) ^ 1, status, kTimeoutProducer)) break;
        uint8_t* kd = smem + kKOff + s * kTileBytes;
        mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        tma_load_3d(kd, &tmK, &k_full[s], 0, h, (jb + i) * kBN);
        tma_load_3d(kd + kBox, &tmK, &k_full[s], 64, h, (jb + i) * kBN);
      }
    } else if (lane == 1) {
      for (int i = 0; i < nblk; ++i) {
        const int s = i % kVStages;
        if (!mbar_wait_park(&v_empty[s], ((i / kVStages) & 1) ^ 1, status, kTimeoutProducer)) break;
        uint8_t* vd = smem + kVOff + s * kTileBytes;
        mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        tma_load_3d(vd, &tmVt, &v_full[s], (jb + i) * kBN, 0, h);
        tma_load_3d(vd + kBox, &tmVt, &v_full[s], (jb + i) * kBN + 64, 0, h);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer (lane 0) ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(kBM, kBN, /*bf16*/ 1);
      bool ok = mbar_wait_park(q_full, 0, status, kTimeoutMma);
      tc_fence_after();
      const uint32_t qa = smem_u32(smem + kQOff);
      auto issue_s = [&](int i, int g) {  // S_g = Q_g K_i^T, then signal the softmax of tile g
        const uint32_t ka = smem_u32(smem + kKOff + (i % kKStages) * kTileBytes);
        const uint32_t qg = qa + g * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t box = (kk >> 2) * kBox;
          mma_f16(tmem_base + g * kBN, sw128_kmajor_desc(qg + box) + 2 * (kk & 3),
                  sw128_kmajor_desc(ka + box) + 2 * (kk & 3), idesc, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[g]);
      };
      auto issue_pv = [&](int i, int g) {  // O_g += P_g V_i with P_g in TMEM (8 columns per 16 keys)
        const uint32_t va = smem_u32(smem + kVOff + (i % kVStages) * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t box = (kk >> 2) * kBox;
          mma_f16_ts(tmem_base + 256 + g * kD, tmem_base + g * kBN + kk * 8,
                     sw128_kmajor_desc(va + box) + 2 * (kk & 3), idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
      };
      auto wait_pv_inputs = [&](int i, int g, bool need_v) -> bool {
        if (need_v && !mbar_wait_park(&v_full[i % kVStages], (i / kVStages) & 1, status, kTimeoutMma)) return false;
        if (!mbar_wait_park(&p_full[g], i & 1, status, kTimeoutMma)) return false;
        tc_fence_after();
        return true;
      };
      for (int i = 0; i < nblk && ok; ++i) {
        const int ks = i % kKStages;
        ok = mbar_wait_park(&k_full[ks], (i / kKStages) & 1, status, kTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        stamp(i, 8);
        if (i > 0) {
          ok = wait_pv_inputs(i - 1, 0, true);
          if (!ok) break;
          stamp(i, 9);
          issue_pv(i - 1, 0);
        }
        issue_s(i, 0);
        stamp(i, 10);
        if (i > 0) {
          ok = wait_pv_inputs(i - 1, 1, false);
          if (!ok) break;
          stamp(i, 11);
          issue_pv(i - 1, 1);
          mma_commit(&v_empty[(i - 1) % kVStages]);
        }
        issue_s(i, 1);
        stamp(i, 12);
        mma_commit(&k_empty[ks]);
      }
      if (ok) {
        const int i = nblk - 1;
        ok = wait_pv_inputs(i, 0, true);
        if (ok) {
          issue_pv(i, 0);
          mma_commit(&o_done[0]);
          ok = wait_pv_inputs(i, 1, false);
        }
        if (ok) {
          issue_pv(i, 1);
          mma_commit(&o_done[1]);
          mma_commit(&v_empty[i % kVStages]);
        }
      }
      mma_commit(drained);
      (void)mbar_wait_park(drained, 0, nullptr, 0);
    }
    __syncwarp();
   }
  } else {
    // ---------------- softmax warpgroups: warpgroup g owns query tile g ----------------
    regs_raise<kSoftmaxRegs>();
    const int g = warp >> 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_col = tmem_base + g * kBN + lane_addr;
    const uint32_t o_col = tmem_base + 256 + g * kD + lane_addr;
    const bool tr = lane == 0 && quarter == 0;  // first warp of each warpgroup
    const int ev = 4 * g;
    // Turn taking: warpgroup g runs the exponentials of a block only after the other warpgroup finished those of
    // its previous block (named barriers kBarTurn + g, 256 threads: g's 128 wait, the other's 128 arrive), so the
    // two tiles' exponential phases alternate at the full rate of the exp units instead of overlapping at half
    // of it, and the tensor core works on one tile while the other tile's softmax runs. Every warp takes part in
    // every turn even after a failed wait (it then skips the work), so no warp is left waiting on a barrier.
    const bool turns = (options & kOptNoTurns) == 0;
    if (turns && g == 1) named_arrive(kBarTurn, 2 * kBM);  // warpgroup 0 goes first
    float m_run = -INFINITY;  // running max of scale * log2(e) * s
    float l_run = 0.0f;
    bool ok = true;
    for (int i = 0; i < nblk; ++i) {
      uint32_t r[2][64];
      float mx = 0.0f;
      if (ok) {
        if (lane == 0) ok = mbar_wait_park(&s_full[g], i & 1, status, kTimeoutEpilogue);
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      if (ok) {
        if (tr) stamp(i, ev + 0);
        tc_fence_after();
        tmem_ld_32x32b_x64(s_col, r[0]);
        tmem_ld_32x32b_x64(s_col + 64, r[1]);
        tmem_wait_ld();
        const int valid = Tk - (jb + i) * kBN;
        if (valid < kBN) {  // last block: keys past Tk do not exist
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (c >= valid) r[c >> 6][c & 63] = __float_as_uint(-INFINITY);
        }
        // row max with 16 independent partial maxima (a single running max would be a 128-long dependent chain)
        float pm[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) pm[k] = __uint_as_float(r[0][k]);
#pragma unroll
        for (int c = 16; c < kBN; ++c) pm[c & 15] = fmaxf(pm[c & 15], __uint_as_float(r[c >> 6][c & 63]));
#pragma unroll
        for (int w = 8; w > 0; w >>= 1)
#pragma unroll
          for (int k = 0; k < w; ++k) pm[k] = fmaxf(pm[k], pm[k + w]);
        mx = pm[0] * scale_log2;
        if (tr) stamp(i, ev + 1);
      }
      if (turns) named_sync(kBarTurn + g, 2 * kBM);
      if (ok) {
        if (i == 0) {
          m_run = mx;
        } else {
          // O_g holds the blocks before i: the S MMA of block i was issued after their P V MMAs, so they are
          // complete once S_g(i) is. Rescale rows whose maximum moved by more than the threshold.
          const bool need = mx > m_run + kRescaleThreshold;
          if (__any_sync(0xffffffffu, need)) {
            const float alpha = need ? fast_exp2(m_run - mx) : 1.0f;
#pragma unroll
            for (int c = 0; c < kD; c += 32) {
              uint32_t o[32];
              tmem_ld_32x32b_x32(o_col + c, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st_32x32b_x32(o_col + c, o);
            }
            l_run *= alpha;
            if (need) m_run = mx;
          }
        }
        uint32_t pk[2][32];
        l_run += softmax_row<kPolyEvery>(r, scale_log2, m_run, pk);
        tmem_st_32x32b_x32(s_col, pk[0]);
        tmem_st_32x32b_x32(s_col + 32, pk[1]);
        if (tr) stamp(i, ev + 2);
      }
      if (turns) named_arrive(kBarTurn + (1 - g), 2 * kBM);
      if (ok) {
        tmem_wait_st();
        if (tr) stamp(i, ev + 3);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g]);
      }
    }
    if (turns && g == 0) named_sync(kBarTurn, 2 * kBM);  // the other warpgroup's last turn
    if (ok) {
      if (lane == 0) ok = mbar_wait_park(&o_done[g], 0, status, kTimeoutEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (ok) {
      tc_fence_after();
      const int q = q0 + g * kBM + row;
      const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      const bool partial = part_o != nullptr;
#pragma unroll
      for (int c0 = 0; c0 < kD; c0 += 32) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(o_col + c0, o);
        tmem_wait_ld();
        if (q < Tq && partial) {
          float4* dst = reinterpret_cast<float4*>(part_o + ((static_cast<int64_t>(range) * Tq + q) * H + h) * kD + c0);
#pragma unroll
          for (int c = 0; c < 32; c += 4)
            dst[c / 4] = make_float4(__uint_as_float(o[c]) * inv_l, __uint_as_float(o[c + 1]) * inv_l,
                                     __uint_as_float(o[c + 2]) * inv_l, __uint_as_float(o[c + 3]) * inv_l);
        } else if (q < Tq) {
          __nv_bfloat16* orow = out + static_cast<int64_t>(q) * out_row + static_cast<int64_t>(h) * kD + c0;
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(o[c + e]) * inv_l;
            *reinterpret_cast<uint4*>(orow + c) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                             pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
          }
        }
      }
      if (partial && q < Tq)
        part_lse[(static_cast<int64_t>(range) * Tq + q) * H + h] = l_run > 0.0f ? m_run + __log2f(l_run) : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem_base, kTmemCols);
}

// Combines the key ranges of each (query, head) row: out = sum_z w_z O_z / sum_z w_z with w_z = 2^(lse_z - max lse),
// where O_z is range z's normalized output and lse_z its log2-sum-exp. One warp per row, four columns per lane.
__global__ void merge_ranges_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse, int ranges,
                                    int Tq, int H, __nv_bfloat16* __restrict__ out, int64_t out_row) {
  const int64_t rowid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (rowid >= static_cast<int64_t>(Tq) * H) return;
  const int lane = threadIdx.x & 31;
  const int q = static_cast<int>(rowid / H), h = static_cast<int>(rowid % H);
  const int64_t plane = static_cast<int64_t>(Tq) * H;
  float mx = -INFINITY;
  for (int z = 0; z < ranges; ++z) mx = fmaxf(mx, part_lse[z * plane + rowid]);
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  float wsum = 0.0f;
  for (int z = 0; z < ranges; ++z) {
    const float lse = part_lse[z * plane + rowid];
    const float w = lse == -INFINITY ? 0.0f : fast_exp2(lse - mx);
    const float4 o = reinterpret_cast<const float4*>(part_o + (z * plane + rowid) * kD)[lane];
    acc[0] = fmaf(w, o.x, acc[0]);
    acc[1] = fmaf(w, o.y, acc[1]);
    acc[2] = fmaf(w, o.z, acc[2]);
    acc[3] = fmaf(w, o.w, acc[3]);
    wsum += w;
  }
  const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
  __nv_bfloat16* orow = out + static_cast<int64_t>(q) * out_row + static_cast<int64_t>(h) * kD + 4 * lane;
  *reinterpret_cast<uint2*>(orow) = make_uint2(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv));
}

// V [Tk, H, 128] (token stride sv, head stride 128) -> V^T [H, 128, tk_pad] with zero padding.
__global__ void transpose_v_kernel(const __nv_bfloat16* __restrict__ v, int64_t sv, int Tk, int tk_pad,
                                   __nv_bfloat16* __restrict__ vt) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int h = blockIdx.z;
  const int t0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int t = t0 + i;
    tile[i][threadIdx.x] = t < Tk ? v[static_cast<int64_t>(t) * sv + h * kD + d0 + threadIdx.x] : __float2bfloat16(0.0f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int t = t0 + threadIdx.x;
    if (t < tk_pad) vt[(static_cast<int64_t>(h) * kD + d0 + i) * tk_pad + t] = tile[threadIdx.x][i];
  }
}

// Key ranges per (query pair, head): the count with the least estimated time, the kernel's time scaling with the
// inverse of how well its CTAs fill the last wave of SMs and each extra range adding the merge pass (FP32 partials
// written and read once at ~4 TB/s, plus a launch). Each range keeps at least 3 key blocks.
int choose_ranges(int pairs, int heads, int tq, int tk, int sms) {
  const int items = pairs * heads;
  const int blocks = (tk + kBN - 1) / kBN;
  const double kernel_s = 4.0 * tq * static_cast<double>(tk) * kD * heads / 1.0e15;  // at ~1 PFLOP/s
  auto estimate = [&](int ranges) {
    const long long ctas = static_cast<long long>(items) * ranges;
    const long long waves = (ctas + sms - 1) / sms;
    const double fill = static_cast<double>(ctas) / static_cast<double>(waves * sms);
    const double merge_s = ranges > 1 ? ranges * static_cast<double>(tq) * heads * kD * 8.0 / 4.0e12 + 5.0e-6 : 0.0;
    return kernel_s / fill + merge_s;
  };
  int best = 1;
  double best_s = estimate(1);
  for (int r = 2; r <= 4 && blocks / r >= 3; ++r) {
    const double t = estimate(r);
    if (t < 0.97 * best_s) {
      best = r;
      best_s = t;
    }
  }
  return best;
}

}  // namespace attn

void attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& out, double scale,
                   const c10::optional<at::Tensor>& status, int64_t options, const c10::optional<at::Tensor>& trace) {
  check_cuda_tensor(q, "q");
  check_cuda_tensor(k, "k");
  check_cuda_tensor(v, "v");
  check_cuda_tensor(out, "out");
  const at::Tensor* all[4] = {&q, &k, &v, &out};
  for (const at::Tensor* t : all) {
    RC_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 3, "attention takes bf16 [T, H, 128] tensors");
    RC_CHECK(t->size(2) == attn::kD && t->stride(2) == 1 && t->stride(1) == attn::kD,
             "head_dim must be 128 with heads contiguous within a token row");
    RC_CHECK((t->stride(0) * 2) % 16 == 0, "token rows must be 16-byte multiples");
  }
  const int Tq = static_cast<int>(q.size(0)), H = static_cast<int>(q.size(1)), Tk = static_cast<int>(k.size(0));
  RC_CHECK(k.size(1) == H && v.size(1) == H && v.size(0) == Tk, "q, k, v disagree on heads or keys");
  RC_CHECK(out.size(0) == Tq && out.size(1) == H && out.is_contiguous(), "out must be a contiguous [Tq, H, 128]");
  RC_CHECK(Tq > 0 && Tk > 0, "empty attention");
  if (trace.has_value())
    RC_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                 trace->numel() >= attn::kTraceBlocks * attn::kTraceEvents,
             "trace must be a contiguous int64 CUDA tensor of at least 512 entries");
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.get_device()).stream();
  const int tk_pad = (Tk + 7) / 8 * 8;
  at::Tensor vt = at::empty({H, attn::kD, tk_pad}, q.options());
  attn::transpose_v_kernel<<<dim3((tk_pad + 31) / 32, attn::kD / 32, H), dim3(32, 8), 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), v.stride(0), Tk, tk_pad,
      reinterpret_cast<__nv_bfloat16*>(vt.data_ptr()));
  RC_CUDA(cudaGetLastError());
  CUtensorMap tmQ = make_tmap_3d(q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, attn::kD, H, Tq, attn::kD * 2,
                                 q.stride(0) * 2, 64, 1, attn::kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tmK = make_tmap_3d(k.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, attn::kD, H, Tk, attn::kD * 2,
                                 k.stride(0) * 2, 64, 1, attn::kBN, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tmVt = make_tmap_3d(vt.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, tk_pad, attn::kD, H,
                                  static_cast<uint64_t>(tk_pad) * 2, static_cast<uint64_t>(tk_pad) * attn::kD * 2, 64,
                                  attn::kD, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  using Kernel = decltype(&attn::attention_fwd_kernel<0>);
  static const Kernel variants[2] = {attn::attention_fwd_kernel<0>, attn::attention_fwd_kernel<8>};
  static bool configured = false;
  static int sms = 0;
  if (!configured) {
    for (Kernel kernel : variants) {
      RC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::kSmemBytes));
      // the register split inside the kernel assumes the launch holds exactly kLaunchRegs per thread
      cudaFuncAttributes attr;
      RC_CUDA(cudaFuncGetAttributes(&attr, kernel));
      RC_CHECK(attr.numRegs == attn::kLaunchRegs, "attention kernel compiled to " + std::to_string(attr.numRegs) +
                                                      " registers per thread; its register split needs " +
                                                      std::to_string(attn::kLaunchRegs));
    }
    RC_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, q.get_device()));
    configured = true;
  }
  const Kernel kernel = variants[(options & attn::kOptPoly) ? 1 : 0];
  const int pairs = (Tq + attn::kTilesPerCta * attn::kBM - 1) / (attn::kTilesPerCta * attn::kBM);
  const int blocks = (Tk + attn::kBN - 1) / attn::kBN;
  int ranges = static_cast<int>(options & attn::kOptSplitMask);
  if (ranges == 0) ranges = attn::choose_ranges(pairs, H, Tq, Tk, sms);
  ranges = std::min(ranges, blocks);
  const int per_range = (blocks + ranges - 1) / ranges;
  ranges = (blocks + per_range - 1) / per_range;  // no empty range
  at::Tensor part_o, part_lse;
  if (ranges > 1) {
    part_o = at::empty({ranges, Tq, H, attn::kD}, q.options().dtype(at::kFloat));
    part_lse = at::empty({ranges, Tq, H}, q.options().dtype(at::kFloat));
  }
  const float scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  dim3 grid(pairs, H, ranges);
  kernel<<<grid, attn::kThreads, attn::kSmemBytes, stream>>>(
      tmQ, tmK, tmVt, Tq, Tk, H, scale_log2, per_range, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      out.stride(0), ranges > 1 ? part_o.data_ptr<float>() : nullptr,
      ranges > 1 ? part_lse.data_ptr<float>() : nullptr, status_ptr(status), static_cast<int>(options),
      (options & attn::kOptTrace) && trace.has_value() ? reinterpret_cast<long long*>(trace->data_ptr<int64_t>()) : nullptr);
  RC_CUDA(cudaGetLastError());
  if (ranges > 1) {
    const int64_t rows = static_cast<int64_t>(Tq) * H;
    attn::merge_ranges_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(
        part_o.data_ptr<float>(), part_lse.data_ptr<float>(), ranges, Tq, H,
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0));
    RC_CUDA(cudaGetLastError());
  }
}

}  // namespace rc
