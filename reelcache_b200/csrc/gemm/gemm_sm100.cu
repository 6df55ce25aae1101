// Persistent warp-specialized tcgen05 GEMM for sm_100a: D[M, N] = A[M, K] * B[N, K]^T with bf16
// operands (both K-major, i.e. torch's x @ W^T for a Linear weight W[N, K]), fp32 accumulation in
// TMEM, and a fused epilogue (bias, tanh-GELU, gated residual, fp32 or bf16 output).
//
// Roles (320 threads, one CTA per SM):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [BN x 64] per stage, 128-byte swizzle.
//   warp 1      TMEM owner and MMA issuer (one elected lane issues tcgen05.mma, 4 per K block).
//   warps 2..9  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32*(w%4)..+31; the two
//               warps of one lane quarter take alternate 32-column chunks), fused math, vectorized global
//               stores. The chunk's bias, gate and residual are loaded with 16-byte loads before its
//               TMEM read, so their latency overlaps it.
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the epilogue of tile t
// overlaps the main loop of tile t+1.
#include <cstdlib>
#include <string>

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace rc {
namespace gemm {

enum Epilogue : int {
  kStore = 0,         // D = acc
  kBias = 1,          // D = acc + bias[n]
  kBiasGelu = 2,      // D = gelu_tanh(acc + bias[n])
  kBiasGateResid = 3, // D = resid[m, n] + (acc + bias[n]) * gate[n]   (D may alias resid)
};

struct EpiParams {
  void* out;              // [M, ldo] bf16 or fp32
  const __nv_bfloat16* bias;  // [N] or null
  const float* gate;      // [N] or null (gate = 1)
  const __nv_bfloat16* resid; // [M, ldr] or null
  int64_t ldo;
  int64_t ldr;
  float alpha;            // scale applied to acc before bias
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kGroupM = 8;
// Shared memory for operand stages: the 227 KB a CTA may hold, less alignment slack and the barriers.
constexpr int kStageBudget = 227 * 1024 - 1024 - 256;

template <int BN>
struct Config {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kStageBudget / kStageBytes > 10 ? 10 : kStageBudget / kStageBytes;
  static constexpr int kTmemCols = (2 * BN) <= 256 ? 256 : 512;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// tanh-approximated GELU; tanh from the hardware approximation (relative error below 2^-10, far under the
// bfloat16 rounding of the output).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);  // sqrt(2/pi) (x + 0.044715 x^3)
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * x * (1.0f + t);
}

__device__ __forceinline__ float bf16_lo(uint32_t pair) { return __uint_as_float(pair << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t pair) { return __uint_as_float(pair & 0xffff0000u); }

// 32 consecutive bfloat16 values as 16 packed pairs; ``vec``: four 16-byte loads (aligned, all in range),
// else element loads of the first ``valid`` values (the rest zero).
template <bool kReadOnly>
__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* p, bool vec, int valid, uint32_t (&out)[16]) {
  if (vec) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = kReadOnly ? __ldg(q + i) : q[i];
      out[4 * i] = u.x;
      out[4 * i + 1] = u.y;
      out[4 * i + 2] = u.z;
      out[4 * i + 3] = u.w;
    }
  } else {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t lo = 2 * j < valid ? h[2 * j] : 0u;
      const uint32_t hi = 2 * j + 1 < valid ? h[2 * j + 1] : 0u;
      out[j] = lo | (hi << 16);
    }
  }
}

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m_idx, int& n_idx) {
  const int per_group = kGroupM * num_n;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - group * per_group;
  m_idx = first_m + r % gsize;
  n_idx = r / gsize;
}

// Epilogue of one accumulator tile: this warp's alternate 32-column chunks (``half``, ``half + 2``, ...) of its
// 32 TMEM lanes (``quarter``); ``row`` is this thread's output row, ``n_base`` the tile's first column.
template <int BN, int EPI, bool OUT_F32>
__device__ __forceinline__ void epilogue_tile(uint32_t acc_tmem, int quarter, int half, int row, bool row_ok,
                                              int n_base, int N, const EpiParams& ep) {
#pragma unroll 1
  for (int c = half; c < BN / 32; c += 2) {
    const int n0 = n_base + c * 32;
    if (n0 >= N) break;  // uniform across the warp
    const int valid = min(32, N - n0);
    uint32_t bias2[16], res2[16];
    float g[32];
    if (EPI != kStore && ep.bias != nullptr)
      load_bf16x32<true>(ep.bias + n0, valid == 32 && aligned16(ep.bias + n0), valid, bias2);
    if (EPI == kBiasGateResid) {
      const __nv_bfloat16* rrow = ep.resid + static_cast<int64_t>(row) * ep.ldr + n0;
      if (row_ok) load_bf16x32<false>(rrow, valid == 32 && aligned16(rrow), valid, res2);
      if (ep.gate != nullptr) {
        if (valid == 32 && aligned16(ep.gate + n0)) {
          const float4* q = reinterpret_cast<const float4*>(ep.gate + n0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 u = __ldg(q + i);
            g[4 * i] = u.x;
            g[4 * i + 1] = u.y;
            g[4 * i + 2] = u.z;
            g[4 * i + 3] = u.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) g[j] = j < valid ? ep.gate[n0 + j] : 0.0f;
        }
      }
    }
    uint32_t raw[32];
    tmem_ld_32x32b_x32(acc_tmem + c * 32 + (static_cast<uint32_t>(quarter * 32) << 16), raw);
    tmem_wait_ld();
    if (!row_ok) continue;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]) * ep.alpha;
    if (EPI != kStore && ep.bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        v[2 * j] += bf16_lo(bias2[j]);
        v[2 * j + 1] += bf16_hi(bias2[j]);
      }
    }
    if (EPI == kBiasGelu) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
    }
    if (EPI == kBiasGateResid) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float g0 = ep.gate != nullptr ? g[2 * j] : 1.0f;
        const float g1 = ep.gate != nullptr ? g[2 * j + 1] : 1.0f;
        v[2 * j] = fmaf(v[2 * j], g0, bf16_lo(res2[j]));
        v[2 * j + 1] = fmaf(v[2 * j + 1], g1, bf16_hi(res2[j]));
      }
    }
    if (OUT_F32) {
      float* orow = reinterpret_cast<float*>(ep.out) + static_cast<int64_t>(row) * ep.ldo + n0;
      if (valid == 32 && aligned16(orow)) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(orow + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < valid) orow[j] = v[j];
      }
    } else {
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(ep.out) + static_cast<int64_t>(row) * ep.ldo + n0;
      if (valid == 32 && aligned16(orow)) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 pk;
          pk.x = pack_bf16x2(v[j], v[j + 1]);
          pk.y = pack_bf16x2(v[j + 2], v[j + 3]);
          pk.z = pack_bf16x2(v[j + 4], v[j + 5]);
          pk.w = pack_bf16x2(v[j + 6], v[j + 7]);
          *reinterpret_cast<uint4*>(orow + j) = pk;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < valid) orow[j] = __float2bfloat16(v[j]);
      }
    }
  }
}

template <int BN, int EPI, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, EpiParams ep, int* status) {
  using Cfg = Config<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drained = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(drained, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int m_idx, n_idx;
        tile_coords(t, num_m, num_n, m_idx, n_idx);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * Cfg::kStageBytes;
          uint8_t* b_dst = a_dst + Cfg::kABytes;
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(a_dst, &tmA, &full[stage], kb * kBK, m_idx * kBM);
          tma_load_2d(b_dst, &tmB, &full[stage], kb * kBK, n_idx * BN);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = make_idesc_f16(kBM, BN, /*bf16*/ 1);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (lane == 0) ok = mbar_wait(&acc_empty[buf], acc_phase ^ 1, status, kTimeoutMma);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * BN;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (lane == 0) ok = mbar_wait(&full[stage], phase, status, kTimeoutMma);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + stage * Cfg::kStageBytes);
          const uint32_t b_addr = a_addr + Cfg::kABytes;
          const uint64_t adesc = sw128_kmajor_desc(a_addr);
          const uint64_t bdesc = sw128_kmajor_desc(b_addr);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // Advancing 16 bf16 (32 bytes) along K inside the swizzle atom: +2 in the >>4 address.
            mma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) mma_commit(&acc_full[buf]);
      __syncwarp();
    }
    // Drain: wait (bounded) until every MMA this thread issued has completed before TMEM is freed.
    if (lane == 0) {
      mma_commit(drained);
      (void)mbar_wait(drained, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    // ---------------- Epilogue ----------------
    const int quarter = warp & 3;         // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;     // this warp's alternate 32-column chunks: half, half + 2, ...
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      int m_idx, n_idx;
      tile_coords(t, num_m, num_n, m_idx, n_idx);
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&acc_full[buf], acc_phase, status, kTimeoutEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int row = m_idx * kBM + quarter * 32 + lane;
      const bool row_ok = row < M;
      epilogue_tile<BN, EPI, OUT_F32>(tmem_base + buf * BN, quarter, half, row, row_ok, n_idx * BN, N, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}


// ---------------------------------------------------------------------------------------------
// Paired-CTA variant: a cluster of two CTAs computes a 256 x BN tile with tcgen05.mma.cta_group::2.
// CTA r of the pair loads A rows [256 m + 128 r, +128) and B rows [BN n + BN/2 r, +BN/2) into its own
// shared memory (no multicast); the leader's MMA reads both CTAs' halves and accumulates rows 128 r.. of
// the tile into CTA r's TMEM (all BN columns). Per SM this moves 16 KB of A and BN/2 x 128 B of B per
// 64-deep K block instead of 16 KB + BN x 128 B, which is what bounds the single-CTA kernel (its operand
// stream from L2 runs near the L2-to-SM bandwidth).
//
// Barriers: full[s] (leader) counts both CTAs' TMA bytes, the leader's producer posting the expected
// total; empty[s] and acc_full[b] exist in both CTAs and receive one MMA commit each from the leader;
// acc_empty[b] (leader) counts the epilogue warps of both CTAs. Every wait is bounded; a CTA that gives
// up still reaches the closing cluster barrier, so its peer is never left waiting on it there.
// ---------------------------------------------------------------------------------------------

constexpr int kPairBM = 256;

template <int BN>
struct PairConfig {
  static constexpr int kABytes = kBM * kBK * 2;              // this CTA's 128 rows of A
  static constexpr int kBBytes = (BN / 2) * kBK * 2;         // this CTA's BN / 2 rows of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kStageBudget / kStageBytes > 10 ? 10 : kStageBudget / kStageBytes;
  static constexpr int kTmemCols = (2 * BN) <= 256 ? 256 : 512;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
};

template <int BN, int EPI, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tn_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M,
                        int N, int K, EpiParams ep, int* status) {
  using Cfg = PairConfig<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drained = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_m = (M + kPairBM - 1) / kPairBM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);
    }
    mbar_init(drained, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM of both allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs: this CTA's halves) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += num_pairs) {
        int m_idx, n_idx;
        tile_coords(t, num_m, num_n, m_idx, n_idx);
        const int a_row = m_idx * kPairBM + static_cast<int>(rank) * kBM;
        const int b_row = n_idx * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_spin(&empty[stage], phase ^ 1, status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = cluster_addr(&full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          uint8_t* a_dst = smem + stage * Cfg::kStageBytes;
          tma_load_2d_pair(a_dst, &tmA, leader_full, kb * kBK, a_row);
          tma_load_2d_pair(a_dst + Cfg::kABytes, &tmB, leader_full, kb * kBK, b_row);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader) {
      constexpr uint32_t idesc = make_idesc_f16(kPairBM, BN, /*bf16*/ 1);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += num_pairs, ++local) {
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (lane == 0) ok = mbar_wait_cluster(&acc_empty[buf], acc_phase ^ 1, status, kTimeoutMma);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (lane == 0) ok = mbar_wait_cluster(&full[stage], phase, status, kTimeoutMma);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(smem + stage * Cfg::kStageBytes);
            const uint64_t adesc = sw128_kmajor_desc(a_addr);
            const uint64_t bdesc = sw128_kmajor_desc(a_addr + Cfg::kABytes);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              mma_f16_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            mma_commit_pair(cluster_addr(&empty[stage], 0));
            mma_commit_pair(cluster_addr(&empty[stage], 1));
          }
          __syncwarp();
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (lane == 0) {
          mma_commit_pair(cluster_addr(&acc_full[buf], 0));
          mma_commit_pair(cluster_addr(&acc_full[buf], 1));
        }
        __syncwarp();
      }
      if (lane == 0) {
        mma_commit_pair(cluster_addr(drained, 0));
        (void)mbar_wait(drained, 0, nullptr, 0);
      }
      __syncwarp();
    }
  } else {
    // ---------------- Epilogue (both CTAs: this CTA's 128 rows of each tile) ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t leader_acc_empty0 = cluster_addr(&acc_empty[0], 0);
    const uint32_t leader_acc_empty1 = cluster_addr(&acc_empty[1], 0);
    int local = 0;
    for (int t = pair; t < num_tiles; t += num_pairs, ++local) {
      int m_idx, n_idx;
      tile_coords(t, num_m, num_n, m_idx, n_idx);
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&acc_full[buf], acc_phase, status, kTimeoutEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int row = m_idx * kPairBM + static_cast<int>(rank) * kBM + quarter * 32 + lane;
      epilogue_tile<BN, EPI, OUT_F32>(tmem_base + buf * BN, quarter, half, row, row < M, n_idx * BN, N, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(buf ? leader_acc_empty1 : leader_acc_empty0);
    }
  }

  tc_fence_before();
  cluster_sync_all();  // the leader's MMAs (reading both CTAs' shared memory, writing both TMEMs) are drained
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
}

template <int BN, int EPI, bool OUT_F32>
void launch(const at::Tensor& A, const at::Tensor& B, int M, int N, int K, const EpiParams& ep, int* status,
            cudaStream_t stream) {
  using Cfg = Config<BN>;
  CUtensorMap tmA = make_tmap_2d(A.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, A.stride(0) * 2, kBK, kBM,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tmB = make_tmap_2d(B.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, B.stride(0) * 2, kBK, BN,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  auto kernel = gemm_tn_kernel<BN, EPI, OUT_F32>;
  static bool configured = false;  // per template instance
  if (!configured) {
    RC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    configured = true;
  }
  const int num_tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int grid = std::min(num_tiles, sm_count(A.get_device()));
  kernel<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(tmA, tmB, M, N, K, ep, status);
  RC_CUDA(cudaGetLastError());
}

template <int BN, int EPI, bool OUT_F32>
void launch_pair(const at::Tensor& A, const at::Tensor& B, int M, int N, int K, const EpiParams& ep, int* status,
                 cudaStream_t stream) {
  using Cfg = PairConfig<BN>;
  CUtensorMap tmA = make_tmap_2d(A.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, A.stride(0) * 2, kBK, kBM,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tmB = make_tmap_2d(B.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, B.stride(0) * 2, kBK,
                                 BN / 2, CU_TENSOR_MAP_SWIZZLE_128B);
  auto kernel = gemm_tn_pair_kernel<BN, EPI, OUT_F32>;
  static bool configured = false;  // per template instance
  if (!configured) {
    RC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    configured = true;
  }
  const int num_tiles = ((M + kPairBM - 1) / kPairBM) * ((N + BN - 1) / BN);
  const int pairs = std::min(num_tiles, sm_count(A.get_device()) / 2);
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(2 * pairs);
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = Cfg::kSmemBytes;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeClusterDimension;
  attribute[0].val.clusterDim.x = 2;
  attribute[0].val.clusterDim.y = 1;
  attribute[0].val.clusterDim.z = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  RC_CUDA(cudaLaunchKernelEx(&config, kernel, tmA, tmB, M, N, K, ep, status));
}

// N tile of the paired kernel: the least work lost to partial waves over the 74 CTA pairs.
int pick_bn_pair(int M, int N, int pairs) {
  const int candidates[3] = {128, 192, 256};
  int best = 256;
  double best_cost = 1e30;
  const int num_m = (M + kPairBM - 1) / kPairBM;
  for (int bn : candidates) {
    const long tiles = static_cast<long>(num_m) * ((N + bn - 1) / bn);
    const long waves = (tiles + pairs - 1) / pairs;
    const double cost = static_cast<double>(waves) * bn * (1.0 + 32.0 / bn);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

// The paired kernel is opt-in (REELCACHE_GEMM_PAIRS=1) for GEMMs of at least two 256-row tiles. Measured on
// one B200 on the DiT's shapes (4680 rows) it is 6 % faster on the QKV projection (N 4608) and 4-16 % slower
// on the N = 1536 and N = 8960 projections, where the 19 row tiles of 256 leave partial waves over 74 pairs;
// with neither the L2 (31-37 % of peak) nor the TMA stream limiting the single-CTA kernel, halving the B
// stream per SM does not pay for that.
constexpr int kPairMinRows = 512;

bool use_pairs(int M) {
  static const bool enabled = [] {
    const char* v = std::getenv("REELCACHE_GEMM_PAIRS");
    return v != nullptr && std::string(v) == "1";
  }();
  return enabled && M >= kPairMinRows;
}

// Picks the N tile that wastes the least work over the 148-SM waves.
int pick_bn(int M, int N, int sms) {
  const int candidates[3] = {128, 192, 256};
  int best = 256;
  double best_cost = 1e30;
  const int num_m = (M + kBM - 1) / kBM;
  for (int bn : candidates) {
    const int num_n = (N + bn - 1) / bn;
    const long tiles = static_cast<long>(num_m) * num_n;
    const long waves = (tiles + sms - 1) / sms;
    // cost ~ waves * per-tile time (proportional to bn) + small penalty for narrow tiles (B re-reads)
    double cost = static_cast<double>(waves) * bn * (1.0 + 16.0 / bn);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

template <int EPI, bool OUT_F32>
void dispatch_bn(int bn, bool pairs, const at::Tensor& A, const at::Tensor& B, int M, int N, int K,
                 const EpiParams& ep, int* status, cudaStream_t stream) {
  if (pairs) {
    switch (bn) {
      case 128: launch_pair<128, EPI, OUT_F32>(A, B, M, N, K, ep, status, stream); break;
      case 192: launch_pair<192, EPI, OUT_F32>(A, B, M, N, K, ep, status, stream); break;
      default: launch_pair<256, EPI, OUT_F32>(A, B, M, N, K, ep, status, stream); break;
    }
    return;
  }
  switch (bn) {
    case 128: launch<128, EPI, OUT_F32>(A, B, M, N, K, ep, status, stream); break;
    case 192: launch<192, EPI, OUT_F32>(A, B, M, N, K, ep, status, stream); break;
    default: launch<256, EPI, OUT_F32>(A, B, M, N, K, ep, status, stream); break;
  }
}

}  // namespace gemm

// out[M, N] = epilogue(alpha * A[M, K] @ B[N, K]^T). A and B bf16 with unit stride along K.
void gemm_bf16_tn(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epilogue,
                  const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& gate,
                  const c10::optional<at::Tensor>& resid, double alpha, int64_t bn,
                  const c10::optional<at::Tensor>& status) {
  check_cuda_tensor(A, "A");
  check_cuda_tensor(B, "B");
  check_cuda_tensor(out, "out");
  RC_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "A and B must be bfloat16");
  RC_CHECK(A.dim() == 2 && B.dim() == 2 && out.dim() == 2, "A, B and out must be 2-D");
  RC_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && out.stride(1) == 1, "inner dimensions must be contiguous");
  const int M = static_cast<int>(A.size(0));
  const int K = static_cast<int>(A.size(1));
  const int N = static_cast<int>(B.size(0));
  RC_CHECK(B.size(1) == K, "A and B disagree on K");
  RC_CHECK(out.size(0) == M && out.size(1) == N, "out must be [M, N]");
  RC_CHECK(K % 8 == 0, "K must be a multiple of 8 (16-byte TMA rows)");
  RC_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  const bool out_f32 = out.scalar_type() == at::kFloat;
  RC_CHECK(out_f32 || out.scalar_type() == at::kBFloat16, "out must be float32 or bfloat16");
  c10::cuda::CUDAGuard guard(A.device());
  gemm::EpiParams ep;
  ep.out = out.data_ptr();
  ep.ldo = out.stride(0);
  ep.alpha = static_cast<float>(alpha);
  ep.bias = nullptr;
  ep.gate = nullptr;
  ep.resid = nullptr;
  ep.ldr = 0;
  if (bias.has_value() && bias->defined()) {
    RC_CHECK(bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() && bias->numel() == N,
             "bias must be a contiguous bfloat16 [N] vector");
    ep.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (gate.has_value() && gate->defined()) {
    RC_CHECK(gate->scalar_type() == at::kFloat && gate->is_contiguous() && gate->numel() == N,
             "gate must be a contiguous float32 [N] vector");
    ep.gate = gate->data_ptr<float>();
  }
  if (epilogue == gemm::kBiasGateResid) {
    RC_CHECK(resid.has_value() && resid->defined(), "gated residual epilogue needs resid");
    RC_CHECK(resid->scalar_type() == at::kBFloat16 && resid->dim() == 2 && resid->stride(1) == 1 &&
                 resid->size(0) == M && resid->size(1) == N,
             "resid must be a bfloat16 [M, N] matrix with unit inner stride");
    RC_CHECK(!out_f32, "gated residual epilogue writes bfloat16");
    ep.resid = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
    ep.ldr = resid->stride(0);
  }
  int* st = status_ptr(status);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(A.get_device()).stream();
  const int sms = sm_count(A.get_device());
  const bool pairs = gemm::use_pairs(M);
  const int tile_n = bn > 0 ? static_cast<int>(bn) : (pairs ? gemm::pick_bn_pair(M, N, sms / 2) : gemm::pick_bn(M, N, sms));
  RC_CHECK(tile_n == 128 || tile_n == 192 || tile_n == 256, "bn must be 128, 192 or 256");
  switch (epilogue) {
    case gemm::kStore:
      if (out_f32)
        gemm::dispatch_bn<gemm::kStore, true>(tile_n, pairs, A, B, M, N, K, ep, st, stream);
      else
        gemm::dispatch_bn<gemm::kStore, false>(tile_n, pairs, A, B, M, N, K, ep, st, stream);
      break;
    case gemm::kBias:
      if (out_f32)
        gemm::dispatch_bn<gemm::kBias, true>(tile_n, pairs, A, B, M, N, K, ep, st, stream);
      else
        gemm::dispatch_bn<gemm::kBias, false>(tile_n, pairs, A, B, M, N, K, ep, st, stream);
      break;
    case gemm::kBiasGelu:
      gemm::dispatch_bn<gemm::kBiasGelu, false>(tile_n, pairs, A, B, M, N, K, ep, st, stream);
      break;
    case gemm::kBiasGateResid:
      gemm::dispatch_bn<gemm::kBiasGateResid, false>(tile_n, pairs, A, B, M, N, K, ep, st, stream);
      break;
    default:
      RC_CHECK(false, "unknown epilogue");
  }
}

}  // namespace rc
