// Flash-attention forward for sm_100a: out = softmax(scale * Q K^T) V per head, bf16 in / bf16 out, head_dim 128,
// fp32 accumulation in TMEM. Q [Tq, H, 128], K and V [Tk, H, 128] (token rows of any 16-byte-multiple stride,
// heads contiguous within a row); out [Tq, H, 128] contiguous.
//
// One CTA per (128-query tile, head), 320 threads:
//   warp 0      TMA producer: lane 0 loads Q once (two 64-column boxes) and the K_j tiles of 128 keys, lane 1 the
//               V^T_j tiles, each into a 2-stage ring (K freed after S_j = Q K_j^T, V after O += P_j V_j).
//   warp 1      TMEM owner and MMA issuer: S_0, S_1, then S_{j+2} as soon as S_j has been read out and
//               O_{j%2} += P_j V_j as soon as P_j is written.
//   warps 2..9  two softmax warpgroups (one thread per query row; TMEM lane = row). Warpgroup g takes the KV
//               blocks j = g, g + 2, ... with its own S_g and O_g in TMEM, so two warps share each SM
//               sub-partition's exp pipe and hide each other's TMEM-load latency. Per block: load S_j (128 fp32),
//               free S_g, online softmax in the log2 domain with *lazy rescaling* (the running max only moves
//               when the block maximum exceeds it by more than 8, i.e. p <= 256; then the row's O_g is rescaled
//               in TMEM after the warpgroup's previous P V completed), write P_j (bf16) into shared memory in the
//               128-byte-swizzled K-major layout the MMA reads. Warpgroup 0 finally merges the two partial
//               results (max, sum, O) and stores bf16 rows.
// V is transposed once per call into V^T [H, 128, Tk_pad] so both GEMMs read K-major operands.
// Every wait is bounded (2 s): on expiry a status code is recorded, the loops stop, the MMA warp drains its
// MMAs (bounded) and TMEM is freed.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_bf16.h>

#include <cmath>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace rc {
namespace attn {

constexpr int kD = 128;
constexpr int kBM = 128;       // queries per CTA
constexpr int kBN = 128;       // keys per block
constexpr int kThreads = 320;  // producer, MMA, two softmax warpgroups
constexpr int kBox = 128 * 64 * 2;          // one [128 rows x 64 cols] bf16 box: 16 KB
constexpr int kTileBytes = 2 * kBox;        // a 128 x 128 operand tile: 32 KB
constexpr int kStages = 2;
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kTileBytes;
constexpr int kVOff = kKOff + kStages * kTileBytes;
constexpr int kPOff = kVOff + kStages * kTileBytes;   // one P tile per warpgroup
constexpr int kBarOff = kPOff + 2 * kTileBytes;
constexpr int kXOff = kBarOff + 256;                   // merge exchange: m[128], l[128], flag
constexpr int kSmemBytes = kXOff + 2 * 128 * 4 + 64 + 1024;
constexpr uint32_t kTmemCols = 512;       // S_g at 128 g, O_g at 256 + 128 g
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for x <= 0 on the FMA/ALU pipes (half of the softmax exponentials, so the exp pipe is not the bound):
// x = n + f with n = rint(x) taken from the low mantissa bits of x + 1.5 * 2^23 (Cody-Waite style reduction),
// f in [-0.5, 0.5], 2^f by a cubic least-squares fit at Chebyshev nodes (relative error < 8e-5, far below the
// bfloat16 rounding of P), and 2^n added to the exponent field. x is clamped at -125 (the result stays normal).
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -125.0f);
  const float t = __fadd_rn(x, 12582912.0f);
  const float n = __fsub_rn(t, 12582912.0f);
  const float f = __fsub_rn(x, n);
  const float p = fmaf(fmaf(fmaf(0.05508868f, f, 0.24260405f), f, 0.69327623f), f, 0.99992895f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

// Two non-negative finite floats -> bfloat16x2, round to nearest even, on the integer pipe.
__device__ __forceinline__ uint32_t pack_bf16x2_alu(float a, float b) {
  uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
  ua += 0x7FFFu + ((ua >> 16) & 1u);
  ub += 0x7FFFu + ((ub >> 16) & 1u);
  return __byte_perm(ua, ub, 0x7632);
}

__device__ __forceinline__ void pair_barrier() {  // both softmax warpgroups (256 threads), barrier id 1
  asm volatile("bar.sync 1, 256;" ::: "memory");
}

// Softmax warpgroup g handles the KV blocks j = g, g + 2, g + 4, ... with its own S_g and O_g in TMEM; warpgroup 0
// merges both partial results at the end.
__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmVt, int Tq, int Tk, int H, float scale_log2,
                         __nv_bfloat16* __restrict__ out, int64_t out_row, int* status, int ablate) {
  // ablate (measurement only): bit 0 skips the softmax arithmetic (P = 0), bit 1 stops reloading K/V after the
  // first kStages blocks (stages are reused as loaded), bit 2 skips the P V MMAs, bit 3 skips the S loads from
  // TMEM, bit 4 the P stores and bit 5 the proxy fence (the last three only with bit 0), bit 6 the S MMAs after
  // the first two blocks.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [kStages]
  uint64_t* k_empty = bars + 3;   // [kStages]
  uint64_t* v_full = bars + 5;    // [kStages]
  uint64_t* v_empty = bars + 7;   // [kStages]
  uint64_t* s_full = bars + 9;    // [2] per warpgroup
  uint64_t* s_free = bars + 11;   // [2]
  uint64_t* p_full = bars + 13;   // [2]
  uint64_t* o_done = bars + 15;   // [2]
  uint64_t* drained = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  float* x_m = reinterpret_cast<float*>(smem + kXOff);
  float* x_l = x_m + 128;
  int* x_flag = reinterpret_cast<int*>(x_l + 128);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * kBM;
  const int h = blockIdx.y;
  const int nblk = (Tk + kBN - 1) / kBN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int b = 0; b < kStages; ++b) {
      mbar_init(&k_full[b], 1);
      mbar_init(&k_empty[b], 1);
      mbar_init(&v_full[b], 1);
      mbar_init(&v_empty[b], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&s_free[g], 4);
      mbar_init(&p_full[g], 4);
      mbar_init(&o_done[g], 1);
    }
    mbar_init(drained, 1);
    *x_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmVt);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: lane 0 streams Q and K, lane 1 streams V^T (independent orders) ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_3d(smem + kQOff, &tmQ, q_full, 0, h, q0);
      tma_load_3d(smem + kQOff + kBox, &tmQ, q_full, 64, h, q0);
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages;
        if (!mbar_wait_park(&k_empty[s], ((j / kStages) & 1) ^ 1, status, kTimeoutProducer)) break;
        if ((ablate & 2) && j >= kStages) {
          mbar_arrive(&k_full[s]);
          continue;
        }
        uint8_t* kd = smem + kKOff + s * kTileBytes;
        mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        tma_load_3d(kd, &tmK, &k_full[s], 0, h, j * kBN);
        tma_load_3d(kd + kBox, &tmK, &k_full[s], 64, h, j * kBN);
      }
    } else if (lane == 1) {
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages;
        if (!mbar_wait_park(&v_empty[s], ((j / kStages) & 1) ^ 1, status, kTimeoutProducer)) break;
        if ((ablate & 2) && j >= kStages) {
          mbar_arrive(&v_full[s]);
          continue;
        }
        uint8_t* vd = smem + kVOff + s * kTileBytes;
        mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        tma_load_3d(vd, &tmVt, &v_full[s], j * kBN, 0, h);
        tma_load_3d(vd + kBox, &tmVt, &v_full[s], j * kBN + 64, 0, h);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: S_0, S_1, then per block j: S_{j+2}, O_{j%2} += P_j V_j ----------------
    constexpr uint32_t idesc = make_idesc_f16(kBM, kBN, /*bf16*/ 1);
    bool ok = true;
    if (lane == 0) ok = mbar_wait_park(q_full, 0, status, kTimeoutMma);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    auto issue_s = [&](int j) -> bool {  // S_{j%2} = Q K_j^T
      const int s = j % kStages, g = j & 1;
      bool good = true;
      if (lane == 0) good = mbar_wait_park(&k_full[s], (j / kStages) & 1, status, kTimeoutMma) &&
                            mbar_wait_park(&s_free[g], ((j >> 1) & 1) ^ 1, status, kTimeoutMma);
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_u32(smem + kQOff);
        const uint32_t ka = smem_u32(smem + kKOff + s * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          if ((ablate & 64) && j >= 2) break;
          const uint32_t box = (kk >> 2) * kBox;
          mma_f16(tmem_base + g * kBN, sw128_kmajor_desc(qa + box) + 2 * (kk & 3),
                  sw128_kmajor_desc(ka + box) + 2 * (kk & 3), idesc, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[g]);
        mma_commit(&k_empty[s]);
      }
      __syncwarp();
      return true;
    };
    // S_{j+2} is issued as soon as warpgroup (j % 2) has moved S_j into registers, so its next scores are ready
    // when it finishes P_j; O += P_j V_j follows P_j. Event order: S_0, S_1, then for j = 0, 1, ...:
    // [S_j freed -> S_{j+2}], [P_{j-1} written -> O += P_{j-1} V_{j-1}].
    auto issue_pv = [&](int j) -> bool {
      const int s = j % kStages, g = j & 1;
      bool good = true;
      if (lane == 0) good = mbar_wait_park(&p_full[g], (j >> 1) & 1, status, kTimeoutMma) &&
                            mbar_wait_park(&v_full[s], (j / kStages) & 1, status, kTimeoutMma);
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t pa = smem_u32(smem + kPOff + g * kTileBytes);
        const uint32_t va = smem_u32(smem + kVOff + s * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          if (ablate & 4) break;
          const uint32_t box = (kk >> 2) * kBox;
          mma_f16(tmem_base + 256 + g * kBN, sw128_kmajor_desc(pa + box) + 2 * (kk & 3),
                  sw128_kmajor_desc(va + box) + 2 * (kk & 3), idesc, (j >= 2 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&o_done[g]);
        mma_commit(&v_empty[s]);
      }
      __syncwarp();
      return true;
    };
    if (ok && nblk > 0) ok = issue_s(0);
    if (ok && nblk > 1) ok = issue_s(1);
    for (int j = 0; j <= nblk && ok; ++j) {
      if (j + 2 < nblk && !issue_s(j + 2)) {  // waits for S_j to be freed (issue_s waits on s_free)
        ok = false;
        break;
      }
      if (j >= 1 && !issue_pv(j - 1)) {
        ok = false;
        break;
      }
    }
    if (lane == 0) {
      mma_commit(drained);
      (void)mbar_wait_park(drained, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax warpgroups ----------------
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_col = tmem_base + g * kBN + lane_addr;
    const uint32_t o_col = tmem_base + 256 + g * kBN + lane_addr;
    uint8_t* pbase = smem + kPOff + g * kTileBytes;
    float m_run = -INFINITY;  // running max of scale * log2(e) * s
    float l_run = 0.0f;
    bool ok = true;
    int count = 0;  // blocks processed by this warpgroup
    for (int j = g; j < nblk && ok; j += 2, ++count) {
      const uint32_t ph = count & 1;
      if (lane == 0) ok = mbar_wait_park(&s_full[g], ph, status, kTimeoutEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      uint32_t r[2][64];
      if (ablate & 8) {
#pragma unroll
        for (int c = 0; c < 64; ++c) r[0][c] = r[1][c] = static_cast<uint32_t>(c + j);
      } else {
        tmem_ld_32x32b_x64(s_col, r[0]);
        tmem_ld_32x32b_x64(s_col + 64, r[1]);
        tmem_wait_ld();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[g]);
      if (ablate & 1) {
        if (count > 0) {
          if (lane == 0) ok = mbar_wait_park(&o_done[g], (count - 1) & 1, status, kTimeoutEpilogue);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
        }
        if (!(ablate & 16)) {
#pragma unroll
          for (int chunk = 0; chunk < kBN / 8; ++chunk)
            *reinterpret_cast<uint4*>(pbase + (chunk >> 3) * kBox + row * 128 + (((chunk & 7) ^ (row & 7)) << 4)) =
                make_uint4(r[0][chunk], 0u, 0u, 0u);
        }
        l_run = 1.0f;
        m_run = 0.0f;
        if (!(ablate & 32)) fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g]);
        continue;
      }
      const int valid = Tk - j * kBN;
      if (valid < kBN) {  // last block: keys past Tk do not exist
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (c >= valid) r[c >> 6][c & 63] = __float_as_uint(-INFINITY);
      }
      // row max with 16 independent partial maxima (a single running max would be a 128-long dependent chain)
      float pm[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) pm[k] = __uint_as_float(r[k >> 6][k & 63]);
#pragma unroll
      for (int c = 16; c < kBN; ++c) pm[c & 15] = fmaxf(pm[c & 15], __uint_as_float(r[c >> 6][c & 63]));
#pragma unroll
      for (int w = 8; w > 0; w >>= 1)
#pragma unroll
        for (int k = 0; k < w; ++k) pm[k] = fmaxf(pm[k], pm[k + w]);
      const float mx = pm[0] * scale_log2;
      if (count > 0) {
        // O_g += P V of this warpgroup's previous block must be complete before P_g is rewritten (and before
        // O_g's rows are rescaled)
        if (lane == 0) ok = mbar_wait_park(&o_done[g], (count - 1) & 1, status, kTimeoutEpilogue);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        const bool need = mx > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? fast_exp2(m_run - mx) : 1.0f;
#pragma unroll
          for (int c = 0; c < kD; c += 16) {
            uint32_t o[16];
            tmem_ld_32x32b_x16(o_col + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_32x32b_x16(o_col + c, o);
          }
          tmem_wait_st();
          l_run *= alpha;
          if (need) m_run = mx;
        }
      } else {
        m_run = mx;
      }
      // P_j = exp2(scale_log2 * s - m_run) as bf16 in the swizzled K-major layout; row sum in fp32
      const float neg_m = -m_run;
      float ps[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};  // independent partial row sums
#pragma unroll
      for (int chunk = 0; chunk < kBN / 8; ++chunk) {  // 16-byte chunks of 8 keys
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = chunk * 8 + 2 * e;
          const float p0 = fast_exp2(fmaf(__uint_as_float(r[c >> 6][c & 63]), scale_log2, neg_m));
          const float p1 = fast_exp2(fmaf(__uint_as_float(r[(c + 1) >> 6][(c + 1) & 63]), scale_log2, neg_m));
          ps[(2 * e) & 7] += p0;
          ps[(2 * e + 1) & 7] += p1;
          w[e] = pack_bf16x2(p0, p1);
        }
        const int box = chunk >> 3;
        const int cc = chunk & 7;
        *reinterpret_cast<uint4*>(pbase + box * kBox + row * 128 + ((cc ^ (row & 7)) << 4)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
      l_run += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
    }
    // wait for this warpgroup's last O_g += P V
    if (ok && count > 0) {
      if (lane == 0) ok = mbar_wait_park(&o_done[g], (count - 1) & 1, status, kTimeoutEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (g == 1) {
      x_m[row] = m_run;
      x_l[row] = l_run;
      if (!ok && lane == 0) atomicOr(x_flag, 1);
    }
    pair_barrier();
    const bool all_ok = ok && (*x_flag == 0);
    if (g == 0 && all_ok) {
      tc_fence_after();
      const float m_b = x_m[row], l_b = x_l[row];
      const bool has_b = nblk > 1;
      const float m = has_b ? fmaxf(m_run, m_b) : m_run;
      const float a = fast_exp2(m_run - m);
      const float b = has_b ? fast_exp2(m_b - m) : 0.0f;
      const float l = l_run * a + l_b * b;
      const float inv_a = l > 0.0f ? a / l : 0.0f;
      const float inv_b = l > 0.0f ? b / l : 0.0f;
      const int q = q0 + row;
      __nv_bfloat16* orow = out + static_cast<int64_t>(q) * out_row + static_cast<int64_t>(h) * kD;
#pragma unroll
      for (int c0 = 0; c0 < kD; c0 += 32) {
        uint32_t oa[32], ob[32];
        tmem_ld_32x32b_x32(o_col + c0, oa);
        if (has_b) tmem_ld_32x32b_x32(o_col + kBN + c0, ob);
        tmem_wait_ld();
        if (q < Tq) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              v[e] = __uint_as_float(oa[c + e]) * inv_a + (has_b ? __uint_as_float(ob[c + e]) * inv_b : 0.0f);
            *reinterpret_cast<uint4*>(orow + c0 + c) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                                  pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
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

}  // namespace attn

void attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& out, double scale,
                   const c10::optional<at::Tensor>& status, int64_t ablate) {
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
  static bool configured = false;
  if (!configured) {
    RC_CUDA(cudaFuncSetAttribute(attn::attention_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 attn::kSmemBytes));
    configured = true;
  }
  const float scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  dim3 grid((Tq + attn::kBM - 1) / attn::kBM, H);
  attn::attention_fwd_kernel<<<grid, attn::kThreads, attn::kSmemBytes, stream>>>(
      tmQ, tmK, tmVt, Tq, Tk, H, scale_log2, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0),
      status_ptr(status), static_cast<int>(ablate));
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
