// Fused restore GEMM for sm_100a (the B200 counterpart of the reference's Triton
// `_fused_restore_kernel`, reelcache/restore_kernels.py:1446-1516):
//
//   native slot <- cast(RoPE(dequantize(pixels) @ Q[:rank]))
//
// computed as  acc = A @ Bt^T  with  A[n, k] = p[n, k] - 128  (exact FP16, unpack.cu) and
// Bt = hi/lo FP16 split of s[k] * Q[k, c] * 2^e (prep.cu), then  y = acc * 2^-e + bias[c]  with the
// per-channel bias sum_k (o[k] + 128 s[k]) Q[k, c]; "fp16x2" runs both halves, "fp16" the hi half.
//
// One persistent launch covers a group of jobs (one job = one chunk's K or V of one layer).
// Work item = (job, 128-token tile, 256-channel tile); each CTA owns a contiguous range of items.
// Roles (320 threads, one CTA per SM):
//   warp 0      TMA producer: per K block the A tile [128 x 64] and the B tile [256 x 64] (hi half,
//               then the lo half in a second pass); 128-byte swizzle, no multicast; 3 stages of 48 KB.
//   warp 1      TMEM owner and MMA issuer (4 x tcgen05.mma kind::f16 per K block).
//   warps 2..9  epilogue: warp w reads TMEM lane quarter (w % 4) and one 128-column half of the tile;
//               applies scale + bias and interleaved-pair RoPE, casts, and writes each 32 x 32 block
//               to a 64-byte-swizzled SMEM buffer that a TMA bulk store (double-buffered per warp)
//               copies into the native cache slot; layouts whose channels are not contiguous take
//               per-thread strided stores instead.
// RoPE and bias operands live in shared memory per job: the 3-axis (frame, row, column) tables are
// separable, so a job needs only its T x Pt + H x Ph + W x Pw (cos, sin) entries, not one row per
// token; the 8 epilogue warps load them cooperatively when the job changes (mbarrier handshake,
// bounded waits). Lanes of a warp hold consecutive tokens, so the frame and row sections are
// broadcast reads and the column section is conflict-free. Dense (non-separable) tables fall back to
// per-token FP32 rows [tokens, pairs] read from global memory.
// Accumulators are double-buffered in TMEM (2 x 256 columns) so the epilogue of one tile overlaps
// the main loop of the next. The launch parameters (tensor maps included) are built once on the host
// (restore_build) and launched any number of times (restore_run).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <vector>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace rc {
namespace restore {

constexpr int kMaxJobs = 16;
constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 3;
constexpr int kEpilogueWarps = 8;
constexpr int kThreads = (2 + kEpilogueWarps) * 32;
constexpr int kATileBytes = kBM * kBK * 2;   // 16 KB
constexpr int kBTileBytes = kBN * kBK * 2;   // 32 KB
constexpr int kStageBytes = kATileBytes + kBTileBytes;
constexpr int kOutBufBytes = 32 * 32 * 2;    // one 32 x 32 16-bit output block
constexpr int kOutBytes = kEpilogueWarps * 2 * kOutBufBytes;
constexpr int kRopeEntries = 5120;          // (cos, sin) float2 entries of one job's separable tables
constexpr int kBiasSmem = 2048;             // channels whose bias is staged in shared memory
constexpr int kSmemBytes = kStages * kStageBytes + kOutBytes + kRopeEntries * 8 + kBiasSmem * 4 + 1024 + 256;
static_assert(kSmemBytes <= 232448, "shared memory budget of one CTA");
constexpr int kTmemCols = 512;

enum OutDtype : int { kOutBF16 = 0, kOutF16 = 1, kOutF32 = 2 };
enum RopeMode : int { kRopeNone = 0, kRopeTokens = 1, kRopePacked = 2 };

struct JobDesc {
  void* dst;                // element (token 0, head 0, dim 0) of the destination slot
  const float* bias;        // [channels]
  const float* cos;         // kRopeTokens: per-token tables [tokens, pairs] fp32;
  const float* sin;         // kRopePacked: cos = (cos, sin) pairs of the T, H, W sections back to back
  int64_t dst_ts, dst_hs, dst_ds;  // destination element strides (token, head, dim)
  int tokens, kblocks, passes;     // passes: 2 = hi + lo, 1 = hi only
  int a_kblocks, b_kblocks;        // K blocks held by the A / B operands (coordinates wrap)
  int out_dtype, channels, head_dim, n_tiles, work_begin;
  int rope, pairs, tma_store;
  int sec_t, sec_th;               // kRopePacked: pairs [0, sec_t) frame, [sec_t, sec_th) row, rest column
  int grid_h, grid_w, off_h, off_w, entries;
  int bias_smem;                   // bias staged in shared memory (channels <= kBiasSmem)
  float inverse;
};

struct Params {
  CUtensorMap a_maps[kMaxJobs];  // A [tokens, k_pad] fp16, box 64 x 128
  CUtensorMap b_maps[kMaxJobs];  // Bt [channels, k_pad or 2 k_pad] fp16, box 64 x 256
  CUtensorMap o_maps[kMaxJobs];  // destination [tokens, channels] 16-bit, box 32 x 32, 64-byte swizzle
  JobDesc jobs[kMaxJobs];
  int num_jobs;
  int total_work;
};

__device__ __forceinline__ void decode_work(const Params& p, int w, int& j, int& m_tile, int& n_tile) {
  j = 0;
#pragma unroll 1
  for (int i = 1; i < p.num_jobs; ++i)
    if (w >= p.jobs[i].work_begin) j = i;
  const int local = w - p.jobs[j].work_begin;
  m_tile = local / p.jobs[j].n_tiles;
  n_tile = local - m_tile * p.jobs[j].n_tiles;
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) restore_kernel(const __grid_constant__ Params p, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* out_smem = smem + kStages * kStageBytes;
  float2* rope_smem = reinterpret_cast<float2*>(out_smem + kOutBytes);
  float* bias_smem = reinterpret_cast<float*>(rope_smem + kRopeEntries);
  uint64_t* full = reinterpret_cast<uint64_t*>(bias_smem + kBiasSmem);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* tab_free = acc_empty + 2;   // every epilogue thread is done with the current job's tables
  uint64_t* tab_ready = tab_free + 1;   // every epilogue thread has stored its share of the next ones
  uint64_t* drained = tab_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Each CTA owns a contiguous range of work items: consecutive tiles mostly share one job's tensor
  // maps (descriptor-cache hits) and A tile (L2 hits).
  const int work_lo = static_cast<int>((static_cast<int64_t>(p.total_work) * blockIdx.x) / gridDim.x);
  const int work_hi = static_cast<int>((static_cast<int64_t>(p.total_work) * (blockIdx.x + 1)) / gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpilogueWarps);
    }
    mbar_init(tab_free, kEpilogueWarps * 32);
    mbar_init(tab_ready, kEpilogueWarps * 32);
    mbar_init(drained, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
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
      int last_job = -1;
      for (int w = work_lo; w < work_hi && ok; ++w) {
        int j, m_tile, n_tile;
        decode_work(p, w, j, m_tile, n_tile);
        const JobDesc& jb = p.jobs[j];
        if (j != last_job) {
          tma_prefetch_desc(&p.a_maps[j]);
          tma_prefetch_desc(&p.b_maps[j]);
          last_job = j;
        }
        const int steps = jb.kblocks * jb.passes;
        for (int s = 0; s < steps; ++s) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          // 8-bit sources: A [N, k_pad] is read twice, B [C, 2 k_pad] holds the hi then the lo half.
          // Float sources: A [N, 2 k_pad] holds hi then lo, B [C, k_pad] is read twice.
          tma_load_2d(a_dst, &p.a_maps[j], &full[stage], (s % jb.a_kblocks) * kBK, m_tile * kBM);
          tma_load_2d(a_dst + kATileBytes, &p.b_maps[j], &full[stage], (s % jb.b_kblocks) * kBK, n_tile * kBN);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = make_idesc_f16(kBM, kBN, /*f16*/ 0);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int w = work_lo; w < work_hi && ok; ++w, ++local) {
      int j, m_tile, n_tile;
      decode_work(p, w, j, m_tile, n_tile);
      const int steps = p.jobs[j].kblocks * p.jobs[j].passes;
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (lane == 0) ok = mbar_wait(&acc_empty[buf], acc_phase ^ 1, status, kTimeoutMma);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * kBN;
      for (int s = 0; s < steps; ++s) {
        if (lane == 0) ok = mbar_wait(&full[stage], phase, status, kTimeoutMma);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t base = smem_u32(smem + stage * kStageBytes);
          const uint64_t adesc = sw128_kmajor_desc(base);
          const uint64_t bdesc = sw128_kmajor_desc(base + kATileBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (s > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) mma_commit(&acc_full[buf]);
      __syncwarp();
    }
    if (lane == 0) {
      mma_commit(drained);
      (void)mbar_wait(drained, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    // ---------------- Epilogue (8 warps) ----------------
    const int quarter = warp & 3;
    const int col_half = (warp - 2) >> 2;
    const int et = threadIdx.x - 64;  // 0 .. 255 among the epilogue threads
    uint8_t* my_out = out_smem + (warp - 2) * 2 * kOutBufBytes;
    int local = 0;
    int block = 0;  // output blocks written by this warp (selects the staging buffer)
    int table_job = -1, table_loads = 0;
    for (int w = work_lo; w < work_hi; ++w, ++local) {
      int j, m_tile, n_tile;
      decode_work(p, w, j, m_tile, n_tile);
      const JobDesc& jb = p.jobs[j];
      if (j != table_job) {
        // Job change (the same tile sequence for all 8 warps): wait until every epilogue thread is
        // done with the previous job's shared tables, store this job's share, publish.
        bool ok = true;
        if (table_loads > 0) {
          mbar_arrive(tab_free);
          ok = mbar_wait(tab_free, (table_loads - 1) & 1, status, kTimeoutEpilogue);
        }
        if (__all_sync(0xffffffffu, ok)) {
          if (jb.rope == kRopePacked) {
            const float2* src = reinterpret_cast<const float2*>(jb.cos);
            for (int i = et; i < jb.entries; i += kEpilogueWarps * 32) rope_smem[i] = __ldg(src + i);
          }
          if (jb.bias_smem) {
            for (int i = et; i < jb.channels; i += kEpilogueWarps * 32) bias_smem[i] = __ldg(jb.bias + i);
          }
          mbar_arrive(tab_ready);
          ok = mbar_wait(tab_ready, table_loads & 1, status, kTimeoutEpilogue);
        }
        if (!__all_sync(0xffffffffu, ok)) break;
        table_job = j;
        ++table_loads;
      }
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int row0 = m_tile * kBM + quarter * 32;
      const int token = row0 + lane;
      const bool valid = token < jb.tokens;
      const int tok = valid ? token : 0;
      // kRopePacked: entry of pair q is base(q) + q with one base per section
      int base_t = 0, base_h = 0, base_w = 0;
      if (jb.rope == kRopePacked) {
        const int hw = jb.grid_h * jb.grid_w;
        const int f = tok / hw;
        const int rem = tok - f * hw;
        const int y = rem / jb.grid_w;
        const int x = rem - y * jb.grid_w;
        base_t = f * jb.sec_t;
        base_h = jb.off_h + y * (jb.sec_th - jb.sec_t) - jb.sec_t;
        base_w = jb.off_w + x * (jb.pairs - jb.sec_th) - jb.sec_th;
      }
      const float* cos_row = jb.cos + static_cast<int64_t>(tok) * jb.pairs;
      const float* sin_row = jb.sin + static_cast<int64_t>(tok) * jb.pairs;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&acc_full[buf], acc_phase, status, kTimeoutEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < kBN / 64; ++c) {
        const int n0 = n_tile * kBN + col_half * (kBN / 2) + c * 32;
        if (n0 >= jb.channels) break;  // uniform: channels is a multiple of 32 (checked on the host)
        uint32_t raw[32];
        tmem_ld_32x32b_x32(tmem_base + buf * kBN + col_half * (kBN / 2) + c * 32 +
                               (static_cast<uint32_t>(quarter * 32) << 16),
                           raw);
        float bias[32];
        if (jb.bias_smem) {
          const float4* bias4 = reinterpret_cast<const float4*>(bias_smem + n0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 b = bias4[i];
            bias[4 * i] = b.x; bias[4 * i + 1] = b.y; bias[4 * i + 2] = b.z; bias[4 * i + 3] = b.w;
          }
        } else {
          const float4* bias4 = reinterpret_cast<const float4*>(jb.bias + n0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 b = __ldg(bias4 + i);
            bias[4 * i] = b.x; bias[4 * i + 1] = b.y; bias[4 * i + 2] = b.z; bias[4 * i + 3] = b.w;
          }
        }
        const int pair0 = (n0 % jb.head_dim) >> 1;
        float cs[16], sn[16];
        if (jb.rope == kRopePacked) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int q = pair0 + i;
            const int e = q + (q < jb.sec_t ? base_t : (q < jb.sec_th ? base_h : base_w));
            const float2 v = rope_smem[e];
            cs[i] = v.x;
            sn[i] = v.y;
          }
        } else if (jb.rope == kRopeTokens && valid) {
          const float4* c4 = reinterpret_cast<const float4*>(cos_row + pair0);
          const float4* s4 = reinterpret_cast<const float4*>(sin_row + pair0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 cv = __ldg(c4 + i);
            const float4 sv = __ldg(s4 + i);
            cs[4 * i] = cv.x; cs[4 * i + 1] = cv.y; cs[4 * i + 2] = cv.z; cs[4 * i + 3] = cv.w;
            sn[4 * i] = sv.x; sn[4 * i + 1] = sv.y; sn[4 * i + 2] = sv.z; sn[4 * i + 3] = sv.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            cs[i] = 1.0f;
            sn[i] = 0.0f;
          }
        }
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = fmaf(__uint_as_float(raw[i]), jb.inverse, bias[i]);
        if (jb.rope != kRopeNone) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float e = v[2 * i];
            const float o = v[2 * i + 1];
            v[2 * i] = e * cs[i] - o * sn[i];
            v[2 * i + 1] = e * sn[i] + o * cs[i];
          }
        }
        if (jb.tma_store) {
          // 32 x 32 16-bit block -> 64-byte-swizzled staging buffer -> TMA bulk store.
          uint8_t* ob = my_out + (block & 1) * kOutBufBytes;
          if (lane == 0) bulk_wait_read<1>();  // the store that used this buffer two blocks ago has read it
          __syncwarp();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = jb.out_dtype == kOutBF16 ? pack_bf16x2(v[2 * i], v[2 * i + 1]) : pack_f16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t phys = static_cast<uint32_t>(q) ^ ((static_cast<uint32_t>(lane) >> 1) & 3u);
            *reinterpret_cast<uint4*>(ob + lane * 64 + phys * 16) =
                make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < jb.tokens) {
            tma_store_2d(&p.o_maps[j], ob, n0, row0);
            bulk_commit();
          }
          ++block;
          continue;
        }
        if (!valid) continue;
        const int head = n0 / jb.head_dim;
        const int d0 = n0 - head * jb.head_dim;
        const int64_t base = static_cast<int64_t>(token) * jb.dst_ts + static_cast<int64_t>(head) * jb.dst_hs +
                             static_cast<int64_t>(d0) * jb.dst_ds;
        if (jb.out_dtype == kOutF32) {
          float* out = reinterpret_cast<float*>(jb.dst) + base;
          if (jb.dst_ds == 1 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(out + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
            for (int i = 0; i < 32; ++i) out[static_cast<int64_t>(i) * jb.dst_ds] = v[i];
          }
        } else {
          uint16_t* out = reinterpret_cast<uint16_t*>(jb.dst) + base;
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = jb.out_dtype == kOutBF16 ? pack_bf16x2(v[2 * i], v[2 * i + 1]) : pack_f16x2(v[2 * i], v[2 * i + 1]);
          if (jb.dst_ds == 1 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<uint4*>(out + 2 * i) = make_uint4(pk[i], pk[i + 1], pk[i + 2], pk[i + 3]);
          } else {
            for (int i = 0; i < 16; ++i) {
              out[static_cast<int64_t>(2 * i) * jb.dst_ds] = static_cast<uint16_t>(pk[i] & 0xffffu);
              out[static_cast<int64_t>(2 * i + 1) * jb.dst_ds] = static_cast<uint16_t>(pk[i] >> 16);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    // every bulk store must have finished reading its staging buffer before the CTA exits
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

}  // namespace restore

// Builds the launch parameters of one fused restore over <= 16 jobs (tensor maps encoded once) and
// returns them as a CPU byte tensor for restore_run. `jobs` is a CPU int64 [n, 40] table (field
// order: reelcache_b200/ops/restore.py, RestoreProgram.prepare); `a_ops` the per-job A operands and
// `b_ops` the prepared B operands; `inverse` the exact inverse prescales (CPU float32 [n]).
at::Tensor restore_build(const at::Tensor& jobs, const std::vector<at::Tensor>& a_ops, const std::vector<at::Tensor>& b_ops,
                         const at::Tensor& inverse) {
  RC_CHECK(jobs.device().is_cpu() && jobs.scalar_type() == at::kLong && jobs.dim() == 2 && jobs.size(1) == 40,
           "jobs must be a CPU int64 [num_jobs, 40] table");
  const int n = static_cast<int>(jobs.size(0));
  RC_CHECK(n >= 1 && n <= restore::kMaxJobs, "between 1 and 16 jobs per launch");
  RC_CHECK(static_cast<int>(a_ops.size()) == n && static_cast<int>(b_ops.size()) == n, "one A and B operand per job");
  RC_CHECK(inverse.device().is_cpu() && inverse.scalar_type() == at::kFloat && inverse.numel() == n,
           "inverse must be a CPU float32 [num_jobs] vector");
  at::Tensor blob = at::zeros({static_cast<int64_t>(sizeof(restore::Params))}, at::TensorOptions().dtype(at::kByte));
  restore::Params& p = *reinterpret_cast<restore::Params*>(blob.data_ptr<uint8_t>());
  const int64_t* f = jobs.data_ptr<int64_t>();
  const float* inv = inverse.data_ptr<float>();
  int work = 0;
  const int device = a_ops[0].get_device();
  for (int i = 0; i < n; ++i) {
    const int64_t* r = f + i * 40;
    restore::JobDesc& jb = p.jobs[i];
    const at::Tensor& a = a_ops[i];
    const at::Tensor& b = b_ops[i];
    RC_CHECK(a.is_cuda() && a.scalar_type() == at::kHalf && a.dim() == 2 && a.stride(1) == 1,
             "A operands must be CUDA float16 [tokens, k_pad] with unit inner stride");
    RC_CHECK(b.is_cuda() && b.scalar_type() == at::kHalf && b.dim() == 2 && b.stride(1) == 1,
             "B operands must be CUDA float16 [channels, 2 * k_pad] with unit inner stride");
    RC_CHECK(a.get_device() == device && b.get_device() == device, "all operands must share a device");
    jb.dst = reinterpret_cast<void*>(r[0]);
    jb.bias = reinterpret_cast<const float*>(r[1]);
    jb.cos = reinterpret_cast<const float*>(r[2]);
    jb.sin = reinterpret_cast<const float*>(r[3]);
    jb.dst_ts = r[4];
    jb.dst_hs = r[5];
    jb.dst_ds = r[6];
    jb.tokens = static_cast<int>(r[7]);
    jb.passes = static_cast<int>(r[8]);
    jb.out_dtype = static_cast<int>(r[12]);
    jb.channels = static_cast<int>(r[13]);
    jb.head_dim = static_cast<int>(r[14]);
    jb.rope = static_cast<int>(r[15]);
    jb.pairs = static_cast<int>(r[17]);
    jb.sec_t = static_cast<int>(r[18]);
    jb.sec_th = static_cast<int>(r[18] + r[19]);
    jb.entries = static_cast<int>(r[20]);
    jb.grid_h = static_cast<int>(r[10]);
    jb.grid_w = static_cast<int>(r[11]);
    jb.off_h = static_cast<int>(r[9] * r[18]);
    jb.off_w = static_cast<int>(r[9] * r[18] + r[10] * r[19]);
    jb.inverse = inv[i];
    const int64_t k_pad = std::min(a.size(1), b.size(1));
    RC_CHECK(k_pad % 64 == 0 && (a.size(1) == k_pad || a.size(1) == 2 * k_pad) &&
                 (b.size(1) == k_pad || b.size(1) == 2 * k_pad),
             "operand K extents must be k_pad or 2 * k_pad (k_pad a multiple of 64)");
    RC_CHECK(a.size(0) == jb.tokens && b.size(0) == jb.channels, "operand extents disagree with the job");
    RC_CHECK(jb.passes == 1 || jb.passes == 2, "passes must be 1 or 2");
    RC_CHECK(jb.channels % 32 == 0 && jb.head_dim % 32 == 0 && jb.channels % jb.head_dim == 0,
             "channels and head_dim must be multiples of 32");
    RC_CHECK(reinterpret_cast<uintptr_t>(jb.bias) % 16 == 0, "bias must be 16-byte aligned");
    RC_CHECK(jb.rope >= restore::kRopeNone && jb.rope <= restore::kRopePacked, "unknown RoPE mode");
    RC_CHECK(jb.rope != restore::kRopeTokens ||
                 (reinterpret_cast<uintptr_t>(jb.cos) % 16 == 0 && reinterpret_cast<uintptr_t>(jb.sin) % 16 == 0 &&
                  jb.pairs * 2 == jb.head_dim),
             "RoPE token tables must be 16-byte aligned [tokens, head_dim / 2] float32 rows");
    if (jb.rope == restore::kRopePacked) {
      RC_CHECK(jb.pairs * 2 == jb.head_dim && jb.sec_t >= 0 && jb.sec_th >= jb.sec_t && jb.sec_th <= jb.pairs,
               "RoPE sections must split head_dim / 2 pairs");
      RC_CHECK(jb.grid_h >= 1 && jb.grid_w >= 1 && r[9] * r[10] * r[11] == jb.tokens, "grid must cover the tokens");
      RC_CHECK(jb.entries == r[9] * r[18] + r[10] * r[19] + r[11] * (jb.pairs - jb.sec_th) &&
                   jb.entries <= restore::kRopeEntries && reinterpret_cast<uintptr_t>(jb.cos) % 8 == 0,
               "packed RoPE tables: T*Pt + H*Ph + W*Pw (cos, sin) entries, at most 5120, 8-byte aligned");
    }
    jb.bias_smem = jb.channels <= restore::kBiasSmem;
    jb.kblocks = static_cast<int>(k_pad / restore::kBK);
    jb.a_kblocks = static_cast<int>(a.size(1) / restore::kBK);
    jb.b_kblocks = static_cast<int>(b.size(1) / restore::kBK);
    RC_CHECK(jb.passes == 1 || (jb.a_kblocks + jb.b_kblocks == 3 * jb.kblocks), "two passes need one doubled operand");
    jb.n_tiles = (jb.channels + restore::kBN - 1) / restore::kBN;
    jb.work_begin = work;
    work += ((jb.tokens + restore::kBM - 1) / restore::kBM) * jb.n_tiles;
    p.a_maps[i] = make_tmap_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.size(1), a.size(0), a.stride(0) * 2,
                               restore::kBK, restore::kBM, CU_TENSOR_MAP_SWIZZLE_128B);
    p.b_maps[i] = make_tmap_2d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b.size(1), b.size(0), b.stride(0) * 2,
                               restore::kBK, restore::kBN, CU_TENSOR_MAP_SWIZZLE_128B);
    // TMA stores need channels contiguous inside each token row (BTHD / THD caches)
    jb.tma_store = jb.out_dtype != restore::kOutF32 && jb.dst_ds == 1 && jb.dst_hs == jb.head_dim &&
                   reinterpret_cast<uintptr_t>(jb.dst) % 16 == 0 && (jb.dst_ts * 2) % 16 == 0;
    if (jb.tma_store)
      p.o_maps[i] = make_tmap_2d(jb.dst, jb.out_dtype == restore::kOutBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                 2, jb.channels, jb.tokens, jb.dst_ts * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  p.num_jobs = n;
  p.total_work = work;
  return blob;
}

void restore_run(const at::Tensor& blob, int64_t device, const c10::optional<at::Tensor>& status) {
  RC_CHECK(blob.device().is_cpu() && blob.scalar_type() == at::kByte &&
               blob.numel() == static_cast<int64_t>(sizeof(restore::Params)),
           "restore_run takes the byte tensor returned by restore_build");
  const restore::Params& p = *reinterpret_cast<const restore::Params*>(blob.data_ptr<uint8_t>());
  const int dev = static_cast<int>(device);
  c10::cuda::CUDAGuard guard(dev);
  static bool configured[64] = {false};
  if (!configured[dev]) {
    RC_CUDA(cudaFuncSetAttribute(restore::restore_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 restore::kSmemBytes));
    configured[dev] = true;
  }
  const int grid = std::min(p.total_work, sm_count(dev));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  restore::restore_kernel<<<grid, restore::kThreads, restore::kSmemBytes, stream>>>(p, status_ptr(status));
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
