// Fused restore kernel for sm_100a (the B200 counterpart of the reference's Triton
// `_fused_restore_kernel`, reelcache/restore_kernels.py:1446-1516):
//
//   native slot <- cast(RoPE(dequantize(unpack(pixels)) @ Q[:rank]))
//
// One persistent launch covers a group of jobs (one job = one chunk's K or V of one layer).
// Work item = (job, 128-token tile, 256-channel tile). Roles (448 threads, one CTA per SM):
//   warp 0      TMA producer of the basis tile Qt[256 channels x 64 rank] (fp16, 128-byte swizzle,
//               no multicast) from the transposed, zero-padded device basis of the job.
//   warp 1      TMEM owner + MMA issuer: per 64-rank block, 4 x tcgen05.mma kind::f16 for the high
//               FP16 half of the coefficients and 4 for the low half (precision "fp16x2").
//   warps 2..9  epilogue: warp w reads TMEM lane quarter (w % 4) and one 128-column half of the tile;
//               multiplies by the exact inverse prescale, applies interleaved-pair RoPE on the three
//               (t, h, w) sections from FP32 cos/sin tables (stored [pairs, rows]; loaded one
//               32-column chunk ahead), casts and stores into the native [T, H, D] / [H, T, D] slot.
//   warps 10..13 gather producers (thread = token row): read 64 rank columns of a dense uint8
//               [N, K_pad] coefficient matrix as four 16-byte vectors (decoded pictures are first
//               unpacked into that layout by csrc/restore/unpack.cu) or an fp32 matrix, dequantize
//               exactly as `float(pixel) * scale + offset` with two roundings, prescale by an exact
//               power of two, split into FP16 hi + lo and write both K-major 128-byte-swizzled A tiles.
// Three pipeline stages of {A_hi 16 KB, A_lo 16 KB, B 32 KB}; accumulators double-buffered in TMEM.
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
constexpr int kGatherWarps = 4;
constexpr int kEpilogueWarps = 8;
constexpr int kGatherThreads = kGatherWarps * 32;
constexpr int kGatherWarp0 = 2 + kEpilogueWarps;
constexpr int kThreads = (kGatherWarp0 + kGatherWarps) * 32;  // 14 warps
constexpr int kATileBytes = kBM * kBK * 2;   // 16 KB
constexpr int kBTileBytes = kBN * kBK * 2;   // 32 KB
constexpr int kStageBytes = 2 * kATileBytes + kBTileBytes;
constexpr int kTableBytes = 2 * 2 * kBK * 4 + 16;  // double-buffered {scale, offset} + abort flags
constexpr int kSmemBytes = kStages * kStageBytes + kTableBytes + 1024 + 256;
constexpr int kTmemCols = 512;

enum SourceKind : int { kMatrixU8 = 1, kMatrixF32 = 2 };
enum OutDtype : int { kOutBF16 = 0, kOutF16 = 1, kOutF32 = 2 };

struct JobDesc {
  const uint8_t* src;       // picture buffer base, or the coefficient matrix
  const int64_t* pic_off;   // [segments * frames]: byte offset of this matrix's rectangle on each picture
  const float* scale;       // [rank] per-column affine (uint8 sources)
  const float* offset;      // [rank]
  void* dst;                // element (token 0, head 0, dim 0) of the destination slot
  const float* cos;         // RoPE tables [rows, head_dim / 2] fp32 (null: no rotation)
  const float* sin;
  int64_t src_row_stride;   // matrix sources: elements between token rows
  int64_t plane_stride;     // pictures: bytes between planes
  int64_t pic_row_stride;   // pictures: bytes between picture rows
  int64_t dst_ts, dst_hs, dst_ds;  // destination element strides (token, head, dim)
  int src_kind, tokens, rank, kblocks;
  int frames, height, width;        // token grid (height * width tokens per frame)
  int planes, grid_cols, slots;     // mosaic: planes per picture, cell columns, channels per segment
  int out_dtype, channels, head_dim, n_tiles, m_tiles, work_begin;
  int rope, rope_dense, rope_rs, row_t, row_h, row_w, sec_t, sec_h;
  int split;                // 1: fp16x2 (hi + lo products), 0: fp16 (hi only)
  float prescale, inverse;
};

struct Params {
  CUtensorMap maps[kMaxJobs];  // Qt[channels, rank_pad] fp16 per job
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

// Per-K-block affine table (scale, offset of the 64 rank columns), built by the first 64 gather
// threads and double-buffered across K blocks.
struct ColumnTable {
  float scale[kBK];
  float offset[kBK];
};

__device__ __forceinline__ void build_table(const JobDesc& jb, int k0, int t, ColumnTable* tab) {
  if (t >= kBK) return;
  const int k = k0 + t;
  float sc = 0.0f, of = 0.0f;
  if (k < jb.rank && jb.src_kind == kMatrixU8) {
    sc = __ldg(jb.scale + k);
    of = __ldg(jb.offset + k);
  }
  tab->scale[t] = sc;
  tab->offset[t] = of;
}

__device__ __forceinline__ void split_store(const float (&v)[8], float prescale, int row, int col, uint8_t* a_hi,
                                            uint8_t* a_lo) {
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float s0 = v[2 * e] * prescale;
    const float s1 = v[2 * e + 1] * prescale;
    const __half h0 = __float2half_rn(s0);
    const __half h1 = __float2half_rn(s1);
    const __half l0 = __float2half_rn(s0 - __half2float(h0));
    const __half l1 = __float2half_rn(s1 - __half2float(h1));
    hi[e] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
    lo[e] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
  }
  const uint32_t off = sw128_offset_16bit(row, col);
  *reinterpret_cast<uint4*>(a_hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4*>(a_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Dequantize + split one token row (64 rank columns) of a [128 x 64] coefficient block into the
// hi/lo A tiles. uint8 sources are read as 4 x 16-byte vectors (rows padded to 64 columns).
__device__ __forceinline__ void gather_row(const JobDesc& jb, const ColumnTable* tab, int row, int m0, int k0,
                                           uint8_t* a_hi, uint8_t* a_lo) {
  const int token = m0 + row;
  const bool valid = token < jb.tokens;
  if (jb.src_kind == kMatrixU8) {
    uint4 raw[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    if (valid) {
      const uint4* rowp = reinterpret_cast<const uint4*>(jb.src + static_cast<int64_t>(token) * jb.src_row_stride + k0);
#pragma unroll
      for (int i = 0; i < 4; ++i) raw[i] = __ldg(rowp + i);
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 q = raw[c >> 1];
      const uint32_t w0 = (c & 1) ? q.z : q.x;
      const uint32_t w1 = (c & 1) ? q.w : q.y;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t byte = ((e < 4 ? w0 : w1) >> ((e & 3) * 8)) & 0xffu;
        const int kk = c * 8 + e;
        v[e] = valid ? __fadd_rn(__fmul_rn(static_cast<float>(byte), tab->scale[kk]), tab->offset[kk]) : 0.0f;
      }
      split_store(v, jb.prescale, row, c * 8, a_hi, a_lo);
    }
  } else {
    const float* rowp = reinterpret_cast<const float*>(jb.src) + static_cast<int64_t>(token) * jb.src_row_stride + k0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int kk = c * 8 + e;
        v[e] = (valid && k0 + kk < jb.rank) ? __ldg(rowp + kk) : 0.0f;
      }
      split_store(v, jb.prescale, row, c * 8, a_hi, a_lo);
    }
  }
}

__device__ __forceinline__ void gather_barrier() {
  asm volatile("bar.sync 1, %0;" ::"r"(kGatherThreads) : "memory");
}

__global__ void __maxnreg__(128) restore_kernel(const __grid_constant__ Params p, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drained = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1 + kGatherWarps);  // TMA expect_tx arrival + one arrival per gather warp
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpilogueWarps);
    }
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
    // ---------------- TMA producer (basis) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < p.total_work && ok; w += gridDim.x) {
        int j, m_tile, n_tile;
        decode_work(p, w, j, m_tile, n_tile);
        const JobDesc& jb = p.jobs[j];
        for (int kb = 0; kb < jb.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* b_dst = smem + stage * kStageBytes + 2 * kATileBytes;
          mbar_arrive_expect_tx(&full[stage], kBTileBytes);
          tma_load_2d(b_dst, &p.maps[j], &full[stage], kb * kBK, n_tile * kBN);
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
    for (int w = blockIdx.x; w < p.total_work && ok; w += gridDim.x, ++local) {
      int j, m_tile, n_tile;
      decode_work(p, w, j, m_tile, n_tile);
      const int kblocks = p.jobs[j].kblocks;
      const int split = p.jobs[j].split;
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (lane == 0) ok = mbar_wait(&acc_empty[buf], acc_phase ^ 1, status, kTimeoutMma);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * kBN;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (lane == 0) ok = mbar_wait(&full[stage], phase, status, kTimeoutMma);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t base = smem_u32(smem + stage * kStageBytes);
          const uint64_t ahi = sw128_kmajor_desc(base);
          const uint64_t alo = sw128_kmajor_desc(base + kATileBytes);
          const uint64_t bdesc = sw128_kmajor_desc(base + 2 * kATileBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16(d_tmem, ahi + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          if (split) {
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) mma_f16(d_tmem, alo + 2 * k, bdesc + 2 * k, idesc, 1u);
          }
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
  } else if (warp < kGatherWarp0) {
    // ---------------- Epilogue (8 warps) ----------------
    // Warp e = warp - 2 reads TMEM lane quarter (warp % 4) and the column half (e / 4) of the tile.
    const int quarter = warp & 3;
    const int col_half = (warp - 2) >> 2;
    int local = 0;
    for (int w = blockIdx.x; w < p.total_work; w += gridDim.x, ++local) {
      int j, m_tile, n_tile;
      decode_work(p, w, j, m_tile, n_tile);
      const JobDesc& jb = p.jobs[j];
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int token = m_tile * kBM + quarter * 32 + lane;
      const bool valid = token < jb.tokens;
      int frame = 0, y = 0, x = 0;
      if (valid) {
        const int per_frame = jb.height * jb.width;
        frame = token / per_frame;
        const int rem = token - frame * per_frame;
        y = rem / jb.width;
        x = rem - y * jb.width;
      }
      const int row_t = jb.rope_dense ? jb.row_t + token : jb.row_t + frame;
      const int row_h = jb.row_h + y;
      const int row_w = jb.row_w + x;
      // RoPE factors of the next 32-column chunk, loaded one chunk ahead (first one before the wait).
      float cs_next[16], sn_next[16];
      auto load_rope = [&](int chunk, float (&cs)[16], float (&sn)[16]) {
        const int n0 = n_tile * kBN + col_half * (kBN / 2) + chunk * 32;
        const int d0 = n0 % jb.head_dim;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int pair = (d0 >> 1) + i;
          const int trow = (jb.rope_dense || pair < jb.sec_t) ? row_t : (pair < jb.sec_t + jb.sec_h ? row_h : row_w);
          const int64_t idx = static_cast<int64_t>(pair) * jb.rope_rs + trow;  // tables stored [pairs, rows]
          cs[i] = (jb.rope && valid && n0 < jb.channels) ? __ldg(jb.cos + idx) : 1.0f;
          sn[i] = (jb.rope && valid && n0 < jb.channels) ? __ldg(jb.sin + idx) : 0.0f;
        }
      };
      load_rope(0, cs_next, sn_next);
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
        float cs[16], sn[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          cs[i] = cs_next[i];
          sn[i] = sn_next[i];
        }
        if (c + 1 < kBN / 64) load_rope(c + 1, cs_next, sn_next);
        tmem_wait_ld();
        if (!valid) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]) * jb.inverse;
        if (jb.rope) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float e = v[2 * i];
            const float o = v[2 * i + 1];
            v[2 * i] = e * cs[i] - o * sn[i];
            v[2 * i + 1] = e * sn[i] + o * cs[i];
          }
        }
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
  } else {
    // ---------------- Gather producers (4 warps, thread = token row) ----------------
    const int gt = threadIdx.x - kGatherWarp0 * 32;  // 0..127
    const int row = gt;
    ColumnTable* tables = reinterpret_cast<ColumnTable*>(smem + kStages * kStageBytes);
    // Abort flags, double-buffered by iteration parity so a flag raised at iteration k+1 is never
    // seen by a warp still finishing iteration k (every gather warp leaves at the same iteration).
    volatile int* abort_flags = reinterpret_cast<volatile int*>(tables + 2);
    if (gt < 2) abort_flags[gt] = 0;
    gather_barrier();
    int stage = 0;
    uint32_t phase = 0;
    int iter = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.total_work && ok; w += gridDim.x) {
      int j, m_tile, n_tile;
      decode_work(p, w, j, m_tile, n_tile);
      const JobDesc& jb = p.jobs[j];
      for (int kb = 0; kb < jb.kblocks; ++kb, ++iter) {
        ColumnTable* tab = tables + (iter & 1);
        build_table(jb, kb * kBK, gt, tab);
        if (lane == 0) {
          ok = mbar_wait(&empty[stage], phase ^ 1, status, kTimeoutGather);
          if (!ok) abort_flags[iter & 1] = 1;
        }
        gather_barrier();  // table and abort flag visible to every gather thread
        ok = abort_flags[iter & 1] == 0;
        if (!ok) break;
        uint8_t* a_hi = smem + stage * kStageBytes;
        gather_row(jb, tab, row, m_tile * kBM, kb * kBK, a_hi, a_hi + kATileBytes);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

}  // namespace restore

// Launches one fused restore over a group of jobs. `jobs` is an int64 CPU tensor [num_jobs, 40] of
// job fields (see reelcache_b200/ops/restore.py for the field order); `bases` the per-job
// transposed zero-padded FP16 bases Qt[channels, rank_pad].
void restore_launch(const at::Tensor& jobs, const std::vector<at::Tensor>& bases, const at::Tensor& prescale,
                    const c10::optional<at::Tensor>& status) {
  RC_CHECK(jobs.device().is_cpu() && jobs.scalar_type() == at::kLong && jobs.dim() == 2 && jobs.size(1) == 40,
           "jobs must be a CPU int64 [num_jobs, 40] table");
  const int n = static_cast<int>(jobs.size(0));
  RC_CHECK(n >= 1 && n <= restore::kMaxJobs, "between 1 and 16 jobs per launch");
  RC_CHECK(static_cast<int>(bases.size()) == n, "one basis per job");
  RC_CHECK(prescale.device().is_cpu() && prescale.scalar_type() == at::kFloat && prescale.numel() == 2 * n,
           "prescale must be a CPU float32 [num_jobs, 2] table");
  const int64_t* f = jobs.data_ptr<int64_t>();
  const float* ps = prescale.data_ptr<float>();
  restore::Params p;
  memset(&p, 0, sizeof(p));
  int work = 0;
  int device = bases[0].get_device();
  for (int i = 0; i < n; ++i) {
    const int64_t* r = f + i * 40;
    restore::JobDesc& jb = p.jobs[i];
    const at::Tensor& qt = bases[i];
    RC_CHECK(qt.is_cuda() && qt.scalar_type() == at::kHalf && qt.dim() == 2 && qt.stride(1) == 1,
             "bases must be CUDA float16 [channels, rank_pad] with unit inner stride");
    RC_CHECK(qt.get_device() == device, "all bases must share a device");
    jb.src = reinterpret_cast<const uint8_t*>(r[0]);
    jb.pic_off = reinterpret_cast<const int64_t*>(r[1]);
    jb.scale = reinterpret_cast<const float*>(r[2]);
    jb.offset = reinterpret_cast<const float*>(r[3]);
    jb.dst = reinterpret_cast<void*>(r[4]);
    jb.cos = reinterpret_cast<const float*>(r[5]);
    jb.sin = reinterpret_cast<const float*>(r[6]);
    jb.src_row_stride = r[7];
    jb.plane_stride = r[8];
    jb.pic_row_stride = r[9];
    jb.dst_ts = r[10];
    jb.dst_hs = r[11];
    jb.dst_ds = r[12];
    jb.src_kind = static_cast<int>(r[13]);
    jb.tokens = static_cast<int>(r[14]);
    jb.rank = static_cast<int>(r[15]);
    jb.frames = static_cast<int>(r[16]);
    jb.height = static_cast<int>(r[17]);
    jb.width = static_cast<int>(r[18]);
    jb.planes = static_cast<int>(r[19]);
    jb.grid_cols = static_cast<int>(r[20]);
    jb.slots = static_cast<int>(r[21]);
    jb.out_dtype = static_cast<int>(r[22]);
    jb.channels = static_cast<int>(r[23]);
    jb.head_dim = static_cast<int>(r[24]);
    jb.rope = static_cast<int>(r[25]);
    jb.rope_dense = static_cast<int>(r[26]);
    jb.rope_rs = static_cast<int>(r[27]);
    jb.row_t = static_cast<int>(r[28]);
    jb.row_h = static_cast<int>(r[29]);
    jb.row_w = static_cast<int>(r[30]);
    jb.sec_t = static_cast<int>(r[31]);
    jb.sec_h = static_cast<int>(r[32]);
    jb.split = static_cast<int>(r[33]);
    jb.prescale = ps[2 * i];
    jb.inverse = ps[2 * i + 1];
    RC_CHECK(jb.tokens >= 1 && jb.rank >= 1, "job needs tokens and rank");
    RC_CHECK(jb.src_kind == restore::kMatrixU8 || jb.src_kind == restore::kMatrixF32,
             "source must be a uint8 or float32 coefficient matrix (pictures are unpacked first)");
    RC_CHECK(jb.src_kind != restore::kMatrixU8 ||
                 (reinterpret_cast<uintptr_t>(jb.src) % 16 == 0 && jb.src_row_stride % 16 == 0 &&
                  jb.src_row_stride >= ((jb.rank + 63) / 64) * 64),
             "uint8 coefficient rows must be 16-byte aligned and padded to a multiple of 64 columns");
    RC_CHECK(jb.channels % 32 == 0 && jb.head_dim % 32 == 0 && jb.channels % jb.head_dim == 0,
             "channels and head_dim must be multiples of 32");
    RC_CHECK(qt.size(0) == jb.channels && qt.size(1) % 64 == 0 && qt.size(1) >= jb.rank,
             "basis must be [channels, rank_pad] with rank_pad a multiple of 64 covering the rank");
    RC_CHECK(jb.frames * jb.height * jb.width == jb.tokens, "grid does not match the token count");
    jb.kblocks = (jb.rank + restore::kBK - 1) / restore::kBK;
    jb.m_tiles = (jb.tokens + restore::kBM - 1) / restore::kBM;
    jb.n_tiles = (jb.channels + restore::kBN - 1) / restore::kBN;
    jb.work_begin = work;
    work += jb.m_tiles * jb.n_tiles;
    p.maps[i] = make_tmap_2d(qt.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, qt.size(1), qt.size(0),
                             qt.stride(0) * 2, restore::kBK, restore::kBN, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  p.num_jobs = n;
  p.total_work = work;
  c10::cuda::CUDAGuard guard(device);
  static bool configured[64] = {false};
  if (!configured[device]) {
    RC_CUDA(cudaFuncSetAttribute(restore::restore_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 restore::kSmemBytes));
    configured[device] = true;
  }
  const int grid = std::min(work, sm_count(device));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device).stream();
  restore::restore_kernel<<<grid, restore::kThreads, restore::kSmemBytes, stream>>>(p, status_ptr(status));
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
