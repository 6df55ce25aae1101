// Sequence-parallel Gram fit: the Gram GEMM over this rank's token shard fused with the reduce-scatter
// of the partial Grams to the matrices' fit owners, over NVLink peer memory (sm_100a).
//
// Under sequence parallelism every rank holds a token shard X_r [n_r, C] of each captured matrix and the
// fit needs G = sum_r X_r^T X_r on the matrix's owner. The library path is a local GEMM per matrix followed
// by a reduce (or all-reduce) over NCCL of the full C x C FP32 Gram. Here one persistent kernel computes,
// for a batch of matrices stacked as X^T [B * C, n_r] (bf16, K-major), every UPPER-TRIANGULAR 128 x 128 tile
// of X_r^T X_r (a Gram is symmetric, so half the tiles and half the NVLink bytes) with the tensor-core
// partials promoted to IEEE FP32 adds every 256 tokens (as gemm_exact.cu does every 128: FP32-level accuracy), and the
// epilogue stores each finished tile straight into the owner's symmetric partial buffer
// partials[rank][slot][C][C] (peer stores when the owner is another rank), so a tile's transfer overlaps
// the MMAs of the next. After a device barrier the owner sums the P partials in rank order (deterministic)
// and mirrors the upper triangle.
//
// Roles as in gemm_exact.cu: warp 0 TMA producer (plain loads of local memory), warp 1 MMA issuer (chunk g
// into TMEM buffer g % 4), warps 2..5 epilogue (IEEE accumulation of the chunk partials, then the stores).
// Every wait is bounded (status word, no trap).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <vector>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace rc {
namespace gram_rs {

constexpr int kMaxPeers = 8;
constexpr int kMaxMatrices = 64;
constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kBK = 64;
constexpr int kChunk = 4;  // K-blocks per TMEM partial (256 tokens: still FP32-level, half the promotions)
constexpr int kBufs = 4;
constexpr int kThreads = 192;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kStages = 6;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
static_assert(kSmemBytes <= 232448, "shared memory budget of one CTA");

struct Params {
  CUtensorMap tm;                // X^T stacked [B * C, n_r] bf16
  int matrices, C, K;            // K = tokens of this rank's shard
  int tiles_per_matrix;          // nt (nt + 1) / 2 upper-triangular tiles, nt = C / 128
  int nt;
  int rank, world, slots;
  float* partials[kMaxPeers];    // owner p's [world][slots][C][C] FP32 partial buffer
  int owner[kMaxMatrices];
  int slot[kMaxMatrices];
};

// Upper-triangular tile index u (row-major over i <= j) -> (i, j).
__device__ __forceinline__ void upper_tile(int u, int nt, int& i, int& j) {
  int row = 0, remaining = u;
  while (remaining >= nt - row) {
    remaining -= nt - row;
    ++row;
  }
  i = row;
  j = row + remaining;
}

__global__ void __launch_bounds__(kThreads, 1) gram_rs_kernel(const __grid_constant__ Params p, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + kBufs;
  uint64_t* drained = acc_empty + kBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.matrices * p.tiles_per_matrix;
  const int kblocks = (p.K + kBK - 1) / kBK;
  const int chunks = (kblocks + kChunk - 1) / kChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drained, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&p.tm);
  if (warp == 1) tmem_alloc(tmem_slot, kBufs * kBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int b = t / p.tiles_per_matrix;
        int ti, tj;
        upper_tile(t - b * p.tiles_per_matrix, p.nt, ti, tj);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(dst, &p.tm, &full[stage], kb * kBK, b * p.C + ti * kBM);
          tma_load_2d(dst + kABytes, &p.tm, &full[stage], kb * kBK, b * p.C + tj * kBN);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = make_idesc_f16(kBM, kBN, /*bf16*/ 1);
    int stage = 0;
    uint32_t phase = 0;
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      for (int c = 0; c < chunks && ok; ++c, ++g) {
        const int buf = g % kBufs;
        const uint32_t acc_phase = (g / kBufs) & 1;
        if (lane == 0) ok = mbar_wait(&acc_empty[buf], acc_phase ^ 1, status, kTimeoutMma);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kBN;
        const int kb_end = min(kblocks, (c + 1) * kChunk);
        for (int kb = c * kChunk; kb < kb_end; ++kb) {
          if (lane == 0) ok = mbar_wait(&full[stage], phase, status, kTimeoutMma);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(smem + stage * kStageBytes);
            const uint64_t adesc = sw128_kmajor_desc(a_addr);
            const uint64_t bdesc = sw128_kmajor_desc(a_addr + kABytes);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              mma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > c * kChunk || k > 0) ? 1u : 0u);
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
    }
    if (lane == 0) {
      mma_commit(drained);
      (void)mbar_wait(drained, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const int b = t / p.tiles_per_matrix;
      int ti, tj;
      upper_tile(t - b * p.tiles_per_matrix, p.nt, ti, tj);
      float acc[kBN];
#pragma unroll
      for (int j = 0; j < kBN; ++j) acc[j] = 0.0f;
      for (int c = 0; c < chunks; ++c, ++g) {
        const int buf = g % kBufs;
        const uint32_t acc_phase = (g / kBufs) & 1;
        if (lane == 0) ok = mbar_wait(&acc_full[buf], acc_phase, status, kTimeoutEpilogue);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + buf * kBN + (static_cast<uint32_t>(quarter * 32) << 16);
        // 32-column slices, the next one's TMEM read in flight while this one is added
        uint32_t raw[2][32];
        tmem_ld_32x32b_x32(taddr, raw[0]);
#pragma unroll
        for (int q = 0; q < kBN / 32; ++q) {
          tmem_wait_ld();
          if (q + 1 < kBN / 32) tmem_ld_32x32b_x32(taddr + (q + 1) * 32, raw[(q + 1) & 1]);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[q * 32 + j] = __fadd_rn(acc[q * 32 + j], __uint_as_float(raw[q & 1][j]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      if (!ok) break;
      // the finished tile goes straight to the matrix's owner (NVLink stores for a peer owner)
      const int row = ti * kBM + quarter * 32 + lane;
      float* dst = p.partials[p.owner[b]] +
                   ((static_cast<int64_t>(p.rank) * p.slots + p.slot[b]) * p.C + row) * p.C + tj * kBN;
#pragma unroll
      for (int j = 0; j < kBN; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kBufs * kBN);
}

}  // namespace gram_rs

// Partial Grams of this rank's shard of every matrix, delivered to the owners: xt = X^T stacked [B * C, n_r]
// bf16 (C a multiple of 128), partials[p] = owner p's FP32 [world, slots, C, C] buffer (peer views),
// owners / slots = int64 [B] on the CPU. Only the upper-triangular 128 x 128 tiles are written.
//
// to_local: every tile goes into this rank's own buffer instead (`partials` = that one buffer, [1, slots, C, C];
// slots[b] numbers the matrices globally, the same on every rank), for the in-switch reduction
// (nvls_reduce.cu), which then reads every rank's copy of a slot through the multicast address.
void gram_reduce_scatter(const at::Tensor& xt, int64_t matrices, const std::vector<at::Tensor>& partials,
                         const at::Tensor& owners, const at::Tensor& slots, int64_t rank,
                         const c10::optional<at::Tensor>& status, bool to_local) {
  using namespace gram_rs;
  check_cuda_tensor(xt, "xt");
  RC_CHECK(xt.scalar_type() == at::kBFloat16 && xt.dim() == 2 && xt.stride(1) == 1 && (xt.stride(0) * 2) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(xt.data_ptr()) % 16 == 0,
           "xt must be a 16-byte aligned bfloat16 [B * C, tokens] matrix with unit inner stride");
  RC_CHECK(matrices >= 1 && matrices <= kMaxMatrices && xt.size(0) % matrices == 0, "1..64 stacked matrices");
  const int C = static_cast<int>(xt.size(0) / matrices);
  RC_CHECK(C % 128 == 0, "channels must be a multiple of 128");
  const int world = to_local ? kMaxPeers : static_cast<int>(partials.size());
  RC_CHECK(!to_local || partials.size() == 1, "to_local takes this rank's own buffer only");
  RC_CHECK(to_local || (world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world),
           "one partial buffer per rank (<= 8)");
  RC_CHECK(owners.device().is_cpu() && owners.scalar_type() == at::kLong && owners.numel() == matrices &&
               slots.device().is_cpu() && slots.scalar_type() == at::kLong && slots.numel() == matrices,
           "owners and slots must be CPU int64 [B]");
  Params p;
  memset(&p, 0, sizeof(p));
  p.matrices = static_cast<int>(matrices);
  p.C = C;
  p.K = static_cast<int>(xt.size(1));
  RC_CHECK(p.K % 8 == 0 && p.K > 0, "tokens must be a positive multiple of 8");
  p.nt = C / 128;
  p.tiles_per_matrix = p.nt * (p.nt + 1) / 2;
  p.rank = to_local ? 0 : static_cast<int>(rank);
  p.world = world;
  const int64_t* own = owners.data_ptr<int64_t>();
  const int64_t* sl = slots.data_ptr<int64_t>();
  int max_slot = 0;
  for (int b = 0; b < matrices; ++b) {
    RC_CHECK(own[b] >= 0 && own[b] < world && sl[b] >= 0, "owner / slot out of range");
    p.owner[b] = static_cast<int>(own[b]);
    p.slot[b] = static_cast<int>(sl[b]);
    max_slot = std::max(max_slot, p.slot[b]);
  }
  for (int r = 0; r < world; ++r) {
    const at::Tensor& t = partials[to_local ? 0 : r];
    RC_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous() && t.dim() == 4 && t.size(0) == (to_local ? 1 : world) &&
                 t.size(2) == C && t.size(3) == C && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
             "partial buffers must be contiguous float32 [world, slots, C, C]");
    RC_CHECK(t.size(1) > max_slot, "a slot index exceeds the partial buffer");
    p.slots = static_cast<int>(t.size(1));
    p.partials[r] = t.data_ptr<float>();
  }
  p.tm = make_tmap_2d(xt.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.K, xt.size(0), xt.stride(0) * 2, kBK, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  c10::cuda::CUDAGuard guard(xt.device());
  static bool configured[64] = {false};
  const int device = xt.get_device();
  if (!configured[device]) {
    RC_CUDA(cudaFuncSetAttribute(gram_rs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    configured[device] = true;
  }
  const int tiles = p.matrices * p.tiles_per_matrix;
  const int grid = std::min(tiles, sm_count(device));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device).stream();
  gram_rs_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p, status_ptr(status));
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
