// FP32-accurate tcgen05 GEMM for sm_100a: D[M, N] = alpha * A[M, K] * B[N, K]^T with bf16 operands
// (both K-major) whose products are exact in FP32, and with the accumulation promoted out of the tensor
// cores every kChunk K-blocks.
//
// Why: the tensor cores' FP32 accumulation is not IEEE round-to-nearest; measured on B200, the relative
// error of a bf16 GEMM with exactly representable inputs grows linearly with K (about 5e-6 at K = 4680,
// 3e-5 at K = 28080, against 2e-7 and 3e-7 for an IEEE FP32 GEMM). Here each TMEM accumulator only ever
// sums kChunk * 64 = 128 K-elements (where the tensor-core error is at the FP32 level), and the epilogue
// warps add the chunk partials into FP32 registers with IEEE adds. With the split-bf16 operands of
// csrc/fit/fitter.cu (FP32 = hi + mid + lo, six cross products as K-concatenated segments) this is an
// FP32 GEMM on the tensor cores.
//
// Roles (192 threads, one CTA per SM, persistent over 128 x 128 tiles, or over (tile, K-split) items when the
// tiles alone fill less than half of the SMs):
//   warp 0      TMA producer (A and B tiles of 64 K per stage, 128-byte swizzle; plain loads).
//   warp 1      TMEM owner and MMA issuer: chunk g of the CTA accumulates into TMEM buffer g % 4
//               (4 x 128 columns), committed to acc_full[g % 4].
//   warps 2..5  epilogue: per chunk, tcgen05.ld of the partial (warp w reads TMEM lanes 32 (w % 4) + 0..31),
//               128 IEEE adds into the running row sums, release of the buffer; at the tile end the sums
//               (times alpha) are stored as FP32.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace rc {
namespace gemm_exact {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kBK = 64;
constexpr int kChunk = 2;           // K-blocks per TMEM partial (128 K-elements)
constexpr int kBufs = 4;            // TMEM partial buffers (4 x 128 fp32 columns = 512)
constexpr int kThreads = 192;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kStages = 6;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
constexpr int kGroupM = 8;

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m_idx, int& n_idx) {
  const int per_group = kGroupM * num_n;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - group * per_group;
  m_idx = first_m + r % gsize;
  n_idx = r / gsize;
}

// Split-K: work item w covers tile w / splits and the chunks [s * per, min(chunks, (s + 1) * per)) of split
// s = w % splits, storing its FP32 partial at out + s * split_stride (one reduction sums the partials).
__device__ __forceinline__ void item_range(int w, int splits, int per, int chunks, int& tile, int& c0, int& c1) {
  tile = w / splits;
  const int s = w - tile * splits;
  c0 = s * per;
  c1 = min(chunks, c0 + per);
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_promoted_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M,
                         int N, int K, float* __restrict__ out, int64_t ldo, float alpha, int* status, int splits,
                         int64_t split_stride) {
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
  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + kBN - 1) / kBN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (K + kBK - 1) / kBK;
  const int chunks = (kblocks + kChunk - 1) / kChunk;
  const int per = (chunks + splits - 1) / splits;
  const int num_items = num_tiles * splits;

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
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
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
      for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
        int t, c0, c1;
        item_range(w, splits, per, chunks, t, c0, c1);
        int m_idx, n_idx;
        tile_coords(t, num_m, num_n, m_idx, n_idx);
        const int kb_stop = min(kblocks, c1 * kChunk);
        for (int kb = c0 * kChunk; kb < kb_stop; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(a_dst, &tmA, &full[stage], kb * kBK, m_idx * kBM);
          tma_load_2d(a_dst + kABytes, &tmB, &full[stage], kb * kBK, n_idx * kBN);
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
    int g = 0;  // chunk counter of this CTA
    bool ok = true;
    for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
      int t, c0, c1;
      item_range(w, splits, per, chunks, t, c0, c1);
      for (int c = c0; c < c1 && ok; ++c, ++g) {
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
    for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
      int t, c0, c1;
      item_range(w, splits, per, chunks, t, c0, c1);
      int m_idx, n_idx;
      tile_coords(t, num_m, num_n, m_idx, n_idx);
      float* part = out + static_cast<int64_t>(w - t * splits) * split_stride;
      float acc[kBN];
#pragma unroll
      for (int j = 0; j < kBN; ++j) acc[j] = 0.0f;
      for (int c = c0; c < c1; ++c, ++g) {
        const int buf = g % kBufs;
        const uint32_t acc_phase = (g / kBufs) & 1;
        if (lane == 0) ok = mbar_wait(&acc_full[buf], acc_phase, status, kTimeoutEpilogue);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + buf * kBN + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
        for (int q = 0; q < kBN / 32; ++q) {
          uint32_t raw[32];
          tmem_ld_32x32b_x32(taddr + q * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[q * 32 + j] = __fadd_rn(acc[q * 32 + j], __uint_as_float(raw[j]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      if (!ok) break;
      const int row = m_idx * kBM + quarter * 32 + lane;
      if (row < M) {
        float* orow = part + static_cast<int64_t>(row) * ldo + n_idx * kBN;
        const int valid = min(kBN, N - n_idx * kBN);
        if (valid == kBN && (reinterpret_cast<uintptr_t>(orow) & 15) == 0) {
#pragma unroll
          for (int j = 0; j < kBN; j += 4)
            *reinterpret_cast<float4*>(orow + j) =
                make_float4(acc[j] * alpha, acc[j + 1] * alpha, acc[j + 2] * alpha, acc[j + 3] * alpha);
        } else {
#pragma unroll
          for (int j = 0; j < kBN; ++j)
            if (j < valid) orow[j] = acc[j] * alpha;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kBufs * kBN);
}

}  // namespace gemm_exact

void gemm_bf16_promoted(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, double alpha,
                        const c10::optional<at::Tensor>& status) {
  check_cuda_tensor(A, "A");
  check_cuda_tensor(B, "B");
  check_cuda_tensor(out, "out");
  RC_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "A and B must be bfloat16");
  RC_CHECK(out.scalar_type() == at::kFloat, "out must be float32");
  RC_CHECK(A.dim() == 2 && B.dim() == 2 && out.dim() == 2, "2-D operands");
  RC_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && out.stride(1) == 1, "unit inner strides");
  const int M = static_cast<int>(A.size(0)), K = static_cast<int>(A.size(1)), N = static_cast<int>(B.size(0));
  RC_CHECK(B.size(1) == K && out.size(0) == M && out.size(1) == N, "shapes");
  RC_CHECK(K % 8 == 0 && M > 0 && N > 0 && K > 0, "K must be a positive multiple of 8");
  RC_CHECK((A.stride(0) * 2) % 16 == 0 && (B.stride(0) * 2) % 16 == 0, "row strides must be 16-byte multiples");
  c10::cuda::CUDAGuard guard(A.device());
  using namespace gemm_exact;
  CUtensorMap tmA = make_tmap_2d(A.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, A.stride(0) * 2, kBK, kBM,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tmB = make_tmap_2d(B.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, B.stride(0) * 2, kBK, kBN,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  static bool configured = false;
  if (!configured) {
    RC_CUDA(cudaFuncSetAttribute(gemm_promoted_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    configured = true;
  }
  const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  const int sms = sm_count(A.get_device());
  const int chunks = ((K + kBK - 1) / kBK + kChunk - 1) / kChunk;
  // Split K when the tiles fill less than half of the SMs: each split keeps >= 2 chunks (256 K-elements), the
  // partials land in a workspace and one deterministic reduction sums them (FP32 adds of FP32-accurate partials).
  int splits = 1;
  if (tiles * 2 <= sms && chunks >= 4) splits = std::min(chunks / 2, (sms + tiles - 1) / tiles);
  if (splits > 1) {
    const int per = (chunks + splits - 1) / splits;
    splits = (chunks + per - 1) / per;  // no empty split
  }
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(A.get_device()).stream();
  if (splits == 1) {
    const int grid = std::min(tiles, sms);
    gemm_promoted_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmA, tmB, M, N, K, out.data_ptr<float>(),
                                                                  out.stride(0), static_cast<float>(alpha),
                                                                  status_ptr(status), 1, 0);
    RC_CUDA(cudaGetLastError());
    return;
  }
  at::Tensor work = at::empty({splits, M, N}, out.options());
  const int grid = std::min(tiles * splits, sms);
  gemm_promoted_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmA, tmB, M, N, K, work.data_ptr<float>(), N,
                                                                static_cast<float>(alpha), status_ptr(status),
                                                                splits, static_cast<int64_t>(M) * N);
  RC_CUDA(cudaGetLastError());
  at::sum_out(out, work, {0});  // one deterministic reduction over the splits
}

}  // namespace rc
