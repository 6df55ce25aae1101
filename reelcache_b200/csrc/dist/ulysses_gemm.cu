// Ulysses all-to-all fused into the projection GEMMs of a context-parallel attention block (sm_100a).
//
// Under Ulysses every rank holds a block of tokens (n_loc rows) before attention and a block of heads
// (Hp = H / P heads, all P * n_loc tokens) inside it. The library path is GEMM -> all_to_all (QKV) and
// all_to_all -> GEMM (output projection). Here each is ONE kernel over NVLink peer memory:
//
//  * scatter (QKV): D = X_loc @ W_qkv^T with W rows ordered [q | k | v] x [head, dim]. The epilogue of
//    every 32-column chunk (one head's 32 dims) stores straight into the owner rank's q/k/v buffer
//    [rows_all, Hp, d] at row (rank * n_loc + m): the transfer of a tile overlaps the MMAs of the next.
//  * gather (out-projection): Y_loc = O_gathered @ W_o^T where column block k of O belongs to the rank
//    owning head k / d. Every N tile of an M tile needs the same A rows, so a remote A tile must cross
//    NVLink once, not once per N tile: before their epilogue work, the epilogue warps of every CTA copy
//    (vector loads from the peer, stores to a local staging buffer) the units (M tile, remote owner) dealt
//    to them, M tiles first, and publish each with a release increment of that M tile's flag. The TMA
//    producer reads this rank's own columns straight from its attention output and the remote columns
//    from the staging buffer once the M tile's flag is complete (acquire + proxy fence, bounded wait), so
//    the copy of later M tiles overlaps the MMAs of earlier ones. The launch is cooperative (every CTA
//    resident), so a producer never waits for a copy that cannot run. The epilogue is local (bf16 store,
//    or the FP32 residual update x += gate * (acc + bias)).
//
// Roles (192 threads, one CTA per SM, persistent over tiles): warp 0 TMA producer, warp 1 TMEM owner
// and MMA issuer, warps 2..5 epilogue (warp w reads TMEM lanes 32 * (w % 4)). Accumulators are
// double-buffered in TMEM. Every wait is bounded (status word, no trap).
//
// peer_barrier: one CTA; thread p stores the epoch into rank p's flag slot [rank] (release, system
// scope) and then waits (bounded) until its own slot [p] holds the epoch. Kernels before it on the
// stream (the scatter stores) are complete and visible before the flag is written.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <vector>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace rc {
namespace ulysses {

constexpr int kMaxPeers = 8;
constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kStages = 4;
constexpr int kTmemCols = 512;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
static_assert(kSmemBytes <= 232448, "shared memory budget of one CTA");

enum Mode : int { kScatter = 0, kGather = 1 };
enum Epi : int { kEpiStore = 0, kEpiResidF32 = 1 };

struct Params {
  CUtensorMap tm_a[kMaxPeers];  // scatter: [0] = local X [M, K]; gather: owner p's O [rows_all, kcols_owner]
  CUtensorMap tm_b;             // W [N, K]
  int M, N, K;
  int world, rank;
  // gather: A rows start at a_row0 (= rank * n_loc) in every owner's buffer; K columns per owner
  int a_row0, kcols_owner;
  // scatter: dst[s][p] = row 0 of section s (q, k, v) in owner p's buffer [rows_all, Hp, d]
  __nv_bfloat16* dst[3][kMaxPeers];
  int dst_row0;                 // first destination row of local row 0 (rank * n_loc)
  int sec_cols;                 // H * d: columns of one section
  int head_dim, heads_per_rank;
  // gather staging: remote owners' columns of this rank's rows, copied once per call
  CUtensorMap tm_stage;         // stage [rows_pad, K]
  const __nv_bfloat16* src[kMaxPeers];  // owner p's attention output [rows_all, kcols_owner]
  __nv_bfloat16* stage;
  int* tile_flags;              // [flag_tiles] per-M-tile copy counters (monotonic across calls)
  int flag_tiles;
  int flag_target;              // value of a complete M tile's counter after this call
  // epilogue
  const __nv_bfloat16* bias;    // [N] or null
  const float* gate;            // [N] or null (kEpiResidF32)
  void* out;                    // gather + kEpiStore: bf16 [M, ldo]; kEpiResidF32: fp32 [M, ldo] updated in place
  int64_t ldo;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m_idx, int& n_idx) {
  constexpr int kGroupM = 8;
  const int per_group = kGroupM * num_n;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - group * per_group;
  m_idx = first_m + r % gsize;
  n_idx = r / gsize;
}

// Bounded wait until *flag >= target (acquire, GPU scope); false (status recorded) on timeout.
__device__ __forceinline__ bool wait_flag(const int* flag, int target, int* status) {
  const uint64_t start = globaltimer_ns();
#pragma unroll 1
  for (uint32_t iter = 0;; ++iter) {
    int seen;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(seen) : "l"(flag) : "memory");
    if (seen - target >= 0) return true;
    if ((iter & 255u) == 255u && (globaltimer_ns() - start > kWaitLimitNs || status_set(status))) {
      record_status(status, kTimeoutGather);
      return false;
    }
    __nanosleep(32);
  }
}

template <int MODE, int EPI>
__global__ void __launch_bounds__(kThreads, 1) ulysses_gemm_kernel(const __grid_constant__ Params p, int* status) {
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
  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = (p.N + kBN - 1) / kBN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
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
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_b);
      const int maps = MODE == kGather ? p.world : 1;
      for (int i = 0; i < maps; ++i) tma_prefetch_desc(&p.tm_a[i]);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int staged_m = -1;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int m_idx, n_idx;
        tile_coords(t, num_m, num_n, m_idx, n_idx);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * kStageBytes;
          uint8_t* b_dst = a_dst + kABytes;
          if (MODE == kGather) {
            // K block kb of the gathered O lives in owner k0 / kcols_owner (kcols_owner % 64 == 0)
            const int k0 = kb * kBK;
            const int owner = k0 / p.kcols_owner;
            if (owner != p.rank && m_idx != staged_m) {  // remote columns of this M tile: wait for their copies
              if (!wait_flag(p.tile_flags + m_idx, p.flag_target, status)) {
                ok = false;  // nothing armed: the MMA warp stops on the status word
                break;
              }
              asm volatile("fence.proxy.async.global;" ::: "memory");
              staged_m = m_idx;
            }
            mbar_arrive_expect_tx(&full[stage], kStageBytes);
            if (owner == p.rank)
              tma_load_2d(a_dst, &p.tm_a[owner], &full[stage], k0 - owner * p.kcols_owner, p.a_row0 + m_idx * kBM);
            else
              tma_load_2d(a_dst, &p.tm_stage, &full[stage], k0, m_idx * kBM);
          } else {
            mbar_arrive_expect_tx(&full[stage], kStageBytes);
            tma_load_2d(a_dst, &p.tm_a[0], &full[stage], kb * kBK, m_idx * kBM);
          }
          tma_load_2d(b_dst, &p.tm_b, &full[stage], kb * kBK, n_idx * kBN);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = make_idesc_f16(kBM, kBN, /*bf16*/ 1);
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
      const uint32_t d_tmem = tmem_base + buf * kBN;
      for (int kb = 0; kb < kblocks; ++kb) {
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
            mma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
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
    if (lane == 0) {  // every issued MMA has completed before TMEM is released
      mma_commit(drained);
      (void)mbar_wait(drained, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    // ---------------- Epilogue ----------------
    const int quarter = warp & 3;
    if (MODE == kGather && p.world > 1) {
      // Copy phase: units (M tile, remote owner), M tiles first, dealt round-robin over the CTAs.
      const int et = threadIdx.x - 64;  // 0 .. 127
      const int vecs_per_row = p.kcols_owner / 8;
      const int units = p.flag_tiles * (p.world - 1);
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int m = u / (p.world - 1);
        const int j = u - m * (p.world - 1);
        const int owner = j < p.rank ? j : j + 1;
        const int rows = max(0, min(kBM, p.M - m * kBM));
        const uint4* src = reinterpret_cast<const uint4*>(p.src[owner] + static_cast<int64_t>(p.a_row0 + m * kBM) *
                                                                             p.kcols_owner);
        __nv_bfloat16* dst_base = p.stage + static_cast<int64_t>(m * kBM) * p.K + owner * p.kcols_owner;
        const int total = rows * vecs_per_row;
#pragma unroll 1
        for (int v0 = et; v0 < total; v0 += 128 * 8) {
          uint4 buf[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int v = v0 + i * 128;
            if (v < total) buf[i] = src[v];  // NVLink loads, eight in flight per thread
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int v = v0 + i * 128;
            if (v < total) {
              const int r = v / vecs_per_row;
              const int c = v - r * vecs_per_row;
              *reinterpret_cast<uint4*>(dst_base + static_cast<int64_t>(r) * p.K + c * 8) = buf[i];
            }
          }
        }
        // the unit's stores are visible to TMA loads of other CTAs before the flag says so
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (et == 0) asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.tile_flags + m) : "memory");
      }
    }
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
      const bool row_ok = row < p.M;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        const int n0 = n_idx * kBN + c * 32;
        if (n0 >= p.N) break;  // uniform across the warp (N % 32 == 0)
        uint32_t raw[32];
        tmem_ld_32x32b_x32(tmem_base + buf * kBN + c * 32 + (static_cast<uint32_t>(quarter * 32) << 16), raw);
        tmem_wait_ld();
        if (!row_ok) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
        if (p.bias != nullptr) {
          const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + n0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 w = __ldg(b4 + q);
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 pair = *reinterpret_cast<const __nv_bfloat162*>(&words[e]);
              v[8 * q + 2 * e] += __bfloat162float(pair.x);
              v[8 * q + 2 * e + 1] += __bfloat162float(pair.y);
            }
          }
        }
        if (MODE == kScatter) {
          // 32 columns = 32 dims of one head of one section: 64 contiguous bytes at the owner
          const int s = n0 / p.sec_cols;
          const int within = n0 - s * p.sec_cols;
          const int head = within / p.head_dim;
          const int dim0 = within - head * p.head_dim;
          const int owner = head / p.heads_per_rank;
          const int lh = head - owner * p.heads_per_rank;
          __nv_bfloat16* dst = p.dst[s][owner] +
                               (static_cast<int64_t>(p.dst_row0 + row) * p.heads_per_rank + lh) * p.head_dim + dim0;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk;
            pk.x = pack_bf16x2(v[j], v[j + 1]);
            pk.y = pack_bf16x2(v[j + 2], v[j + 3]);
            pk.z = pack_bf16x2(v[j + 4], v[j + 5]);
            pk.w = pack_bf16x2(v[j + 6], v[j + 7]);
            *reinterpret_cast<uint4*>(dst + j) = pk;  // NVLink store when owner != rank
          }
        } else if (EPI == kEpiResidF32) {
          float* orow = reinterpret_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 x = *reinterpret_cast<float4*>(orow + j);
            const float4 g = p.gate != nullptr ? __ldg(reinterpret_cast<const float4*>(p.gate + n0 + j))
                                               : make_float4(1.f, 1.f, 1.f, 1.f);
            x.x = fmaf(g.x, v[j], x.x);
            x.y = fmaf(g.y, v[j + 1], x.y);
            x.z = fmaf(g.z, v[j + 2], x.z);
            x.w = fmaf(g.w, v[j + 3], x.w);
            *reinterpret_cast<float4*>(orow + j) = x;
          }
        } else {
          __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk;
            pk.x = pack_bf16x2(v[j], v[j + 1]);
            pk.y = pack_bf16x2(v[j + 2], v[j + 3]);
            pk.z = pack_bf16x2(v[j + 4], v[j + 5]);
            pk.w = pack_bf16x2(v[j + 6], v[j + 7]);
            *reinterpret_cast<uint4*>(orow + j) = pk;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// Bounded flag barrier across ranks over peer memory (see the file comment).
__global__ void peer_barrier_kernel(int* const* flags, int rank, int world, int epoch, int* status) {
  const int peer = threadIdx.x;
  if (peer >= world) return;
  int* remote = flags[peer] + rank;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
  const int* mine = flags[rank] + peer;
  const uint64_t start = globaltimer_ns();
#pragma unroll 1
  for (uint32_t iter = 0;; ++iter) {
    int seen;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(seen) : "l"(mine) : "memory");
    if (seen - epoch >= 0) break;  // epochs only grow (wrap-safe comparison)
    if ((iter & 255u) == 255u) {
      if (globaltimer_ns() - start > kWaitLimitNs || status_set(status)) {
        record_status(status, kTimeoutPeer);
        break;
      }
    }
    __nanosleep(64);
  }
}

}  // namespace ulysses

namespace {

void check_bf16_matrix(const at::Tensor& t, const char* name) {
  check_cuda_tensor(t, name);
  RC_CHECK(t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 && (t.stride(0) * 2) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
           std::string(name) + " must be a 16-byte aligned bfloat16 matrix with unit inner stride");
}

void launch_ulysses(const ulysses::Params& p, int mode, int epi, int device, int* status) {
  using namespace ulysses;
  static bool configured[64] = {false};
  if (!configured[device]) {
    RC_CUDA(cudaFuncSetAttribute(ulysses_gemm_kernel<kScatter, kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSmemBytes));
    RC_CUDA(cudaFuncSetAttribute(ulysses_gemm_kernel<kGather, kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSmemBytes));
    RC_CUDA(cudaFuncSetAttribute(ulysses_gemm_kernel<kGather, kEpiResidF32>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    configured[device] = true;
  }
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + kBN - 1) / kBN);
  const int grid = std::min(tiles, sm_count(device));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device).stream();
  if (mode == kScatter) {
    ulysses_gemm_kernel<kScatter, kEpiStore><<<grid, kThreads, kSmemBytes, stream>>>(p, status);
  } else {
    // cooperative: every CTA is resident, so a producer's wait for another CTA's copy always ends
    const void* fn = epi == kEpiResidF32 ? reinterpret_cast<const void*>(ulysses_gemm_kernel<kGather, kEpiResidF32>)
                                         : reinterpret_cast<const void*>(ulysses_gemm_kernel<kGather, kEpiStore>);
    Params copy = p;
    void* args[2] = {&copy, &status};
    RC_CUDA(cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kThreads), args, kSmemBytes, stream));
  }
  RC_CUDA(cudaGetLastError());
}

}  // namespace

// QKV projection with the Ulysses scatter fused in: x [n_loc, K] (this rank's tokens), w [3 * H * d, K],
// dst_{q,k,v}[p] = owner p's buffer [rows, Hp, d] (peer views; the local one for p == rank); this rank's
// rows go to rows rank * n_loc + (0 .. n_loc) of every owner's buffers.
void ulysses_qkv(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                 const std::vector<at::Tensor>& dst_q, const std::vector<at::Tensor>& dst_k,
                 const std::vector<at::Tensor>& dst_v, int64_t rank, int64_t head_dim,
                 const c10::optional<at::Tensor>& status) {
  using namespace ulysses;
  check_bf16_matrix(x, "x");
  check_bf16_matrix(w, "w");
  const int world = static_cast<int>(dst_q.size());
  RC_CHECK(world >= 1 && world <= kMaxPeers && dst_k.size() == dst_q.size() && dst_v.size() == dst_q.size(),
           "one q, k and v destination per rank (at most 8 ranks)");
  RC_CHECK(rank >= 0 && rank < world, "rank out of range");
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(w.size(0));
  RC_CHECK(w.size(1) == K && K % 8 == 0, "x and w disagree on K (a multiple of 8)");
  RC_CHECK(N % 3 == 0 && head_dim % 32 == 0 && (N / 3) % head_dim == 0, "w rows must be 3 x heads x head_dim");
  const int heads = static_cast<int>(N / 3 / head_dim);
  RC_CHECK(heads % world == 0, "heads must divide evenly across the ranks");
  const int hp = heads / world;
  Params p;
  memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.world = world;
  p.rank = static_cast<int>(rank);
  p.sec_cols = N / 3;
  p.head_dim = static_cast<int>(head_dim);
  p.heads_per_rank = hp;
  p.dst_row0 = static_cast<int>(rank) * M;
  const std::vector<at::Tensor>* sections[3] = {&dst_q, &dst_k, &dst_v};
  for (int s = 0; s < 3; ++s)
    for (int r = 0; r < world; ++r) {
      const at::Tensor& d = (*sections[s])[r];
      RC_CHECK(d.scalar_type() == at::kBFloat16 && d.is_contiguous() && d.dim() == 3 && d.size(1) == hp &&
                   d.size(2) == head_dim && d.size(0) >= (rank + 1) * M &&
                   reinterpret_cast<uintptr_t>(d.data_ptr()) % 16 == 0,
               "destinations must be contiguous 16-byte aligned bfloat16 [rows >= world * n_loc, Hp, d]");
      p.dst[s][r] = reinterpret_cast<__nv_bfloat16*>(d.data_ptr());
    }
  if (bias.has_value() && bias->defined()) {
    RC_CHECK(bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() && bias->numel() == N &&
                 reinterpret_cast<uintptr_t>(bias->data_ptr()) % 16 == 0,
             "bias must be a contiguous 16-byte aligned bfloat16 [N] vector");
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  p.tm_a[0] = make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, x.stride(0) * 2, kBK, kBM,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  p.tm_b = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, w.stride(0) * 2, kBK, kBN,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  c10::cuda::CUDAGuard guard(x.device());
  launch_ulysses(p, kScatter, kEpiStore, x.get_device(), status_ptr(status));
}

// Output projection with the Ulysses gather fused in: o_owners[p] = owner p's attention output
// [rows_all, Hp * d] (peer views), w [N, H * d]; this rank's n_loc rows (rows rank * n_loc ..) of the
// gathered output times w^T, then out = bf16 result [n_loc, N] (epilogue 0) or out (fp32 [n_loc, N])
// += gate * (acc + bias) (epilogue 1).
void ulysses_out(const std::vector<at::Tensor>& o_owners, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                 const c10::optional<at::Tensor>& gate, at::Tensor& out, int64_t rank, int64_t n_loc,
                 int64_t epilogue, const at::Tensor& stage, const at::Tensor& tile_flags, int64_t call,
                 const c10::optional<at::Tensor>& status) {
  using namespace ulysses;
  check_bf16_matrix(w, "w");
  const int world = static_cast<int>(o_owners.size());
  RC_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "one attention output per rank (<= 8)");
  const int N = static_cast<int>(w.size(0)), K = static_cast<int>(w.size(1));
  RC_CHECK(K % world == 0 && (K / world) % kBK == 0, "each owner's columns must be a multiple of 64");
  const int kcols = K / world;
  Params p;
  memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(n_loc);
  p.N = N;
  p.K = K;
  p.world = world;
  p.rank = static_cast<int>(rank);
  p.a_row0 = static_cast<int>(rank * n_loc);
  p.kcols_owner = kcols;
  RC_CHECK(N % 32 == 0, "N must be a multiple of 32");
  for (int r = 0; r < world; ++r) {
    const at::Tensor& o = o_owners[r];
    check_bf16_matrix(o, "attention output");
    RC_CHECK(o.size(1) == kcols && o.size(0) >= (rank + 1) * n_loc, "attention outputs must be [rows_all, K / world]");
    p.tm_a[r] = make_tmap_2d(o.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kcols, o.size(0), o.stride(0) * 2, kBK,
                             kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  p.tm_b = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, w.stride(0) * 2, kBK, kBN,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  for (int r = 0; r < world; ++r) {
    p.src[r] = reinterpret_cast<const __nv_bfloat16*>(o_owners[r].data_ptr());
    RC_CHECK(o_owners[r].is_contiguous(), "attention outputs must be contiguous");
  }
  const int num_m = static_cast<int>((n_loc + kBM - 1) / kBM);
  check_bf16_matrix(stage, "stage");
  RC_CHECK(stage.size(1) == K && stage.size(0) >= static_cast<int64_t>(num_m) * kBM && stage.is_contiguous(),
           "stage must be a contiguous bfloat16 [>= ceil(n_loc / 128) * 128, K] buffer");
  check_cuda_tensor(tile_flags, "tile_flags");
  RC_CHECK(tile_flags.scalar_type() == at::kInt && tile_flags.dim() == 1 && tile_flags.numel() >= num_m,
           "tile_flags must be a CUDA int32 vector with one counter per M tile");
  RC_CHECK(call >= 1 && call * (world - 1) < (1ll << 30), "call counts from 1");
  p.stage = reinterpret_cast<__nv_bfloat16*>(stage.data_ptr());
  p.tile_flags = tile_flags.data_ptr<int>();
  p.flag_tiles = static_cast<int>(tile_flags.numel());
  p.flag_target = static_cast<int>(call * (world - 1));
  p.tm_stage = make_tmap_2d(stage.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, stage.size(0), stage.stride(0) * 2,
                            kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (bias.has_value() && bias->defined()) {
    RC_CHECK(bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() && bias->numel() == N &&
                 reinterpret_cast<uintptr_t>(bias->data_ptr()) % 16 == 0,
             "bias must be a contiguous 16-byte aligned bfloat16 [N] vector");
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  check_cuda_tensor(out, "out");
  RC_CHECK(out.dim() == 2 && out.size(0) == n_loc && out.size(1) == N && out.stride(1) == 1 &&
               (out.stride(0) * out.element_size()) % 16 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "out must be a 16-byte aligned [n_loc, N] matrix with unit inner stride");
  if (epilogue == kEpiResidF32) {
    RC_CHECK(out.scalar_type() == at::kFloat, "the residual epilogue updates a float32 out");
    if (gate.has_value() && gate->defined()) {
      RC_CHECK(gate->scalar_type() == at::kFloat && gate->is_contiguous() && gate->numel() == N &&
                   reinterpret_cast<uintptr_t>(gate->data_ptr()) % 16 == 0,
               "gate must be a contiguous 16-byte aligned float32 [N] vector");
      p.gate = gate->data_ptr<float>();
    }
  } else {
    RC_CHECK(epilogue == kEpiStore && out.scalar_type() == at::kBFloat16, "epilogue 0 stores bfloat16");
  }
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  c10::cuda::CUDAGuard guard(w.device());
  launch_ulysses(p, kGather, static_cast<int>(epilogue), w.get_device(), status_ptr(status));
}

// Device-side barrier over peer flag words: flags is a CUDA int64 tensor of the ranks' flag addresses
// (each rank's int32 [world] slots, mapped on this device); epoch grows by one per barrier.
void peer_barrier(const at::Tensor& flags, int64_t rank, int64_t epoch, const c10::optional<at::Tensor>& status) {
  check_cuda_tensor(flags, "flags");
  RC_CHECK(flags.scalar_type() == at::kLong && flags.dim() == 1 && flags.numel() >= 1 && flags.numel() <= 32,
           "flags must be a CUDA int64 vector of <= 32 flag addresses");
  const int world = static_cast<int>(flags.numel());
  RC_CHECK(rank >= 0 && rank < world, "rank out of range");
  c10::cuda::CUDAGuard guard(flags.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(flags.get_device()).stream();
  ulysses::peer_barrier_kernel<<<1, 32, 0, stream>>>(reinterpret_cast<int* const*>(flags.data_ptr<int64_t>()),
                                                     static_cast<int>(rank), world, static_cast<int>(epoch),
                                                     status_ptr(status));
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
