// Basis preparation for the fused restore GEMM (sm_100a).
//
// The restore computes, per token n and channel c,
//   y[n, c] = sum_k (p[n, k] * s[k] + o[k]) * Q[k, c]
//           = sum_k (p[n, k] - 128) * (s[k] * Q[k, c])  +  sum_k (o[k] + 128 s[k]) * Q[k, c]
// with p the 8-bit pixel, (s, o) the column's affine and Q the FP16 basis. The first term runs on
// the tensor cores with the exact FP16 operand (p - 128) and the B operand s[k] * Q[k, c] * 2^e split
// into FP16 hi + lo (two products, FP32 accumulation; 2^e is the job's exact power-of-two prescale);
// the second is a per-channel bias. This kernel writes, per job, Bt[c, 0:K_pad] = hi,
// Bt[c, K_pad:2 K_pad] = lo (K-major for TMA, zero beyond the rank) and bias[c] (FP64 accumulation,
// fixed order: deterministic).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cuda_fp16.h>

#include "../common/host.h"
#include "restore_one.h"

namespace rc {
namespace prep {

constexpr int kMaxJobs = 48;
constexpr int kThreads = 256;
constexpr int kVec = 8;                          // channels per thread (one 16-byte basis load)
constexpr int kGroups = 32;                      // channel groups per block: one warp spans 256 channels
constexpr int kChannels = kGroups * kVec;        // channels per block
constexpr int kKLanes = kThreads / kGroups;      // 8: warp w handles K rows w*8 .. w*8+7 of every 64

struct Job {
  const __half* q;       // [R, C] basis rows
  const float* scale;    // [rank]
  const float* offset;   // [rank]
  __half* bt;            // [C, 2 * k_pad]
  float* bias;           // [C]
  int64_t q_stride;      // elements between basis rows
  int rank, k_pad, channels;
  float prescale;
  int vec;               // basis rows 16-byte aligned: one 16-byte load per thread and row
};

struct Params {
  Job jobs[kMaxJobs];
};

// One warp reads 512 contiguous bytes of a basis row (a basis in a peer's memory then crosses NVLink in
// whole lines); each thread owns 8 channels and, per 64-row K block, 8 consecutive K rows, so it writes
// one 16-byte hi and one 16-byte lo chunk of each of its 8 Bt rows. The bias of a channel accumulates in
// FP64 in a fixed order: ascending K within a lane, then lanes 0..7.
__global__ void __launch_bounds__(kThreads) prep_kernel(const __grid_constant__ Params p) {
  const Job& jb = p.jobs[blockIdx.y];
  const int c0 = blockIdx.x * kChannels + (threadIdx.x % kGroups) * kVec;
  if (blockIdx.x * kChannels >= jb.channels) return;
  const int lane_k = threadIdx.x / kGroups;
  __shared__ double partial[kKLanes][kChannels];
  double acc[kVec];
#pragma unroll
  for (int j = 0; j < kVec; ++j) acc[j] = 0.0;
  const bool live = c0 < jb.channels;
  for (int k0 = lane_k * 8; k0 < jb.k_pad; k0 += kKLanes * 8) {
    float v[8][kVec];  // [k][channel]
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = k0 + i;
      float q[kVec];
#pragma unroll
      for (int j = 0; j < kVec; ++j) q[j] = 0.0f;
      if (live && k < jb.rank) {
        const __half* row = jb.q + static_cast<int64_t>(k) * jb.q_stride + c0;
        if (jb.vec) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(row));
          const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int j = 0; j < kVec / 2; ++j) {
            const float2 f = __half22float2(h2[j]);
            q[2 * j] = f.x;
            q[2 * j + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < kVec; ++j)
            if (c0 + j < jb.channels) q[j] = __half2float(row[j]);
        }
        const float s = jb.scale[k];
        const double shift = static_cast<double>(jb.offset[k]) + 128.0 * static_cast<double>(s);
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          v[i][j] = (s * jb.prescale) * q[j];
          acc[j] += shift * static_cast<double>(q[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < kVec; ++j) v[i][j] = 0.0f;
      }
    }
    if (live) {
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        if (c0 + j >= jb.channels) break;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const __half h0 = __float2half_rn(v[i][j]);
          const __half h1 = __float2half_rn(v[i + 1][j]);
          const __half l0 = __float2half_rn(v[i][j] - __half2float(h0));
          const __half l1 = __float2half_rn(v[i + 1][j] - __half2float(h1));
          hi[i / 2] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
          lo[i / 2] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
        }
        __half* out = jb.bt + static_cast<int64_t>(c0 + j) * 2 * jb.k_pad;
        *reinterpret_cast<uint4*>(out + k0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(out + jb.k_pad + k0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
    }
  }
  const int local_c = (threadIdx.x % kGroups) * kVec;
#pragma unroll
  for (int j = 0; j < kVec; ++j) partial[lane_k][local_c + j] = acc[j];
  __syncthreads();
  const int c = blockIdx.x * kChannels + threadIdx.x;  // kThreads == kChannels: one thread per channel
  if (c < jb.channels) {
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < kKLanes; ++i) sum += partial[i][threadIdx.x];
    jb.bias[c] = static_cast<float>(sum);
  }
}

static_assert(kThreads == kChannels, "the bias reduction assigns one thread per channel");

}  // namespace prep

// jobs: CPU int64 [n, 10]: q, scale, offset, bt, bias, q_stride, rank, k_pad, channels, prescale bits
// (float32 bit pattern in the low 32 bits).
void prep_launch(const at::Tensor& jobs, int64_t device) {
  RC_CHECK(jobs.device().is_cpu() && jobs.scalar_type() == at::kLong && jobs.dim() == 2 && jobs.size(1) == 10,
           "jobs must be a CPU int64 [n, 10] table");
  const int n = static_cast<int>(jobs.size(0));
  RC_CHECK(n >= 1 && n <= prep::kMaxJobs, "between 1 and 48 prep jobs per launch");
  prep::Params p;
  memset(&p, 0, sizeof(p));
  const int64_t* f = jobs.data_ptr<int64_t>();
  int max_channels = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t* r = f + i * 10;
    prep::Job& jb = p.jobs[i];
    jb.q = reinterpret_cast<const __half*>(r[0]);
    jb.scale = reinterpret_cast<const float*>(r[1]);
    jb.offset = reinterpret_cast<const float*>(r[2]);
    jb.bt = reinterpret_cast<__half*>(r[3]);
    jb.bias = reinterpret_cast<float*>(r[4]);
    jb.q_stride = r[5];
    jb.rank = static_cast<int>(r[6]);
    jb.k_pad = static_cast<int>(r[7]);
    jb.channels = static_cast<int>(r[8]);
    const uint32_t bits = static_cast<uint32_t>(r[9] & 0xffffffffll);
    memcpy(&jb.prescale, &bits, 4);
    RC_CHECK(jb.k_pad % 64 == 0 && jb.rank <= jb.k_pad && jb.rank >= 1, "k_pad must be a multiple of 64 >= rank");
    RC_CHECK(reinterpret_cast<uintptr_t>(jb.bt) % 16 == 0, "prepared basis must be 16-byte aligned");
    jb.vec = reinterpret_cast<uintptr_t>(jb.q) % 16 == 0 && jb.q_stride % 8 == 0 && jb.channels % 8 == 0;
    max_channels = std::max(max_channels, jb.channels);
  }
  c10::cuda::CUDAGuard guard(static_cast<int>(device));
  dim3 grid((max_channels + prep::kChannels - 1) / prep::kChannels, n);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(static_cast<int>(device)).stream();
  prep::prep_kernel<<<grid, prep::kThreads, 0, stream>>>(p);
  RC_CUDA(cudaGetLastError());
}

// Allocation-free launch of one job (restore_one.h).
const char* prep_one(const __half* q, int64_t q_stride, const float* scale, const float* offset, __half* bt,
                     float* bias, int rank, int k_pad, int channels, float prescale, cudaStream_t stream) {
  if (k_pad % 64 != 0 || rank < 1 || rank > k_pad || channels < 1) return "prep: bad job geometry";
  if (reinterpret_cast<uintptr_t>(bt) % 16 != 0) return "prep: prepared basis must be 16-byte aligned";
  prep::Params p;
  memset(&p, 0, sizeof(p));
  prep::Job& jb = p.jobs[0];
  jb.q = q;
  jb.scale = scale;
  jb.offset = offset;
  jb.bt = bt;
  jb.bias = bias;
  jb.q_stride = q_stride;
  jb.rank = rank;
  jb.k_pad = k_pad;
  jb.channels = channels;
  jb.prescale = prescale;
  jb.vec = reinterpret_cast<uintptr_t>(q) % 16 == 0 && q_stride % 8 == 0 && channels % 8 == 0;
  dim3 grid((channels + prep::kChannels - 1) / prep::kChannels, 1);
  prep::prep_kernel<<<grid, prep::kThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? nullptr : "prep: launch failed";
}

}  // namespace rc
