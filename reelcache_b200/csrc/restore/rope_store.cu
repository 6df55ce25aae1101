// Dense install kernel for sm_100a (the counterpart of the reference's `_rope_store_kernel`,
// reelcache/restore_kernels.py:1556-1586): an uncompressed canonical [N, C] matrix (RAW archive,
// GPU/host raw tier, decoded dense history) is rotated with the engine's interleaved-pair RoPE
// (optional), cast and stored through arbitrary (token, head, dim) strides into the native cache.
// Memory-bound: each thread moves 8 channels (16-byte loads of bf16/f16 sources).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace rc {
namespace dense {

constexpr int kMaxJobs = 48;
constexpr int kThreads = 256;

struct Job {
  const void* src;
  void* dst;
  const float* cos;
  const float* sin;
  int64_t src_ts;           // elements between source token rows (channel stride 1)
  int64_t dst_ts, dst_hs, dst_ds;
  int src_dtype, out_dtype; // 0 bf16, 1 f16, 2 f32
  int tokens, channels, head_dim;
  int height, width;
  int rope, rope_dense, rope_rs, row_t, row_h, row_w, sec_t, sec_h;
};

struct Params {
  Job jobs[kMaxJobs];
  int num_jobs;
};

__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dtype) {
  if (dtype == 0) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__global__ void __launch_bounds__(kThreads) rope_store_kernel(const __grid_constant__ Params p) {
  const Job& jb = p.jobs[blockIdx.y];
  const int groups = jb.channels >> 3;  // 8 channels per thread
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t total = static_cast<int64_t>(jb.tokens) * groups;
  if (item >= total) return;
  const int token = static_cast<int>(item / groups);
  const int c0 = static_cast<int>(item - static_cast<int64_t>(token) * groups) * 8;
  float v[8];
  const int64_t sbase = static_cast<int64_t>(token) * jb.src_ts + c0;
  if (jb.src_dtype != 2 && (reinterpret_cast<uintptr_t>(jb.src) & 15) == 0 && (sbase & 7) == 0) {
    const uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(jb.src) + sbase);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (jb.src_dtype == 0) {
        v[2 * i] = __uint_as_float((w[i] & 0xffffu) << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      } else {
        v[2 * i] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] & 0xffffu)));
        v[2 * i + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] >> 16)));
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = load_elem(jb.src, sbase + i, jb.src_dtype);
  }
  const int head = c0 / jb.head_dim;
  const int d0 = c0 - head * jb.head_dim;
  if (jb.rope) {
    const int per_frame = jb.height * jb.width;
    const int frame = token / per_frame;
    const int rem = token - frame * per_frame;
    const int y = rem / jb.width;
    const int x = rem - y * jb.width;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int pair = (d0 >> 1) + i;
      int row;
      if (jb.rope_dense) row = jb.row_t + token;
      else if (pair < jb.sec_t) row = jb.row_t + frame;
      else if (pair < jb.sec_t + jb.sec_h) row = jb.row_h + y;
      else row = jb.row_w + x;
      const int64_t idx = static_cast<int64_t>(pair) * jb.rope_rs + row;  // tables stored [pairs, rows]
      const float cs = jb.cos[idx];
      const float sn = jb.sin[idx];
      const float e = v[2 * i], o = v[2 * i + 1];
      v[2 * i] = e * cs - o * sn;
      v[2 * i + 1] = e * sn + o * cs;
    }
  }
  const int64_t dbase = static_cast<int64_t>(token) * jb.dst_ts + static_cast<int64_t>(head) * jb.dst_hs +
                        static_cast<int64_t>(d0) * jb.dst_ds;
  if (jb.out_dtype == 2) {
    float* out = reinterpret_cast<float*>(jb.dst) + dbase;
    for (int i = 0; i < 8; ++i) out[static_cast<int64_t>(i) * jb.dst_ds] = v[i];
  } else {
    uint16_t* out = reinterpret_cast<uint16_t*>(jb.dst) + dbase;
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      pk[i] = jb.out_dtype == 0 ? pack_bf16x2(v[2 * i], v[2 * i + 1]) : pack_f16x2(v[2 * i], v[2 * i + 1]);
    if (jb.dst_ds == 1 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
      *reinterpret_cast<uint4*>(out) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    } else {
      for (int i = 0; i < 4; ++i) {
        out[static_cast<int64_t>(2 * i) * jb.dst_ds] = static_cast<uint16_t>(pk[i] & 0xffffu);
        out[static_cast<int64_t>(2 * i + 1) * jb.dst_ds] = static_cast<uint16_t>(pk[i] >> 16);
      }
    }
  }
}

}  // namespace dense

// jobs: CPU int64 [n, 24]: src, dst, cos, sin, src_ts, dst_ts, dst_hs, dst_ds, src_dtype, out_dtype,
// tokens, channels, head_dim, height, width, rope, rope_dense, rope_rs, row_t, row_h, row_w, sec_t,
// sec_h, device.
void rope_store_launch(const at::Tensor& jobs) {
  RC_CHECK(jobs.device().is_cpu() && jobs.scalar_type() == at::kLong && jobs.dim() == 2 && jobs.size(1) == 24,
           "jobs must be a CPU int64 [n, 24] table");
  const int n = static_cast<int>(jobs.size(0));
  RC_CHECK(n >= 1 && n <= dense::kMaxJobs, "between 1 and 48 dense jobs per launch");
  dense::Params p;
  memset(&p, 0, sizeof(p));
  const int64_t* f = jobs.data_ptr<int64_t>();
  int64_t max_items = 0;
  const int device = static_cast<int>(f[23]);
  for (int i = 0; i < n; ++i) {
    const int64_t* r = f + i * 24;
    dense::Job& jb = p.jobs[i];
    jb.src = reinterpret_cast<const void*>(r[0]);
    jb.dst = reinterpret_cast<void*>(r[1]);
    jb.cos = reinterpret_cast<const float*>(r[2]);
    jb.sin = reinterpret_cast<const float*>(r[3]);
    jb.src_ts = r[4];
    jb.dst_ts = r[5];
    jb.dst_hs = r[6];
    jb.dst_ds = r[7];
    jb.src_dtype = static_cast<int>(r[8]);
    jb.out_dtype = static_cast<int>(r[9]);
    jb.tokens = static_cast<int>(r[10]);
    jb.channels = static_cast<int>(r[11]);
    jb.head_dim = static_cast<int>(r[12]);
    jb.height = static_cast<int>(r[13]);
    jb.width = static_cast<int>(r[14]);
    jb.rope = static_cast<int>(r[15]);
    jb.rope_dense = static_cast<int>(r[16]);
    jb.rope_rs = static_cast<int>(r[17]);
    jb.row_t = static_cast<int>(r[18]);
    jb.row_h = static_cast<int>(r[19]);
    jb.row_w = static_cast<int>(r[20]);
    jb.sec_t = static_cast<int>(r[21]);
    jb.sec_h = static_cast<int>(r[22]);
    RC_CHECK(jb.channels % 8 == 0 && jb.head_dim % 8 == 0, "channels and head_dim must be multiples of 8");
    max_items = std::max<int64_t>(max_items, static_cast<int64_t>(jb.tokens) * (jb.channels / 8));
  }
  p.num_jobs = n;
  c10::cuda::CUDAGuard guard(device);
  dim3 grid(static_cast<unsigned>((max_items + dense::kThreads - 1) / dense::kThreads), n);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device).stream();
  dense::rope_store_kernel<<<grid, dense::kThreads, 0, stream>>>(p);
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
