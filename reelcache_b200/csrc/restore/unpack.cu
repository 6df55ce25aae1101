// Coefficient unpack for sm_100a (the counterpart of the reference's `_unpack_kernel`,
// reelcache/restore_kernels.py:1517-1555): gathers each job's 8-bit coefficient pixels -- from the
// reelcache.channel_tiles.v1 mosaic of decoded pictures, or from a dense uint8 [N, >= rank] matrix --
// into the fused restore GEMM's A operand: a row-major FP16 matrix [N, K_pad] of centered pixels
// (p - 128, exact in FP16), zero beyond the rank.
//
// One thread produces 8 consecutive rank columns of one token (one 16-byte store). Threads of a
// warp hold consecutive tokens, so each pixel load of the warp reads neighbouring bytes of one
// picture row (or one 8-byte slice per row of a dense matrix).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cuda_fp16.h>

#include "../common/host.h"
#include "restore_one.h"

namespace rc {
namespace unpack {

constexpr int kMaxJobs = 48;
constexpr int kThreads = 256;

struct Job {
  const int64_t* pic_addr;   // pictures: [segments * frames] absolute address of the rectangle origin
  const int32_t* col_off;    // pictures: [k_pad] byte offset of column k's cell in a picture (-1: none)
  const int32_t* col_seg;    // pictures: [k_pad] segment of column k
  const uint8_t* matrix;     // dense source [tokens, >= rank] (null for pictures)
  __half* out;               // [tokens, k_pad]
  int64_t row_stride;        // pictures: picture row stride; dense: matrix row stride (bytes)
  int tokens, k_pad, rank, frames, height, width;
  int vec8;                  // dense, rows >= k_pad bytes apart: 2 = 16-byte aligned rows (unpack_dense16),
                             // 1 = 8-byte aligned (one 8-byte load per thread), 0 = byte loads
  int run_len;               // dense gather (0: none): token t reads source row
  int64_t run_stride;        //   (t / run_len) * run_stride + run_offset + t % run_len
  int64_t run_offset;        //   (a rank's column or row block of a frame grid)
};

// The dense source row a job's token reads: itself, or its place in the job's runs.
__device__ __forceinline__ int64_t source_row(const Job& jb, int token) {
  if (jb.run_len == 0) return token;
  const int run = token / jb.run_len;
  return static_cast<int64_t>(run) * jb.run_stride + jb.run_offset + (token - run * jb.run_len);
}

struct Params {
  Job jobs[kMaxJobs];
};

__device__ __forceinline__ uint32_t centered_pair(uint32_t a, uint32_t b) {
  const __half2 h = __halves2half2(__int2half_rn(static_cast<int>(a) - 128), __int2half_rn(static_cast<int>(b) - 128));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Dense sources with 16-byte aligned rows at least k_pad bytes apart: one thread per 16 consecutive
// columns of one token, lanes walking along a row first, so a warp loads whole 64-byte row segments
// (full sectors: a source in a peer's memory crosses NVLink once, without over-fetch) and stores 32
// contiguous bytes per thread.
__device__ __forceinline__ void unpack_dense16(const Job& jb, int64_t item) {
  const int groups = jb.k_pad >> 4;
  if (item >= static_cast<int64_t>(jb.tokens) * groups) return;
  const int token = static_cast<int>(item / groups);
  const int group = static_cast<int>(item - static_cast<int64_t>(token) * groups);
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(jb.matrix + source_row(jb, token) * jb.row_stride +
                                                         group * 16));
  const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int k = group * 16 + 2 * i;
    const uint32_t word = words[i >> 1];
    const uint32_t a = k < jb.rank ? (word >> (16 * (i & 1))) & 0xffu : 128u;
    const uint32_t b = k + 1 < jb.rank ? (word >> (16 * (i & 1) + 8)) & 0xffu : 128u;
    w[i] = centered_pair(a, b);
  }
  uint4* out = reinterpret_cast<uint4*>(jb.out + static_cast<int64_t>(token) * jb.k_pad + group * 16);
  out[0] = make_uint4(w[0], w[1], w[2], w[3]);
  out[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__global__ void __launch_bounds__(kThreads) unpack_kernel(const __grid_constant__ Params p) {
  const Job& jb = p.jobs[blockIdx.y];
  if (jb.vec8 == 2) {
    unpack_dense16(jb, static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x);
    return;
  }
  const int groups = jb.k_pad >> 3;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (item >= static_cast<int64_t>(jb.tokens) * groups) return;
  const int group = static_cast<int>(item / jb.tokens);  // token fastest within a warp
  const int token = static_cast<int>(item - static_cast<int64_t>(group) * jb.tokens);
  uint32_t px[8];
  bool live[8];
  if (jb.matrix != nullptr) {
    const uint8_t* rowp = jb.matrix + source_row(jb, token) * jb.row_stride + group * 8;
    if (jb.vec8) {
      // one 8-byte load: a source in a peer's memory (the sequence-parallel restore) then costs one
      // NVLink request per 8 coefficients instead of eight byte loads
      const uint2 raw = __ldg(reinterpret_cast<const uint2*>(rowp));
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        live[i] = group * 8 + i < jb.rank;
        const uint32_t word = i < 4 ? raw.x : raw.y;
        px[i] = live[i] ? (word >> (8 * (i & 3))) & 0xffu : 128u;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        live[i] = group * 8 + i < jb.rank;
        px[i] = live[i] ? __ldg(rowp + i) : 128u;
      }
    }
  } else {
    const int per_frame = jb.height * jb.width;
    const int frame = token / per_frame;
    const int rem = token - frame * per_frame;
    const int y = rem / jb.width;
    const int64_t pix = static_cast<int64_t>(y) * jb.row_stride + (rem - y * jb.width);
    int cur_seg = -1;
    const uint8_t* base = nullptr;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = group * 8 + i;
      const int off = __ldg(jb.col_off + k);
      live[i] = off >= 0;
      px[i] = 128u;
      if (live[i]) {
        const int seg = __ldg(jb.col_seg + k);
        if (seg != cur_seg) {
          cur_seg = seg;
          base = reinterpret_cast<const uint8_t*>(__ldg(jb.pic_addr + seg * jb.frames + frame) + pix);
        }
        px[i] = __ldg(base + off);
      }
    }
  }
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // columns beyond the rank hold 0 (their centered pixel would be 0 too: px = 128)
    w[i] = centered_pair(px[2 * i], px[2 * i + 1]);
  }
  *reinterpret_cast<uint4*>(jb.out + static_cast<int64_t>(token) * jb.k_pad + group * 8) = make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace unpack

// jobs: CPU int64 [n, 12 or 15]: pic_addr, col_off, col_seg, matrix, out, row_stride, tokens, k_pad, rank,
// frames, height, width[, run_len, run_stride, run_offset]. Pointers are device addresses on `device`.
void unpack_launch(const at::Tensor& jobs, int64_t device) {
  RC_CHECK(jobs.device().is_cpu() && jobs.scalar_type() == at::kLong && jobs.dim() == 2 &&
               (jobs.size(1) == 12 || jobs.size(1) == 15),
           "jobs must be a CPU int64 [n, 12 or 15] table");
  const int width = static_cast<int>(jobs.size(1));
  const int n = static_cast<int>(jobs.size(0));
  RC_CHECK(n >= 1 && n <= unpack::kMaxJobs, "between 1 and 48 unpack jobs per launch");
  unpack::Params p;
  memset(&p, 0, sizeof(p));
  const int64_t* f = jobs.data_ptr<int64_t>();
  int64_t max_items = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t* r = f + i * width;
    unpack::Job& jb = p.jobs[i];
    jb.pic_addr = reinterpret_cast<const int64_t*>(r[0]);
    jb.col_off = reinterpret_cast<const int32_t*>(r[1]);
    jb.col_seg = reinterpret_cast<const int32_t*>(r[2]);
    jb.matrix = reinterpret_cast<const uint8_t*>(r[3]);
    jb.out = reinterpret_cast<__half*>(r[4]);
    jb.row_stride = r[5];
    jb.tokens = static_cast<int>(r[6]);
    jb.k_pad = static_cast<int>(r[7]);
    jb.rank = static_cast<int>(r[8]);
    jb.frames = static_cast<int>(r[9]);
    jb.height = static_cast<int>(r[10]);
    jb.width = static_cast<int>(r[11]);
    if (width == 15 && r[12] > 0) {
      RC_CHECK(jb.matrix != nullptr && r[13] >= 0 && r[14] >= 0, "row runs apply to dense sources");
      jb.run_len = static_cast<int>(r[12]);
      jb.run_stride = r[13];
      jb.run_offset = r[14];
    }
    jb.vec8 = 0;
    if (jb.matrix != nullptr && jb.row_stride >= jb.k_pad) {
      const uintptr_t base = reinterpret_cast<uintptr_t>(jb.matrix);
      if (base % 16 == 0 && jb.row_stride % 16 == 0) jb.vec8 = 2;
      else if (base % 8 == 0 && jb.row_stride % 8 == 0) jb.vec8 = 1;
    }
    RC_CHECK(jb.k_pad % 64 == 0 && jb.k_pad > 0 && jb.rank <= jb.k_pad, "k_pad must be a multiple of 64 >= rank");
    RC_CHECK(reinterpret_cast<uintptr_t>(jb.out) % 16 == 0, "unpack output must be 16-byte aligned");
    RC_CHECK(jb.matrix != nullptr || jb.frames * jb.height * jb.width == jb.tokens, "grid does not match the tokens");
    max_items = std::max<int64_t>(max_items, static_cast<int64_t>(jb.tokens) * (jb.k_pad / 8));
  }
  c10::cuda::CUDAGuard guard(static_cast<int>(device));
  dim3 grid(static_cast<unsigned>((max_items + unpack::kThreads - 1) / unpack::kThreads), n);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(static_cast<int>(device)).stream();
  unpack::unpack_kernel<<<grid, unpack::kThreads, 0, stream>>>(p);
  RC_CUDA(cudaGetLastError());
}

// Allocation-free launch of one dense uint8 job (restore_one.h).
const char* unpack_u8_one(const uint8_t* matrix, int64_t row_stride, __half* out, int tokens, int k_pad, int rank,
                          cudaStream_t stream) {
  if (k_pad % 64 != 0 || k_pad <= 0 || rank < 1 || rank > k_pad || tokens < 1) return "unpack: bad job geometry";
  if (reinterpret_cast<uintptr_t>(out) % 16 != 0) return "unpack: output must be 16-byte aligned";
  unpack::Params p;
  memset(&p, 0, sizeof(p));
  unpack::Job& jb = p.jobs[0];
  jb.matrix = matrix;
  jb.out = out;
  jb.row_stride = row_stride;
  jb.tokens = tokens;
  jb.k_pad = k_pad;
  jb.rank = rank;
  jb.frames = 1;
  jb.height = 1;
  jb.width = tokens;
  const int64_t items = static_cast<int64_t>(tokens) * (k_pad / 8);
  dim3 grid(static_cast<unsigned>((items + unpack::kThreads - 1) / unpack::kThreads), 1);
  unpack::unpack_kernel<<<grid, unpack::kThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? nullptr : "unpack: launch failed";
}

}  // namespace rc
