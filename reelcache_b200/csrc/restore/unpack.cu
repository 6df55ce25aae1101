// Picture unpack for sm_100a (the counterpart of the reference's `_unpack_kernel`,
// reelcache/restore_kernels.py:1517-1555): gathers the 8-bit coefficient pixels of each job's
// reelcache.channel_tiles.v1 mosaic into a dense row-major uint8 matrix [N, K_pad] (zero beyond the
// rank), the operand layout the fused restore GEMM streams with 16-byte loads.
//
// One thread produces 16 consecutive rank columns of one token (one 16-byte store). Threads of a
// warp hold consecutive tokens, so every pixel load of the warp reads neighbouring bytes of one
// picture row. The per-column cell offsets and segments come from a host-built table.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "../common/host.h"

namespace rc {
namespace unpack {

constexpr int kMaxJobs = 48;
constexpr int kThreads = 256;

struct Job {
  const int64_t* pic_addr;   // [segments * frames] absolute address of the matrix rectangle origin
  const int32_t* col_off;    // [k_pad] byte offset of column k's cell inside a picture (-1 beyond rank)
  const int32_t* col_seg;    // [k_pad] segment of column k
  uint8_t* out;              // [tokens, k_pad]
  int64_t row_stride;        // picture row stride (bytes)
  int tokens, k_pad, frames, height, width;
};

struct Params {
  Job jobs[kMaxJobs];
};

__global__ void __launch_bounds__(kThreads) unpack_kernel(const __grid_constant__ Params p) {
  const Job& jb = p.jobs[blockIdx.y];
  const int groups = jb.k_pad >> 4;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (item >= static_cast<int64_t>(jb.tokens) * groups) return;
  // token fastest: a warp covers 32 consecutive tokens of one 16-column group
  const int group = static_cast<int>(item / jb.tokens);
  const int token = static_cast<int>(item - static_cast<int64_t>(group) * jb.tokens);
  const int per_frame = jb.height * jb.width;
  const int frame = token / per_frame;
  const int rem = token - frame * per_frame;
  const int y = rem / jb.width;
  const int64_t pix = static_cast<int64_t>(y) * jb.row_stride + (rem - y * jb.width);
  uint32_t words[4] = {0u, 0u, 0u, 0u};
  int cur_seg = -1;
  const uint8_t* base = nullptr;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int k = group * 16 + i;
    const int off = __ldg(jb.col_off + k);
    uint32_t v = 0u;
    if (off >= 0) {
      const int seg = __ldg(jb.col_seg + k);
      if (seg != cur_seg) {
        cur_seg = seg;
        base = reinterpret_cast<const uint8_t*>(__ldg(jb.pic_addr + seg * jb.frames + frame) + pix);
      }
      v = __ldg(base + off);
    }
    words[i >> 2] |= v << ((i & 3) * 8);
  }
  *reinterpret_cast<uint4*>(jb.out + static_cast<int64_t>(token) * jb.k_pad + group * 16) =
      make_uint4(words[0], words[1], words[2], words[3]);
}

}  // namespace unpack

// jobs: CPU int64 [n, 10]: pic_addr, col_off, col_seg, out, row_stride, tokens, k_pad, frames,
// height, width. All pointers device addresses on the current device.
void unpack_launch(const at::Tensor& jobs, int64_t device) {
  RC_CHECK(jobs.device().is_cpu() && jobs.scalar_type() == at::kLong && jobs.dim() == 2 && jobs.size(1) == 10,
           "jobs must be a CPU int64 [n, 10] table");
  const int n = static_cast<int>(jobs.size(0));
  RC_CHECK(n >= 1 && n <= unpack::kMaxJobs, "between 1 and 48 unpack jobs per launch");
  unpack::Params p;
  memset(&p, 0, sizeof(p));
  const int64_t* f = jobs.data_ptr<int64_t>();
  int64_t max_items = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t* r = f + i * 10;
    unpack::Job& jb = p.jobs[i];
    jb.pic_addr = reinterpret_cast<const int64_t*>(r[0]);
    jb.col_off = reinterpret_cast<const int32_t*>(r[1]);
    jb.col_seg = reinterpret_cast<const int32_t*>(r[2]);
    jb.out = reinterpret_cast<uint8_t*>(r[3]);
    jb.row_stride = r[4];
    jb.tokens = static_cast<int>(r[5]);
    jb.k_pad = static_cast<int>(r[6]);
    jb.frames = static_cast<int>(r[7]);
    jb.height = static_cast<int>(r[8]);
    jb.width = static_cast<int>(r[9]);
    RC_CHECK(jb.k_pad % 16 == 0 && jb.k_pad > 0, "k_pad must be a positive multiple of 16");
    RC_CHECK(reinterpret_cast<uintptr_t>(jb.out) % 16 == 0, "unpack output must be 16-byte aligned");
    RC_CHECK(jb.frames * jb.height * jb.width == jb.tokens, "grid does not match the token count");
    max_items = std::max<int64_t>(max_items, static_cast<int64_t>(jb.tokens) * (jb.k_pad / 16));
  }
  c10::cuda::CUDAGuard guard(static_cast<int>(device));
  dim3 grid(static_cast<unsigned>((max_items + unpack::kThreads - 1) / unpack::kThreads), n);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(static_cast<int>(device)).stream();
  unpack::unpack_kernel<<<grid, unpack::kThreads, 0, stream>>>(p);
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
