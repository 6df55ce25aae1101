// NVLS (NVLink SHARP) reduction of symmetric partial buffers through the NVSwitch, sm_100a.
//
// Every rank holds its FP32 partial of a matrix at the same offset of its symmetric buffer; the buffer is bound to
// an NVLink multicast object, so one address (the multicast address) names the copy on every GPU. An owner reads
// that address with multimem.ld_reduce: the switch fetches the element from every GPU bound to the object, adds
// them and returns the sum, so each partial crosses NVLink once, from its GPU to the switch, and the owner receives
// one reduced stream -- the traffic of an in-switch reduce-scatter, with no peer loads and no sum kernel.
//
// The caller orders this after every rank wrote its partials (a device barrier on the stream before the launch).
// Only the upper-triangular 128 x 128 tiles of each C x C matrix are reduced (the partials are Grams); the
// caller mirrors them. The switch adds the ranks' values in an order of its own, so results may differ in the
// last bit from a rank-ordered sum.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "../common/host.h"

namespace rc {
namespace nvls {

constexpr int kTile = 128;
constexpr int kThreads = 256;

// Sum over every GPU bound to the multicast object of the four floats at `mc` (16-byte aligned multicast address).
__device__ __forceinline__ float4 ld_reduce_add_v4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

// One CTA per (matrix, upper tile): out[m] tile (ti, tj) = sum over GPUs of buffer[offsets[m] + tile].
__global__ void __launch_bounds__(kThreads) reduce_upper_kernel(const float* __restrict__ mc_base,
                                                                const int64_t* __restrict__ offsets,
                                                                float* __restrict__ out, int C) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");  // the partials' writers released them before our barrier
  const int nt = C / kTile;
  const int per_matrix = nt * (nt + 1) / 2;
  const int m = blockIdx.x / per_matrix;
  int t = blockIdx.x % per_matrix;
  int ti = 0;
  while (t >= nt - ti) {  // upper tiles of row ti: (ti, ti) .. (ti, nt - 1)
    t -= nt - ti;
    ++ti;
  }
  const int tj = ti + t;
  const float* src = mc_base + offsets[m];
  float* dst = out + static_cast<int64_t>(m) * C * C;
  for (int idx = threadIdx.x; idx < kTile * (kTile / 4); idx += kThreads) {
    const int row = ti * kTile + idx / (kTile / 4);
    const int col = tj * kTile + (idx % (kTile / 4)) * 4;
    const int64_t at = static_cast<int64_t>(row) * C + col;
    *reinterpret_cast<float4*>(dst + at) = ld_reduce_add_v4(src + at);
  }
}

}  // namespace nvls

// out[m] (FP32 [count, C, C], upper 128 x 128 tiles written) = sum over the multicast group of the C x C partial at
// element offset offsets[m] of the symmetric buffer whose multicast address is `mc_ptr` (`buffer_elems` floats).
void nvls_reduce_upper(int64_t mc_ptr, int64_t buffer_elems, const at::Tensor& offsets, at::Tensor& out, int64_t C) {
  RC_CHECK(mc_ptr != 0 && mc_ptr % 16 == 0, "a 16-byte aligned multicast address is required");
  RC_CHECK(C > 0 && C % nvls::kTile == 0, "C must be a positive multiple of 128");
  check_cuda_tensor(out, "out");
  RC_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.dim() == 3 && out.size(1) == C &&
               out.size(2) == C,
           "out must be a contiguous float32 [count, C, C]");
  RC_CHECK(offsets.scalar_type() == at::kLong && offsets.dim() == 1 && offsets.numel() == out.size(0),
           "one int64 element offset per output matrix");
  const at::Tensor host = offsets.cpu();
  const int64_t* off = host.data_ptr<int64_t>();
  for (int64_t m = 0; m < host.numel(); ++m)
    RC_CHECK(off[m] >= 0 && off[m] % 4 == 0 && off[m] + C * C <= buffer_elems,
             "a partial's offset lies outside the symmetric buffer or breaks 16-byte alignment");
  const int count = static_cast<int>(out.size(0));
  if (count == 0) return;
  const at::Tensor dev_offsets = host.to(out.device());
  c10::cuda::CUDAGuard guard(out.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(out.get_device()).stream();
  const int nt = static_cast<int>(C / nvls::kTile);
  const int blocks = count * nt * (nt + 1) / 2;
  nvls::reduce_upper_kernel<<<blocks, nvls::kThreads, 0, stream>>>(
      reinterpret_cast<const float*>(mc_ptr), dev_offsets.data_ptr<int64_t>(), out.data_ptr<float>(),
      static_cast<int>(C));
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
