// Device finalization of coefficient tiles for sm_100a (the counterpart of the reference's torch
// `quantize_device` path, reelcache/node_packets.py:156-188 and the covering affine of
// reelcache/_hevc.py:400-474):
//
//   colminmax: per-column extrema lo[k], hi[k] of FP32 coefficients P[N, r] (exact; NaN/Inf flagged)
//   quantize:  pixel = clip(rint((double(v) - double(offset[k])) / double(scale[k])), 0, 255)
//              (0 where scale == 0), the same IEEE FP64 arithmetic as the host path, so device and
//              host pixels are bitwise equal.
// The covering affine itself (a handful of FP32/FP64 operations per column) is computed on the host
// from the D2H-copied extrema.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cfloat>

#include "../common/host.h"

namespace rc {
namespace quant {

constexpr int kCols = 32;
constexpr int kRowsPerBlock = 8;

// grid: (ceil(r / 32), row_splits); block (32, 8). Writes partial extrema per row split.
__global__ void colminmax_kernel(const float* __restrict__ p, int64_t ld, int n, int r, int rows_per_split,
                                 float* __restrict__ lo_part, float* __restrict__ hi_part, int* __restrict__ bad) {
  const int col = blockIdx.x * kCols + threadIdx.x;
  const int row0 = blockIdx.y * rows_per_split;
  const int row1 = min(n, row0 + rows_per_split);
  float lo = FLT_MAX, hi = -FLT_MAX;
  bool finite = true;
  if (col < r) {
    for (int row = row0 + threadIdx.y; row < row1; row += kRowsPerBlock) {
      const float v = p[static_cast<int64_t>(row) * ld + col];
      finite &= isfinite(v);
      lo = fminf(lo, v);
      hi = fmaxf(hi, v);
    }
  }
  __shared__ float slo[kRowsPerBlock][kCols];
  __shared__ float shi[kRowsPerBlock][kCols];
  slo[threadIdx.y][threadIdx.x] = lo;
  shi[threadIdx.y][threadIdx.x] = hi;
  if (!finite) atomicExch(bad, 1);
  __syncthreads();
  if (threadIdx.y == 0 && col < r) {
    for (int i = 1; i < kRowsPerBlock; ++i) {
      lo = fminf(lo, slo[i][threadIdx.x]);
      hi = fmaxf(hi, shi[i][threadIdx.x]);
    }
    lo_part[static_cast<int64_t>(blockIdx.y) * r + col] = lo;
    hi_part[static_cast<int64_t>(blockIdx.y) * r + col] = hi;
  }
}

// one thread per element; out has row stride ldo (bytes)
__global__ void quantize_kernel(const float* __restrict__ p, int64_t ld, int n, int r, const float* __restrict__ scale,
                                const float* __restrict__ offset, uint8_t* __restrict__ out, int64_t ldo) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(n) * r) return;
  const int row = static_cast<int>(idx / r);
  const int col = static_cast<int>(idx - static_cast<int64_t>(row) * r);
  const float s = scale[col];
  double ratio = 0.0;
  if (s > 0.0f) ratio = __ddiv_rn(__dsub_rn(static_cast<double>(p[static_cast<int64_t>(row) * ld + col]),
                                             static_cast<double>(offset[col])),
                                   static_cast<double>(s));
  double q = rint(ratio);
  q = fmin(fmax(q, 0.0), 255.0);
  out[static_cast<int64_t>(row) * ldo + col] = static_cast<uint8_t>(q);
}

}  // namespace quant

// lo, hi: float32 [r] outputs; returns nothing; bad: int32 [1] nonfinite flag (device).
void colminmax(const at::Tensor& p, at::Tensor& lo, at::Tensor& hi, at::Tensor& bad) {
  RC_CHECK(p.is_cuda() && p.scalar_type() == at::kFloat && p.dim() == 2 && p.stride(1) == 1,
           "coefficients must be a CUDA float32 [N, r] matrix with unit column stride");
  const int n = static_cast<int>(p.size(0));
  const int r = static_cast<int>(p.size(1));
  c10::cuda::CUDAGuard guard(p.device());
  const int splits = std::max(1, std::min(64, n / 256));
  const int rows_per_split = (n + splits - 1) / splits;
  auto lo_part = at::empty({splits, r}, p.options());
  auto hi_part = at::empty({splits, r}, p.options());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(p.get_device()).stream();
  dim3 grid((r + quant::kCols - 1) / quant::kCols, splits);
  dim3 block(quant::kCols, quant::kRowsPerBlock);
  quant::colminmax_kernel<<<grid, block, 0, stream>>>(p.data_ptr<float>(), p.stride(0), n, r, rows_per_split,
                                                      lo_part.data_ptr<float>(), hi_part.data_ptr<float>(),
                                                      bad.data_ptr<int>());
  RC_CUDA(cudaGetLastError());
  lo.copy_(std::get<0>(lo_part.min(0)));
  hi.copy_(std::get<0>(hi_part.max(0)));
}

void quantize_columns(const at::Tensor& p, const at::Tensor& scale, const at::Tensor& offset, at::Tensor& out) {
  RC_CHECK(p.is_cuda() && p.scalar_type() == at::kFloat && p.dim() == 2 && p.stride(1) == 1,
           "coefficients must be a CUDA float32 [N, r] matrix with unit column stride");
  RC_CHECK(out.is_cuda() && out.scalar_type() == at::kByte && out.dim() == 2 && out.stride(1) == 1 &&
               out.size(0) == p.size(0) && out.size(1) >= p.size(1),
           "out must be a CUDA uint8 [N, >= r] matrix");
  RC_CHECK(scale.numel() == p.size(1) && offset.numel() == p.size(1) && scale.scalar_type() == at::kFloat &&
               offset.scalar_type() == at::kFloat && scale.is_contiguous() && offset.is_contiguous(),
           "scale/offset must be contiguous float32 [r] vectors");
  c10::cuda::CUDAGuard guard(p.device());
  const int n = static_cast<int>(p.size(0));
  const int r = static_cast<int>(p.size(1));
  const int64_t total = static_cast<int64_t>(n) * r;
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(p.get_device()).stream();
  quant::quantize_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      p.data_ptr<float>(), p.stride(0), n, r, scale.data_ptr<float>(), offset.data_ptr<float>(), out.data_ptr<uint8_t>(),
      out.stride(0));
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
