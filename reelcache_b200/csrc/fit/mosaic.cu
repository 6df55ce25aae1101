// Device channel-tile mosaic for sm_100a (the device side of the reference's node-packet finalization,
// reelcache/node_packets.py:176 mosaic_device, with the reelcache.channel_tiles.v1 geometry of
// reelcache/_hevc.py:517-612): quantized coefficients u8 [frames * height * width, rank] -> canvas
// u8 [segments * frames, planes, image_h, image_w]. Segment s holds channels [s * slots, (s + 1) * slots);
// slot i of a segment sits in plane i % planes, grid cell (i / planes) of a columns-wide grid. Padding and
// unused cells are zero. One thread per canvas byte: coalesced writes, gathered reads.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "../common/host.h"

namespace rc {
namespace fit {

struct MosaicGeometry {
  int frames, height, width, rank, planes, columns, rows, image_h, image_w, slots, segments;
};

__global__ void mosaic_kernel(const uint8_t* __restrict__ pixels, int64_t ld, MosaicGeometry g,
                              uint8_t* __restrict__ canvas, int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  int64_t rest = idx;
  const int x = static_cast<int>(rest % g.image_w);
  rest /= g.image_w;
  const int y = static_cast<int>(rest % g.image_h);
  rest /= g.image_h;
  const int plane = static_cast<int>(rest % g.planes);
  rest /= g.planes;
  const int frame = static_cast<int>(rest % g.frames);
  const int segment = static_cast<int>(rest / g.frames);
  uint8_t value = 0;
  const int cell_row = y / g.height, cell_col = x / g.width;
  if (cell_row < g.rows && cell_col < g.columns) {
    const int slot = (cell_row * g.columns + cell_col) * g.planes + plane;
    const int channel = segment * g.slots + slot;
    if (slot < g.slots && channel < g.rank) {
      const int64_t token = (static_cast<int64_t>(frame) * g.height + (y - cell_row * g.height)) * g.width +
                            (x - cell_col * g.width);
      value = pixels[token * ld + channel];
    }
  }
  canvas[idx] = value;
}

}  // namespace fit

void mosaic_u8(const at::Tensor& pixels, at::Tensor& canvas, const std::vector<int64_t>& geometry) {
  check_cuda_tensor(pixels, "pixels");
  check_cuda_tensor(canvas, "canvas");
  RC_CHECK(pixels.scalar_type() == at::kByte && canvas.scalar_type() == at::kByte, "u8 pixels and canvas");
  RC_CHECK(pixels.dim() == 2 && pixels.stride(1) == 1 && canvas.is_contiguous(), "pixels [N, >= rank], dense canvas");
  RC_CHECK(geometry.size() == 11, "geometry: frames, height, width, rank, planes, columns, rows, image_h, image_w, "
                                  "slots, segments");
  fit::MosaicGeometry g{static_cast<int>(geometry[0]), static_cast<int>(geometry[1]), static_cast<int>(geometry[2]),
                        static_cast<int>(geometry[3]), static_cast<int>(geometry[4]), static_cast<int>(geometry[5]),
                        static_cast<int>(geometry[6]), static_cast<int>(geometry[7]), static_cast<int>(geometry[8]),
                        static_cast<int>(geometry[9]), static_cast<int>(geometry[10])};
  RC_CHECK(pixels.size(0) == int64_t(g.frames) * g.height * g.width && pixels.size(1) >= g.rank, "pixel shape");
  RC_CHECK(g.rows * g.height <= g.image_h && g.columns * g.width <= g.image_w, "grid exceeds the canvas");
  const int64_t total = int64_t(g.segments) * g.frames * g.planes * g.image_h * g.image_w;
  RC_CHECK(canvas.numel() == total, "canvas size differs from the geometry");
  if (total == 0) return;
  c10::cuda::CUDAGuard guard(pixels.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(pixels.get_device()).stream();
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  fit::mosaic_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(pixels.data_ptr<uint8_t>(),
                                                                            pixels.stride(0), g,
                                                                            canvas.data_ptr<uint8_t>(), total);
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
