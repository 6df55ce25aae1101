// Host-side fast paths of the restore staging engine and the coefficient-stream tools: parallel
// positioned reads into (pinned) host memory with the GIL released, and Annex-B start-code scanning
// of HEVC streams (the counterparts of the reference's ctypes pread loop,
// reelcache/restore_staging.py:336, and its memmem NAL scan, reelcache/accel_c.py:346-357).
#include <ATen/ATen.h>
#include <fcntl.h>
#include <pybind11/pybind11.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace rc {

// Reads sizes[i] bytes at file offset offsets[i] of paths[i] into the host address dest[i], on up to
// `threads` threads (largest requests first). Returns the bytes read; raises on any short read.
int64_t pread_many(const std::vector<std::string>& paths, const std::vector<int64_t>& offsets,
                   const std::vector<int64_t>& sizes, const std::vector<int64_t>& dest, int64_t threads) {
  const size_t n = paths.size();
  if (offsets.size() != n || sizes.size() != n || dest.size() != n)
    throw std::runtime_error("reelcache_b200: pread_many takes equal-length paths/offsets/sizes/dest");
  std::vector<size_t> order(n);
  for (size_t i = 0; i < n; ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](size_t a, size_t b) { return sizes[a] > sizes[b]; });
  std::atomic<size_t> next{0};
  std::atomic<int64_t> total{0};
  std::vector<std::string> errors(static_cast<size_t>(std::max<int64_t>(1, threads)));
  auto worker = [&](int id) {
    while (true) {
      const size_t k = next.fetch_add(1);
      if (k >= n) return;
      const size_t i = order[k];
      const int fd = ::open(paths[i].c_str(), O_RDONLY | O_CLOEXEC);
      if (fd < 0) {
        errors[id] = "cannot open " + paths[i] + ": " + std::strerror(errno);
        return;
      }
      int64_t done = 0;
      char* out = reinterpret_cast<char*>(dest[i]);
      while (done < sizes[i]) {
        const ssize_t got = ::pread(fd, out + done, static_cast<size_t>(sizes[i] - done), offsets[i] + done);
        if (got < 0 && errno == EINTR) continue;
        if (got <= 0) break;
        done += got;
      }
      ::close(fd);
      if (done != sizes[i]) {
        errors[id] = "short read of " + paths[i];
        return;
      }
      total.fetch_add(done);
    }
  };
  {
    pybind11::gil_scoped_release release;
    const int count = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(threads, static_cast<int64_t>(n))));
    std::vector<std::thread> pool;
    for (int t = 1; t < count; ++t) pool.emplace_back(worker, t);
    worker(0);
    for (auto& th : pool) th.join();
  }
  for (const auto& e : errors)
    if (!e.empty()) throw std::runtime_error("reelcache_b200: " + e);
  return total.load();
}

// Byte offsets of every Annex-B start code 00 00 01 in a CPU uint8 tensor (a 4-byte 00 00 00 01 code is
// reported at its last three bytes, as a plain pattern search does).
std::vector<int64_t> start_codes(const at::Tensor& data) {
  if (!data.device().is_cpu() || data.scalar_type() != at::kByte || !data.is_contiguous())
    throw std::runtime_error("reelcache_b200: start_codes takes a contiguous CPU uint8 tensor");
  const uint8_t* p = data.data_ptr<uint8_t>();
  const int64_t n = data.numel();
  std::vector<int64_t> out;
  int64_t i = 0;
  while (i + 3 <= n) {
    const void* hit = std::memchr(p + i + 2, 1, static_cast<size_t>(n - i - 2));
    if (hit == nullptr) break;
    const int64_t k = static_cast<const uint8_t*>(hit) - p;  // candidate 01 at k
    if (p[k - 1] == 0 && p[k - 2] == 0) out.push_back(k - 2);
    i = k - 1;
  }
  return out;
}

namespace {

std::runtime_error integrity(const std::string& message) {
  return std::runtime_error("integrity: " + message);
}

}  // namespace

// The NAL-unit table of an Annex-B HEVC stream: int64 [n, 3] rows (offset of the unit's header, length without
// trailing zero bytes, nal_unit_type), with the stream checks of the Python reader (a leading 3- or 4-byte start
// code, a 2-byte header per unit, a clear forbidden bit). A malformed stream throws "integrity: ...". Runs without
// the GIL (the counterpart of the reference's native nal_units, native/reelcache_native/src/lib.rs:28-69).
at::Tensor nal_units(const at::Tensor& data) {
  const std::vector<int64_t> starts = start_codes(data);
  const uint8_t* p = data.data_ptr<uint8_t>();
  const int64_t n = data.numel();
  if (starts.empty() || starts[0] > 1 || (starts[0] == 1 && p[0] != 0))
    throw integrity("an Annex-B HEVC stream must begin with a 3- or 4-byte start code");
  at::Tensor table = at::empty({static_cast<int64_t>(starts.size()), 3}, at::kLong);
  int64_t* row = table.data_ptr<int64_t>();
  for (size_t i = 0; i < starts.size(); ++i) {
    const int64_t begin = starts[i] + 3;
    const bool last = i + 1 == starts.size();
    int64_t end = last ? n : starts[i + 1];
    while (!last && end > begin && p[end - 1] == 0) --end;  // zero bytes before the next start code
    if (end - begin < 2)
      throw integrity("NAL unit at byte " + std::to_string(begin) + " is shorter than its 2-byte header");
    const uint8_t header = p[begin];
    if (header & 0x80) throw integrity("NAL unit at byte " + std::to_string(begin) + " sets the forbidden zero bit");
    row[3 * i] = begin;
    row[3 * i + 1] = end - begin;
    row[3 * i + 2] = (header >> 1) & 0x3F;
  }
  return table;
}

// Channel tiles back to coefficients: images uint8 [segments * frames, planes, image_h, image_w] (segment-major,
// then frame) of a channel-tile layout -> values uint8 [frames * height * width, rank]. Channel c lives in segment
// c / slots at cell index i = c % slots: plane i % planes, tile row (i / planes) / columns, tile column
// (i / planes) % columns. Runs without the GIL (the reference's native unpack_tile, lib.rs:71-140, per layout).
at::Tensor unmosaic_all(const at::Tensor& images, int64_t frames, int64_t height, int64_t width, int64_t rank,
                        int64_t columns, int64_t planes, int64_t slots) {
  if (!images.device().is_cpu() || images.scalar_type() != at::kByte || !images.is_contiguous() || images.dim() != 4)
    throw std::runtime_error("reelcache_b200: unmosaic_all takes a contiguous CPU uint8 [pictures, planes, h, w]");
  if (frames < 1 || height < 1 || width < 1 || rank < 1 || columns < 1 || planes < 1 || slots < 1)
    throw std::runtime_error("reelcache_b200: unmosaic_all needs positive layout dimensions");
  const int64_t segments = (rank + slots - 1) / slots;
  const int64_t rows_needed = ((std::min(rank, slots) + planes - 1) / planes + columns - 1) / columns;
  const int64_t ih = images.size(2), iw = images.size(3);
  if (images.size(0) != segments * frames || images.size(1) != planes || ih < rows_needed * height ||
      iw < columns * width)
    throw std::runtime_error("reelcache_b200: the pictures do not hold this channel-tile layout");
  std::vector<int64_t> base(static_cast<size_t>(rank));
  for (int64_t c = 0; c < rank; ++c) {
    const int64_t s = c / slots, index = c % slots;
    const int64_t plane = index % planes, cell = index / planes;
    const int64_t y0 = (cell / columns) * height, x0 = (cell % columns) * width;
    base[c] = ((s * frames) * planes + plane) * ih * iw + y0 * iw + x0;
  }
  at::Tensor out = at::empty({frames * height * width, rank}, at::kByte);
  const uint8_t* src = images.data_ptr<uint8_t>();
  uint8_t* dst = out.data_ptr<uint8_t>();
  const int64_t picture = planes * ih * iw;
  for (int64_t f = 0; f < frames; ++f)
    for (int64_t y = 0; y < height; ++y)
      for (int64_t x = 0; x < width; ++x) {
        const int64_t offset = f * picture + y * iw + x;
        uint8_t* d = dst + ((f * height + y) * width + x) * rank;
        for (int64_t c = 0; c < rank; ++c) d[c] = src[base[c] + offset];
      }
  return out;
}

}  // namespace rc
