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

}  // namespace rc
