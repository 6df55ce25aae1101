// Allocation-free restore entry point: see noalloc.h for the contract.
//
// The scratch operands of the restore pipeline (the unpacked A operand, the prepared B operand and
// the per-channel bias) live in one file-scope device array instead of per-call allocations; the
// three launches take their parameters by value from this call's stack.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <mutex>

#include "noalloc.h"
#include "restore_one.h"

namespace rc {
namespace {

constexpr int kMaxDevices = 64;

// The one scratch area per device (file-scope device storage: reserved at module load, never
// allocated or freed by a call).
static __device__ __align__(256) unsigned char g_noalloc_scratch[RC_NOALLOC_SCRATCH_BYTES];

unsigned char* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_setup_lock;

int fail(char* error, size_t error_len, int code, const char* what) {
  if (error != nullptr && error_len > 0) snprintf(error, error_len, "rc_restore_u8_noalloc: %s", what);
  return code;
}

uint64_t align256(uint64_t n) { return (n + 255) & ~uint64_t(255); }

// Exponent e bringing bound * 2^e into (2^13, 2^14] (0 for a zero or non-finite bound), clamped to
// +-100: the same rule as reelcache_b200.ops.restore.prescale_exponent.
int prescale_exponent(double bound) {
  if (!(bound > 0.0) || !std::isfinite(bound)) return 0;
  const double b = bound > 1e-30 ? bound : 1e-30;
  int e = 14 - static_cast<int>(std::ceil(std::log2(b)));
  if (e < -100) e = -100;
  if (e > 100) e = 100;
  return e;
}

// Per-device setup (first call): the scratch address and the restore kernel's shared memory.
const char* setup(int device) {
  std::lock_guard<std::mutex> guard(g_setup_lock);
  if (g_scratch_addr[device] != nullptr) return nullptr;
  int current = -1;
  if (cudaGetDevice(&current) != cudaSuccess) return "no current CUDA device";
  if (current != device && cudaSetDevice(device) != cudaSuccess) return "cannot select the device";
  void* addr = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
  const char* error = err == cudaSuccess ? restore_one_setup(device) : "cudaGetSymbolAddress of the scratch failed";
  if (current != device) cudaSetDevice(current);
  if (error != nullptr) return error;
  g_scratch_addr[device] = static_cast<unsigned char*>(addr);
  return nullptr;
}

}  // namespace
}  // namespace rc

extern "C" int rc_restore_u8_noalloc(const RcRestoreU8Job* job, int device, void* stream, char* error,
                                     size_t error_len) {
  using namespace rc;
  if (device < 0 || device >= kMaxDevices) return fail(error, error_len, RC_NOALLOC_BAD_ARGUMENT, "bad device");
  if (const char* why = setup(device)) return fail(error, error_len, RC_NOALLOC_CUDA_ERROR, why);
  if (job == nullptr) return RC_NOALLOC_OK;  // setup only
  const RcRestoreU8Job& j = *job;
  if (j.coefficients == nullptr || j.basis == nullptr || j.scale == nullptr || j.offset == nullptr ||
      j.destination == nullptr)
    return fail(error, error_len, RC_NOALLOC_BAD_ARGUMENT, "null operand pointer");
  if (j.tokens < 1 || j.tokens >= (1 << 24) || j.rank < 1 || j.rank > 8192 || j.coeff_stride < j.rank ||
      j.basis_stride < j.channels || j.channels < 32 || j.channels % 32 != 0 || j.head_dim < 32 ||
      j.head_dim % 32 != 0 || j.channels % j.head_dim != 0 || (j.passes != 1 && j.passes != 2) || j.out_dtype < 0 ||
      j.out_dtype > 2)
    return fail(error, error_len, RC_NOALLOC_BAD_ARGUMENT, "job geometry out of range");
  const int64_t k_pad = (j.rank + 63) / 64 * 64;
  const uint64_t a_bytes = align256(static_cast<uint64_t>(j.tokens) * k_pad * 2);
  const uint64_t b_bytes = align256(static_cast<uint64_t>(j.channels) * 2 * k_pad * 2);
  const uint64_t bias_bytes = align256(static_cast<uint64_t>(j.channels) * 4);
  if (a_bytes + b_bytes + bias_bytes > RC_NOALLOC_SCRATCH_BYTES) {
    char what[160];
    snprintf(what, sizeof(what), "job needs %llu bytes of scratch, above the fixed %u",
             static_cast<unsigned long long>(a_bytes + b_bytes + bias_bytes), RC_NOALLOC_SCRATCH_BYTES);
    return fail(error, error_len, RC_NOALLOC_TOO_LARGE, what);
  }
  unsigned char* base = g_scratch_addr[device];
  __half* a = reinterpret_cast<__half*>(base);
  __half* bt = reinterpret_cast<__half*>(base + a_bytes);
  float* bias = reinterpret_cast<float*>(base + a_bytes + b_bytes);
  const int e = prescale_exponent(j.scale_basis_bound);
  const float prescale = std::ldexp(1.0f, e);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int current = -1;
  if (cudaGetDevice(&current) != cudaSuccess) return fail(error, error_len, RC_NOALLOC_CUDA_ERROR, "no device");
  if (current != device && cudaSetDevice(device) != cudaSuccess)
    return fail(error, error_len, RC_NOALLOC_CUDA_ERROR, "cannot select the device");
  const char* why = unpack_u8_one(static_cast<const uint8_t*>(j.coefficients), j.coeff_stride, a,
                                  static_cast<int>(j.tokens), static_cast<int>(k_pad), static_cast<int>(j.rank), s);
  if (why == nullptr)
    why = prep_one(static_cast<const __half*>(j.basis), j.basis_stride, static_cast<const float*>(j.scale),
                   static_cast<const float*>(j.offset), bt, bias, static_cast<int>(j.rank), static_cast<int>(k_pad),
                   static_cast<int>(j.channels), prescale, s);
  if (why == nullptr) {
    RestoreOneArgs r;
    r.a = a;
    r.bt = bt;
    r.bias = bias;
    r.dst = j.destination;
    r.dst_ts = j.dst_token_stride;
    r.dst_hs = j.dst_head_stride;
    r.dst_ds = j.dst_dim_stride;
    r.tokens = static_cast<int>(j.tokens);
    r.k_pad = static_cast<int>(k_pad);
    r.passes = static_cast<int>(j.passes);
    r.out_dtype = static_cast<int>(j.out_dtype);
    r.channels = static_cast<int>(j.channels);
    r.head_dim = static_cast<int>(j.head_dim);
    r.rope_pack = j.rope_pack;
    r.grid_t = static_cast<int>(j.grid_t);
    r.grid_h = static_cast<int>(j.grid_h);
    r.grid_w = static_cast<int>(j.grid_w);
    r.sec_t = static_cast<int>(j.sec_t);
    r.sec_h = static_cast<int>(j.sec_h);
    r.rope_entries = static_cast<int>(j.rope_entries);
    r.inverse = std::ldexp(1.0f, -e);
    r.status = j.status;
    why = restore_launch_one(r, device, s);
  }
  if (current != device) cudaSetDevice(current);
  if (why != nullptr) return fail(error, error_len, RC_NOALLOC_CUDA_ERROR, why);
  return RC_NOALLOC_OK;
}
