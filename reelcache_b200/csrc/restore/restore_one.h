// Internal interface of the single-job, allocation-free launches of the restore pipeline (unpack,
// basis preparation, fused restore GEMM). The no-allocation entry point (noalloc.cu) builds every
// launch parameter on the stack and calls these; they allocate nothing, throw nothing and return a
// static error description (nullptr on success).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rc {

// One u8-sourced restore job after its scratch operands are laid out.
struct RestoreOneArgs {
  const __half* a;            // [tokens, k_pad] centered pixels (unpack output)
  const __half* bt;           // [channels, 2 * k_pad] prepared basis (hi | lo)
  const float* bias;          // [channels]
  void* dst;                  // element (token 0, head 0, dim 0) of the destination slot
  int64_t dst_ts, dst_hs, dst_ds;
  int tokens, k_pad, passes, out_dtype, channels, head_dim;
  const void* rope_pack;      // separable (cos, sin) pairs, 16-byte aligned, storage of even length; null: none
  int grid_t, grid_h, grid_w, sec_t, sec_h, rope_entries;
  float inverse;              // 2^-e of the job's prescale
  int* status;                // device status word (nullable)
};

const char* unpack_u8_one(const uint8_t* matrix, int64_t row_stride, __half* out, int tokens, int k_pad, int rank,
                          cudaStream_t stream);
const char* prep_one(const __half* q, int64_t q_stride, const float* scale, const float* offset, __half* bt,
                     float* bias, int rank, int k_pad, int channels, float prescale, cudaStream_t stream);
const char* restore_one_setup(int device);
const char* restore_launch_one(const RestoreOneArgs& args, int device, cudaStream_t stream);

}  // namespace rc
