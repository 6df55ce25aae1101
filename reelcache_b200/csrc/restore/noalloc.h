/* Allocation-free restore entry point (C ABI).
 *
 * This interface has no counterpart in the reference implementation. It restores one
 * 8-bit-coefficient job -- unpack, basis preparation and the fused sm_100a restore GEMM with its
 * RoPE epilogue, the same kernels and parameters as the Python entry point
 * reelcache_b200.restore_kernels.reconstruct (backend "fused") -- without allocating anything:
 * its intermediate operands live in one fixed device scratch area of RC_NOALLOC_SCRATCH_BYTES
 * bytes, and every launch parameter is built on the caller's stack.
 *
 * It exists for callers that must not allocate: a host engine in C/C++ that owns all device
 * memory itself (a caching allocator it does not control would fragment or grow its pool), code
 * that runs while another component has the allocator locked or is trimming device memory under
 * pressure, and latency-critical restore paths where an allocation (cudaMalloc synchronizes the
 * device; a caching allocator may block or call into the driver) cannot be afforded.
 *
 * Contract:
 *  - The first call on a device performs setup (resolves the scratch address with
 *    cudaGetSymbolAddress, reserves the kernel's shared memory, resolves the tensor-map encoder).
 *    Make that first call (a call with job == NULL only performs setup) before any stream
 *    capture begins.
 *  - Scratch need: align256(tokens * k_pad * 2) + align256(channels * 4 * k_pad) +
 *    align256(channels * 4) bytes, k_pad = rank rounded up to a multiple of 64. Larger jobs are
 *    rejected (return RC_NOALLOC_TOO_LARGE) before anything is launched.
 *  - Nothing in the scratch has to start at zero: every call writes all the scratch it reads.
 *    The optional status word (job->status) must start at zero; a kernel that gave up a bounded
 *    wait sets it nonzero.
 *  - Calls on one device share the one scratch area: two calls whose GPU work can overlap (on
 *    different streams, or from different threads without ordering) race on it. Issue them on one
 *    stream, or order them with events.
 *  - All pointers are device pointers on `device` except `error`. Work is enqueued on `stream`
 *    (a cudaStream_t; NULL is the legacy default stream); the call returns without waiting.
 */
#ifndef REELCACHE_B200_NOALLOC_H
#define REELCACHE_B200_NOALLOC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RC_NOALLOC_SCRATCH_BYTES (32u << 20)

#define RC_NOALLOC_OK 0
#define RC_NOALLOC_BAD_ARGUMENT 1
#define RC_NOALLOC_TOO_LARGE 2
#define RC_NOALLOC_CUDA_ERROR 3

typedef struct RcRestoreU8Job {
  const void* coefficients;    /* uint8 [tokens, >= rank], row stride coeff_stride bytes */
  int64_t coeff_stride;
  int64_t tokens;
  int64_t rank;
  const void* basis;           /* float16 [>= rank, channels] rows, row stride basis_stride elements */
  int64_t basis_stride;
  const void* scale;           /* float32 [rank]: coefficient k = pixel * scale[k] + offset[k] */
  const void* offset;          /* float32 [rank] */
  double scale_basis_bound;    /* max_k |scale[k]| * max |basis|: selects the exact power-of-two prescale */
  void* destination;           /* element (token 0, head 0, dim 0) of the native cache slot */
  int64_t dst_token_stride;    /* element strides of the slot */
  int64_t dst_head_stride;
  int64_t dst_dim_stride;
  int64_t out_dtype;           /* 0 bfloat16, 1 float16, 2 float32 */
  int64_t channels;            /* heads * head_dim (multiple of 32) */
  int64_t head_dim;            /* multiple of 32 */
  const void* rope_pack;       /* NULL: no rotation; else separable (cos, sin) float32 pairs */
  int64_t grid_t, grid_h, grid_w;        /* token grid (frames, rows, columns) */
  int64_t sec_t, sec_h;                  /* pairs of the frame and row sections */
  int64_t rope_entries;                  /* grid_t*sec_t + grid_h*sec_h + grid_w*(head_dim/2-sec_t-sec_h) */
  int64_t passes;              /* 1: one FP16 product (bfloat16 slots), 2: hi + lo products */
  int* status;                 /* NULL or a zero-initialized device word for bounded-wait failures */
} RcRestoreU8Job;

/* Returns RC_NOALLOC_OK or an error code; on error writes a message into error[0..error_len). */
int rc_restore_u8_noalloc(const RcRestoreU8Job* job, int device, void* stream, char* error, size_t error_len);

#ifdef __cplusplus
}
#endif

#endif /* REELCACHE_B200_NOALLOC_H */
