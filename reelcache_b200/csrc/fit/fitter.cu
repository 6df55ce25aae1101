// Fitter kernels for sm_100a: the numerical building blocks of rank selection that the reference runs
// through cuBLAS SGEMM, cuSOLVER and Triton (reelcache/exact_blas.py, reelcache/cusolver_eigh.py,
// reelcache/accel_b.py:318-455).
//
//   split_bf16x3     FP32 matrix -> bfloat16 hi/mid/lo parts laid out as K-concatenated segments, so one
//                    tcgen05 bf16 GEMM over the concatenated K evaluates the six leading cross products
//                    hh + hm + mh + mm + hl + lh of an FP32 product (24+ significant bits per operand,
//                    FP32 accumulation in TMEM): an FP32-accurate GEMM on the tensor cores.
//   jacobi_eigh      batched symmetric eigendecomposition (FP32, n <= 160): cyclic two-sided Jacobi with
//                    the round-robin parallel ordering, one CTA per matrix, matrix and eigenvectors resident
//                    in shared memory; rotations skipped below max(tol * sqrt(|a_pp a_qq|), eps * ||A||_F);
//                    converged when a sweep rotates nothing (bounded sweep count, status per matrix).
//   sq_partials      per 8-row block: sum (x/s)^2, sum ((x-r)/s)^2 and a non-finite flag, FP32 squares
//                    summed per thread then reduced in FP64 (deterministic).
//   fingerprint      exact int64 modular checksums of the bit patterns of a 16/32-bit matrix (linear and
//                    quadratic terms of 16-bit parts with column and row weights), one warp per row.
//   dot2_gemm        P = X R^T with compensated dot products (Ogita, Rump and Oishi, "Accurate sum and dot
//                    product", SIAM J. Sci. Comput. 26(6), 2005: TwoProduct by FMA, TwoSum), FP32 result.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_bf16.h>

#include <cfloat>
#include <cstdint>

#include "../common/host.h"

namespace rc {
namespace fit {

// ---------------------------------------------------------------------------------------------------
// split_bf16x3
// ---------------------------------------------------------------------------------------------------

constexpr int kSplitTile = 32;

// x: logical [R, K] FP32 with element strides (sr, sk). out: bf16 [R, ldo]; segment s (s < nseg) covers
// columns [s * kp, s * kp + K) and holds part ((pattern >> 2s) & 3) of each element (0 hi, 1 mid, 2 lo);
// columns [s * kp + K, (s + 1) * kp) are zero. grid (ceil(K/32), ceil(R/32)), block (32, 8).
__global__ void split_bf16x3_kernel(const float* __restrict__ x, int64_t sr, int64_t sk, int R, int K, int kp,
                                    __nv_bfloat16* __restrict__ out, int64_t ldo, int nseg, uint32_t pattern) {
  __shared__ float tile[kSplitTile][kSplitTile + 1];  // [r][k]
  const int k0 = blockIdx.x * kSplitTile;
  const int r0 = blockIdx.y * kSplitTile;
  const int tx = threadIdx.x, ty = threadIdx.y;
  if (sk == 1) {
    for (int i = ty; i < kSplitTile; i += 8) {
      const int r = r0 + i, k = k0 + tx;
      tile[i][tx] = (r < R && k < K) ? x[static_cast<int64_t>(r) * sr + k] : 0.0f;
    }
  } else {
    for (int i = ty; i < kSplitTile; i += 8) {
      const int r = r0 + tx, k = k0 + i;
      tile[tx][i] = (r < R && k < K) ? x[static_cast<int64_t>(r) * sr + static_cast<int64_t>(k) * sk] : 0.0f;
    }
  }
  __syncthreads();
  const int k = k0 + tx;
  if (k >= kp) return;
  for (int i = ty; i < kSplitTile; i += 8) {
    const int r = r0 + i;
    if (r >= R) break;
    const float v = tile[i][tx];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(hi);  // exact: v minus its rounding to 8 significant bits
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(mid);
    const __nv_bfloat16 lo = __float2bfloat16_rn(r2);
    __nv_bfloat16* row = out + static_cast<int64_t>(r) * ldo;
    for (int s = 0; s < nseg; ++s) {
      const uint32_t part = (pattern >> (2 * s)) & 3u;
      row[static_cast<int64_t>(s) * kp + k] = part == 0 ? hi : (part == 1 ? mid : lo);
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// jacobi_eigh
// ---------------------------------------------------------------------------------------------------

constexpr int kJacobiMaxN = 160;
constexpr int kJacobiThreads = 512;

enum JacobiInfo : int { kConverged = 0, kSweepLimit = 1, kNonFinite = 2 };

// Pair i of round r of the round-robin ordering of m (even) indices: every index once per round,
// every unordered pair once per m - 1 rounds.
__device__ __forceinline__ void rr_pair(int m, int r, int i, int& p, int& q) {
  if (i == 0) {
    p = m - 1;
    q = r;
  } else {
    p = (r + i) % (m - 1);
    q = (r - i + (m - 1)) % (m - 1);
  }
  if (p > q) {
    const int t = p;
    p = q;
    q = t;
  }
}

// in: [batch, n, n] FP32 symmetric (lower and upper both read; symmetrized on load).
// values: [batch, n] ascending; vectors: [batch, n, n] with vectors[b, :, j] the j-th eigenvector.
// info[b]: kConverged / kSweepLimit / kNonFinite; sweeps[b]: sweeps run.
__global__ void __launch_bounds__(kJacobiThreads, 1)
    jacobi_eigh_kernel(const float* __restrict__ in, int n, float* __restrict__ values, float* __restrict__ vectors,
                       int* __restrict__ info, int* __restrict__ sweeps_out, int max_sweeps, float tol) {
  extern __shared__ float smem[];
  const int m = (n + 1) & ~1;  // even number of indices (index n is a dummy when n is odd)
  const int ld = m + 1;        // odd row stride: column walks hit distinct banks
  float* A = smem;
  float* V = A + m * ld;
  float* cs_c = V + m * ld;
  float* cs_s = cs_c + m / 2;
  float* red = cs_s + m / 2;     // [kJacobiThreads / 32] reduction scratch
  int* pair_p = reinterpret_cast<int*>(red + kJacobiThreads / 32);
  int* pair_q = pair_p + m / 2;
  int* flags = pair_q + m / 2;   // [0] rotations this sweep, [1] non-finite seen, [2] rank scratch base
  int* rank = flags + 4;         // [m]
  const int tid = threadIdx.x;
  const int b = blockIdx.x;
  const float* a_in = in + static_cast<int64_t>(b) * n * n;

  float local_sq = 0.0f;
  bool local_bad = false;
  for (int idx = tid; idx < m * m; idx += kJacobiThreads) {
    const int i = idx / m, j = idx % m;
    float v = 0.0f;
    if (i < n && j < n) {
      v = 0.5f * (a_in[i * n + j] + a_in[j * n + i]);
      local_bad |= !(fabsf(v) <= FLT_MAX);
    }
    A[i * ld + j] = v;
    V[i * ld + j] = (i == j) ? 1.0f : 0.0f;
    local_sq += v * v;
  }
  if (tid == 0) {
    flags[0] = 0;
    flags[1] = 0;
  }
  // block reduction of ||A||_F^2
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) local_sq += __shfl_xor_sync(0xffffffffu, local_sq, off);
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = local_sq;
  if (local_bad) atomicOr(&flags[1], 1);
  __syncthreads();
  float fro2 = 0.0f;
  for (int w = 0; w < kJacobiThreads / 32; ++w) fro2 += red[w];
  const bool bad = flags[1] != 0;
  const float abs_floor = 1.1920929e-07f * sqrtf(fro2);  // FP32 epsilon * ||A||_F

  int sweep = 0;
  int status = bad ? kNonFinite : kSweepLimit;
  const int half = m / 2;
  while (!bad && sweep < max_sweeps) {
    __syncthreads();
    if (tid == 0) flags[0] = 0;
    for (int round = 0; round < m - 1; ++round) {
      __syncthreads();
      if (tid < half) {
        int p, q;
        rr_pair(m, round, tid, p, q);
        float c = 1.0f, s = 0.0f;
        if (q < n) {
          const float apq = A[p * ld + q];
          const float app = A[p * ld + p];
          const float aqq = A[q * ld + q];
          const float thresh = fmaxf(tol * sqrtf(fabsf(app) * fabsf(aqq)), abs_floor);
          if (fabsf(apq) > thresh) {
            const double theta = (static_cast<double>(aqq) - app) / (2.0 * apq);
            const double t = (theta >= 0.0 ? 1.0 : -1.0) / (fabs(theta) + sqrt(theta * theta + 1.0));
            const double cd = 1.0 / sqrt(t * t + 1.0);
            c = static_cast<float>(cd);
            s = static_cast<float>(t * cd);
            atomicAdd(&flags[0], 1);
          }
        }
        pair_p[tid] = p;
        pair_q[tid] = q;
        cs_c[tid] = c;
        cs_s[tid] = s;
      }
      __syncthreads();
      // rows p, q of A  <-  J^T A
      for (int idx = tid; idx < half * m; idx += kJacobiThreads) {
        const int pi = idx / m, j = idx % m;
        const float s = cs_s[pi];
        if (s == 0.0f) continue;
        const float c = cs_c[pi];
        const int p = pair_p[pi], q = pair_q[pi];
        const float ap = A[p * ld + j], aq = A[q * ld + j];
        A[p * ld + j] = c * ap - s * aq;
        A[q * ld + j] = s * ap + c * aq;
      }
      __syncthreads();
      // columns p, q of A and V  <-  (.) J
      for (int idx = tid; idx < half * m; idx += kJacobiThreads) {
        const int pi = idx / m, i = idx % m;
        const float s = cs_s[pi];
        if (s == 0.0f) continue;
        const float c = cs_c[pi];
        const int p = pair_p[pi], q = pair_q[pi];
        const float ap = A[i * ld + p], aq = A[i * ld + q];
        A[i * ld + p] = c * ap - s * aq;
        A[i * ld + q] = s * ap + c * aq;
        const float vp = V[i * ld + p], vq = V[i * ld + q];
        V[i * ld + p] = c * vp - s * vq;
        V[i * ld + q] = s * vp + c * vq;
      }
      __syncthreads();
      // the annihilated entries are exactly zero
      if (tid < half && cs_s[tid] != 0.0f) {
        const int p = pair_p[tid], q = pair_q[tid];
        A[p * ld + q] = 0.0f;
        A[q * ld + p] = 0.0f;
      }
    }
    __syncthreads();
    ++sweep;
    if (flags[0] == 0) {
      status = kConverged;
      break;
    }
  }
  __syncthreads();
  // ascending order: rank of each diagonal entry (ties broken by index)
  for (int i = tid; i < n; i += kJacobiThreads) {
    const float di = A[i * ld + i];
    int r = 0;
    for (int j = 0; j < n; ++j) {
      const float dj = A[j * ld + j];
      r += (dj < di) || (dj == di && j < i);
    }
    rank[i] = r;
  }
  __syncthreads();
  float* vals = values + static_cast<int64_t>(b) * n;
  float* vecs = vectors + static_cast<int64_t>(b) * n * n;
  for (int i = tid; i < n; i += kJacobiThreads) vals[rank[i]] = A[i * ld + i];
  for (int idx = tid; idx < n * n; idx += kJacobiThreads) {
    const int row = idx / n, i = idx % n;
    vecs[row * n + rank[i]] = V[row * ld + i];
  }
  if (tid == 0) {
    info[b] = status;
    sweeps_out[b] = sweep;
  }
}

inline int jacobi_smem_bytes(int n) {
  const int m = (n + 1) & ~1;
  const int ld = m + 1;
  return static_cast<int>(sizeof(float)) * (2 * m * ld + m + kJacobiThreads / 32) +
         static_cast<int>(sizeof(int)) * (m + 4 + m);
}

// ---------------------------------------------------------------------------------------------------
// sq_partials
// ---------------------------------------------------------------------------------------------------

constexpr int kSqRows = 8;
constexpr int kSqThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  return static_cast<float>(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}

// out[block] = {sum (x/s)^2, sum ((x - r)/s)^2, non-finite flag} over rows [8 block, 8 block + 8).
template <typename TX, typename TR, bool HAS_R, bool DIV>
__global__ void __launch_bounds__(kSqThreads)
    sq_partials_kernel(const TX* __restrict__ x, int64_t sx0, int64_t sx1, const TR* __restrict__ r, int64_t sr0,
                       int64_t sr1, int rows, int cols, float scale, double* __restrict__ out) {
  __shared__ double red[2][kSqThreads / 32];
  __shared__ int bad_any;
  const int tid = threadIdx.x;
  if (tid == 0) bad_any = 0;
  float ax = 0.0f, ad = 0.0f;
  bool bad = false;
  const int row0 = blockIdx.x * kSqRows;
  double dx = 0.0, dd = 0.0;
  for (int i = 0; i < kSqRows; ++i) {
    const int row = row0 + i;
    if (row >= rows) break;
    for (int c = tid; c < cols; c += kSqThreads) {
      const float v = to_f32(x[static_cast<int64_t>(row) * sx0 + static_cast<int64_t>(c) * sx1]);
      bad |= !(fabsf(v) <= FLT_MAX);
      const float xs = DIV ? __fdiv_rn(v, scale) : v;
      ax = __fmaf_rn(xs, xs, ax);
      if (HAS_R) {
        const float rv = to_f32(r[static_cast<int64_t>(row) * sr0 + static_cast<int64_t>(c) * sr1]);
        float d = v - rv;
        if (DIV) d = __fdiv_rn(d, scale);
        ad = __fmaf_rn(d, d, ad);
      }
    }
    // FP32 per row and thread, FP64 across rows
    dx += ax;
    dd += ad;
    ax = 0.0f;
    ad = 0.0f;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    dx += __shfl_xor_sync(0xffffffffu, dx, off);
    dd += __shfl_xor_sync(0xffffffffu, dd, off);
  }
  __syncthreads();
  if (bad) atomicOr(&bad_any, 1);
  if ((tid & 31) == 0) {
    red[0][tid >> 5] = dx;
    red[1][tid >> 5] = dd;
  }
  __syncthreads();
  if (tid == 0) {
    double sx = 0.0, sd = 0.0;
    for (int w = 0; w < kSqThreads / 32; ++w) {
      sx += red[0][w];
      sd += red[1][w];
    }
    out[blockIdx.x * 3] = sx;
    out[blockIdx.x * 3 + 1] = sd;
    out[blockIdx.x * 3 + 2] = bad_any ? 1.0 : 0.0;
  }
}

// ---------------------------------------------------------------------------------------------------
// fingerprint partials
// ---------------------------------------------------------------------------------------------------

constexpr int kFpRowsPerBlock = 8;  // one warp per row

__device__ __forceinline__ long long pymod(long long a, long long p) {
  long long r = a % p;
  return r < 0 ? r + p : r;
}

// bits: [rows, cols] int16 (WIDE = false) or int32 (WIDE = true) bit patterns. Per row: for each 16-bit part
// (the value, or low/high halves of a 32-bit pattern) and combination (column multiplier a, row multiplier b,
// square): S = sum_c term(c) * ((c * a + 7) % 1021 + 1), then (S mod p) * ((row * b + 3) % 1019 + 1).
// out[block, 6]: those products summed over the block's rows (exact int64).
template <bool WIDE>
__global__ void fingerprint_kernel(const void* __restrict__ bits_ptr, int64_t s0, int64_t s1, int rows, int cols,
                                   int64_t row_start, long long prime, long long* __restrict__ out) {
  __shared__ long long acc[kFpRowsPerBlock][6];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kFpRowsPerBlock + warp;
  long long s[6] = {0, 0, 0, 0, 0, 0};
  if (row < rows) {
    for (int c = lane; c < cols; c += 32) {
      const long long w0 = (static_cast<long long>(c) * 37 + 7) % 1021 + 1;
      const long long w1 = (static_cast<long long>(c) * 613 + 7) % 1021 + 1;
      const long long w2 = (static_cast<long long>(c) * 1 + 7) % 1021 + 1;
      const int64_t off = static_cast<int64_t>(row) * s0 + static_cast<int64_t>(c) * s1;
      if (WIDE) {
        const long long v = static_cast<const int32_t*>(bits_ptr)[off];
        const long long low = v & 0xFFFF;
        const long long high = v >> 16;
        s[0] += low * w0;
        s[1] += low * w1;
        s[2] += low * low * w2;
        s[3] += high * w0;
        s[4] += high * w1;
        s[5] += high * high * w2;
      } else {
        const long long v = static_cast<const int16_t*>(bits_ptr)[off];
        s[0] += v * w0;
        s[1] += v * w1;
        s[2] += v * v * w2;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 6; ++k) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s[k] += __shfl_xor_sync(0xffffffffu, s[k], off);
  }
  if (lane == 0) {
    if (row < rows) {
      const long long grow = row_start + row;
      const long long r0 = (grow * 101 + 3) % 1019 + 1;
      const long long r1 = (grow * 211 + 3) % 1019 + 1;
      const long long r2 = (grow * 17 + 3) % 1019 + 1;
      acc[warp][0] = pymod(s[0], prime) * r0;
      acc[warp][1] = pymod(s[1], prime) * r1;
      acc[warp][2] = pymod(s[2], prime) * r2;
      acc[warp][3] = WIDE ? pymod(s[3], prime) * r0 : 0;
      acc[warp][4] = WIDE ? pymod(s[4], prime) * r1 : 0;
      acc[warp][5] = WIDE ? pymod(s[5], prime) * r2 : 0;
    } else {
      for (int k = 0; k < 6; ++k) acc[warp][k] = 0;
    }
  }
  __syncthreads();
  if (threadIdx.x < 6) {
    long long t = 0;
    for (int w = 0; w < kFpRowsPerBlock; ++w) t += acc[w][threadIdx.x];
    out[blockIdx.x * 6 + threadIdx.x] = t;
  }
}

// ---------------------------------------------------------------------------------------------------
// dot2_gemm
// ---------------------------------------------------------------------------------------------------

constexpr int kD2Tile = 64;
constexpr int kD2K = 16;

// out[n, r] = X[n, c] . R[r, c]^T (both FP32, unit inner stride) with Dot2 accumulation in k order.
// block (16, 16): each thread owns a 4 x 4 patch of the 64 x 64 tile.
__global__ void __launch_bounds__(256)
    dot2_gemm_kernel(const float* __restrict__ X, int64_t ldx, const float* __restrict__ R, int64_t ldr,
                     float* __restrict__ out, int64_t ldo, int n, int r, int c) {
  __shared__ float xs[kD2K][kD2Tile + 4];
  __shared__ float rs[kD2K][kD2Tile + 4];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int tid = ty * 16 + tx;
  const int m0 = blockIdx.x * kD2Tile, n0 = blockIdx.y * kD2Tile;
  float hi[4][4], lo[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hi[i][j] = 0.0f;
      lo[i][j] = 0.0f;
    }
  for (int k0 = 0; k0 < c; k0 += kD2K) {
    // 64 rows x 16 k of each operand: 1024 values, 4 per thread
    for (int e = tid; e < kD2Tile * kD2K; e += 256) {
      const int row = e / kD2K, kk = e % kD2K;
      const int k = k0 + kk;
      xs[kk][row] = (m0 + row < n && k < c) ? X[static_cast<int64_t>(m0 + row) * ldx + k] : 0.0f;
      rs[kk][row] = (n0 + row < r && k < c) ? R[static_cast<int64_t>(n0 + row) * ldr + k] : 0.0f;
    }
    __syncthreads();
    const int kmax = min(kD2K, c - k0);
    for (int kk = 0; kk < kmax; ++kk) {
      float a[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = rs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float p = __fmul_rn(a[i], bv[j]);
          const float e = __fmaf_rn(a[i], bv[j], -p);  // TwoProduct error term
          const float s = __fadd_rn(hi[i][j], p);       // TwoSum
          const float v = __fsub_rn(s, hi[i][j]);
          const float t = __fadd_rn(__fsub_rn(hi[i][j], __fsub_rn(s, v)), __fsub_rn(p, v));
          hi[i][j] = s;
          lo[i][j] = __fadd_rn(lo[i][j], __fadd_rn(t, e));
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = m0 + ty * 4 + i;
    if (row >= n) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = n0 + tx * 4 + j;
      if (col < r) out[static_cast<int64_t>(row) * ldo + col] = __fadd_rn(hi[i][j], lo[i][j]);
    }
  }
}

}  // namespace fit

// ---------------------------------------------------------------------------------------------------
// host entry points
// ---------------------------------------------------------------------------------------------------

void split_bf16x3(const at::Tensor& x, at::Tensor& out, int64_t kp, const std::vector<int64_t>& parts) {
  check_cuda_tensor(x, "x");
  check_cuda_tensor(out, "out");
  RC_CHECK(x.scalar_type() == at::kFloat && x.dim() == 2, "x must be a 2-D float32 matrix");
  RC_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.stride(1) == 1, "out must be 2-D bf16");
  const int R = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1));
  const int nseg = static_cast<int>(parts.size());
  RC_CHECK(nseg >= 1 && nseg <= 16, "1..16 segments");
  RC_CHECK(kp >= K && out.size(0) == R && out.size(1) >= nseg * kp, "out too small for the segments");
  RC_CHECK(x.stride(1) == 1 || x.stride(0) == 1, "x needs one unit stride");
  uint32_t pattern = 0;
  for (int s = 0; s < nseg; ++s) {
    RC_CHECK(parts[s] >= 0 && parts[s] <= 2, "parts are 0 (hi), 1 (mid) or 2 (lo)");
    pattern |= static_cast<uint32_t>(parts[s]) << (2 * s);
  }
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.get_device()).stream();
  dim3 grid((static_cast<int>(kp) + fit::kSplitTile - 1) / fit::kSplitTile, (R + fit::kSplitTile - 1) / fit::kSplitTile);
  fit::split_bf16x3_kernel<<<grid, dim3(32, 8), 0, stream>>>(
      x.data_ptr<float>(), x.stride(0), x.stride(1), R, K, static_cast<int>(kp),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), nseg, pattern);
  RC_CUDA(cudaGetLastError());
}

void jacobi_eigh(const at::Tensor& a, at::Tensor& values, at::Tensor& vectors, at::Tensor& info, at::Tensor& sweeps,
                 int64_t max_sweeps, double tol) {
  check_cuda_tensor(a, "a");
  RC_CHECK(a.scalar_type() == at::kFloat && a.dim() == 3 && a.is_contiguous(), "a must be contiguous [B, n, n] fp32");
  const int B = static_cast<int>(a.size(0)), n = static_cast<int>(a.size(1));
  RC_CHECK(a.size(2) == n && n >= 1 && n <= fit::kJacobiMaxN, "Jacobi kernel takes 1 <= n <= 160");
  RC_CHECK(values.is_contiguous() && values.scalar_type() == at::kFloat && values.numel() == int64_t(B) * n, "values");
  RC_CHECK(vectors.is_contiguous() && vectors.scalar_type() == at::kFloat && vectors.numel() == int64_t(B) * n * n,
           "vectors");
  RC_CHECK(info.is_contiguous() && info.scalar_type() == at::kInt && info.numel() == B, "info");
  RC_CHECK(sweeps.is_contiguous() && sweeps.scalar_type() == at::kInt && sweeps.numel() == B, "sweeps");
  RC_CHECK(max_sweeps >= 1 && max_sweeps <= 100, "max_sweeps in [1, 100]");
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(a.get_device()).stream();
  const int smem = fit::jacobi_smem_bytes(n);
  RC_CUDA(cudaFuncSetAttribute(fit::jacobi_eigh_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  fit::jacobi_eigh_kernel<<<B, fit::kJacobiThreads, smem, stream>>>(
      a.data_ptr<float>(), n, values.data_ptr<float>(), vectors.data_ptr<float>(), info.data_ptr<int>(),
      sweeps.data_ptr<int>(), static_cast<int>(max_sweeps), static_cast<float>(tol));
  RC_CUDA(cudaGetLastError());
}

template <typename TX>
static void sq_dispatch_r(const at::Tensor& x, const c10::optional<at::Tensor>& r, float scale, at::Tensor& out,
                          cudaStream_t stream, int blocks) {
  const int rows = static_cast<int>(x.size(0)), cols = static_cast<int>(x.size(1));
  const TX* xp = reinterpret_cast<const TX*>(x.data_ptr());
  double* op = out.data_ptr<double>();
  const bool div = scale != 0.0f;
  if (!r.has_value() || !r->defined()) {
    if (div)
      fit::sq_partials_kernel<TX, TX, false, true><<<blocks, fit::kSqThreads, 0, stream>>>(
          xp, x.stride(0), x.stride(1), xp, 0, 0, rows, cols, scale, op);
    else
      fit::sq_partials_kernel<TX, TX, false, false><<<blocks, fit::kSqThreads, 0, stream>>>(
          xp, x.stride(0), x.stride(1), xp, 0, 0, rows, cols, 1.0f, op);
    return;
  }
  RC_CHECK(r->scalar_type() == at::kFloat, "the reconstruction must be float32");
  const float* rp = r->data_ptr<float>();
  if (div)
    fit::sq_partials_kernel<TX, float, true, true><<<blocks, fit::kSqThreads, 0, stream>>>(
        xp, x.stride(0), x.stride(1), rp, r->stride(0), r->stride(1), rows, cols, scale, op);
  else
    fit::sq_partials_kernel<TX, float, true, false><<<blocks, fit::kSqThreads, 0, stream>>>(
        xp, x.stride(0), x.stride(1), rp, r->stride(0), r->stride(1), rows, cols, 1.0f, op);
}

void sq_partials(const at::Tensor& x, const c10::optional<at::Tensor>& r, double scale, at::Tensor& out) {
  check_cuda_tensor(x, "x");
  RC_CHECK(x.dim() == 2, "x must be 2-D");
  const int rows = static_cast<int>(x.size(0));
  const int blocks = (rows + fit::kSqRows - 1) / fit::kSqRows;
  RC_CHECK(out.scalar_type() == at::kDouble && out.is_contiguous() && out.numel() >= int64_t(blocks) * 3,
           "out must hold [ceil(rows / 8), 3] float64");
  if (r.has_value() && r->defined())
    RC_CHECK(r->dim() == 2 && r->size(0) == x.size(0) && r->size(1) == x.size(1), "r must match x");
  if (blocks == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.get_device()).stream();
  const float s = static_cast<float>(scale);
  switch (x.scalar_type()) {
    case at::kFloat:
      sq_dispatch_r<float>(x, r, s, out, stream, blocks);
      break;
    case at::kBFloat16:
      sq_dispatch_r<__nv_bfloat16>(x, r, s, out, stream, blocks);
      break;
    case at::kHalf:
      sq_dispatch_r<__half>(x, r, s, out, stream, blocks);
      break;
    default:
      RC_CHECK(false, "x must be float32, bfloat16 or float16");
  }
  RC_CUDA(cudaGetLastError());
}

void fingerprint_partials(const at::Tensor& bits, at::Tensor& out, int64_t row_start, int64_t prime) {
  check_cuda_tensor(bits, "bits");
  RC_CHECK(bits.dim() == 2, "bits must be 2-D");
  const bool wide = bits.scalar_type() == at::kInt;
  RC_CHECK(wide || bits.scalar_type() == at::kShort, "bits must be an int16 or int32 view");
  const int rows = static_cast<int>(bits.size(0)), cols = static_cast<int>(bits.size(1));
  RC_CHECK(cols <= (1 << 14) && rows <= (1 << 22), "fingerprint geometry exceeds its overflow-free range");
  const int blocks = (rows + fit::kFpRowsPerBlock - 1) / fit::kFpRowsPerBlock;
  RC_CHECK(out.scalar_type() == at::kLong && out.is_contiguous() && out.numel() >= int64_t(blocks) * 6,
           "out must hold [ceil(rows / 8), 6] int64");
  if (blocks == 0) return;
  c10::cuda::CUDAGuard guard(bits.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(bits.get_device()).stream();
  if (wide)
    fit::fingerprint_kernel<true><<<blocks, 32 * fit::kFpRowsPerBlock, 0, stream>>>(
        bits.data_ptr(), bits.stride(0), bits.stride(1), rows, cols, row_start, prime, reinterpret_cast<long long*>(out.data_ptr<int64_t>()));
  else
    fit::fingerprint_kernel<false><<<blocks, 32 * fit::kFpRowsPerBlock, 0, stream>>>(
        bits.data_ptr(), bits.stride(0), bits.stride(1), rows, cols, row_start, prime, reinterpret_cast<long long*>(out.data_ptr<int64_t>()));
  RC_CUDA(cudaGetLastError());
}

void dot2_gemm(const at::Tensor& x, const at::Tensor& rows, at::Tensor& out) {
  check_cuda_tensor(x, "x");
  check_cuda_tensor(rows, "rows");
  RC_CHECK(x.scalar_type() == at::kFloat && rows.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat,
           "dot2_gemm takes float32 operands");
  RC_CHECK(x.dim() == 2 && rows.dim() == 2 && x.stride(1) == 1 && rows.stride(1) == 1 && out.stride(1) == 1,
           "unit inner strides");
  const int n = static_cast<int>(x.size(0)), c = static_cast<int>(x.size(1)), r = static_cast<int>(rows.size(0));
  RC_CHECK(rows.size(1) == c && out.size(0) == n && out.size(1) == r, "shapes");
  if (n == 0 || r == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.get_device()).stream();
  dim3 grid((n + fit::kD2Tile - 1) / fit::kD2Tile, (r + fit::kD2Tile - 1) / fit::kD2Tile);
  fit::dot2_gemm_kernel<<<grid, dim3(16, 16), 0, stream>>>(x.data_ptr<float>(), x.stride(0), rows.data_ptr<float>(),
                                                           rows.stride(0), out.data_ptr<float>(), out.stride(0), n, r,
                                                           c);
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
