// DiT block elementwise kernels for sm_100a (memory-bound; one warp per token row, FP32 statistics):
//
//   ln_modulate      y = LayerNorm(x) * (1 + scale) + shift          (AdaLN; optional affine weight/bias)
//   qkv_norm_rope    from the fused QKV projection [T, 3C]: q = RoPE(RMSNorm(q) * wq),
//                    k_pre = RMSNorm(k) * wk (normalized pre-RoPE K, the archival capture),
//                    k = RoPE(k_pre) and v written straight into the KV-cache slots
//   rms_norm         y = RMSNorm(x) * w over the full row (cross-attention q / context k)
//
// RMSNorm spans all heads (Wan's qk-norm over the model width). RoPE rotates interleaved pairs with
// per-token FP32 cos/sin tables [T, head_dim / 2].
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cuda_bf16.h>

#include "../common/host.h"

namespace rc {
namespace norms {

constexpr int kMaxVec = 8;  // up to 8 x 16 bytes (64 bf16) per lane: rows up to 2048 channels

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Eight consecutive FP32 parameters p[c0 .. c0 + 8) with two 16-byte read-only loads (p 16-byte aligned,
// c0 a multiple of 8; the launchers check the alignment).
__device__ __forceinline__ void load_f32x8(const float* __restrict__ p, int c0, float* out) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p + c0));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + c0) + 1);
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// x, y: [rows, C] bf16 (row strides ldx, ldy); shift/scale: fp32 [C] (null = 0); weight/bias: fp32 [C]
template <int VEC>
__global__ void ln_modulate_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_bfloat16* __restrict__ y,
                                   int64_t ldy, int rows, int C, const float* __restrict__ shift,
                                   const float* __restrict__ scale, const float* __restrict__ weight,
                                   const float* __restrict__ bias, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[VEC * 8];
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * ldx);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C) unpack8(src[i * 32 + lane], v + i * 8);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i * 8 + e] = 0.0f;
  }
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < VEC * 8; ++i) s += v[i];
  const float mean = warp_sum(s) / C;
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[i * 8 + e] - mean;
        q += d * d;
      }
  }
  const float rstd = rsqrtf(warp_sum(q) / C + eps);
  uint4* dst = reinterpret_cast<uint4*>(y + static_cast<int64_t>(row) * ldy);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c0 = (i * 32 + lane) * 8;
    if (c0 >= C) continue;
    float o[8], wt[8], bs[8], sc[8], sh[8];
    if (weight != nullptr) {
      load_f32x8(weight, c0, wt);
      load_f32x8(bias, c0, bs);
    }
    if (scale != nullptr) load_f32x8(scale, c0, sc);
    if (shift != nullptr) load_f32x8(shift, c0, sh);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float t = (v[i * 8 + e] - mean) * rstd;
      if (weight != nullptr) t = fmaf(t, wt[e], bs[e]);
      if (scale != nullptr) t = fmaf(t, sc[e], t);
      o[e] = shift != nullptr ? t + sh[e] : t;
    }
    dst[i * 32 + lane] = pack8(o);
  }
}

// RMS-normalize one row of C channels held as VEC x 8 values per lane; returns the normalized values
template <int VEC>
__device__ __forceinline__ void rms_row(float* v, int C, int lane, const float* __restrict__ w, float eps) {
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < VEC * 8; ++i) q += v[i] * v[i];
  const float r = rsqrtf(warp_sum(q) / C + eps);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c0 = (i * 32 + lane) * 8;
    if (c0 >= C) continue;  // C is a multiple of 8: a lane's 8 channels are all in range or all out
    float wt[8];
    load_f32x8(w, c0, wt);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[i * 8 + e] = v[i * 8 + e] * r * wt[e];
  }
}

template <int VEC>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, int C, int lane, float* v) {
  const uint4* src = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C) unpack8(src[i * 32 + lane], v + i * 8);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i * 8 + e] = 0.0f;
  }
}

template <int VEC>
__device__ __forceinline__ void store_row(__nv_bfloat16* p, int C, int lane, const float* v) {
  uint4* dst = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < C) dst[i * 32 + lane] = pack8(v + i * 8);
  }
}

// rotate interleaved pairs: channel c (even) pairs with c + 1, pair index (c % head_dim) / 2
template <int VEC>
__device__ __forceinline__ void rope_row(float* v, int C, int lane, int head_dim, const float* __restrict__ cs,
                                         const float* __restrict__ sn) {
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c0 = (i * 32 + lane) * 8;
    if (c0 >= C) continue;
    const int pair0 = (c0 % head_dim) >> 1;
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs + pair0));
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(sn + pair0));
    const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float c = cv[e], s = sv[e];
      const float a = v[i * 8 + 2 * e], b = v[i * 8 + 2 * e + 1];
      v[i * 8 + 2 * e] = a * c - b * s;
      v[i * 8 + 2 * e + 1] = a * s + b * c;
    }
  }
}

// One warp per token: qkv row [3C] -> q_out [C], k_pre [C], k_cache [C], v_cache [C]
template <int VEC>
__global__ void qkv_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld_qkv, int rows, int C,
                                     int head_dim, const float* __restrict__ wq, const float* __restrict__ wk,
                                     const float* __restrict__ cos_tok, const float* __restrict__ sin_tok,
                                     __nv_bfloat16* __restrict__ q_out, int64_t ld_q,
                                     __nv_bfloat16* __restrict__ k_pre, int64_t ld_kp,
                                     __nv_bfloat16* __restrict__ k_cache, int64_t ld_k,
                                     __nv_bfloat16* __restrict__ v_cache, int64_t ld_v, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* src = qkv + static_cast<int64_t>(row) * ld_qkv;
  const float* cs = cos_tok + static_cast<int64_t>(row) * (head_dim / 2);
  const float* sn = sin_tok + static_cast<int64_t>(row) * (head_dim / 2);
  float v[VEC * 8];
  // q
  load_row<VEC>(src, C, lane, v);
  rms_row<VEC>(v, C, lane, wq, eps);
  rope_row<VEC>(v, C, lane, head_dim, cs, sn);
  store_row<VEC>(q_out + static_cast<int64_t>(row) * ld_q, C, lane, v);
  // k
  load_row<VEC>(src + C, C, lane, v);
  rms_row<VEC>(v, C, lane, wk, eps);
  if (k_pre != nullptr) store_row<VEC>(k_pre + static_cast<int64_t>(row) * ld_kp, C, lane, v);
  rope_row<VEC>(v, C, lane, head_dim, cs, sn);
  store_row<VEC>(k_cache + static_cast<int64_t>(row) * ld_k, C, lane, v);
  // v
  load_row<VEC>(src + 2 * C, C, lane, v);
  store_row<VEC>(v_cache + static_cast<int64_t>(row) * ld_v, C, lane, v);
}

template <int VEC>
__global__ void rms_norm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_bfloat16* __restrict__ y,
                                int64_t ldy, int rows, int C, const float* __restrict__ w, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[VEC * 8];
  load_row<VEC>(x + static_cast<int64_t>(row) * ldx, C, lane, v);
  rms_row<VEC>(v, C, lane, w, eps);
  store_row<VEC>(y + static_cast<int64_t>(row) * ldy, C, lane, v);
}

// Per-head RMSNorm and / or interleaved-pair RoPE of [tokens, heads, head_dim] rows (LongCat's q / k): one warp
// per (token, head); lane l holds head_dim / 32 consecutive elements, so every rotated pair stays in one lane.
template <int PER>
__global__ void head_norm_rope_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_ts, int64_t x_hs,
                                      __nv_bfloat16* __restrict__ y, int64_t y_ts, int64_t y_hs, int tokens,
                                      int heads, const float* __restrict__ w, const float* __restrict__ cos_tok,
                                      const float* __restrict__ sin_tok, float eps) {
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= tokens * heads) return;
  const int token = item / heads;
  const int head = item - token * heads;
  constexpr int kHeadDim = PER * 32;
  const __nv_bfloat16* src = x + static_cast<int64_t>(token) * x_ts + static_cast<int64_t>(head) * x_hs + lane * PER;
  float v[PER];
#pragma unroll
  for (int i = 0; i < PER; i += 2) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + i));
    v[i] = f.x;
    v[i + 1] = f.y;
  }
  if (w != nullptr) {
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, offset);
    const float r = rsqrtf(ss / kHeadDim + eps);
#pragma unroll
    for (int i = 0; i < PER; ++i) v[i] = v[i] * r * __ldg(w + lane * PER + i);
  }
  if (cos_tok != nullptr) {
    const float* cs = cos_tok + static_cast<int64_t>(token) * (kHeadDim / 2) + lane * (PER / 2);
    const float* sn = sin_tok + static_cast<int64_t>(token) * (kHeadDim / 2) + lane * (PER / 2);
#pragma unroll
    for (int i = 0; i < PER / 2; ++i) {
      const float c = __ldg(cs + i), s = __ldg(sn + i);
      const float a = v[2 * i], b = v[2 * i + 1];
      v[2 * i] = a * c - b * s;
      v[2 * i + 1] = a * s + b * c;
    }
  }
  __nv_bfloat16* dst = y + static_cast<int64_t>(token) * y_ts + static_cast<int64_t>(head) * y_hs + lane * PER;
#pragma unroll
  for (int i = 0; i < PER; i += 2)
    *reinterpret_cast<__nv_bfloat162*>(dst + i) = __floats2bfloat162_rn(v[i], v[i + 1]);
}

}  // namespace norms

namespace {
const float* opt_f32(const c10::optional<at::Tensor>& t, int64_t n, const char* name) {
  if (!t.has_value() || !t->defined()) return nullptr;
  RC_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == n &&
               reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
           std::string(name) + " must be a contiguous, 16-byte aligned CUDA float32 vector of the row width");
  return t->data_ptr<float>();
}

void check_rows(const at::Tensor& t, const char* name) {
  RC_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
               t.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
           std::string(name) + " must be a 16-byte aligned CUDA bfloat16 [rows, C] matrix");
}
}  // namespace

#define RC_VEC_DISPATCH(C, KERNEL, ...)                                        \
  do {                                                                         \
    const int vec = ((C) + 255) / 256;                                         \
    RC_CHECK((C) % 8 == 0 && vec >= 1 && vec <= norms::kMaxVec, "row width must be a multiple of 8, <= 2048"); \
    switch (vec) {                                                             \
      case 1: KERNEL<1><<<grid, 256, 0, stream>>>(__VA_ARGS__); break;         \
      case 2: KERNEL<2><<<grid, 256, 0, stream>>>(__VA_ARGS__); break;         \
      case 3: KERNEL<3><<<grid, 256, 0, stream>>>(__VA_ARGS__); break;         \
      case 4: KERNEL<4><<<grid, 256, 0, stream>>>(__VA_ARGS__); break;         \
      case 5: KERNEL<5><<<grid, 256, 0, stream>>>(__VA_ARGS__); break;         \
      case 6: KERNEL<6><<<grid, 256, 0, stream>>>(__VA_ARGS__); break;         \
      case 7: KERNEL<7><<<grid, 256, 0, stream>>>(__VA_ARGS__); break;         \
      default: KERNEL<8><<<grid, 256, 0, stream>>>(__VA_ARGS__); break;        \
    }                                                                          \
    RC_CUDA(cudaGetLastError());                                               \
  } while (0)

void ln_modulate(const at::Tensor& x, at::Tensor& y, const c10::optional<at::Tensor>& shift,
                 const c10::optional<at::Tensor>& scale, const c10::optional<at::Tensor>& weight,
                 const c10::optional<at::Tensor>& bias, double eps) {
  check_rows(x, "x");
  check_rows(y, "y");
  const int rows = static_cast<int>(x.size(0));
  const int C = static_cast<int>(x.size(1));
  RC_CHECK(y.size(0) == rows && y.size(1) == C, "y must match x");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.get_device()).stream();
  dim3 grid((rows + 7) / 8);
  RC_VEC_DISPATCH(C, norms::ln_modulate_kernel, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                  reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0), rows, C, opt_f32(shift, C, "shift"),
                  opt_f32(scale, C, "scale"), opt_f32(weight, C, "weight"), opt_f32(bias, C, "bias"),
                  static_cast<float>(eps));
}

void qkv_norm_rope(const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& cos_tok,
                   const at::Tensor& sin_tok, at::Tensor& q_out, const c10::optional<at::Tensor>& k_pre,
                   at::Tensor& k_cache, at::Tensor& v_cache, int64_t head_dim, double eps) {
  check_rows(qkv, "qkv");
  check_rows(q_out, "q_out");
  check_rows(k_cache, "k_cache");
  check_rows(v_cache, "v_cache");
  const int rows = static_cast<int>(qkv.size(0));
  const int C = static_cast<int>(qkv.size(1) / 3);
  RC_CHECK(qkv.size(1) == 3 * C && q_out.size(1) == C && k_cache.size(1) == C && v_cache.size(1) == C &&
               q_out.size(0) == rows && k_cache.size(0) == rows && v_cache.size(0) == rows,
           "qkv is [T, 3C]; outputs are [T, C]");
  RC_CHECK(cos_tok.is_cuda() && cos_tok.scalar_type() == at::kFloat && cos_tok.is_contiguous() &&
               cos_tok.size(0) == rows && cos_tok.size(1) * 2 == head_dim && sin_tok.sizes() == cos_tok.sizes() &&
               sin_tok.is_contiguous() && reinterpret_cast<uintptr_t>(cos_tok.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(sin_tok.data_ptr()) % 16 == 0 && head_dim % 8 == 0,
           "cos/sin must be 16-byte aligned float32 [T, head_dim / 2] per-token tables");
  __nv_bfloat16* kp = nullptr;
  int64_t ld_kp = 0;
  if (k_pre.has_value() && k_pre->defined()) {
    check_rows(*k_pre, "k_pre");
    kp = reinterpret_cast<__nv_bfloat16*>(k_pre->data_ptr());
    ld_kp = k_pre->stride(0);
  }
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(qkv.get_device()).stream();
  dim3 grid((rows + 7) / 8);
  RC_VEC_DISPATCH(C, norms::qkv_norm_rope_kernel, reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                  qkv.stride(0), rows, C, static_cast<int>(head_dim), opt_f32(wq, C, "wq"), opt_f32(wk, C, "wk"),
                  cos_tok.data_ptr<float>(), sin_tok.data_ptr<float>(),
                  reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), q_out.stride(0), kp, ld_kp,
                  reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()), k_cache.stride(0),
                  reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), v_cache.stride(0), static_cast<float>(eps));
}

void rms_norm(const at::Tensor& x, at::Tensor& y, const at::Tensor& w, double eps) {
  check_rows(x, "x");
  check_rows(y, "y");
  const int rows = static_cast<int>(x.size(0));
  const int C = static_cast<int>(x.size(1));
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.get_device()).stream();
  dim3 grid((rows + 7) / 8);
  RC_VEC_DISPATCH(C, norms::rms_norm_kernel, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                  reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0), rows, C, opt_f32(w, C, "w"),
                  static_cast<float>(eps));
}

void head_norm_rope(const at::Tensor& x, at::Tensor& y, const c10::optional<at::Tensor>& w,
                    const c10::optional<at::Tensor>& cos_tok, const c10::optional<at::Tensor>& sin_tok, double eps) {
  RC_CHECK(x.is_cuda() && y.is_cuda() && x.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16 &&
               x.dim() == 3 && y.dim() == 3 && x.sizes() == y.sizes() && x.stride(2) == 1 && y.stride(2) == 1,
           "x and y must be CUDA bfloat16 [tokens, heads, head_dim] with unit inner stride");
  const int tokens = static_cast<int>(x.size(0)), heads = static_cast<int>(x.size(1));
  const int head_dim = static_cast<int>(x.size(2));
  RC_CHECK(head_dim == 64 || head_dim == 128 || head_dim == 256, "head_dim must be 64, 128 or 256");
  RC_CHECK(x.stride(0) % 2 == 0 && x.stride(1) % 2 == 0 && y.stride(0) % 2 == 0 && y.stride(1) % 2 == 0 &&
               reinterpret_cast<uintptr_t>(x.data_ptr()) % 4 == 0 && reinterpret_cast<uintptr_t>(y.data_ptr()) % 4 == 0,
           "rows must be 4-byte aligned");
  const float* wp = opt_f32(w, head_dim, "w");
  RC_CHECK(cos_tok.has_value() == sin_tok.has_value(), "cos and sin come together");
  const float* cp = nullptr;
  const float* sp = nullptr;
  if (cos_tok.has_value() && cos_tok->defined()) {
    RC_CHECK(cos_tok->is_cuda() && cos_tok->scalar_type() == at::kFloat && cos_tok->is_contiguous() &&
                 sin_tok->is_contiguous() && cos_tok->numel() == static_cast<int64_t>(tokens) * (head_dim / 2) &&
                 sin_tok->numel() == cos_tok->numel(),
             "cos / sin must be contiguous CUDA float32 [tokens, head_dim / 2]");
    cp = cos_tok->data_ptr<float>();
    sp = sin_tok->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.get_device()).stream();
  const int64_t items = static_cast<int64_t>(tokens) * heads;
  if (items == 0) return;
  dim3 grid(static_cast<unsigned>((items + 7) / 8));
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  switch (head_dim) {
    case 64:
      norms::head_norm_rope_kernel<2><<<grid, 256, 0, stream>>>(xp, x.stride(0), x.stride(1), yp, y.stride(0),
                                                                y.stride(1), tokens, heads, wp, cp, sp, (float)eps);
      break;
    case 128:
      norms::head_norm_rope_kernel<4><<<grid, 256, 0, stream>>>(xp, x.stride(0), x.stride(1), yp, y.stride(0),
                                                                y.stride(1), tokens, heads, wp, cp, sp, (float)eps);
      break;
    default:
      norms::head_norm_rope_kernel<8><<<grid, 256, 0, stream>>>(xp, x.stride(0), x.stride(1), yp, y.stride(0),
                                                                y.stride(1), tokens, heads, wp, cp, sp, (float)eps);
  }
  RC_CUDA(cudaGetLastError());
}

}  // namespace rc
