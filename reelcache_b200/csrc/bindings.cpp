// Python bindings of the reelcache_b200 native extension (CUDA kernels for sm_100a and the C++
// host fast paths).
#include <torch/extension.h>

#include <vector>

namespace rc {
int64_t pread_many(const std::vector<std::string>& paths, const std::vector<int64_t>& offsets,
                   const std::vector<int64_t>& sizes, const std::vector<int64_t>& dest, int64_t threads);
std::vector<int64_t> start_codes(const at::Tensor& data);
at::Tensor nal_units(const at::Tensor& data);
at::Tensor unmosaic_all(const at::Tensor& images, int64_t frames, int64_t height, int64_t width, int64_t rank,
                        int64_t columns, int64_t planes, int64_t slots);
void gemm_bf16_tn(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epilogue,
                  const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& gate,
                  const c10::optional<at::Tensor>& resid, double alpha, int64_t bn,
                  const c10::optional<at::Tensor>& status);
at::Tensor restore_build(const at::Tensor& jobs, const std::vector<at::Tensor>& a_ops,
                         const std::vector<at::Tensor>& b_ops, const at::Tensor& inverse);
void restore_run(const at::Tensor& blob, int64_t device, const c10::optional<at::Tensor>& status, int64_t options);
void prep_launch(const at::Tensor& jobs, int64_t device);
void colminmax(const at::Tensor& p, at::Tensor& lo, at::Tensor& hi, at::Tensor& bad);
void ln_modulate(const at::Tensor& x, at::Tensor& y, const c10::optional<at::Tensor>& shift,
                 const c10::optional<at::Tensor>& scale, const c10::optional<at::Tensor>& weight,
                 const c10::optional<at::Tensor>& bias, double eps);
void qkv_norm_rope(const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& cos_tok,
                   const at::Tensor& sin_tok, at::Tensor& q_out, const c10::optional<at::Tensor>& k_pre,
                   at::Tensor& k_cache, at::Tensor& v_cache, int64_t head_dim, double eps);
void rms_norm(const at::Tensor& x, at::Tensor& y, const at::Tensor& w, double eps);
void head_norm_rope(const at::Tensor& x, at::Tensor& y, const c10::optional<at::Tensor>& w,
                    const c10::optional<at::Tensor>& cos_tok, const c10::optional<at::Tensor>& sin_tok, double eps);
void quantize_columns(const at::Tensor& p, const at::Tensor& scale, const at::Tensor& offset, at::Tensor& out);
void rope_store_launch(const at::Tensor& jobs);
void unpack_launch(const at::Tensor& jobs, int64_t device);
void split_bf16x3(const at::Tensor& x, at::Tensor& out, int64_t kp, const std::vector<int64_t>& parts);
void jacobi_eigh(const at::Tensor& a, at::Tensor& values, at::Tensor& vectors, at::Tensor& info, at::Tensor& sweeps,
                 int64_t max_sweeps, double tol);
void sq_partials(const at::Tensor& x, const c10::optional<at::Tensor>& r, double scale, at::Tensor& out);
void fingerprint_partials(const at::Tensor& bits, at::Tensor& out, int64_t row_start, int64_t prime);
void dot2_gemm(const at::Tensor& x, const at::Tensor& rows, at::Tensor& out);
void attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& out, double scale,
                   const c10::optional<at::Tensor>& status, int64_t options, const c10::optional<at::Tensor>& trace);
void mosaic_u8(const at::Tensor& pixels, at::Tensor& canvas, const std::vector<int64_t>& geometry);
void gemm_bf16_promoted(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, double alpha,
                        const c10::optional<at::Tensor>& status);
void ulysses_qkv(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                 const std::vector<at::Tensor>& dst_q, const std::vector<at::Tensor>& dst_k,
                 const std::vector<at::Tensor>& dst_v, int64_t rank, int64_t head_dim,
                 const c10::optional<at::Tensor>& status);
void ulysses_out(const std::vector<at::Tensor>& o_owners, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                 const c10::optional<at::Tensor>& gate, at::Tensor& out, int64_t rank, int64_t n_loc,
                 int64_t epilogue, const at::Tensor& stage, const at::Tensor& tile_flags, int64_t call,
                 const c10::optional<at::Tensor>& status);
void peer_barrier(const at::Tensor& flags, int64_t rank, int64_t epoch, const c10::optional<at::Tensor>& status);
void nvls_reduce_upper(int64_t mc_ptr, int64_t buffer_elems, const at::Tensor& offsets, at::Tensor& out, int64_t C);
void gram_reduce_scatter(const at::Tensor& xt, int64_t matrices, const std::vector<at::Tensor>& partials,
                         const at::Tensor& owners, const at::Tensor& slots, int64_t rank,
                         const c10::optional<at::Tensor>& status, bool to_local);
}  // namespace rc

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "reelcache_b200 native kernels (sm_100a) and host fast paths";
  m.def("gemm_bf16_tn", &rc::gemm_bf16_tn, "out = epilogue(alpha * A @ B^T) on tcgen05", py::arg("A"),
        py::arg("B"), py::arg("out"), py::arg("epilogue") = 0, py::arg("bias") = py::none(),
        py::arg("gate") = py::none(), py::arg("resid") = py::none(), py::arg("alpha") = 1.0, py::arg("bn") = 0,
        py::arg("status") = py::none());
  m.def("ulysses_qkv", &rc::ulysses_qkv, "QKV projection GEMM with the Ulysses head scatter fused (peer stores)",
        py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("dst_q"), py::arg("dst_k"), py::arg("dst_v"),
        py::arg("rank"), py::arg("head_dim"), py::arg("status") = py::none());
  m.def("ulysses_out", &rc::ulysses_out, "output projection GEMM with the Ulysses token gather fused (peer TMA loads)",
        py::arg("o_owners"), py::arg("w"), py::arg("bias"), py::arg("gate"), py::arg("out"), py::arg("rank"),
        py::arg("n_loc"), py::arg("epilogue"), py::arg("stage"), py::arg("tile_flags"), py::arg("call"),
        py::arg("status") = py::none());
  m.def("nvls_reduce_upper", &rc::nvls_reduce_upper,
        "in-switch (NVLS multimem.ld_reduce) sum of symmetric C x C partials, upper 128 x 128 tiles",
        py::arg("mc_ptr"), py::arg("buffer_elems"), py::arg("offsets"), py::arg("out"), py::arg("C"));
  m.def("peer_barrier", &rc::peer_barrier, "bounded device-side barrier over peer flag words", py::arg("flags"),
        py::arg("rank"), py::arg("epoch"), py::arg("status") = py::none());
  m.def("gram_reduce_scatter", &rc::gram_reduce_scatter,
        "upper-triangular partial Grams of this rank's token shard stored into the owners' buffers (peer stores)",
        py::arg("xt"), py::arg("matrices"), py::arg("partials"), py::arg("owners"), py::arg("slots"), py::arg("rank"),
        py::arg("status") = py::none(), py::arg("to_local") = false);
  m.def("restore_build", &rc::restore_build, "launch parameters of a fused restore over <= 48 jobs",
        py::arg("jobs"), py::arg("a_ops"), py::arg("b_ops"), py::arg("inverse"));
  m.def("restore_run", &rc::restore_run, "launch a fused restore from restore_build parameters", py::arg("blob"),
        py::arg("device"), py::arg("status") = py::none(), py::arg("options") = 0);
  m.def("colminmax", &rc::colminmax, "per-column extrema of FP32 coefficients", py::arg("p"), py::arg("lo"),
        py::arg("hi"), py::arg("bad"));
  m.def("quantize_columns", &rc::quantize_columns, "FP64 rint quantization of coefficients to uint8",
        py::arg("p"), py::arg("scale"), py::arg("offset"), py::arg("out"));
  m.def("ln_modulate", &rc::ln_modulate, "y = LayerNorm(x) * (1 + scale) + shift", py::arg("x"), py::arg("y"),
        py::arg("shift") = py::none(), py::arg("scale") = py::none(), py::arg("weight") = py::none(),
        py::arg("bias") = py::none(), py::arg("eps") = 1e-6);
  m.def("qkv_norm_rope", &rc::qkv_norm_rope, "q/k RMSNorm + RoPE from fused qkv into q and KV-cache slots",
        py::arg("qkv"), py::arg("wq"), py::arg("wk"), py::arg("cos_tok"), py::arg("sin_tok"), py::arg("q_out"),
        py::arg("k_pre"), py::arg("k_cache"), py::arg("v_cache"), py::arg("head_dim"), py::arg("eps") = 1e-6);
  m.def("head_norm_rope", &rc::head_norm_rope, "per-head RMSNorm and / or interleaved RoPE of [T, H, D]",
        py::arg("x"), py::arg("y"), py::arg("w"), py::arg("cos_tok"), py::arg("sin_tok"), py::arg("eps"));
  m.def("rms_norm", &rc::rms_norm, "y = RMSNorm(x) * w", py::arg("x"), py::arg("y"), py::arg("w"),
        py::arg("eps") = 1e-6);
  m.def("prep_launch", &rc::prep_launch, "scaled hi/lo basis + bias preparation over <= 48 jobs", py::arg("jobs"),
        py::arg("device"));
  m.def("rope_store_launch", &rc::rope_store_launch, "dense RoPE + cast + strided store over <= 48 jobs",
        py::arg("jobs"));
  m.def("unpack_launch", &rc::unpack_launch, "mosaic pictures -> dense uint8 [N, K_pad] over <= 48 jobs",
        py::arg("jobs"), py::arg("device"));
  m.def("pread_many", &rc::pread_many, "parallel positioned reads into host memory (GIL released)",
        py::arg("paths"), py::arg("offsets"), py::arg("sizes"), py::arg("dest"), py::arg("threads") = 8);
  m.def("start_codes", &rc::start_codes, "Annex-B start-code offsets of a CPU uint8 tensor", py::arg("data"));
  m.def("nal_units", &rc::nal_units, "NAL-unit table [n, 3] (offset, length, type) of an Annex-B stream (GIL released)",
        py::arg("data"), py::call_guard<py::gil_scoped_release>());
  m.def("unmosaic_all", &rc::unmosaic_all, "channel-tile pictures back to [tokens, rank] coefficients (GIL released)",
        py::arg("images"), py::arg("frames"), py::arg("height"), py::arg("width"), py::arg("rank"), py::arg("columns"),
        py::arg("planes"), py::arg("slots"), py::call_guard<py::gil_scoped_release>());
  m.def("split_bf16x3", &rc::split_bf16x3, "FP32 -> K-concatenated bf16 hi/mid/lo segments", py::arg("x"),
        py::arg("out"), py::arg("kp"), py::arg("parts"));
  m.def("jacobi_eigh", &rc::jacobi_eigh, "batched FP32 Jacobi eigendecomposition (n <= 160)", py::arg("a"),
        py::arg("values"), py::arg("vectors"), py::arg("info"), py::arg("sweeps"), py::arg("max_sweeps"),
        py::arg("tol"));
  m.def("sq_partials", &rc::sq_partials, "FP64 partial sums of (x/s)^2 and ((x-r)/s)^2 per 8 rows", py::arg("x"),
        py::arg("r"), py::arg("scale"), py::arg("out"));
  m.def("fingerprint_partials", &rc::fingerprint_partials, "exact int64 fingerprint partials per 8 rows",
        py::arg("bits"), py::arg("out"), py::arg("row_start"), py::arg("prime"));
  m.def("gemm_bf16_promoted", &rc::gemm_bf16_promoted,
        "out = alpha * A @ B^T (bf16, K-major) with TMEM partials promoted to FP32 registers every 128 K",
        py::arg("A"), py::arg("B"), py::arg("out"), py::arg("alpha") = 1.0, py::arg("status") = py::none());
  m.def("attention_fwd", &rc::attention_fwd, "flash-attention forward on tcgen05 (bf16, head_dim 128)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"), py::arg("scale"), py::arg("status") = py::none(),
        py::arg("options") = 0, py::arg("trace") = py::none());
  m.def("mosaic_u8", &rc::mosaic_u8, "channel-tile mosaic of u8 coefficients into a canvas", py::arg("pixels"),
        py::arg("canvas"), py::arg("geometry"));
  m.def("dot2_gemm", &rc::dot2_gemm, "compensated FP32 GEMM out = x @ rows^T", py::arg("x"), py::arg("rows"),
        py::arg("out"));
}
